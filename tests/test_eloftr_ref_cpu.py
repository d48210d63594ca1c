# SPDX-License-Identifier: Unlicense
"""The reference's own Efficient LoFTR device stage, run here: its
pth_open, eloftr_load, eloftr_alloc and eloftr_match with its ops.c and
OpenCL kernels, unchanged, on the CPU (oracle/_ref/libref_cpu.so over
oracle/cl_backend_emul.c; the test skips when it has not been built),
against the ELoFTR oracle (oracle/eloftr_ref.py), on the seeded synthetic
weights and a band-limited 64 x 64 grey pair shifted by 8 pixels. The
reference's own debug dumps (eloftr.c:638-681) pin every stage of the
oracle: backbone, transformer and fusion features each within relative
L2 1e-5; then the same coarse matches in the same order, confidences and
refined keypoints within 1e-5. CPU only (about 30 s: the emulation runs
every work-item as C on the host)."""

import ctypes as C
import os
import tempfile
from pathlib import Path

import numpy as np
import pytest

from coreg import synth
from oracle import eloftr_ref

LIB = Path(__file__).resolve().parents[1] / "oracle" / "_ref" / "libref_cpu.so"
CACHE = Path(os.environ.get("COREG_CACHE", Path(tempfile.gettempdir()) / "coreg_cache"))


@pytest.fixture(scope="module")
def ref():
    if not LIB.exists():
        pytest.skip("oracle/_ref/libref_cpu.so not built (make -C oracle)")
    lib = C.CDLL(str(LIB))
    P, I, FL = C.c_void_p, C.c_int, C.c_float
    lib.ref_eloftr_run.restype = I
    lib.ref_eloftr_run.argtypes = [C.c_char_p, P, P, I, I, FL, I, P, P, P, P, C.c_char_p]
    return lib


def test_eloftr_stage_matches_the_reference(ref, tmp_path):
    wpath = synth.write_eloftr_weights(CACHE / "weights", 0)
    H = W = 64
    rng = np.random.default_rng(5)
    base = synth.band_limited(rng, H + 8, W + 8, 3.0) / 255.0
    g0 = np.ascontiguousarray(base[8:, 8:], np.float32)
    g1 = np.ascontiguousarray(base[:H, :W], np.float32)
    cap = 1024
    mi = np.zeros(cap, np.int32)
    mj = np.zeros(cap, np.int32)
    mc = np.zeros(cap, np.float32)
    kp = np.zeros((cap, 4), np.float32)
    n = ref.ref_eloftr_run(str(wpath).encode(), g0.ctypes.data, g1.ctypes.data, H, W, 1.0, cap,
                           mi.ctypes.data, mj.ctypes.data, mc.ctypes.data, kp.ctypes.data,
                           str(tmp_path).encode())
    model = eloftr_ref.Model(synth.read_safetensors(wpath), pos_scale=1.0)
    want_i, want_j, want_c, want_kp, dumps = model.run(g0, g1)
    for name, want in dumps.items():
        got = np.fromfile(tmp_path / f"tile001_eloftr_{name}.f32", np.float32)
        want = np.asarray(want, np.float32).ravel()
        assert got.shape == want.shape, name
        assert np.linalg.norm(got - want) / np.linalg.norm(want) <= 1e-5, name
    assert n == len(want_i) > 0
    assert np.array_equal(mi[:n], want_i)
    assert np.array_equal(mj[:n], want_j)
    assert np.abs(mc[:n] - want_c).max() <= 1e-5
    assert np.abs(kp[:n] - want_kp).max() <= 1e-5
