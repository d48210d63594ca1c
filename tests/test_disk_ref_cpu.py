# SPDX-License-Identifier: Unlicense
"""The reference's own DISK device stage, run here: its pth_open,
disk_load, disk_alloc and disk_detect with its ops.c and OpenCL kernels,
unchanged, on the CPU (oracle/_ref/libref_cpu.so over
oracle/cl_backend_emul.c; the test skips when it has not been built),
against the DISK oracle (oracle/disk_ref.py), on the seeded synthetic
weights and a band-limited 48 x 48 image (44 x 44 valid). This pins the
oracle's U-Net, NMS, selection and descriptors to the reference itself:
network output relative L2 <= 1e-5, the same keypoints in the same
order, scores and descriptors within 1e-5. CPU only (about 25 s: the
emulation runs every work-item as C on the host)."""

import ctypes as C
import os
import tempfile
from pathlib import Path

import numpy as np
import pytest

from coreg import synth
from oracle import disk_ref

LIB = Path(__file__).resolve().parents[1] / "oracle" / "_ref" / "libref_cpu.so"
CACHE = Path(os.environ.get("COREG_CACHE", Path(tempfile.gettempdir()) / "coreg_cache"))


@pytest.fixture(scope="module")
def ref():
    if not LIB.exists():
        pytest.skip("oracle/_ref/libref_cpu.so not built (make -C oracle)")
    lib = C.CDLL(str(LIB))
    P, I, FL = C.c_void_p, C.c_int, C.c_float
    lib.ref_disk_run.restype = I
    lib.ref_disk_run.argtypes = [C.c_char_p, P, I, I, I, I, I, FL, P, P, P, P, P]
    return lib


def test_disk_stage_matches_the_reference(ref):
    wpath = synth.write_disk_weights(CACHE / "weights", 0)
    H = W = 48
    h = w = 44
    n = 32
    rng = np.random.default_rng(1)
    img = (np.stack([synth.band_limited(rng, H, W, 2.0) for _ in range(3)]) / 255.0)
    img = np.ascontiguousarray(img, np.float32)
    xy = np.zeros((n, 2), np.int32)
    score = np.zeros(n, np.float32)
    desc = np.zeros((n, disk_ref.DESC), np.float32)
    net = np.zeros((disk_ref.DESC + 1, H, W), np.float32)
    k = ref.ref_disk_run(str(wpath).encode(), img.ctypes.data, H, W, h, w, n, 0.0, None,
                         xy.ctypes.data, score.ctypes.data, desc.ctypes.data, net.ctypes.data)
    out, want_xy, want_score, want_desc = disk_ref.detect(img, synth.read_safetensors(wpath), h,
                                                          w, n)
    assert np.linalg.norm(net - out) / np.linalg.norm(out) <= 1e-5
    assert k == len(want_xy) > 5
    assert np.array_equal(xy[:k], want_xy)
    assert np.abs(score[:k] - want_score).max() <= 1e-5
    assert np.abs(desc[:k] - want_desc).max() <= 1e-5
