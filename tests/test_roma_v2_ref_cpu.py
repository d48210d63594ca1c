# SPDX-License-Identifier: Unlicense
"""The reference's own RoMa v2 refiners, run here: its roma_load_v2,
roma_alloc, vgg2 and refiners2 (the second pass, at the tile's size) with
its ops.c and OpenCL kernels, unchanged, on the CPU
(oracle/_ref/libref_cpu.so over oracle/cl_backend_emul.c; the test skips
when it has not been built), against the RoMa oracle's vgg and refiners2
(oracle/roma_ref.py, float64), on seeded synthetic refiner weights, a
band-limited 48 x 48 image pair and a smooth warp on a 24 x 24 grid. This
pins the oracle's wiring of RoMa v2's refiners to the reference: the
feature pyramid and projections, the resampling between scales, the
precision reset, each refiner's input concatenation, local correlation,
depthwise-pointwise stack, heads and update. Warp within 1e-5 (in
normalized coordinates, under 1e-3 px), confidence within relative L2
1e-5."""

import ctypes as C
import os
import tempfile
import types
from pathlib import Path

import numpy as np
import pytest
import torch

from coreg import synth
from oracle import roma_ref as R

LIB = Path(__file__).resolve().parents[1] / "oracle" / "_ref" / "libref_cpu.so"
CACHE = Path(os.environ.get("COREG_CACHE", Path(tempfile.gettempdir()) / "coreg_cache"))


@pytest.fixture(scope="module")
def ref():
    if not LIB.exists():
        pytest.skip("oracle/_ref/libref_cpu.so not built (make -C oracle)")
    lib = C.CDLL(str(LIB))
    P, I = C.c_void_p, C.c_int
    lib.ref_roma_v2_refiners.restype = None
    lib.ref_roma_v2_refiners.argtypes = [C.c_char_p, P, P, I, I, I, I, P, P, P, P]
    return lib


def oracle_refiners(v2, imgs, H, W, h, w, flow, conf):
    """The oracle's second pass: vgg2 features of both images, then
    Runner.refiners2 with the precision cleared."""
    model = types.SimpleNamespace(imagenet=True, vgg2=R.Model._vgg(v2, "refiner_features.layers",
                                                                     3),
                                  ref2=[R.Model._refiner2(R.Model, v2, j) for j in range(3)])
    run = R.Runner.__new__(R.Runner)
    run.m, run.dt, run.dumps = model, torch.float64, {}
    P2 = [[None, None] for _ in range(3)]

    def keep(s):
        def f(x, k):
            r = model.ref2[s]
            P2[s][k] = run.t(r["proj_w"]) @ x.reshape(x.shape[0], -1) + run.t(r["proj_b"])[:, None]
        return f

    for k in range(2):
        img = run.t(R.prepare(imgs[k], H, W, True))
        run.vgg(img, k, P2, [keep(2 - blk) for blk in range(3)], model.vgg2)
    fl, cf, _, _ = run.refiners2(1, H, W, h, w, run.t(flow).reshape(2, -1),
                                 run.t(conf).reshape(4, -1), True, P2)
    return fl.numpy(), cf.numpy()


def test_roma_v2_refiners_match_the_reference(ref):
    path = CACHE / "weights" / "romav2_refiners_only_seed0.safetensors"
    v2 = synth.roma_v2_weights(0)
    if not path.exists():
        path.parent.mkdir(parents=True, exist_ok=True)
        tmp = path.with_suffix(".tmp")
        synth.write_safetensors(tmp, v2)
        tmp.rename(path)
    H = W = 48
    h = w = 24
    rng = np.random.default_rng(3)
    imgs = [np.ascontiguousarray(np.stack([synth.band_limited(rng, H, W, 2.0) for _ in range(3)])
                                 / 255.0, np.float32) for _ in range(2)]
    gy, gx = np.meshgrid((np.arange(h) + 0.5) / h * 2 - 1, (np.arange(w) + 0.5) / w * 2 - 1,
                         indexing="ij")
    flow = np.stack([gx + 0.05 + 0.03 * np.sin(3 * gy), gy - 0.04 + 0.02 * np.cos(2 * gx)])
    flow = np.ascontiguousarray(flow, np.float32)
    conf = np.ascontiguousarray(rng.normal(0, 1, (4, h, w)), np.float32)
    got_f = np.zeros((2, H * W), np.float32)
    got_c = np.zeros((4, H * W), np.float32)
    ref.ref_roma_v2_refiners(str(path).encode(), imgs[0].ctypes.data, imgs[1].ctypes.data, H, W,
                             h, w, flow.ctypes.data, conf.ctypes.data, got_f.ctypes.data,
                             got_c.ctypes.data)
    want_f, want_c = oracle_refiners(v2, imgs, H, W, h, w, flow, conf)
    assert np.isfinite(got_f).all() and np.isfinite(got_c).all()
    assert np.abs(got_f - want_f).max() <= 1e-5
    assert np.linalg.norm(got_c - want_c) / np.linalg.norm(want_c) <= 1e-5
