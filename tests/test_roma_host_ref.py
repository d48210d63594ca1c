# SPDX-License-Identifier: Unlicense
"""RoMa's host-side arithmetic in the oracle (oracle/roma_ref.py) against
the reference's own roma.c, compiled where it lies behind the harness
oracle/roma_host_ref.c into oracle/_ref/libroma_host_ref.so by
oracle/Makefile (the tests skip when it has not been built). CPU only.

* gp_solve (roma.c:772-836): the Gaussian process's float64 Cholesky solve
  of (K + 0.1 I) X = F on cosine-kernel matrices, up to the full coarse
  size (n = 1600 tokens, d = 512 basis columns). The reference rounds X to
  float32; the oracle's float64 X rounds to the same floats.
* prepare (roma.c:1159-1186): the antialiased bicubic input resampling,
  with and without the ImageNet normalization: bit-exact.
* interp_pos (roma.c:261-298): DINOv2's position table interpolated to the
  40 x 40 coarse grid: bit-exact."""

import ctypes as C
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import roma_ref

LIB = Path(__file__).resolve().parents[1] / "oracle" / "_ref" / "libroma_host_ref.so"


@pytest.fixture(scope="module")
def ref():
    if not LIB.exists():
        pytest.skip("oracle/_ref/libroma_host_ref.so not built (make -C oracle)")
    lib = C.CDLL(str(LIB))
    P, I = C.c_void_p, C.c_int
    lib.ref_gp_solve.argtypes = [P, I, P, I]
    lib.ref_prepare.argtypes = [P, I, I, P, I, I, I]
    lib.ref_interp_pos.restype = C.POINTER(C.c_float)
    lib.ref_interp_pos.argtypes = [P]
    return lib


def cos_kernel(rng, n, dim=512, smooth=0.0):
    f = rng.standard_normal((n, dim))
    if smooth:
        f = smooth * np.cumsum(f, 0) / np.sqrt(np.arange(1, n + 1))[:, None] + (1 - smooth) * f
    fn = f / np.linalg.norm(f, axis=1, keepdims=True)
    return np.exp((fn @ fn.T - 1.0) / 0.2).astype(np.float32)


@pytest.mark.parametrize("n,d,smooth", [(300, 64, 0.0), (800, 128, 0.9), (1600, 512, 0.5)])
def test_gp_solve_matches_reference(ref, n, d, smooth):
    rng = np.random.default_rng(n)
    K = cos_kernel(rng, n, smooth=smooth)
    F = rng.standard_normal((n, d)).astype(np.float32)
    want = F.copy()
    ref.ref_gp_solve(K.ctypes.data, n, want.ctypes.data, d)
    got = roma_ref.gp_solve(torch.from_numpy(K), torch.from_numpy(F)).numpy()
    assert np.linalg.norm(got - want) / np.linalg.norm(want) <= 1e-6
    assert np.mean(got.astype(np.float32) == want) >= 0.999


@pytest.mark.parametrize("H,W,h,w,imagenet", [(1024, 1024, 560, 560, 1), (300, 457, 560, 560, 0),
                                              (864, 864, 864, 864, 1), (97, 131, 40, 28, 1)])
def test_prepare_matches_reference(ref, H, W, h, w, imagenet):
    img = np.random.default_rng(H + w).random((3, H, W)).astype(np.float32)
    want = np.empty((3, h, w), np.float32)
    ref.ref_prepare(img.ctypes.data, H, W, want.ctypes.data, h, w, imagenet)
    got = roma_ref.prepare(img, h, w, bool(imagenet))
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_interp_pos_matches_reference(ref):
    c16 = 560 // 14
    assert ref.ref_roma_coarse() == 560
    pos = np.random.default_rng(5).standard_normal((1 + 37 * 37, 1024)).astype(np.float32)
    p = ref.ref_interp_pos(pos.ctypes.data)
    want = np.ctypeslib.as_array(p, ((1 + c16 * c16) * 1024,)).reshape(-1, 1024).copy()
    libc = C.CDLL(None)
    libc.free.argtypes = [C.c_void_p]
    libc.free(C.cast(p, C.c_void_p))
    got = roma_ref.interp_pos(pos, c16)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
