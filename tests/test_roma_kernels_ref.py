# SPDX-License-Identifier: Unlicense
"""The RoMa kernels of the oracle (oracle/roma_ref.py) against the
reference's own OpenCL kernels (roma_kernels.cl), compiled where they lie
as C through oracle/cl_emul.h and run on the CPU with the reference's
work-group sizes (oracle/_ref/libroma_cl_ref.so, built by oracle/Makefile;
the tests skip when it has not been built). CPU only.

Kernels: roma_row_norm and roma_cos_exp (the Gaussian process's kernel
matrices), roma_cls_to_flow (softmax over the 64 x 64 anchors, first
argmax, the clamped five-neighbour mean: modes in corners and on edges
included), roma_warp_sample (bilinear, zero padding, zero at non-finite
warps), roma_local_corr (r = 0..3, warps partly outside and not finite),
roma_disp, roma_update, roma2_update (softplus above and below its
threshold of 20) and roma_dwconv5 (ragged maps, ReLU). The bound is float
rounding: relative L2 <= 1e-6 (the emulation's exp and sqrt are the C
library's, which OpenCL allows to differ by a few units in the last
place)."""

import ctypes as C
import types
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import roma_ref as R

LIB = Path(__file__).resolve().parents[1] / "oracle" / "_ref" / "libroma_cl_ref.so"
P, I, FL = C.c_void_p, C.c_int, C.c_float


@pytest.fixture(scope="module")
def ref():
    if not LIB.exists():
        pytest.skip("oracle/_ref/libroma_cl_ref.so not built (make -C oracle)")
    lib = C.CDLL(str(LIB))
    sig = {
        "ref_row_norm": [P, I, I, P], "ref_cos_exp": [P, P, P, I, I, FL, FL],
        "ref_cls_to_flow": [P, I, I, I, I, P, P], "ref_warp_sample": [P, I, I, I, P, P, I],
        "ref_local_corr": [P, P, I, I, I, I, P, P, I], "ref_disp": [P, I, I, FL, FL, P],
        "ref_update": [P, P, P, I, FL, FL, FL], "ref_update2": [P, P, P, I, FL, FL],
        "ref_dwconv5": [P, I, I, I, P, P, P],
    }
    for name, args in sig.items():
        getattr(lib, name).restype = None
        getattr(lib, name).argtypes = args
    return lib


@pytest.fixture(scope="module")
def run():
    r = types.SimpleNamespace(dt=torch.float32)
    r.t = lambda a: torch.as_tensor(np.asarray(a)).to(torch.float32)
    return r


def rel(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30)


def ptr(a):
    return a.ctypes.data


def warp(rng, n, lo=-1.2, hi=1.2):
    f = rng.uniform(lo, hi, (2, n)).astype(np.float32)
    f[0, 3] = np.nan
    f[1, 7] = np.inf
    return f


def test_gp_kernel_matrices(ref):
    rng = np.random.default_rng(0)
    N, M, D = 60, 70, 512
    A = rng.standard_normal((N, D)).astype(np.float32)
    B = rng.standard_normal((M, D)).astype(np.float32)
    na, nb = np.zeros(N, np.float32), np.zeros(M, np.float32)
    ref.ref_row_norm(ptr(A), N, D, ptr(na))
    ref.ref_row_norm(ptr(B), M, D, ptr(nb))
    ta, tb = torch.from_numpy(A), torch.from_numpy(B)
    assert rel(na, ta.norm(dim=1)) <= 1e-6 and rel(nb, tb.norm(dim=1)) <= 1e-6
    S = (A @ B.T).astype(np.float32)
    got = S.copy()
    ref.ref_cos_exp(ptr(got), ptr(na), ptr(nb), N, M, R.GP_T, R.COS_EPS)
    want = R.cos_exp(torch.from_numpy(S), ta.norm(dim=1), tb.norm(dim=1)).numpy()
    assert rel(got, want) <= 1e-6


def test_cls_to_flow(ref, run):
    rng = np.random.default_rng(1)
    n = 60
    L = (rng.standard_normal((n, R.NCLS + 1)) * 3).astype(np.float32)
    L[:6, :R.NCLS] = -5
    for t, c in enumerate((0, R.NCLS - 1, R.CLS_RES - 1, R.NCLS - R.CLS_RES, 1, R.CLS_RES)):
        L[t, c] = 10  # modes in the corners and next to them: clamped neighbours
    flow, cert = np.zeros((2, n), np.float32), np.zeros(n, np.float32)
    ref.ref_cls_to_flow(ptr(L), R.NCLS + 1, R.NCLS, R.CLS_RES, n, ptr(flow), ptr(cert))
    wf, wc = R.Runner.cls_to_flow(run, torch.from_numpy(L))
    assert rel(flow, wf.numpy()) <= 1e-6
    assert np.array_equal(cert, wc.numpy())


def test_warp_sample(ref, run):
    rng = np.random.default_rng(2)
    C_, H, W = 16, 12, 14
    n = H * W
    f = rng.standard_normal((C_, H, W)).astype(np.float32)
    flow = warp(rng, n)
    got = np.zeros((C_ + 3, n), np.float32)
    ref.ref_warp_sample(ptr(f), C_, H, W, ptr(flow), ptr(got), 3)
    want = R.Runner.sample(run, torch.from_numpy(f), H, W, torch.from_numpy(flow)).numpy()
    assert rel(got[3:], want) <= 1e-6
    assert not got[3:, 3].any() and not got[3:, 7].any()


@pytest.mark.parametrize("r", [0, 1, 2, 3])
def test_local_corr(ref, run, r):
    rng = np.random.default_rng(3 + r)
    C_, H, W = 32, 11, 13
    n = H * W
    f1 = rng.standard_normal((C_, n)).astype(np.float32)
    f2 = rng.standard_normal((C_, H, W)).astype(np.float32)
    flow = warp(rng, n, -1.4, 1.4)
    side = 2 * r + 1
    got = np.zeros((side * side, n), np.float32)
    ref.ref_local_corr(ptr(f1), ptr(f2), C_, H, W, r, ptr(flow), ptr(got), 0)
    want = R.Runner.local_corr(run, torch.from_numpy(f1), torch.from_numpy(f2), H, W, r,
                               torch.from_numpy(flow)).numpy()
    assert rel(got, want) <= 1e-6


def test_disp_and_updates(ref):
    rng = np.random.default_rng(4)
    H, W = 9, 15
    n = H * W
    flow = rng.uniform(-1, 1, (2, n)).astype(np.float32)
    got = np.zeros((2, n), np.float32)
    ref.ref_disp(ptr(flow), H, W, 1.25, 0.7, ptr(got))
    gx, gy = R.Runner.grid(H, W, torch.float32)
    want = R.disp(torch.from_numpy(flow), gx, gy, np.float32(1.25), np.float32(0.7)).numpy()
    assert rel(got, want) <= 1e-6

    d = rng.standard_normal((3, n)).astype(np.float32)
    fl, ce = flow.copy(), rng.standard_normal(n).astype(np.float32)
    wfl, wce = R.update(torch.from_numpy(fl), torch.from_numpy(ce), torch.from_numpy(d), 2.0,
                        560.0, 560.0)
    ref.ref_update(ptr(fl), ptr(ce), ptr(d), n, 2.0, 560.0, 560.0)
    assert rel(fl, wfl) <= 1e-6 and rel(ce, wce) <= 1e-6

    d6 = (rng.standard_normal((6, n)) * 12).astype(np.float32)  # softplus both sides of 20
    fl, cf = flow.copy(), rng.standard_normal((4, n)).astype(np.float32)
    wfl, wcf = R.update2(torch.from_numpy(fl), torch.from_numpy(cf), torch.from_numpy(d6), 864.0,
                         864.0)
    ref.ref_update2(ptr(fl), ptr(cf), ptr(d6), n, 864.0, 864.0)
    assert rel(fl, wfl) <= 1e-6 and rel(cf, wcf) <= 1e-6


@pytest.mark.parametrize("C_,H,W", [(8, 37, 29), (3, 16, 16), (5, 20, 7)])
def test_dwconv5(ref, run, C_, H, W):
    rng = np.random.default_rng(C_ * H)
    x = rng.standard_normal((C_, H, W)).astype(np.float32)
    w = rng.standard_normal((C_, 1, 5, 5)).astype(np.float32)
    b = rng.standard_normal(C_).astype(np.float32)
    got = np.zeros((C_, H, W), np.float32)
    ref.ref_dwconv5(ptr(x), C_, H, W, ptr(w), ptr(b), ptr(got))
    want = R.Runner.conv(run, torch.from_numpy(x), w, b, pad=2, act="relu", groups=C_).numpy()
    assert rel(got, want) <= 1e-6
