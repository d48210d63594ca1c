# SPDX-License-Identifier: Unlicense
"""The Gaussian process's solve on the device (roma_gp_solve,
include/roma_ops.h) against the reference's own host solve (gp_solve,
roma.c:772-836, compiled from its roma.c into oracle/_ref/
libroma_host_ref.so) (GPU).

Both factor K + 0.1 I in double and round X to float, in different
orders, so X must agree to relative L2 1e-6 on the GP's kernel matrices
(the cosine kernel of the build's features, temperature 0.2), sizes that
do and do not fill the 64-row blocks, up to the full 1600 tokens x 512
basis columns; a matrix that is not positive definite is reported."""

import ctypes as C
from pathlib import Path

import numpy as np
import pytest

import coreg
from coreg import handle

LIB = Path(__file__).resolve().parents[1] / "oracle" / "_ref" / "libroma_host_ref.so"


@pytest.fixture(scope="module")
def ref():
    if not LIB.exists():
        pytest.skip("oracle/_ref/libroma_host_ref.so not built (make -C oracle)")
    lib = C.CDLL(str(LIB))
    lib.ref_gp_solve.argtypes = [C.c_void_p, C.c_int, C.c_void_p, C.c_int]
    return lib


def cos_kernel(rng, n, dim=512, smooth=0.0):
    f = rng.standard_normal((n, dim))
    if smooth:
        f = smooth * np.cumsum(f, 0) / np.sqrt(np.arange(1, n + 1))[:, None] + (1 - smooth) * f
    fn = f / np.linalg.norm(f, axis=1, keepdims=True)
    return np.exp((fn @ fn.T - 1.0) / 0.2).astype(np.float32)


def solve(dev, K, F):
    n, d = F.shape
    Kb, Fb, Xb = dev.upload(K), dev.upload(F), dev.zeros(n * d)
    flag = dev.lib.roma_gp_solve(dev.ops_p, handle(Kb), n, handle(Fb), d, 0.1, handle(Xb))
    coreg.check(dev.lib)
    return flag, Xb.read(count=n * d).reshape(n, d)


@pytest.mark.gpu
@pytest.mark.parametrize("n,d,smooth", [(300, 64, 0.0), (1037, 128, 0.9), (1600, 512, 0.5),
                                        (64, 512, 0.3), (41, 16, 0.0)])
def test_gp_solve_matches_reference(dev, ref, n, d, smooth):
    rng = np.random.default_rng(n + d)
    K = cos_kernel(rng, n, smooth=smooth)
    F = rng.standard_normal((n, d)).astype(np.float32)
    want = F.copy()
    ref.ref_gp_solve(K.ctypes.data, n, want.ctypes.data, d)
    flag, got = solve(dev, K, F)
    assert flag == 0
    e = np.linalg.norm(got - want) / np.linalg.norm(want)
    assert e <= 1e-6, e


@pytest.mark.gpu
def test_gp_solve_reports_not_positive_definite(dev):
    n, d = 130, 8
    K = -np.eye(n, dtype=np.float32)
    flag, _ = solve(dev, K, np.ones((n, d), np.float32))
    assert flag == 1
    # The context stays usable.
    rng = np.random.default_rng(3)
    flag, _ = solve(dev, cos_kernel(rng, 70), rng.standard_normal((70, 4)).astype(np.float32))
    assert flag == 0
