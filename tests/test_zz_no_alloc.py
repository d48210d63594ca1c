# SPDX-License-Identifier: Unlicense
"""ops_gemm_noalloc (include/ops_b200.h) against ops_gemm through the C-ABI
(GPU).

The variant stages the bfloat16 operands in the library's fixed scratch
array instead of a cudaMalloc'd buffer. It must give the results of
ops_gemm on the same inputs, call after call, while the context's own
staging buffer (o->scratch16) stays unallocated. The file is named to run
last, after the other tests have used the device, and also passes alone in
a fresh process."""

import numpy as np
import pytest

import coreg
from coreg import Opnd, handle

# Same packing and the same kernels as ops_gemm: identical results up to
# float32 rounding.
TOL = 1e-6

CASES = [
    # M, N, K, nb, act, residual: tensor-core tiles (nb 1), then the
    # batched bfloat16 SIMT tiles with a residual.
    (256, 192, 320, 1, coreg.ACT_GELU, False),
    (130, 96, 72, 2, coreg.ACT_RELU, True),
]


@pytest.fixture(scope="module")
def dev16():
    d = coreg.Device(0, precision=coreg.OPS_BF16)
    yield d
    d.close()


def rel_l2(a, b):
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def run(dev, fn, M, N, K, nb, act, residual, x):
    A, B, bias = (dev.upload(x[k]) for k in ("a", "b", "bias"))
    Cb = dev.upload(x["r"]) if residual else dev.zeros(nb * M * N)
    fn(dev.ops_p, M, N, K, Opnd(handle(A), 0, K, M * K, 0), Opnd(handle(B), 0, K, N * K, 0), 1,
       Opnd(handle(Cb), 0, N, M * N, 0), nb, 1, handle(bias), 0,
       handle(Cb) if residual else None, 0, 0.75, act, 0.0)
    coreg.check(dev.lib)
    return Cb.read(count=nb * M * N)


def inputs(seed, M, N, K, nb):
    rng = np.random.default_rng(seed)
    return {
        "a": rng.standard_normal(nb * M * K, dtype=np.float32),
        "b": (rng.standard_normal(nb * N * K, dtype=np.float32) / np.sqrt(K)).astype(np.float32),
        "bias": rng.standard_normal(N, dtype=np.float32),
        "r": rng.standard_normal(nb * M * N, dtype=np.float32),
    }


@pytest.mark.gpu
def test_noalloc_matches_ops_gemm_two_calls(dev16):
    lib = dev16.lib
    assert lib.ops_gemm_noalloc_max_bytes() == 16 << 20
    xs = [inputs(100 + i, *c[:4]) for i, c in enumerate(CASES)]
    # Two calls of the variant in a row, then ops_gemm on the same inputs.
    got = [run(dev16, lib.ops_gemm_noalloc, *c, x) for c, x in zip(CASES, xs)]
    # The variant never grew the context's staging buffer.
    assert dev16.ops.scratch16_bytes == 0
    for c, x, g in zip(CASES, xs, got):
        want = run(dev16, lib.ops_gemm, *c, x)
        assert np.isfinite(g).all()
        assert rel_l2(g, want) <= TOL, (c, rel_l2(g, want))
    # A repeat of the first product after the array held the second one's
    # operands.
    M, N, K, nb, act, residual = CASES[0]
    x = inputs(100, M, N, K, nb)
    again = run(dev16, lib.ops_gemm_noalloc, M, N, K, nb, act, residual, x)
    want = run(dev16, lib.ops_gemm, M, N, K, nb, act, residual, x)
    assert rel_l2(again, want) <= TOL


@pytest.mark.gpu
def test_noalloc_rejects_products_beyond_the_array(dev16):
    lib = dev16.lib
    # 2 (M + N) K bytes of bfloat16 operands: 17.0 MB > 16 MiB. The buffers
    # are full size, so nothing could be read out of bounds.
    M = N = 4096
    K = 1040
    A, B, Cb = dev16.zeros(M * K), dev16.zeros(N * K), dev16.zeros(M * N)
    lib.ops_gemm_noalloc(dev16.ops_p, M, N, K, Opnd(handle(A), 0, K, 0, 0),
                         Opnd(handle(B), 0, K, 0, 0), 1, Opnd(handle(Cb), 0, N, 0, 0), 1, 1,
                         None, 0, None, 0, 1.0, 0, 0.0)
    with pytest.raises(coreg.CoregError, match="scratch array"):
        coreg.check(lib)
    # The context stays usable.
    M, N, K, nb, act, residual = CASES[0]
    x = inputs(7, M, N, K, nb)
    got = run(dev16, lib.ops_gemm_noalloc, M, N, K, nb, act, residual, x)
    want = run(dev16, lib.ops_gemm, M, N, K, nb, act, residual, x)
    assert rel_l2(got, want) <= TOL
