# SPDX-License-Identifier: Unlicense
"""ops_gemm_noalloc (include/ops_b200.h) against ops_gemm and against the
oracle, through the C-ABI (GPU).

The variant stages the bfloat16 operands in the library's fixed scratch
array instead of a cudaMalloc'd buffer. It must pick the same path as
ops_gemm for every shape (bfloat16 tensor-core or float32 tiles), give its
results on the same inputs, call after call, and leave the context's own
staging buffer (o->scratch16) unallocated. Both are checked against the
oracle's gemm (oracle/ops_ref.py, ops.cl:39-284) on the operands the path
uses (rounded to bfloat16 where the context is OPS_BF16). The file is named
to run last, after the other tests have used the device, and also passes
alone in a fresh process."""

import numpy as np
import pytest

import coreg
from coreg import Opnd, handle
from oracle import ops_ref

# Same packing and the same kernels as ops_gemm: identical results up to
# float32 rounding.
TOL_SAME = 1e-6
# Against the float64 oracle on the same (rounded) operands: float32
# accumulation.
TOL_ORACLE = 1e-5

# M, N, K, nb, nb1, act, residual.
CASES_BF16 = [
    (256, 192, 320, 1, 1, coreg.ACT_GELU, False),   # tensor-core tiles
    (130, 96, 72, 2, 1, coreg.ACT_RELU, True),      # batched, residual
    (128, 32, 64, 1, 1, coreg.ACT_NONE, False),     # N < 64: still bfloat16
    (96, 8, 48, 1, 1, coreg.ACT_GELU, True),        # N < 16
    (80, 40, 32, 4, 2, coreg.ACT_NONE, True),       # nb 4 over nb1 2, strided
    (70000, 16, 16, 1, 1, coreg.ACT_NONE, False),   # M beyond 65535 rows
]
CASES_FP32 = [
    (128, 32, 64, 1, 1, coreg.ACT_GELU, False),
    (80, 40, 32, 4, 2, coreg.ACT_RELU, True),
]


def bf16(x):
    u = np.asarray(x, np.float32).view(np.uint32)
    return (((u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000).astype(np.uint32)).view(np.float32)


def rel_l2(a, b):
    a = np.asarray(a, np.float64).reshape(-1)
    b = np.asarray(b, np.float64).reshape(-1)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def layout(M, K, nb, nb1):
    """Leading dimension and batch strides of a padded, strided operand
    (elements): rows K + 8 apart, inner batches s1 apart, outer s0."""
    ld = K + 8
    s1 = M * ld + 24
    s0 = nb1 * s1 + 40
    return ld, s0, s1, (nb // nb1) * s0


def inputs(seed, M, N, K, nb, nb1):
    rng = np.random.default_rng(seed)
    la, lb = layout(M, K, nb, nb1), layout(N, K, nb, nb1)
    return {
        "a": rng.standard_normal(la[3], dtype=np.float32),
        "b": (rng.standard_normal(lb[3], dtype=np.float32) / np.sqrt(K)).astype(np.float32),
        "bias": rng.standard_normal(N, dtype=np.float32),
        "r": rng.standard_normal(nb * M * N, dtype=np.float32),
        "la": la, "lb": lb,
    }


def products(buf, rows, K, nb, nb1, lay):
    """The nb (rows x K) products of a strided operand, as (nb, rows, K)."""
    ld, s0, s1, _ = lay
    out = np.empty((nb, rows, K), np.float32)
    for b in range(nb):
        base = (b // nb1) * s0 + (b % nb1) * s1
        out[b] = buf[base:base + rows * ld].reshape(rows, ld)[:, :K]
    return out


def run(dev, fn, M, N, K, nb, nb1, act, residual, x):
    A, B, bias = (dev.upload(x[k]) for k in ("a", "b", "bias"))
    Cb = dev.upload(x["r"]) if residual else dev.zeros(nb * M * N)
    la, lb = x["la"], x["lb"]
    fn(dev.ops_p, M, N, K, Opnd(handle(A), 0, la[0], la[1], la[2]),
       Opnd(handle(B), 0, lb[0], lb[1], lb[2]), 1,
       Opnd(handle(Cb), 0, N, nb1 * M * N, M * N), nb, nb1, handle(bias), 0,
       handle(Cb) if residual else None, 0, 0.75, act, 0.0)
    coreg.check(dev.lib)
    return Cb.read(count=nb * M * N)


def oracle(M, N, K, nb, nb1, act, residual, x, rounded):
    a = products(x["a"], M, K, nb, nb1, x["la"])
    b = products(x["b"], N, K, nb, nb1, x["lb"])
    if rounded:
        a, b = bf16(a), bf16(b)
    return ops_ref.gemm(a, b, 1, M, N, K, nb=nb, bias=x["bias"],
                        R=x["r"] if residual else None, alpha=0.75, a=act)


def check_cases(dev, cases, rounded, seed0):
    lib = dev.lib
    xs = [inputs(seed0 + i, *c[:5]) for i, c in enumerate(cases)]
    # The variant on every case, one call after another, then ops_gemm on
    # the same inputs.
    got = [run(dev, lib.ops_gemm_noalloc, *c, x) for c, x in zip(cases, xs)]
    # The variant never grew the context's staging buffer.
    assert dev.ops.scratch16_bytes == 0
    for c, x, g in zip(cases, xs, got):
        assert np.isfinite(g).all(), c
        want = run(dev, lib.ops_gemm, *c, x)
        assert rel_l2(g, want) <= TOL_SAME, (c, rel_l2(g, want))
        ref = oracle(*c, x, rounded)
        assert rel_l2(g, ref) <= TOL_ORACLE, (c, rel_l2(g, ref))
    # A repeat of the first product after the array held the others'
    # operands.
    again = run(dev, lib.ops_gemm_noalloc, *cases[0], xs[0])
    assert rel_l2(again, got[0]) <= TOL_SAME


@pytest.fixture(scope="module")
def dev16():
    d = coreg.Device(0, precision=coreg.OPS_BF16)
    yield d
    d.close()


@pytest.mark.gpu
def test_noalloc_bf16_matches_ops_gemm_and_oracle(dev16):
    assert dev16.lib.ops_gemm_noalloc_max_bytes() == 16 << 20
    check_cases(dev16, CASES_BF16, True, 100)


@pytest.mark.gpu
def test_noalloc_fp32_matches_ops_gemm_and_oracle():
    dev = coreg.Device(0, precision=coreg.OPS_FP32)
    try:
        check_cases(dev, CASES_FP32, False, 200)
    finally:
        dev.close()


@pytest.mark.gpu
def test_noalloc_b_as_k_by_n_matches_ops_gemm():
    """B given as K x N (transb 0): both entry points pack it transposed
    and agree; the context's staging buffer stays unallocated."""
    # A context of its own, whose staging buffer no ops_gemm call has grown.
    dev = coreg.Device(0, precision=coreg.OPS_BF16)
    lib = dev.lib
    M, N, K = 128, 300, 64
    rng = np.random.default_rng(11)
    a = rng.standard_normal((M, K), dtype=np.float32)
    b = (rng.standard_normal((K, N), dtype=np.float32) / np.sqrt(K)).astype(np.float32)
    bias = rng.standard_normal(M, dtype=np.float32)
    outs = []
    try:
        for fn in (lib.ops_gemm_noalloc, lib.ops_gemm_noalloc, lib.ops_gemm):
            A, B, Bi, Cb = dev.upload(a), dev.upload(b), dev.upload(bias), dev.zeros(M * N)
            fn(dev.ops_p, M, N, K, Opnd(handle(A), 0, K, 0, 0), Opnd(handle(B), 0, N, 0, 0), 0,
               Opnd(handle(Cb), 0, N, 0, 0), 1, 1, handle(Bi), 1, None, 0, 1.0, coreg.ACT_NONE,
               0.0)
            coreg.check(lib)
            outs.append(Cb.read(count=M * N))
            if len(outs) == 2:
                assert dev.ops.scratch16_bytes == 0
    finally:
        dev.close()
    assert rel_l2(outs[0], outs[2]) <= TOL_SAME and rel_l2(outs[1], outs[2]) <= TOL_SAME
    ref = ops_ref.gemm(bf16(a), bf16(b), 0, M, N, K, bias=bias, biasrow=1)
    assert rel_l2(outs[0], ref) <= TOL_ORACLE


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
    c = CASES_BF16[0]
    x = inputs(7, *c[:5])
    got = run(dev16, lib.ops_gemm_noalloc, *c, x)
    want = run(dev16, lib.ops_gemm, *c, x)
    assert rel_l2(got, want) <= TOL_SAME
