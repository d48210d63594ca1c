# SPDX-License-Identifier: Unlicense
"""The tcgen05 tensor-core GEMM (ops_gemm with precision OPS_BF16, the
reference's gemm contract of ops.cl:39-52) against the oracle evaluated on
the bfloat16-rounded operands (GPU).

Float32 accumulation of bfloat16 products: the result must match the
float64 product of the rounded operands to float32 accumulation error
(relative L2 <= 1e-5); against the float32 operands it is within the
bfloat16 mode bound of the build's contract (relative L2 <= 2e-2)."""

import ctypes as C

import numpy as np
import pytest

import coreg
from coreg import Opnd
from oracle.ops_ref import gemm as ref_gemm

SHAPES = [
    # M, N, K, act, residual
    (128, 256, 64, 0, False),
    (300, 200, 96, 2, True),     # BN 128 tiles, ragged M and N
    (77, 130, 40, 1, False),     # one ragged tile, K below one stage
    (1601, 3072, 1024, 0, False),  # DINOv2 qkv
    (1601, 1024, 4096, 0, True),   # DINOv2 fc2 with the residual
    (1600, 4097, 1024, 0, False),  # decoder to_out (odd N)
    (4900, 1136, 1136, 0, False),  # refiner 1 x 1 at 1/8
    # 256-row tiles (256, 192 and 160 columns, filling whole rounds of SMs)
    (3202, 3072, 1024, 0, False),  # DINOv2 qkv, both images
    (3202, 4096, 1024, 0, True),   # fc1 shape with a residual
    (3300, 2900, 712, 0, True),    # ragged M, N and K (K a multiple of 8 only)
    (9472, 1024, 256, 0, False),   # 148 tiles of 256 x 256
    # narrow outputs: 16-, 32- and 64-column tiles
    (5000, 32, 32, 2, False),      # refiner pointwise at full size (32 channels)
    (746, 6, 32, 0, True),         # refiner heads (warp 2 + confidence 4)
    (300, 48, 128, 1, False),
    (130, 64, 64, 0, True),
    (2000, 12, 64, 0, False),
]


def bf16_round(x):
    u = np.asarray(x, np.float32).view(np.uint32)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000).astype(np.uint32)
    return r.view(np.float32)


@pytest.fixture(scope="module")
def dev16():
    d = coreg.Device(0, precision=coreg.OPS_BF16)
    yield d
    d.close()


@pytest.mark.gpu
@pytest.mark.parametrize("shape", SHAPES, ids=[f"{s[0]}x{s[1]}x{s[2]}" for s in SHAPES])
def test_tc_gemm_matches_rounded_oracle(dev16, shape):
    M, N, K, act, residual = shape
    rng = np.random.default_rng(M * 7 + N * 3 + K)
    a = rng.standard_normal((M, K), dtype=np.float32)
    b = (rng.standard_normal((N, K), dtype=np.float32) / np.sqrt(K)).astype(np.float32)
    bias = rng.standard_normal(N, dtype=np.float32)
    r = rng.standard_normal((M, N), dtype=np.float32)
    A, B, Bi = dev16.upload(a), dev16.upload(b), dev16.upload(bias)
    Cb = dev16.upload(r) if residual else dev16.zeros(M * N)
    lib = dev16.lib
    lib.ops_gemm(dev16.ops_p, M, N, K, Opnd(A.handle, 0, K, 0, 0), Opnd(B.handle, 0, K, 0, 0), 1,
                 Opnd(Cb.handle, 0, N, 0, 0), 1, 1, Bi.handle, 0,
                 Cb.handle if residual else None, 0, 0.75, act, 0.1)
    got = Cb.read(count=M * N).reshape(M, N)
    coreg.check(lib)
    assert lib.coreg_tc_status() == 0
    want = ref_gemm(bf16_round(a), bf16_round(b), 1, M, N, K, bias=bias, R=r if residual else None,
                    alpha=0.75, a=act, slope=0.1)[0]
    err = np.linalg.norm(got - want) / np.linalg.norm(want)
    assert err <= 1e-5, err
    want32 = ref_gemm(a, b, 1, M, N, K, bias=bias, R=r if residual else None, alpha=0.75, a=act,
                      slope=0.1)[0]
    assert np.linalg.norm(got - want32) / np.linalg.norm(want32) <= 2e-2


LAYOUTS = [
    # M, N, K, transb, biasrow: B as K x N (a 1 x 1 convolution's input,
    # an unfolded image) packed transposed; the bias per row (per output
    # channel of ops_conv1x1) in the epilogue.
    (256, 6400, 256, 0, 1),
    (128, 1000, 576, 0, 1),
    (96, 333, 72, 0, 0),
    (300, 200, 96, 1, 1),
    (4000, 2600, 320, 1, 1),       # 256 x 256 tiles with the row bias
]


@pytest.mark.gpu
@pytest.mark.parametrize("shape", LAYOUTS, ids=[f"{s[0]}x{s[1]}x{s[2]}_t{s[3]}_r{s[4]}"
                                                for s in LAYOUTS])
def test_tc_gemm_b_layouts_and_row_bias(dev16, shape):
    M, N, K, transb, biasrow = shape
    rng = np.random.default_rng(M + N + K)
    a = rng.standard_normal((M, K), dtype=np.float32)
    bt = (rng.standard_normal((N, K), dtype=np.float32) / np.sqrt(K)).astype(np.float32)
    b = bt if transb else np.ascontiguousarray(bt.T)
    bias = rng.standard_normal(M if biasrow else N, dtype=np.float32)
    A, B, Bi, Cb = dev16.upload(a), dev16.upload(b), dev16.upload(bias), dev16.zeros(M * N)
    lib = dev16.lib
    lib.ops_gemm(dev16.ops_p, M, N, K, Opnd(A.handle, 0, K, 0, 0),
                 Opnd(B.handle, 0, K if transb else N, 0, 0), transb,
                 Opnd(Cb.handle, 0, N, 0, 0), 1, 1, Bi.handle, biasrow, None, 0, 1.0, 2, 0.0)
    got = Cb.read(count=M * N).reshape(M, N)
    coreg.check(lib)
    assert lib.coreg_tc_status() == 0
    want = ref_gemm(bf16_round(a), bf16_round(bt), 1, M, N, K, bias=bias, biasrow=biasrow,
                    a=2)[0]
    err = np.linalg.norm(got - want) / np.linalg.norm(want)
    assert err <= 1e-5, err


CONVS = [
    # H, W, C, K (the VGG shapes at reduced size, ragged tiles)
    (40, 40, 64, 64),
    (35, 70, 128, 256),
    (72, 136, 64, 128),
    (17, 9, 256, 64),
    # few input channels: explicit im2col + tensor cores in bfloat16 mode
    (40, 40, 3, 64),
    (35, 70, 3, 64),
    (9, 13, 5, 96),
]


@pytest.mark.gpu
@pytest.mark.parametrize("shape", CONVS, ids=[f"{s[0]}x{s[1]}x{s[2]}to{s[3]}" for s in CONVS])
@pytest.mark.parametrize("prec", [coreg.OPS_FP32, coreg.OPS_BF16], ids=["fp32", "bf16"])
def test_conv3x3_channels_last(shape, prec):
    """ops_conv3x3_cl (implicit GEMM; tensor cores with 3-D TMA boxes in
    bfloat16 mode) against the oracle convolution (ops.cl conv2d
    semantics) on the same channels-last data."""
    from oracle.ops_ref import conv2d

    H, W, C_, K = shape
    dev = coreg.Device(0, precision=prec)
    rng = np.random.default_rng(H * W + C_)
    x = rng.standard_normal((H, W, C_), dtype=np.float32)
    w = (rng.standard_normal((K, C_, 3, 3), dtype=np.float32) / np.sqrt(9 * C_)).astype(np.float32)
    b = rng.standard_normal(K, dtype=np.float32)
    X, Wt, B, Y = dev.upload(x), dev.upload(w), dev.upload(b), dev.zeros(H * W * K)
    dev.lib.ops_conv3x3_cl(dev.ops_p, X.handle, H, W, C_, Wt.handle, B.handle, K, 2, 0.0, Y.handle)
    got = Y.read(count=H * W * K).reshape(H, W, K)
    coreg.check(dev.lib)
    assert dev.lib.coreg_tc_status() == 0
    xr, wr = (bf16_round(x), bf16_round(w)) if prec == coreg.OPS_BF16 else (x, w)
    want = conv2d(xr.transpose(2, 0, 1), C_, H, W, wr, b, K, 3, 3, 1, 1, 1, 1, a=2)
    want = want.transpose(1, 2, 0)
    err = np.linalg.norm(got - want) / np.linalg.norm(want)
    assert err <= 1e-5, err
    dev.close()
