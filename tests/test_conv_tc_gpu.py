# SPDX-License-Identifier: Unlicense
"""ops_conv2d's tensor-core path (OPS_BF16 contexts: stride-1 3 x 3 and
5 x 5 convolutions, normalized and PReLU-gated input included, the
reference's conv2d contract of ops.cl:323-448) against the oracle on the
bfloat16-rounded operands (GPU).

The path rounds the weights and the gated input to bfloat16 and
accumulates in float32 on the tensor cores, so the result must match the
float64 convolution of the rounded operands to float32 accumulation
error (relative L2 <= 1e-5); against the float32 operands it must be
within the bfloat16 mode bound of the build's contract (2e-2). Shapes
follow the networks that call it: DISK's 5 x 5 layers (3 -> 16 on the
image, 80 -> 129 normalized, the last layer) and Efficient LoFTR's 3 x 3
backbone and fusion layers, on ragged maps."""

import ctypes as C

import numpy as np
import pytest

import coreg
from coreg import ConvGeom, handle
from oracle import ops_ref

CASES = [
    # C, K, H, W, ksize, normalized, act
    (3, 16, 40, 48, 5, False, coreg.ACT_NONE),
    (80, 129, 36, 52, 5, True, coreg.ACT_NONE),
    (64, 64, 24, 40, 5, True, coreg.ACT_NONE),
    (96, 64, 17, 33, 5, True, coreg.ACT_NONE),
    (64, 64, 32, 32, 3, False, coreg.ACT_RELU),
    (256, 128, 20, 24, 3, False, coreg.ACT_LEAKY),
    (128, 256, 9, 13, 3, False, coreg.ACT_NONE),
]


def bf16(x):
    u = np.asarray(x, np.float32).view(np.uint32)
    return (((u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000).astype(np.uint32)).view(np.float32)


def rel(a, b):
    a = np.asarray(a, np.float64).reshape(-1)
    b = np.asarray(b, np.float64).reshape(-1)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


@pytest.fixture(scope="module")
def dev16():
    d = coreg.Device(0, precision=coreg.OPS_BF16)
    yield d
    d.close()


@pytest.mark.gpu
@pytest.mark.parametrize("case", CASES, ids=[f"{c[0]}to{c[1]}_{c[2]}x{c[3]}_k{c[4]}"
                                             + ("_norm" if c[5] else "") for c in CASES])
def test_conv_tc_matches_rounded_oracle(dev16, case):
    C_, K, H, W, ks, norm, act = case
    rng = np.random.default_rng(C_ * 31 + K + H)
    x = (rng.standard_normal((C_, H, W)) * 2 + 0.5).astype(np.float32)
    w = (rng.standard_normal((K, C_, ks, ks)) / np.sqrt(C_ * ks * ks)).astype(np.float32)
    b = rng.standard_normal(K).astype(np.float32)
    mean = rstd = alpha = None
    if norm:
        mean = x.reshape(C_, -1).mean(1).astype(np.float32)
        rstd = (1.0 / np.sqrt(x.reshape(C_, -1).var(1) + 1e-5)).astype(np.float32)
        alpha = rng.uniform(0.05, 0.5, C_).astype(np.float32)
    bufs = [dev16.upload(v) for v in (x, w, b)]
    nb = [dev16.upload(v) for v in (mean, rstd, alpha)] if norm else [None] * 3
    out = dev16.zeros(K * H * W)
    g = ConvGeom(ks, ks, 1, 1, ks // 2, ks // 2, 1, 1, 1)
    dev16.lib.ops_conv2d(dev16.ops_p, handle(bufs[0]), C_, H, W, handle(bufs[1]),
                         handle(bufs[2]), K, C.byref(g), *(handle(v) for v in nb), act, 0.1,
                         handle(out))
    coreg.check(dev16.lib)
    got = out.read(count=K * H * W)
    # The gate in float32 as the kernel computes it, then rounded.
    xg = x
    if norm:
        xg = (x - mean[:, None, None]) * rstd[:, None, None]
        xg = np.where(xg >= 0, xg, alpha[:, None, None] * xg).astype(np.float32)
    want_r = ops_ref.conv2d(bf16(xg).reshape(-1), C_, H, W, bf16(w).reshape(-1), b, K, ks, ks,
                            1, 1, ks // 2, ks // 2, a=act, slope=0.1)
    assert rel(got, want_r) <= 1e-5, rel(got, want_r)
    want = ops_ref.conv2d(x.reshape(-1), C_, H, W, w.reshape(-1), b, K, ks, ks, 1, 1, ks // 2,
                          ks // 2, mean=mean, rstd=rstd, alpha=alpha, a=act, slope=0.1)
    assert rel(got, want) <= 2e-2, rel(got, want)
