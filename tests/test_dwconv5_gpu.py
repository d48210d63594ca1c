# SPDX-License-Identifier: Unlicense
"""The RoMa refiner's depthwise 5 x 5 convolution (+ bias, ReLU) on
channels-last maps, roma_dwconv5_cl (include/ops_b200.h), against the
oracle's grouped convolution (roma_kernels.cl:256-284 restated; GPU).

float32 mode: relative L2 <= 1e-5. bfloat16 mode (the kernel roma_match
runs): against the oracle on the bfloat16-rounded input, relative L2 <=
5e-3 (float32 arithmetic, the result rounded to bfloat16: about 2e-3)."""

import numpy as np
import pytest

import coreg
from oracle import ops_ref

SHAPES = [
    # H, W, C
    (40, 40, 32),
    (37, 53, 128),   # ragged pixel tiles
    (45, 70, 512),   # eight 64-channel k-blocks
    (200, 208, 128), # at least one 16 x 16 tile per SM: the TMA-fed bfloat16 kernel
    (16, 20, 48),    # a partial 32-channel block
    (9, 9, 8),
    (11, 13, 12),    # C not a multiple of 8: the generic kernel
]


def bf16_round(x):
    u = np.asarray(x, np.float32).view(np.uint32)
    return (((u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000).astype(np.uint32)).view(np.float32)


def oracle(x, w, b, H, W, C):
    chw = np.transpose(x, (2, 0, 1)).reshape(-1)
    y = ops_ref.conv2d(chw, C, H, W, w.reshape(-1), b, C, 5, 5, 1, 1, 2, 2, groups=C,
                       a=ops_ref.ACT_RELU)
    return np.asarray(y).reshape(C, H, W).transpose(1, 2, 0)


@pytest.mark.gpu
@pytest.mark.parametrize("prec", ["fp32", "bf16"])
@pytest.mark.parametrize("shape", SHAPES, ids=[f"{h}x{w}x{c}" for h, w, c in SHAPES])
def test_dwconv5_cl(shape, prec):
    H, W, C = shape
    dev = coreg.Device(0, precision=coreg.OPS_BF16 if prec == "bf16" else coreg.OPS_FP32)
    try:
        rng = np.random.default_rng(H * 100 + W + C)
        x = rng.standard_normal((H, W, C), dtype=np.float32)
        w = (rng.standard_normal((C, 1, 5, 5), dtype=np.float32) / 5).astype(np.float32)
        b = (0.1 * rng.standard_normal(C)).astype(np.float32)
        X, Wt, B, Y = dev.upload(x), dev.upload(w), dev.upload(b), dev.zeros(H * W * C)
        dev.lib.roma_dwconv5_cl(dev.ops_p, X.handle, H, W, C, Wt.handle, B.handle, Y.handle)
        got = Y.read(count=H * W * C).reshape(H, W, C)
        coreg.check(dev.lib)
        if prec == "fp32":
            want = oracle(x, w, b, H, W, C)
            bound = 1e-5
        else:
            want = oracle(bf16_round(x), w, b, H, W, C)
            bound = 5e-3
        err = np.linalg.norm(got - want) / np.linalg.norm(want)
        assert err <= bound, err
    finally:
        dev.close()
