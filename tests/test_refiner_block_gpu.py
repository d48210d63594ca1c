# SPDX-License-Identifier: Unlicense
"""One hidden block of a RoMa refiner, out = W_pw relu(dw5x5(in) + b_dw) +
b_pw on channels-last maps (roma_refiner_block_cl, include/ops_b200.h),
against the oracle: the depthwise convolution of roma_kernels.cl:251-290
and the 1 x 1 convolution after it (roma.c:970-985) in float64 (GPU).

float32 mode (the two kernels one after the other): relative L2 <= 1e-5.
bfloat16 mode with C 32, 64 or 128 (the fused tensor-core kernel that
roma_match runs): the oracle on the bfloat16-rounded input and weights,
with the depthwise result rounded to bfloat16 as the model stores it;
relative L2 <= 5e-3 (the result itself is rounded to bfloat16: about
2e-3). Other widths run the two bfloat16 kernels one after the other."""

import numpy as np
import pytest

import coreg

SHAPES = [
    # H, W, C
    (37, 45, 32),     # ragged tiles (16 x 8 pixels) on both axes
    (20, 50, 64),
    (24, 40, 128),
    (160, 160, 128),  # 200 tiles: more than one per CTA, both accumulators, the rings wrap
    (432, 432, 32),   # a full-size refiner map (scale 2 of the 864 pass)
    (19, 21, 48),     # no fused kernel: the two kernels
]


def bf16_round(x):
    u = np.asarray(x, np.float32).view(np.uint32)
    return (((u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000).astype(np.uint32)).view(np.float32)


def oracle(x, dw_w, dw_b, pw_w, pw_b, mid_round):
    H, W, C = x.shape
    xp = np.zeros((H + 4, W + 4, C))
    xp[2:-2, 2:-2] = x
    k = dw_w.reshape(C, 25).astype(np.float64)
    acc = np.broadcast_to(dw_b.astype(np.float64), (H, W, C)).copy()
    for i in range(5):
        for j in range(5):
            acc += xp[i:i + H, j:j + W] * k[:, 5 * i + j]
    mid = np.maximum(acc, 0.0)
    if mid_round:
        mid = bf16_round(mid.astype(np.float32)).astype(np.float64)
    return mid.reshape(-1, C) @ pw_w.astype(np.float64).T + pw_b


@pytest.mark.gpu
@pytest.mark.parametrize("prec", ["fp32", "bf16"])
@pytest.mark.parametrize("shape", SHAPES, ids=[f"{h}x{w}x{c}" for h, w, c in SHAPES])
def test_refiner_block_cl(shape, prec):
    H, W, C = shape
    if prec == "fp32" and H * W > 40000:
        pytest.skip("the float32 path is covered at the small shapes")
    dev = coreg.Device(0, precision=coreg.OPS_BF16 if prec == "bf16" else coreg.OPS_FP32)
    try:
        rng = np.random.default_rng(H * 1000 + W + C)
        x = rng.standard_normal((H, W, C), dtype=np.float32)
        dw_w = (rng.standard_normal((C, 1, 5, 5), dtype=np.float32) / 5).astype(np.float32)
        dw_b = (0.1 * rng.standard_normal(C)).astype(np.float32)
        pw_w = (rng.standard_normal((C, C), dtype=np.float32) / np.sqrt(C)).astype(np.float32)
        pw_b = (0.1 * rng.standard_normal(C)).astype(np.float32)
        keep = [dev.upload(a) for a in (x, dw_w, dw_b, pw_w, pw_b)]
        Y = dev.zeros(H * W * C)
        dev.lib.roma_refiner_block_cl(dev.ops_p, keep[0].handle, H, W, C, keep[1].handle,
                                      keep[2].handle, keep[3].handle, keep[4].handle, Y.handle)
        got = Y.read(count=H * W * C).reshape(-1, C)
        coreg.check(dev.lib)
        assert dev.lib.coreg_tc_status() == 0
        if prec == "fp32":
            want = oracle(x, dw_w, dw_b, pw_w, pw_b, False)
            bound = 1e-5
        else:
            want = oracle(bf16_round(x), dw_w, dw_b, bf16_round(pw_w), pw_b, True)
            bound = 5e-3
        err = np.linalg.norm(got - want) / np.linalg.norm(want)
        assert err <= bound, err
    finally:
        dev.close()
