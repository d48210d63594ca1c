# SPDX-License-Identifier: Unlicense
"""RoMa's local correlation on channels-last maps, roma_local_corr_cl
(include/ops_b200.h), against the oracle's restatement of
roma_kernels.cl:153-192 (oracle/roma_ref.py; GPU).

float32 mode: relative L2 <= 1e-5. bfloat16 mode (the kernel roma_match
runs): against the oracle on the bfloat16-rounded maps, relative L2 <= 1e-4
(float32 arithmetic on exact bfloat16 inputs)."""

import types

import numpy as np
import pytest
import torch

import coreg
from oracle import roma_ref

CASES = [
    # C, H, W, r: the refiners' radii 7, 3, 2, 1, 0
    (192, 24, 28, 3),
    (48, 40, 36, 1),
    (512, 10, 12, 7),
    (64, 17, 19, 2),
    (16, 21, 23, 0),
    (12, 15, 14, 1),   # C not a multiple of 8: the generic kernel
]


def bf16_round(x):
    u = np.asarray(x, np.float32).view(np.uint32)
    return (((u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000).astype(np.uint32)).view(np.float32)


def oracle(f1, f2, H, W, r, flow):
    """f1, f2 channels-last (H, W, C); flow (2, H, W); out (H, W, side^2)."""
    C = f1.shape[-1]
    run = types.SimpleNamespace(dt=torch.float64)
    a = torch.from_numpy(f1.reshape(-1, C).T.astype(np.float64))
    b = torch.from_numpy(f2.reshape(-1, C).T.astype(np.float64))
    fl = torch.from_numpy(flow.reshape(2, -1).astype(np.float64))
    out = roma_ref.Runner.local_corr(run, a, b, H, W, r, fl)
    return out.numpy().T.reshape(H, W, -1)


@pytest.mark.gpu
@pytest.mark.parametrize("prec", ["fp32", "bf16"])
@pytest.mark.parametrize("case", CASES, ids=[f"C{c}_{h}x{w}_r{r}" for c, h, w, r in CASES])
def test_local_corr_cl(case, prec):
    C, H, W, r = case
    side = 2 * r + 1
    dev = coreg.Device(0, precision=coreg.OPS_BF16 if prec == "bf16" else coreg.OPS_FP32)
    try:
        rng = np.random.default_rng(C + 7 * H + 13 * W + r)
        f1 = rng.standard_normal((H, W, C), dtype=np.float32)
        f2 = rng.standard_normal((H, W, C), dtype=np.float32)
        # Warps around the identity, some beyond the map, one non-finite.
        gx = -1 + (2 * np.arange(W) + 1) / W
        gy = -1 + (2 * np.arange(H) + 1) / H
        flow = np.stack(np.meshgrid(gx, gy)).astype(np.float32)
        flow += rng.uniform(-0.3, 0.3, flow.shape).astype(np.float32)
        flow[0, 0, 0] = np.nan
        A, B, Fl = dev.upload(f1), dev.upload(f2), dev.upload(flow)
        Y = dev.zeros(H * W * side * side)
        dev.lib.roma_local_corr_cl(dev.ops_p, A.handle, B.handle, C, H, W, r, Fl.handle,
                                   Y.handle)
        got = Y.read(count=H * W * side * side).reshape(H, W, side * side)
        coreg.check(dev.lib)
        if prec == "fp32":
            want, bound = oracle(f1, f2, H, W, r, flow), 1e-5
        else:
            want, bound = oracle(bf16_round(f1), bf16_round(f2), H, W, r, flow), 1e-4
        assert np.isfinite(got).all()
        err = np.linalg.norm(got - want) / np.linalg.norm(want)
        assert err <= bound, err
    finally:
        dev.close()
