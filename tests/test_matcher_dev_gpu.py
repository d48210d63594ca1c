# SPDX-License-Identifier: Unlicense
"""RoMa's matcher stages on the device (roma_sample_matches_dev,
roma_dense_field_dev of include/matcher_roma.h) against the host stages
(roma_sample_matches, roma_dense_field), which tests/
test_matcher_host_stage.py pins bit for bit to the reference's own glue
(matcher_roma.c:61-178) (GPU). The device stages must give the same
matches in the same order with the same positions, costs, sd and cycle
distances, and the same dense field, bit for bit, on the host-stage
test's cases: ragged tiles, warps that leave the tile, NaN certainties,
blocks with no valid cell, the cycle distance (a single-column tile
included), spacing 1 and a large spacing."""

import ctypes as C

import numpy as np
import pytest

import coreg
from coreg.roma import MatchList
from test_matcher_host_stage import LIBC, case, ptr, same, sample

CASES = [
    (0, 64, 64, 60, 57, 8, 0.0, False, True, True),
    (1, 64, 80, 64, 80, 8, 0.5, True, True, False),
    (2, 48, 48, 41, 45, 5, 0.2, False, False, True),
    (3, 32, 32, 32, 1, 4, 0.0, False, True, True),
    (4, 40, 40, 33, 39, 1, 0.3, True, True, True),
    (5, 64, 64, 64, 64, 64, 0.0, False, True, True),
    (6, 864, 864, 864, 800, 8, 0.1, True, True, True),
]


@pytest.mark.gpu
@pytest.mark.parametrize("c", CASES, ids=[f"case{c[0]}" for c in CASES])
def test_device_sampling_equals_host(dev, c):
    seed, H, W, h, w, spacing, min_cert, nan_cert, masks, cycle = c
    lib = dev.lib
    flow, cert, sd, bflow, v1, v2 = case(seed, H, W, h, w, nan_cert, masks)
    if w == 1:
        flow[0] = np.float32(1.0 / W - 1.0)
    bf = bflow if cycle else None
    want = sample(lib, flow, cert, sd, bf, h, w, spacing, min_cert, v1, v2)
    bufs = [dev.upload(x) if x is not None else None for x in (flow, cert, sd, bf)]
    ml = MatchList()
    n = lib.roma_sample_matches_dev(dev.ops_p, *(b.ptr if b else None for b in bufs), H, W, h, w,
                                    spacing, min_cert, ptr(v1), ptr(v2), C.byref(ml))
    coreg.check(lib)
    got = [(m.x1, m.y1, m.x2, m.y2, m.cost, m.sd, m.cycle) for m in ml.v[:ml.n]]
    if ml.v:
        LIBC.free(C.cast(ml.v, C.c_void_p))
    assert n == len(got) == len(want) > 0
    for g, r in zip(got, want):
        assert g[:5] == r[:5] and same(g[5], r[5]) and same(g[6], r[6]), (g, r)


@pytest.mark.gpu
@pytest.mark.parametrize("seed,H,W,h,w,masks,with_sd", [
    (0, 64, 64, 60, 57, True, True), (1, 40, 48, 40, 48, False, False),
    (2, 32, 32, 1, 32, True, True), (3, 864, 864, 700, 864, True, True)])
def test_device_field_equals_host(dev, seed, H, W, h, w, masks, with_sd):
    lib = dev.lib
    flow, cert, sd, _, v1, v2 = case(seed, H, W, h, w, False, masks)
    want = [np.empty((h, w), np.float32) for _ in range(4)]
    lib.roma_dense_field(ptr(flow), ptr(cert), ptr(sd) if with_sd else None, H, W, h, w, ptr(v1),
                         ptr(v2), *(x.ctypes.data for x in want))
    got = [np.empty((h, w), np.float32) for _ in range(4)]
    F, Cb, S = dev.upload(flow), dev.upload(cert), dev.upload(sd)
    lib.roma_dense_field_dev(dev.ops_p, F.ptr, Cb.ptr, S.ptr if with_sd else None, H, W, h, w,
                             ptr(v1), ptr(v2), *(x.ctypes.data for x in got))
    coreg.check(lib)
    for a, b in zip(got, want):
        assert np.array_equal(a, b, equal_nan=True)
