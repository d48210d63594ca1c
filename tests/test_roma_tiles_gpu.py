# SPDX-License-Identifier: Unlicense
"""The RoMa tile queue (include/roma_tiles.h) on one GPU with three
pipelines (GPU): every tile's warp, certainty and sd equal, bit for bit,
roma_match of the same tile on a model of its own (tiles are independent
and each pipeline's kernels are deterministic), and the results arrive in
tile-index order although the pipelines finish out of order. A missing
weight file is a recorded error and no queue."""

import threading

import numpy as np
import pytest

import coreg
from coreg.roma import Roma, RomaTiles
from roma_fixtures import tile_pair, weight_paths

H = W = 128
COARSE = 224


@pytest.mark.gpu
@pytest.mark.parametrize("precision", [coreg.OPS_BF16, coreg.OPS_FP32], ids=["bf16", "fp32"])
def test_tiles_in_order_and_equal_to_roma_match(precision):
    main, dino, v2 = weight_paths()
    tiles = [tile_pair(50 + i, H, W)[:2] for i in range(7)]
    dev = coreg.Device(0, precision=precision)
    solo = Roma(dev, main, dino, v2, H=H, W=W, coarse=COARSE)
    try:
        want = [tuple(np.copy(x) for x in solo.match(*t)) for t in tiles]
    finally:
        solo.close()
        dev.close()
    q = RomaTiles([0], 3, precision, main, dino, v2, H=H, W=W, coarse=COARSE)
    got, threads = [], set()

    def get(i, a, b):
        a[...] = tiles[i][0]
        b[...] = tiles[i][1]
        threads.add(threading.get_ident())

    def put(i, flow, cert, sd):
        got.append((i, flow.copy(), cert.copy(), sd.copy()))

    try:
        assert q.pipelines == 3
        assert q.run(len(tiles), get, put) == len(tiles)
        # A second run on the same queue (graphs already built).
        got2 = []
        q.run(3, get, lambda i, f, c, s: got2.append((i, f.copy())))
    finally:
        q.close()
    assert [g[0] for g in got] == list(range(len(tiles)))
    assert len(threads) > 1
    for (i, f, c, s), w in zip(got, want):
        assert np.array_equal(f, w[0], equal_nan=True), i
        assert np.array_equal(c, w[1], equal_nan=True), i
        assert np.array_equal(s, w[2], equal_nan=True), i
    assert [g[0] for g in got2] == [0, 1, 2]
    assert all(np.array_equal(f, want[i][0], equal_nan=True) for i, f in got2)


@pytest.mark.gpu
def test_tiles_missing_weights_is_an_error(tmp_path):
    main, dino, v2 = weight_paths()
    coreg.load().coreg_set_error_mode(coreg.ERRORS_RECORD)
    with pytest.raises(coreg.CoregError, match="roma_tiles_create"):
        RomaTiles([0], 2, coreg.OPS_BF16, tmp_path / "missing.safetensors", dino, v2, H=H, W=W,
                  coarse=COARSE)


def device_count():
    import torch

    return torch.cuda.device_count()


@pytest.mark.gpu
def test_tiles_over_two_devices_in_order():
    """Two devices, two pipelines each: the tiles are dealt across both GPUs
    and come back in order, each equal to a single-device roma_match bit
    for bit (bfloat16; the same kernels on every B200). Skips on a machine
    with one GPU."""
    if device_count() < 2:
        pytest.skip("needs two GPUs")
    main, dino, v2 = weight_paths()
    tiles = [tile_pair(70 + i, H, W)[:2] for i in range(9)]
    dev = coreg.Device(0, precision=coreg.OPS_BF16)
    solo = Roma(dev, main, dino, v2, H=H, W=W, coarse=COARSE)
    try:
        want = [np.copy(solo.match(*t)[0]) for t in tiles]
    finally:
        solo.close()
        dev.close()
    q = RomaTiles([0, 1], 2, coreg.OPS_BF16, main, dino, v2, H=H, W=W, coarse=COARSE)
    got = []

    def get(i, a, b):
        a[...] = tiles[i][0]
        b[...] = tiles[i][1]

    try:
        assert q.pipelines == 4
        assert q.run(len(tiles), get, lambda i, f, c, s: got.append((i, f.copy()))) == len(tiles)
    finally:
        q.close()
    assert [g[0] for g in got] == list(range(len(tiles)))
    for (i, f), w in zip(got, want):
        assert np.array_equal(f, w, equal_nan=True), i
