# SPDX-License-Identifier: Unlicense
"""DISK at the configuration's full size and in bfloat16 mode (GPU).

Configuration 5 runs DISK on 1024 x 1024 RGB tiles with the top 2048
keypoints and matches the descriptors (disk.c:164-253, adalam.c:38-98).
The float64 oracle (oracle/disk_ref.py) takes minutes there, so the full
size is checked through properties that hold whatever the network's
values are, against the network output the device itself produced (read
back through disk_output_dev):
  - every keypoint is a strict 5 x 5 maximum of the heatmap above the
    threshold, off the 2-cell border (disk_kernels.cl:10-35);
  - the keypoints are exactly the n-best rule (disk.c:236-266) applied to
    that heatmap: the candidates above the (n + 1)-th highest, in raster
    order, at most n;
  - scores are the heatmap at the keypoints, descriptors the L2-normalized
    descriptor channels there (disk_kernels.cl:39-60);
  - the device's nearest neighbours of the two tiles' descriptors equal a
    float64 host recomputation wherever the two compared distances differ
    by more than float32 resolves (adalam.c:62-94).
The bfloat16 mode (tensor-core convolutions) is compared with the float64
oracle at 128 x 128: relative L2 within 2e-2 for the heatmap and the
descriptor channels."""

import os
import tempfile
from pathlib import Path

import numpy as np
import pytest

import coreg
from coreg import synth
from oracle import disk_ref

CACHE = Path(os.environ.get("COREG_CACHE", Path(tempfile.gettempdir()) / "coreg_cache"))
DESC = disk_ref.DESC


def weights():
    return synth.write_disk_weights(CACHE / "weights", 0)


def tile_pair(seed, side):
    a, b, _ = synth.scene_pair(seed, side, side)
    return synth.tile_input(a, side, side), synth.tile_input(b, side, side)


def rel(a, b):
    a = np.asarray(a, np.float64).reshape(-1)
    b = np.asarray(b, np.float64).reshape(-1)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def strict_max_mask(heat, thresh):
    """nms5x5 on the whole map, vectorized: strictly above the 24
    neighbours and thresh, 2-cell border excluded."""
    h, w = heat.shape
    c = heat[2:h - 2, 2:w - 2]
    ok = c > thresh
    for dy in range(-2, 3):
        for dx in range(-2, 3):
            if dy or dx:
                ok &= c > heat[2 + dy:h - 2 + dy, 2 + dx:w - 2 + dx]
    mask = np.zeros((h, w), bool)
    mask[2:h - 2, 2:w - 2] = ok
    return mask


def n_best(heat, mask, n):
    """The n-best rule (disk.c:236-266) in raster order, vectorized."""
    cand = np.sort(heat[mask])[::-1]
    cut = cand[min(n, cand.size - 1)] if cand.size else -np.inf
    ys, xs = np.nonzero(mask & (heat > cut))
    return np.stack([xs, ys], 1)[:n]


def check_detection(d, img, n):
    xy, score, desc = d.detect(img, n=n)
    H, W = img.shape[1:]
    out = d.output(H, W)
    heat = out[DESC]
    mask = strict_max_mask(heat, 0.0)
    assert 0 < len(xy) <= n
    assert mask[xy[:, 1], xy[:, 0]].all()
    assert np.array_equal(xy, n_best(heat, mask, n))
    assert np.array_equal(score, heat[xy[:, 1], xy[:, 0]])
    want = disk_ref.gather(out, xy)
    assert np.abs(desc - want).max() <= 1e-6
    assert np.allclose(np.linalg.norm(desc, axis=1), 1.0, atol=1e-5)
    return xy, desc


@pytest.mark.gpu
@pytest.mark.parametrize("precision", [coreg.OPS_FP32, coreg.OPS_BF16], ids=["fp32", "bf16"])
def test_disk_config5_full_size(precision):
    from coreg.disk import Disk, nearest

    side, n = 1024, 2048
    dev = coreg.Device(0, precision=precision)
    d = Disk(dev, weights(), side, side, nmax=n)
    try:
        A, B = tile_pair(21, side)
        _, da = check_detection(d, A, n)
        _, db = check_detection(d, B, n)
        nn12, score, nn21 = nearest(dev, da, db)
        w12, wscore, w21, gap, col_gap = disk_ref.nearest(da, db)
        sure = gap > 1e-5
        assert (~sure).mean() < 0.01
        assert np.array_equal(nn12[sure], w12[sure])
        assert np.array_equal(nn21[col_gap > 1e-5], w21[col_gap > 1e-5])
        # The ratio of two float32 distances |a|^2 + |b|^2 - 2 a.b of unit
        # vectors: each carries an absolute error of about 1e-6 from the
        # cancellation, so near matches (distances of a few 1e-2) see
        # relative errors up to a few 1e-4.
        assert np.max(np.abs(score - wscore) / np.maximum(np.abs(wscore), 1e-6)) < 1e-3
    finally:
        d.close()
        dev.close()


@pytest.mark.gpu
def test_disk_bf16_network_matches_oracle():
    from coreg.disk import Disk

    side = 128
    dev = coreg.Device(0, precision=coreg.OPS_BF16)
    d = Disk(dev, weights(), side, side, nmax=256)
    try:
        img = tile_pair(22, side)[0]
        check_detection(d, img, 256)
        out = d.output(side, side)
        want = disk_ref.unet(img, synth.read_safetensors(weights()))
        e_heat, e_desc = rel(out[DESC], want[DESC]), rel(out[:DESC], want[:DESC])
        assert e_heat <= 2e-2 and e_desc <= 2e-2, (e_heat, e_desc)
    finally:
        d.close()
        dev.close()
