# SPDX-License-Identifier: Unlicense
"""DISK (include/disk.h) and the descriptor-distance stage against the
oracle (oracle/disk_ref.py: disk.c, disk_kernels.cl and adalam.c:38-98
restated; GPU).

float32 throughout, as the reference. The network output must be within
relative L2 1e-5 of the float64 oracle; keypoint positions (NMS, the n-best
selection) and nearest-neighbour indices are integer outputs and must be
identical, except where the oracle's own margin (the gap between the two
values an index decision compares) is below float32 resolution, which the
tests count and bound."""

import os
import tempfile
from pathlib import Path

import numpy as np
import pytest

import coreg
from coreg import synth
from oracle import disk_ref

CACHE = Path(os.environ.get("COREG_CACHE", Path(tempfile.gettempdir()) / "coreg_cache"))


def weights():
    return synth.write_disk_weights(CACHE / "weights", 0)


def image(seed, H, W):
    rng = np.random.default_rng(seed)
    img = np.stack([synth.band_limited(rng, H, W, 2.0) for _ in range(3)]) / 255.0
    return img.astype(np.float32)


def rel(a, b):
    a = np.asarray(a, np.float64).reshape(-1)
    b = np.asarray(b, np.float64).reshape(-1)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


@pytest.fixture(scope="module")
def disk64():
    from coreg.disk import Disk

    dev = coreg.Device(0, precision=coreg.OPS_FP32)
    d = Disk(dev, weights(), 64, 64, nmax=64)
    yield dev, d
    d.close()
    dev.close()


@pytest.mark.gpu
def test_disk_network_and_keypoints_match_oracle(disk64):
    dev, d = disk64
    img = image(1, 64, 64)
    xy, score, desc = d.detect(img, h=60, w=60, n=40)
    out = d.output(64, 64)
    w = synth.read_safetensors(weights())
    want_out, want_xy, want_score, want_desc = disk_ref.detect(img, w, 60, 60, 40)
    assert rel(out, want_out) <= 1e-5, rel(out, want_out)
    assert len(xy) > 0
    assert np.array_equal(xy, want_xy), (xy[:5], want_xy[:5])
    assert rel(score, want_score) <= 1e-5
    assert rel(desc, want_desc) <= 1e-5


@pytest.mark.gpu
def test_disk_valid_mask_and_fewer_candidates(disk64):
    dev, d = disk64
    img = image(2, 64, 64)
    valid = np.ones((64, 64), np.uint8)
    valid[:, :32] = 0
    xy, score, _ = d.detect(img, n=1000, valid=valid)
    w = synth.read_safetensors(weights())
    out = disk_ref.unet(img, w)
    mask = disk_ref.nms_mask(out[disk_ref.DESC], 64, 64, 0.0)
    want_xy, _ = disk_ref.select(out[disk_ref.DESC], mask, 1000, valid)
    assert np.all(xy[:, 0] >= 32)
    assert np.array_equal(xy, want_xy)


@pytest.mark.gpu
@pytest.mark.parametrize("n1,n2", [(300, 257), (2048, 2048)])
def test_desc_nearest_matches_oracle(dev, n1, n2):
    from coreg.disk import nearest

    rng = np.random.default_rng(n1 + n2)
    d1 = rng.standard_normal((n1, 128)).astype(np.float32)
    d2 = rng.standard_normal((n2, 128)).astype(np.float32)
    d1 /= np.linalg.norm(d1, axis=1, keepdims=True)
    d2 /= np.linalg.norm(d2, axis=1, keepdims=True)
    nn12, score, nn21 = nearest(dev, d1, d2)
    w12, wscore, w21, gap, col_gap = disk_ref.nearest(d1, d2)
    # Float32 resolves distances of these unit vectors to about 1e-6.
    sure = gap > 1e-5
    assert np.array_equal(nn12[sure], w12[sure])
    assert (~sure).mean() < 0.01
    assert np.max(np.abs(score - wscore) / np.maximum(np.abs(wscore), 1e-6)) < 1e-4
    sure21 = col_gap > 1e-5
    assert np.array_equal(nn21[sure21], w21[sure21])
