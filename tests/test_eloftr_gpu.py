# SPDX-License-Identifier: Unlicense
"""Efficient LoFTR (include/eloftr.h) against the oracle
(oracle/eloftr_ref.py: eloftr.c and eloftr_kernels.cl restated; GPU), on
seeded random-init weights in the transformers layout and seeded grey
tiles, float32 as the reference.

The reference's dump points (the 1/8 backbone features, the transformer
output, the fine features) must be within relative L2 1e-5 of the float64
oracle; the coarse matches (cell indices, an integer output) must be the
same set; their confidences within 1e-4 and the refined keypoints within
0.01 px. Random-init weights give few confident mutual matches (the
features of a random RepVGG stack share a large common component), so
several tile pairs are matched."""

import os
import tempfile
from pathlib import Path

import numpy as np
import pytest

import coreg
from coreg import synth
from oracle import eloftr_ref

CACHE = Path(os.environ.get("COREG_CACHE", Path(tempfile.gettempdir()) / "coreg_cache"))
H = W = 128


def weights():
    return synth.write_eloftr_weights(CACHE / "weights", 0)


def pair(seed):
    rng = np.random.default_rng(seed)
    g0 = (synth.band_limited(rng, H, W, 3.0) / 255.0).astype(np.float32)
    if seed % 2:
        g1 = np.roll(g0, (8, 8), (0, 1))
    else:
        g1 = np.clip(g0 + 0.02 * rng.standard_normal(g0.shape), 0, 1).astype(np.float32)
    return g0, g1


def rel(a, b):
    a = np.asarray(a, np.float64).reshape(-1)
    b = np.asarray(b, np.float64).reshape(-1)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


@pytest.mark.gpu
def test_eloftr_matches_oracle(tmp_path):
    from coreg.eloftr import Eloftr

    dev = coreg.Device(0, precision=coreg.OPS_FP32)
    net = Eloftr(dev, weights(), H, W)
    model = eloftr_ref.Model(synth.read_safetensors(weights()))
    total = 0
    try:
        for seed in (1, 2, 3, 4):
            g0, g1 = pair(seed)
            mi, mj, mconf, kp = net.match(g0, g1, dump=tmp_path, tile=seed)
            wi, wj, wc, wkp, dumps = model.run(g0, g1)
            for name, want in dumps.items():
                got = np.fromfile(tmp_path / f"tile{seed:03d}_eloftr_{name}.f32", np.float32)
                assert rel(got, want) <= 1e-5, (seed, name, rel(got, want))
            assert np.array_equal(mi, wi) and np.array_equal(mj, wj), (seed, mi, wi, mj, wj)
            if len(mi):
                assert np.max(np.abs(mconf - wc)) <= 1e-4
                assert np.max(np.abs(kp - wkp)) <= 0.01, (kp, wkp)
            total += len(mi)
    finally:
        net.close()
        dev.close()
    assert total >= 1
