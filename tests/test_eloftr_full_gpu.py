# SPDX-License-Identifier: Unlicense
"""Efficient LoFTR at the configuration's full size (GPU): a 640 x 640
grey pair of configuration 2 (coreg.synth.grey_affine_pair), the device
stage through the C-ABI (eloftr_match, eloftr.c:654-681).

float32 mode against the float64 oracle (oracle/eloftr_ref.py, eloftr.c
and eloftr_kernels.cl restated): the reference's dump points (backbone,
transformer, fine features) within relative L2 1e-5, the same coarse
matches (cell indices, an integer output), confidences within 1e-4 and
refined keypoints within 0.01 px.

bfloat16 mode (tensor-core convolutions and products): the dump points
within relative L2 2e-2 of the oracle, and the properties every match set
has: one-to-one cell pairs (mutual nearest), confidences above the 0.2
threshold, cells off the 2-cell border of the 1/8 grid, keypoints inside
the image and within one fine window of their cells."""

import os
import tempfile
from pathlib import Path

import numpy as np
import pytest

import coreg
from coreg import synth
from oracle import eloftr_ref

CACHE = Path(os.environ.get("COREG_CACHE", Path(tempfile.gettempdir()) / "coreg_cache"))
SIDE = 640


def weights():
    return synth.write_eloftr_weights(CACHE / "weights", 0)


def rel(a, b):
    a = np.asarray(a, np.float64).reshape(-1)
    b = np.asarray(b, np.float64).reshape(-1)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


@pytest.fixture(scope="module")
def pair_and_oracle():
    a, b = synth.grey_affine_pair(2, SIDE, SIDE)
    g0, g1 = a.astype(np.float32) / 255.0, b.astype(np.float32) / 255.0
    model = eloftr_ref.Model(synth.read_safetensors(weights()))
    return g0, g1, model.run(g0, g1)


def check_properties(mi, mj, mconf, kp):
    w = h = SIDE // 8
    assert len(set(mi.tolist())) == len(mi) and len(set(mj.tolist())) == len(mj)
    assert (mconf > 0.2).all()
    for idx in (mi, mj):
        x, y = idx % w, idx // w
        assert ((x >= 2) & (x < w - 2) & (y >= 2) & (y < h - 2)).all()
    assert np.isfinite(kp).all()
    assert ((kp >= -4) & (kp <= SIDE + 4)).all()
    # Each keypoint lies within a fine window (8 px) of its cell's centre.
    for k, idx in ((0, mi), (2, mj)):
        cx, cy = (idx % w) * 8 + 4, (idx // w) * 8 + 4
        assert (np.abs(kp[:, k] - cx) <= 12).all() and (np.abs(kp[:, k + 1] - cy) <= 12).all()


@pytest.mark.gpu
@pytest.mark.parametrize("precision", [coreg.OPS_FP32, coreg.OPS_BF16], ids=["fp32", "bf16"])
def test_eloftr_config2_full_size(tmp_path, pair_and_oracle, precision):
    from coreg.eloftr import Eloftr

    g0, g1, (wi, wj, wc, wkp, dumps) = pair_and_oracle
    dev = coreg.Device(0, precision=precision)
    net = Eloftr(dev, weights(), SIDE, SIDE)
    try:
        mi, mj, mconf, kp = net.match(g0, g1, dump=tmp_path, tile=1)
    finally:
        net.close()
        dev.close()
    bound = 1e-5 if precision == coreg.OPS_FP32 else 2e-2
    for name, want in dumps.items():
        got = np.fromfile(tmp_path / f"tile001_eloftr_{name}.f32", np.float32)
        assert rel(got, want) <= bound, (name, rel(got, want))
    check_properties(mi, mj, mconf, kp)
    if precision == coreg.OPS_FP32:
        assert np.array_equal(mi, wi) and np.array_equal(mj, wj), (mi, wi, mj, wj)
        if len(mi):
            assert np.max(np.abs(mconf - wc)) <= 1e-4
            assert np.max(np.abs(kp - wkp)) <= 0.01
