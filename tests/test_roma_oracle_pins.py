# SPDX-License-Identifier: Unlicense
"""The RoMa oracle (oracle/roma_ref.py, the reference's roma.c restated)
pinned to the libraries the RoMa model is built from, on the same seeded
synthetic weights (CPU only, float64):

* the DINOv2 ViT-L/14 encoder (position interpolation roma.c:257-298,
  dino roma.c:717-738, LayerScale folded at load roma.c:155-214) against
  transformers' Dinov2Model: tests/golden/dino_golden.npz from
  tests/golden/make_dino_golden.py (a 112 x 112 image, DINOv2's original
  interpolation of the position table). Table: max |diff| <= 1e-6;
  patch tokens: relative L2 <= 1e-5 (float32 fixture; the oracle folds
  LayerScale into float32 weights as the reference does).
* the VGG19-BN pyramid (load_vgg roma.c:217-239 with its BatchNorm
  folding, vgg roma.c:742-768) against torchvision's vgg19_bn features:
  tests/golden/vgg_golden.npz from tests/golden/make_vgg_golden.py (a
  32 x 32 input, the four block outputs). Relative L2 <= 1e-5 each."""

from pathlib import Path

import numpy as np
import pytest
import torch

from coreg import synth
from oracle import roma_ref

GOLDEN = Path(__file__).resolve().parent / "golden"


@pytest.fixture(scope="module")
def model():
    main, dino, _ = synth.roma_weights(0)
    return roma_ref.Model(main, dino)


def test_dino_encoder_matches_transformers(model):
    g = np.load(GOLDEN / "dino_golden.npz")
    run = roma_ref.Runner(model, coarse=112, dtype=torch.float64)
    assert np.abs(run.pos.numpy() - g["pos"]).max() <= 1e-6
    run.dino(torch.from_numpy(g["img"]).double(), 0)
    got = run.dumps["dino_0"].numpy().T           # (64, 1024) patch tokens
    want = g["out"][1:].astype(np.float64)
    assert np.linalg.norm(got - want) / np.linalg.norm(want) <= 1e-5


def test_vgg_pyramid_matches_torchvision(model):
    g = np.load(GOLDEN / "vgg_golden.npz")
    run = roma_ref.Runner(model, coarse=112, dtype=torch.float64)
    got = {}

    def keep(name):
        def f(x, k):
            got[name] = x.numpy()
        return f

    run.vgg(torch.from_numpy(g["img"]).double(), 0, None,
            [keep("f1"), keep("f2"), keep("f4"), keep("f8")], model.vgg)
    for name in ("f1", "f2", "f4", "f8"):
        want = g[name].astype(np.float64)
        assert got[name].shape == want.shape
        assert np.linalg.norm(got[name] - want) / np.linalg.norm(want) <= 1e-5, name
