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
  32 x 32 input, the four block outputs). Relative L2 <= 1e-5 each.
* the coordinate decoder's five transformer blocks (block roma.c:679-713
  with the decoder's settings roma.c:44-46: 8 heads of 128, no qkv bias,
  LayerNorm eps 1e-5, no LayerScale) against transformers' Dinov2Layer
  configured alike: tests/golden/decoder_golden.npz from
  tests/golden/make_decoder_golden.py (32 tokens). Relative L2 <= 1e-5.
* the input resampling (prepare / resize_axis / pil_cubic,
  roma.c:1106-1186, Pillow's antialiased bicubic restated in double)
  against Pillow's own resize of float ("F" mode) bands: bit-exact, at the
  coarse and fine pass sizes and at odd up / down scalings.
* the local correlation (roma_local_corr, roma_kernels.cl:153-192: whole
  cell dot products around the warp, combined with one set of bilinear
  weights) against the sampling form the refiners were written in: the
  second map bilinearly sampled by torch's grid_sample (align_corners
  False, zero padding) at the warp plus (2r+1)^2 offsets of 2k/W and 2k/H,
  dotted with the first map over sqrt(C). Max |diff| <= 1e-12, warps
  partly outside the map included."""

import math
import types
from pathlib import Path

import numpy as np
import pytest
import torch
import torch.nn.functional as F
from PIL import Image

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


def test_decoder_blocks_match_transformers(model):
    g = np.load(GOLDEN / "decoder_golden.npz")
    run = roma_ref.Runner(model, coarse=112, dtype=torch.float64)
    x = torch.from_numpy(g["x"]).double()
    for b in model.dec:
        x = run.block(x, b, roma_ref.DEC_HEADS, roma_ref.EPS_LN_DEC)
    want = g["out"].astype(np.float64)
    got = x.numpy()
    assert np.linalg.norm(got - want) / np.linalg.norm(want) <= 1e-5


@pytest.mark.parametrize("H,W,h,w", [(1024, 1024, 560, 560), (1024, 1024, 864, 864),
                                     (300, 457, 560, 560), (97, 131, 40, 28),
                                     (864, 864, 864, 864)])
def test_prepare_resampling_matches_pillow(H, W, h, w):
    img = np.random.default_rng(H * 7 + w).random((3, H, W)).astype(np.float32)
    got = roma_ref.prepare(img, h, w, imagenet=False)
    want = np.stack([np.asarray(Image.fromarray(img[c], mode="F").resize((w, h), Image.BICUBIC))
                     for c in range(3)])
    assert got.shape == want.shape
    assert np.array_equal(got, want)


def corr_by_sampling(f1, f2, H, W, r, flow):
    """Local correlation by sampling: f2 at the warp plus whole-cell
    offsets (normalized 2k/W, 2k/H; y-major channel order), dotted with f1."""
    C, side = f1.shape[0], 2 * r + 1
    k = torch.arange(-r, r + 1, dtype=torch.float64)
    oy, ox = torch.meshgrid(2 * k / H, 2 * k / W, indexing="ij")
    grid = torch.stack([flow[0] + ox[..., None], flow[1] + oy[..., None]], -1)
    s = F.grid_sample(f2.reshape(1, C, H, W), grid.reshape(1, side * side, -1, 2),
                      mode="bilinear", padding_mode="zeros", align_corners=False)[0]
    return (s * f1[:, None, :]).sum(0) / math.sqrt(C)


@pytest.mark.parametrize("C,H,W,r", [(16, 12, 14, 0), (16, 12, 14, 1), (8, 9, 11, 3),
                                     (32, 20, 17, 2)])
def test_local_corr_matches_grid_sampling(C, H, W, r):
    g = torch.Generator().manual_seed(C + r)
    n = H * W
    f1 = torch.randn(C, n, generator=g, dtype=torch.float64)
    f2 = torch.randn(C, H, W, generator=g, dtype=torch.float64)
    flow = torch.rand(2, n, generator=g, dtype=torch.float64) * 2.6 - 1.3
    flow[0, :5], flow[1, :5] = -1 + 7 / W, -1 + 5 / H  # exact cell centres
    runner = types.SimpleNamespace(dt=torch.float64)
    got = roma_ref.Runner.local_corr(runner, f1, f2, H, W, r, flow)
    want = corr_by_sampling(f1, f2, H, W, r, flow)
    assert got.shape == want.shape == ((2 * r + 1) ** 2, n)
    assert (got - want).abs().max().item() <= 1e-12
