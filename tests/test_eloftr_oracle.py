# SPDX-License-Identifier: Unlicense
"""The Efficient LoFTR oracle (oracle/eloftr_ref.py, the reference's
eloftr.c restated) pinned to transformers' EfficientLoFTRForKeypointMatching
with the same seeded synthetic weights, on the 128 x 160 grey pair of
tests/golden/eloftr_golden.npz (made by tests/golden/make_eloftr_golden.py).
CPU only.

- Coarse stage (backbone, aggregated attention with RoPE): the model's
  transformer output, relative L2 <= 1e-6, max |diff| <= 1e-4 (the fixture
  is float32; transformers applies RoPE in float32). Coarse matches: the
  same cell pairs, confidences within 1e-5.
- Fine features (the fusion of eloftr.c:575-604): the model's refinement
  layer at 4096 seeded positions per image, same bounds as the coarse
  output.
- Fine matches (eloftr_kernels.cl:146-295, the authors' two-stage
  FineMatching): for 320 cell pairs, the keypoints of the fixture's
  vectorised torch restatement on the model's own fine windows, within
  1e-5 px; the first stage's discrete choices therefore agree."""

from pathlib import Path

import numpy as np
import pytest

from coreg import synth
from oracle import eloftr_ref

GOLDEN = Path(__file__).resolve().parent / "golden" / "eloftr_golden.npz"


@pytest.fixture(scope="module")
def stages():
    g = np.load(GOLDEN)
    m = eloftr_ref.Model(synth.eloftr_weights(0), pos_scale=1.0)
    f0, f1 = m.backbone(g["grey0"]), m.backbone(g["grey1"])
    x0, x1 = m.transformer(f0[2], f1[2])
    return g, m, (f0, f1), (x0, x1)


def close(got, want, rel=1e-6, atol=1e-4):
    want = want.astype(np.float64)
    assert np.linalg.norm(got - want) / np.linalg.norm(want) <= rel
    assert np.abs(got - want).max() <= atol


def test_eloftr_oracle_coarse_stage_matches_transformers(stages):
    g, _, _, (x0, x1) = stages
    close(x0, g["coarse0"])
    close(x1, g["coarse1"])
    mi, mj, mc = eloftr_ref.coarse_match(x0, x1)
    # transformers' matches[1][i]: the second image's cell matched to cell
    # i of the first (-1: none), scores[1][i] its confidence.
    want_i = np.nonzero(g["matches"][1] >= 0)[0]
    assert len(want_i) > 0
    assert list(mi) == list(want_i)
    assert list(mj) == list(g["matches"][1][want_i])
    assert np.allclose(mc, g["scores"][1][want_i], atol=1e-5)


def test_eloftr_oracle_fine_stage_matches_transformers(stages):
    g, m, f, x = stages
    H, W = g["grey0"].shape
    fine = [m.fusion(x[k], f[k][1], f[k][0], H, W) for k in range(2)]
    for k in range(2):
        close(fine[k].reshape(-1)[g["fine_at"]], g["fine_samples"][k])
    w = x[0].shape[2]
    kp = np.array([eloftr_ref.fine_one(fine[0], fine[1], i % w, i // w, j % w, j // w)
                   for i, j in g["pairs"]])
    assert np.abs(kp - g["fine_kp"]).max() <= 1e-5
