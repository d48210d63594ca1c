# SPDX-License-Identifier: Unlicense
"""The Efficient LoFTR oracle (oracle/eloftr_ref.py, the reference's
eloftr.c restated) pinned to transformers' EfficientLoFTRForKeypointMatching
through the coarse stage: the golden fixture (tests/golden/eloftr_golden.npz,
made by tests/golden/make_eloftr_golden.py with the same seeded synthetic
weights) holds that model's transformer output and coarse matches for a
128 x 160 grey pair. CPU only.

Coarse features: relative L2 <= 1e-6, max |diff| <= 1e-4 (the fixture is
float32; transformers applies RoPE in float32). Coarse matches: the same
cell pairs, confidences within 1e-5."""

from pathlib import Path

import numpy as np

from coreg import synth
from oracle import eloftr_ref

GOLDEN = Path(__file__).resolve().parent / "golden" / "eloftr_golden.npz"


def test_eloftr_oracle_coarse_stage_matches_transformers():
    g = np.load(GOLDEN)
    m = eloftr_ref.Model(synth.eloftr_weights(0), pos_scale=1.0)
    f0, f1 = m.backbone(g["grey0"]), m.backbone(g["grey1"])
    x0, x1 = m.transformer(f0[2], f1[2])
    for got, want in ((x0, g["coarse0"]), (x1, g["coarse1"])):
        want = want.astype(np.float64)
        assert np.linalg.norm(got - want) / np.linalg.norm(want) <= 1e-6
        assert np.abs(got - want).max() <= 1e-4
    mi, mj, mc = eloftr_ref.coarse_match(x0, x1)
    # transformers' matches[1][i]: the second image's cell matched to cell
    # i of the first (-1: none), scores[1][i] its confidence.
    want_i = np.nonzero(g["matches"][1] >= 0)[0]
    assert len(want_i) > 0
    assert list(mi) == list(want_i)
    assert list(mj) == list(g["matches"][1][want_i])
    assert np.allclose(mc, g["scores"][1][want_i], atol=1e-5)
