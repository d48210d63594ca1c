# SPDX-License-Identifier: Unlicense
"""Generate tests/golden/eloftr_golden.npz: the Efficient LoFTR coarse stage
(RepVGG backbone, then the four aggregated self / cross attention layers
with RoPE) and the coarse matches, evaluated by transformers' own
EfficientLoFTRForKeypointMatching in float64 (its rotary step runs in
float32, as transformers writes it), with the seeded synthetic weights of
coreg.synth.eloftr_weights(0), which use that model's parameter names.

Input: a 128 x 160 grey pair (band-limited noise from seed 5, the second a
copy shifted by (8, 8) pixels), so that the coarse map is 16 x 20 cells and
the aggregated one 4 x 5. Stores as float32:

    grey0, grey1            the input pair
    coarse0, coarse1        the transformer's output, (256, 16, 20) each
    matches, scores         the model's coarse matches (cell index pairs,
                            -1 where none) and their confidences

The RoPE positions of transformers' model are the cell indices plus one,
i.e. the reference's table with position scale 1.

Needs transformers and torch (present in the build container); run from
the repository root:

    python tests/golden/make_eloftr_golden.py
"""

import sys
from pathlib import Path

import numpy as np
import torch
from transformers import EfficientLoFTRConfig, EfficientLoFTRForKeypointMatching

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT / "i.coregistration.opencl_b200"))

from coreg import synth  # noqa: E402

H, W = 128, 160


def grey_pair():
    rng = np.random.default_rng(5)
    base = synth.band_limited(rng, H + 8, W + 8, 3.0) / 255.0
    return (np.ascontiguousarray(base[8:, 8:], np.float32),
            np.ascontiguousarray(base[:H, :W], np.float32))


def main():
    sd = synth.eloftr_weights(0)
    model = EfficientLoFTRForKeypointMatching(EfficientLoFTRConfig()).double().eval()
    state = {k: torch.from_numpy(np.asarray(v)).double() for k, v in sd.items()}
    res = model.load_state_dict(state, strict=False)
    if res.unexpected_keys or res.missing_keys:
        raise SystemExit(f"weight names differ: missing {res.missing_keys[:5]} "
                         f"unexpected {res.unexpected_keys[:5]}")
    g0, g1 = grey_pair()
    pix = torch.from_numpy(np.stack([g0, g1])).double()[None, :, None]
    with torch.no_grad():
        feats = model.efficientloftr(pix).feature_maps
        out = model(pix)
    coarse = feats[0].reshape(2, 256, H // 8, W // 8).numpy()
    np.savez_compressed(ROOT / "tests" / "golden" / "eloftr_golden.npz",
                        grey0=g0, grey1=g1,
                        coarse0=coarse[0].astype(np.float32), coarse1=coarse[1].astype(np.float32),
                        matches=out.matches[0].numpy().astype(np.int32),
                        scores=out.matching_scores[0].numpy().astype(np.float32))
    print("coarse", coarse.shape, "matches", out.matches.shape)


if __name__ == "__main__":
    main()
