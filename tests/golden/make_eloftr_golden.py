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
    fine_at                 4096 seeded flat indices into a (64, 128, 160)
                            fine map
    fine_samples            the model's fine features (its refinement
                            layer's forward_pyramid on the coarse output and
                            the backbone's 1/4 and 1/2 maps) at fine_at,
                            (2, 4096): one row per image
    pairs                   (320, 2) cell pairs (i, j): every cell i of the
                            first image with the cell j one step right and
                            down in the second (the pair's 8-pixel shift),
                            clipped to the map, so that the windows of the
                            last row and column reach the zero padding
    fine_sel                (320, 2) the first fine stage's window positions
                            (8 x 8 window of the first image, inner 8 x 8 of
                            the second's 10 x 10 window)
    fine_kp                 (320, 4) float64 (x0, y0, x1, y1) in pixels after
                            both fine stages

The fine matches follow the authors' two-stage FineMatching, which the
reference's eloftr_kernels.cl implements and transformers departs from
(its first stage scales by the 56 sliced channels, not all 64, and it pairs
the row and column maxima of different cells). They are computed here,
vectorised in torch, on the model's own unfolded fine windows (8 x 8 with
stride 8 in the first image, 10 x 10 with padding 1 in the second):
first stage, dual softmax of the first 56 channels over sqrt(64) each,
restricted to the inner 8 x 8 of the second window, first maximum; second
stage, the last 8 channels (the second image's over sqrt(8)), the 3 x 3
neighbourhood of the chosen position read with the inner index used as a
10 x 10 one (index -1 wraps to 9), softmax at temperature 10, expectation
added to the second keypoint. Keypoints: 8 x cell + window position - 3.5.

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


def fine_stage(model, feats, coarse):
    """The fine features' samples and the fine matches of every cell."""
    fw, sl, temp = (model.config.fine_kernel_size, model.config.fine_matching_slice_dim,
                    model.config.fine_matching_regress_temperature)
    d, h, w = coarse.shape[1:]
    fine = model.refinement_layer.forward_pyramid(coarse / d ** 0.5, [feats[2], feats[1]])
    at = np.random.default_rng(11).choice(fine[0].numel(), 4096, replace=False)
    samples = fine.reshape(2, -1)[:, at]

    i = torch.arange(h * w)
    j = torch.clamp(i // w + 1, max=h - 1) * w + torch.clamp(i % w + 1, max=w - 1)

    win0 = torch.nn.functional.unfold(fine[0:1], fw, stride=8)[0]
    win1 = torch.nn.functional.unfold(fine[1:2], fw + 2, stride=8, padding=1)[0]
    c = fine.shape[1]
    win0 = win0.reshape(c, fw * fw, -1).permute(2, 1, 0)[i]
    win1 = win1.reshape(c, (fw + 2) ** 2, -1).permute(2, 1, 0)[j]
    s1 = win0[..., :c - sl] @ win1[..., :c - sl].transpose(1, 2) / c
    p = torch.softmax(s1, 1) * torch.softmax(s1, 2)
    p = p.reshape(-1, fw * fw, fw + 2, fw + 2)[..., 1:-1, 1:-1].reshape(len(i), -1)
    best = torch.from_numpy(np.argmax(p.numpy(), 1))
    a, b = best // (fw * fw), best % (fw * fw)
    s2 = win0[..., c - sl:] @ (win1[..., c - sl:] / sl ** 0.5).transpose(1, 2)
    s2 = s2.reshape(-1, fw * fw, fw + 2, fw + 2)
    r = torch.arange(-1, 2)
    m = torch.arange(len(i))[:, None, None]
    nb = s2[m, a[:, None, None], (b // fw)[:, None, None] + r[:, None],
            (b % fw)[:, None, None] + r[None, :]].reshape(-1, 9)
    heat = torch.softmax(nb / temp, -1).reshape(-1, 3, 3)
    ex = (heat.sum(1) * r).sum(-1)
    ey = (heat.sum(2) * r).sum(-1)
    off = fw / 2 - 0.5
    kp = torch.stack([8 * (i % w) + a % fw - off, 8 * (i // w) + a // fw - off,
                      8 * (j % w) + b % fw - off + ex, 8 * (j // w) + b // fw - off + ey], 1)
    return (at.astype(np.int32), samples.numpy().astype(np.float32),
            torch.stack([i, j], 1).numpy().astype(np.int32),
            torch.stack([a, b], 1).numpy().astype(np.int32), kp.numpy())


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
        fine_at, fine_samples, pairs, fine_sel, fine_kp = fine_stage(
            model, feats, feats[0].reshape(2, 256, H // 8, W // 8))
    coarse = feats[0].reshape(2, 256, H // 8, W // 8).numpy()
    np.savez_compressed(ROOT / "tests" / "golden" / "eloftr_golden.npz",
                        grey0=g0, grey1=g1,
                        coarse0=coarse[0].astype(np.float32), coarse1=coarse[1].astype(np.float32),
                        matches=out.matches[0].numpy().astype(np.int32),
                        scores=out.matching_scores[0].numpy().astype(np.float32),
                        fine_at=fine_at, fine_samples=fine_samples, pairs=pairs,
                        fine_sel=fine_sel, fine_kp=fine_kp)
    print("coarse", coarse.shape, "matches", out.matches.shape)


if __name__ == "__main__":
    main()
