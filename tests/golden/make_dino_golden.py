# SPDX-License-Identifier: Unlicense
"""Generate tests/golden/dino_golden.npz: RoMa's DINOv2 ViT-L/14 encoder
(patch embedding, class token, interpolated position embeddings, the 24
blocks with LayerScale, final LayerNorm) evaluated by transformers' own
Dinov2Model in float64, with the seeded synthetic weights of
coreg.synth.roma_weights(0) (the DINOv2 state dict in the original
facebookresearch names, mapped onto transformers' layout below), on a
seeded 112 x 112 image (an 8 x 8 patch grid, so that the fixture stays
small).

Position embeddings: DINOv2's original interpolate_pos_encoding (which the
reference's roma.c follows) resamples the 37 x 37 table with
torch.nn.functional.interpolate(scale_factor=(8 + 0.1) / 37, bicubic,
align_corners=False); transformers' model resamples to a fixed size
instead. So the table is interpolated here with the original call and
loaded as a model whose own grid is 8 x 8, which transformers uses
unresampled. Stores as float32:

    img                     the input (3, 112, 112)
    pos                     the interpolated table (1 + 64, 1024)
    out                     last_hidden_state (1 + 64, 1024)

Needs transformers and torch (present in the build container); run from
the repository root:

    python tests/golden/make_dino_golden.py
"""

import sys
from pathlib import Path

import numpy as np
import torch
import torch.nn.functional as F
from transformers import Dinov2Config, Dinov2Model

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT / "i.coregistration.opencl_b200"))

from coreg import synth  # noqa: E402

GRID, D, DEPTH, HEADS = 8, 1024, 24, 16


def hf_state(dino, pos):
    """transformers' Dinov2Model state dict from the original names."""
    t = lambda a: torch.from_numpy(np.asarray(a, np.float64))
    s = {
        "embeddings.patch_embeddings.projection.weight": t(dino["patch_embed.proj.weight"]),
        "embeddings.patch_embeddings.projection.bias": t(dino["patch_embed.proj.bias"]),
        "embeddings.cls_token": t(dino["cls_token"]),
        "embeddings.position_embeddings": t(pos)[None],
        "layernorm.weight": t(dino["norm.weight"]),
        "layernorm.bias": t(dino["norm.bias"]),
    }
    for i in range(DEPTH):
        b, o = f"blocks.{i}.", f"encoder.layer.{i}."
        qkv_w, qkv_b = t(dino[b + "attn.qkv.weight"]), t(dino[b + "attn.qkv.bias"])
        for j, n in enumerate(("query", "key", "value")):
            s[o + f"attention.attention.{n}.weight"] = qkv_w[j * D:(j + 1) * D]
            s[o + f"attention.attention.{n}.bias"] = qkv_b[j * D:(j + 1) * D]
        for src, dst in (("norm1", "norm1"), ("norm2", "norm2"), ("attn.proj", "attention.output.dense"),
                         ("mlp.fc1", "mlp.fc1"), ("mlp.fc2", "mlp.fc2")):
            s[o + dst + ".weight"] = t(dino[b + src + ".weight"])
            s[o + dst + ".bias"] = t(dino[b + src + ".bias"])
        s[o + "layer_scale1.lambda1"] = t(dino[b + "ls1.gamma"])
        s[o + "layer_scale2.lambda1"] = t(dino[b + "ls2.gamma"])
    return s


def main():
    dino = synth.roma_weights(0)[1]
    raw = torch.from_numpy(np.asarray(dino["pos_embed"], np.float64)).reshape(1, 37 * 37 + 1, D)
    grid = raw[:, 1:].reshape(1, 37, 37, D).permute(0, 3, 1, 2)
    patch = F.interpolate(grid, scale_factor=((GRID + 0.1) / 37, (GRID + 0.1) / 37),
                          mode="bicubic", align_corners=False)
    assert patch.shape[-2:] == (GRID, GRID)
    pos = torch.cat([raw[:, :1], patch.permute(0, 2, 3, 1).reshape(1, -1, D)], 1)[0]

    cfg = Dinov2Config(hidden_size=D, num_hidden_layers=DEPTH, num_attention_heads=HEADS,
                       mlp_ratio=4, patch_size=14, image_size=14 * GRID, layerscale_value=1.0,
                       layer_norm_eps=1e-6, hidden_act="gelu", qkv_bias=True)
    cfg._attn_implementation = "eager"
    model = Dinov2Model(cfg).double().eval()
    res = model.load_state_dict(hf_state(dino, pos.numpy()), strict=False)
    if res.unexpected_keys or set(res.missing_keys) - {"embeddings.mask_token"}:
        raise SystemExit(f"weight names differ: {res.missing_keys[:5]} {res.unexpected_keys[:5]}")
    img = np.random.default_rng(7).standard_normal((3, 14 * GRID, 14 * GRID)).astype(np.float32)
    with torch.no_grad():
        out = model(torch.from_numpy(img).double()[None]).last_hidden_state[0]
    dst = ROOT / "tests" / "golden" / "dino_golden.npz"
    np.savez_compressed(dst, img=img, pos=pos.numpy().astype(np.float32),
                        out=out.numpy().astype(np.float32))
    print(f"{dst} ({dst.stat().st_size} bytes)")


if __name__ == "__main__":
    main()
