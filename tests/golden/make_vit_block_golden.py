# SPDX-License-Identifier: Unlicense
"""Generate tests/golden/vit_block_golden.npz: one DINOv2 transformer block
(the BASELINE config-1 block: pre-LayerNorm eps 1e-6, qkv with bias, GELU
MLP of ratio 4, LayerScale 1e-5) evaluated by transformers' own
Dinov2Layer in float64, at a reduced size (65 tokens, width 128, 4 heads)
so that the fixture stays small. Weights ~N(0, 0.02) from seed 0 (LayerNorm
gains 1 + N(0, 0.02)), tokens ~N(0, 1) from seed 1. Stores the inputs, the
weights and every intermediate tensor as float32:

    ln1, q, k, v, ctx (attention before the output projection), attn
    (output projection), ln2, fc1 (before GELU), mlp (fc2 output), out

Needs transformers and torch (present in the build container); run from
the repository root:

    python tests/golden/make_vit_block_golden.py
"""

from pathlib import Path

import numpy as np
import torch
from transformers import Dinov2Config
from transformers.models.dinov2.modeling_dinov2 import Dinov2Layer

ROOT = Path(__file__).resolve().parents[2]
N, D, HEADS = 65, 128, 4


def main():
    cfg = Dinov2Config(hidden_size=D, num_attention_heads=HEADS, mlp_ratio=4,
                       layerscale_value=1e-5, layer_norm_eps=1e-6, hidden_act="gelu",
                       qkv_bias=True)
    cfg._attn_implementation = "eager"
    layer = Dinov2Layer(cfg).double().eval()
    g = torch.Generator().manual_seed(0)
    with torch.no_grad():
        for name, p in layer.named_parameters():
            if "lambda1" in name:
                p.fill_(1e-5)
            elif name.startswith("norm") and name.endswith("weight"):
                p.copy_(1.0 + 0.02 * torch.randn(p.shape, generator=g, dtype=torch.float64))
            else:
                p.copy_(0.02 * torch.randn(p.shape, generator=g, dtype=torch.float64))
    x = torch.randn(1, N, D, generator=torch.Generator().manual_seed(1), dtype=torch.float64)

    cap = {}

    def hook(name, pick=lambda o: o):
        def f(_m, _i, o):
            cap[name] = pick(o).detach().clone()
        return f

    att = layer.attention.attention
    hooks = [
        layer.norm1.register_forward_hook(hook("ln1")),
        att.query.register_forward_hook(hook("q")),
        att.key.register_forward_hook(hook("k")),
        att.value.register_forward_hook(hook("v")),
        att.register_forward_hook(hook("ctx", lambda o: o[0] if isinstance(o, tuple) else o)),
        layer.attention.output.dense.register_forward_hook(hook("attn")),
        layer.norm2.register_forward_hook(hook("ln2")),
        layer.mlp.fc1.register_forward_hook(hook("fc1")),
        layer.mlp.register_forward_hook(hook("mlp")),
    ]
    with torch.no_grad():
        out = layer(x)
    for h in hooks:
        h.remove()
    cap["out"] = out[0] if isinstance(out, tuple) else out

    f32 = lambda t: t.reshape(t.shape[-2] if t.dim() > 1 else -1, -1).numpy().astype(np.float32)
    res = {"x": f32(x)}
    sd = {k: v.numpy().astype(np.float32) for k, v in layer.state_dict().items()}
    res.update({"w/" + k: v for k, v in sd.items()})
    for k, v in cap.items():
        res["y/" + k] = v.reshape(N, -1).numpy().astype(np.float32)
    dst = ROOT / "tests" / "golden" / "vit_block_golden.npz"
    np.savez_compressed(dst, **res)
    print(f"{len(res)} arrays -> {dst} ({dst.stat().st_size} bytes)")


if __name__ == "__main__":
    main()
