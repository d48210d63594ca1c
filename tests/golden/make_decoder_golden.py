# SPDX-License-Identifier: Unlicense
"""Generate tests/golden/decoder_golden.npz: the five transformer blocks of
RoMa's coordinate decoder (DINOv2-style blocks of width 1024 with 8 heads
of 128, no qkv bias, LayerNorm eps 1e-5, no LayerScale, GELU MLP of ratio
4) evaluated by transformers' own Dinov2Layer in float64 (configured to
that block: qkv_bias False, layer_norm_eps 1e-5, LayerScale 1), with the
seeded synthetic decoder weights of coreg.synth.roma_weights(0), on 32
seeded tokens (so that the fixture stays small). Stores as float32:

    x      the input tokens (32, 1024), N(0, 1) from seed 3
    out    the output of the fifth block (32, 1024)

Needs transformers and torch (present in the build container); run from
the repository root:

    python tests/golden/make_decoder_golden.py
"""

import sys
from pathlib import Path

import numpy as np
import torch
from transformers import Dinov2Config
from transformers.models.dinov2.modeling_dinov2 import Dinov2Layer

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT / "i.coregistration.opencl_b200"))

from coreg import synth  # noqa: E402

N, D, HEADS, DEPTH = 32, 1024, 8, 5


def layer_state(main, i):
    """Dinov2Layer's state dict from the decoder block's original names."""
    t = lambda a: torch.from_numpy(np.asarray(a, np.float64))
    b = f"decoder.embedding_decoder.blocks.{i}."
    qkv = t(main[b + "attn.qkv.weight"])
    s = {}
    for j, n in enumerate(("query", "key", "value")):
        s[f"attention.attention.{n}.weight"] = qkv[j * D:(j + 1) * D]
    for src, dst in (("norm1", "norm1"), ("norm2", "norm2"), ("attn.proj", "attention.output.dense"),
                     ("mlp.fc1", "mlp.fc1"), ("mlp.fc2", "mlp.fc2")):
        s[dst + ".weight"] = t(main[b + src + ".weight"])
        s[dst + ".bias"] = t(main[b + src + ".bias"])
    s["layer_scale1.lambda1"] = torch.ones(D, dtype=torch.float64)
    s["layer_scale2.lambda1"] = torch.ones(D, dtype=torch.float64)
    return s


def main():
    weights = synth.roma_weights(0)[0]
    cfg = Dinov2Config(hidden_size=D, num_attention_heads=HEADS, mlp_ratio=4,
                       layerscale_value=1.0, layer_norm_eps=1e-5, hidden_act="gelu",
                       qkv_bias=False)
    cfg._attn_implementation = "eager"
    x = np.random.default_rng(3).standard_normal((N, D)).astype(np.float32)
    h = torch.from_numpy(x).double()[None]
    with torch.no_grad():
        for i in range(DEPTH):
            layer = Dinov2Layer(cfg).double().eval()
            res = layer.load_state_dict(layer_state(weights, i), strict=True)
            assert not res.missing_keys and not res.unexpected_keys
            h = layer(h)
            h = h[0] if isinstance(h, tuple) else h
    dst = ROOT / "tests" / "golden" / "decoder_golden.npz"
    np.savez_compressed(dst, x=x, out=h[0].numpy().astype(np.float32))
    print(f"{dst} ({dst.stat().st_size} bytes)")


if __name__ == "__main__":
    main()
