# SPDX-License-Identifier: Unlicense
"""One DINOv2 ViT-L transformer block through the ops.h entry points (the
BASELINE config-1 block: 1025 tokens, width 1024, 16 heads of 64, MLP 4096
with GELU, pre-LayerNorm eps 1e-6, LayerScale 1e-5; float32), every
intermediate tensor compared.

The oracle's restatement of the block (oracle/ops_ref.vit_block, roma.c's
block) is pinned to transformers' own Dinov2Layer through
tests/golden/vit_block_golden.npz (reduced size; CPU). The C-ABI path
composes the reference's calls (ops_layernorm, ops_linear, ops_attention,
LayerScale folded into the output projection and fc2 as roma.c:191-201
does) and must match the golden at the reduced size and the oracle at the
config-1 size, relative L2 <= 1e-5 per intermediate (GPU)."""

from pathlib import Path

import numpy as np
import pytest

from oracle import ops_ref

GOLDEN = Path(__file__).resolve().parent / "golden" / "vit_block_golden.npz"
NAMES = ["ln1", "q", "k", "v", "ctx", "attn", "ln2", "fc1", "mlp", "out"]


def rel(a, b):
    a = np.asarray(a, np.float64).reshape(-1)
    b = np.asarray(b, np.float64).reshape(-1)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def golden():
    z = np.load(GOLDEN)
    w = {k[2:]: z[k] for k in z.files if k.startswith("w/")}
    y = {k[2:]: z[k] for k in z.files if k.startswith("y/")}
    return z["x"], w, y


def test_oracle_block_matches_transformers():
    x, w, y = golden()
    r = ops_ref.vit_block(x, w, heads=4)
    for n in NAMES:
        assert rel(r[n], y[n]) <= 1e-6, (n, rel(r[n], y[n]))


def synth_weights(D, heads, seed=0):
    """Config-1 weights: N(0, 0.02) from seed 0, LayerNorm gains 1 + N(0,
    0.02), LayerScale 1e-5, transformers' names."""
    rng = np.random.default_rng(seed)
    n = lambda *s: (0.02 * rng.standard_normal(s)).astype(np.float32)
    pre = "attention.attention."
    return {
        "norm1.weight": 1 + n(D), "norm1.bias": n(D),
        pre + "query.weight": n(D, D), pre + "query.bias": n(D),
        pre + "key.weight": n(D, D), pre + "key.bias": n(D),
        pre + "value.weight": n(D, D), pre + "value.bias": n(D),
        "attention.output.dense.weight": n(D, D), "attention.output.dense.bias": n(D),
        "layer_scale1.lambda1": np.full(D, 1e-5, np.float32),
        "norm2.weight": 1 + n(D), "norm2.bias": n(D),
        "mlp.fc1.weight": n(4 * D, D), "mlp.fc1.bias": n(4 * D),
        "mlp.fc2.weight": n(D, 4 * D), "mlp.fc2.bias": n(D),
        "layer_scale2.lambda1": np.full(D, 1e-5, np.float32),
    }


def ops_block(dev, x, w, heads, eps=1e-6):
    """The block through the C-ABI (float32), each intermediate read back."""
    import coreg
    from coreg import Opnd, handle

    lib, o = dev.lib, dev.ops_p
    N, D = x.shape
    d = D // heads
    # Every uploaded buffer stays referenced until the block is read back:
    # a Buffer frees its device memory when Python drops it.
    keep = []

    def up(a):
        keep.append(dev.upload(np.ascontiguousarray(a, np.float32)))
        return keep[-1]
    pre = "attention.attention."
    X = up(x)
    LN1, LN2 = dev.zeros(N * D), dev.zeros(N * D)
    QKV, CTX, ATT = dev.zeros(N * 3 * D), dev.zeros(N * D), dev.zeros(N * D)
    FC1P, FC1, MLP = dev.zeros(N * 4 * D), dev.zeros(N * 4 * D), dev.zeros(N * D)
    wqkv = up(np.concatenate([w[pre + "query.weight"], w[pre + "key.weight"],
                              w[pre + "value.weight"]]))
    bqkv = up(np.concatenate([w[pre + "query.bias"], w[pre + "key.bias"], w[pre + "value.bias"]]))
    ls1, ls2 = w["layer_scale1.lambda1"], w["layer_scale2.lambda1"]
    wo, bo = w["attention.output.dense.weight"], w["attention.output.dense.bias"]
    w2, b2 = w["mlp.fc2.weight"], w["mlp.fc2.bias"]

    lib.ops_layernorm(o, N, D, handle(X), handle(LN1), handle(up(w["norm1.weight"])),
                      handle(up(w["norm1.bias"])), eps, 0, 0.0)
    lib.ops_linear(o, N, D, 3 * D, handle(LN1), 0, handle(wqkv), handle(bqkv), handle(QKV), 0,
                   0, 0.0, 0)
    lib.ops_attention(o, Opnd(handle(QKV), 0, 3 * D, 0, 0), Opnd(handle(QKV), D, 3 * D, 0, 0),
                      Opnd(handle(QKV), 2 * D, 3 * D, 0, 0), Opnd(handle(CTX), 0, D, 0, 0),
                      N, N, heads, d, 1.0 / np.sqrt(d), None)
    lib.ops_linear(o, N, D, D, handle(CTX), 0, handle(up(wo)), handle(up(bo)), handle(ATT), 0,
                   0, 0.0, 0)
    # The residual stream with LayerScale folded into the projection.
    H = up(x)
    lib.ops_linear(o, N, D, D, handle(CTX), 0, handle(up(wo * ls1[:, None])),
                   handle(up(bo * ls1)), handle(H), 0, 0, 0.0, 1)
    lib.ops_layernorm(o, N, D, handle(H), handle(LN2), handle(up(w["norm2.weight"])),
                      handle(up(w["norm2.bias"])), eps, 0, 0.0)
    w1, b1 = up(w["mlp.fc1.weight"]), up(w["mlp.fc1.bias"])
    lib.ops_linear(o, N, D, 4 * D, handle(LN2), 0, handle(w1), handle(b1), handle(FC1P), 0,
                   0, 0.0, 0)
    lib.ops_linear(o, N, D, 4 * D, handle(LN2), 0, handle(w1), handle(b1), handle(FC1), 0,
                   coreg.ACT_GELU, 0.0, 0)
    lib.ops_linear(o, N, 4 * D, D, handle(FC1), 0, handle(up(w2)), handle(up(b2)), handle(MLP),
                   0, 0, 0.0, 0)
    OUT = dev.zeros(N * D)
    lib.ocl_copy(dev.ocl_p, handle(H), 0, handle(OUT), 0, N * D * 4)
    lib.ops_linear(o, N, 4 * D, D, handle(FC1), 0, handle(up(w2 * ls2[:, None])),
                   handle(up(b2 * ls2)), handle(OUT), 0, 0, 0.0, 1)
    coreg.check(lib)
    rd = lambda b, n: b.read(count=n)
    qkv = rd(QKV, N * 3 * D).reshape(N, 3 * D)
    return {"ln1": rd(LN1, N * D), "q": qkv[:, :D], "k": qkv[:, D:2 * D], "v": qkv[:, 2 * D:],
            "ctx": rd(CTX, N * D), "attn": rd(ATT, N * D), "ln2": rd(LN2, N * D),
            "fc1": rd(FC1P, N * 4 * D), "mlp": rd(MLP, N * D), "out": rd(OUT, N * D)}


@pytest.mark.gpu
def test_block_through_ops_matches_transformers(dev):
    x, w, y = golden()
    got = ops_block(dev, x, w, heads=4)
    for n in NAMES:
        assert rel(got[n], y[n]) <= 1e-5, (n, rel(got[n], y[n]))


@pytest.mark.gpu
def test_config1_block_through_ops_matches_oracle(dev):
    N, D, heads = 1025, 1024, 16
    w = synth_weights(D, heads, seed=0)
    x = np.random.default_rng(1).standard_normal((N, D)).astype(np.float32)
    got = ops_block(dev, x, w, heads)
    want = ops_ref.vit_block(x, w, heads)
    for n in NAMES:
        assert rel(got[n], want[n]) <= 1e-5, (n, rel(got[n], want[n]))
