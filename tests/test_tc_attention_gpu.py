# SPDX-License-Identifier: Unlicense
"""The fused tcgen05 attention (ops_attention_qkv, bfloat16 mode) and its
float32 counterpart against the oracle attention (ops.cl:607-687
semantics) on the transformer shapes of the models (GPU).

bfloat16 mode: operands rounded to bfloat16 and the probabilities too, so
the bound is the build's bfloat16 contract (relative L2 <= 2e-2); it is
checked tighter (1e-2) here. float32 mode: relative L2 <= 1e-5."""

import numpy as np
import pytest

import coreg
from oracle.ops_ref import attention as ref_attention
from test_tc_gemm_gpu import bf16_round

SHAPES = [
    # tokens, channels, heads
    (1601, 1024, 16),   # DINOv2 ViT-L/14 at 560
    (1600, 1024, 8),    # coordinate decoder (head size 128)
    (257, 1024, 16),    # DINOv2 at 224
    (77, 128, 2),       # one partial key block
    (300, 256, 2),      # head size 128, ragged
]


@pytest.mark.gpu
@pytest.mark.parametrize("shape", SHAPES, ids=[f"{s[0]}x{s[1]}h{s[2]}" for s in SHAPES])
@pytest.mark.parametrize("prec", [coreg.OPS_BF16, coreg.OPS_FP32], ids=["bf16", "fp32"])
def test_attention_qkv(shape, prec):
    N, Dm, heads = shape
    d = Dm // heads
    rng = np.random.default_rng(N + Dm + heads)
    qkv = (rng.standard_normal((N, 3 * Dm), dtype=np.float32) * 1.5).astype(np.float32)
    dev = coreg.Device(0, precision=prec)
    X, O = dev.upload(qkv), dev.zeros(N * Dm)
    scale = float(1.0 / np.sqrt(d))
    dev.lib.ops_attention_qkv(dev.ops_p, X.handle, N, Dm, heads, scale, O.handle)
    got = O.read(count=N * Dm).reshape(N, Dm)
    coreg.check(dev.lib)
    assert dev.lib.coreg_tc_status() == 0
    src = bf16_round(qkv) if prec == coreg.OPS_BF16 else qkv
    want = ref_attention(src[:, :Dm], src[:, Dm:2 * Dm], src[:, 2 * Dm:], N, N, heads, d,
                         np.float32(scale))
    err = np.linalg.norm(got - want) / np.linalg.norm(want)
    assert err <= (1e-2 if prec == coreg.OPS_BF16 else 1e-5), err
    dev.close()


GENERIC = [
    # tokens, heads, head size: Efficient LoFTR's aggregated attention (8
    # heads of 32, zero-padded to 64), head sizes 64 and 100 (padded to 128)
    (400, 8, 32),
    (130, 4, 64),
    (90, 2, 100),
]


@pytest.mark.gpu
@pytest.mark.parametrize("shape", GENERIC, ids=[f"{s[0]}h{s[1]}d{s[2]}" for s in GENERIC])
def test_ops_attention_bf16_on_tensor_cores(shape):
    """ops_attention (separate float32 Q, K, V of any leading dimension)
    in a bfloat16 context: the tcgen05 kernels on the packed, zero-padded
    heads, against the oracle on the rounded operands (1e-2, as above)."""
    from coreg import Opnd

    N, heads, d = shape
    Dm = heads * d
    rng = np.random.default_rng(N * heads + d)
    q, k, v = (rng.standard_normal((N, Dm + 8), dtype=np.float32) for _ in range(3))
    dev = coreg.Device(0, precision=coreg.OPS_BF16)
    Q, K, V = dev.upload(q), dev.upload(k), dev.upload(v)
    O = dev.zeros(N * (Dm + 4))
    scale = float(1.0 / np.sqrt(d))
    dev.lib.ops_attention(dev.ops_p, Opnd(Q.handle, 0, Dm + 8, 0, 0), Opnd(K.handle, 0, Dm + 8, 0, 0),
                          Opnd(V.handle, 0, Dm + 8, 0, 0), Opnd(O.handle, 0, Dm + 4, 0, 0), N, N,
                          heads, d, scale, None)
    got = O.read(count=N * (Dm + 4)).reshape(N, Dm + 4)[:, :Dm]
    coreg.check(dev.lib)
    assert dev.lib.coreg_tc_status() == 0
    want = ref_attention(bf16_round(q[:, :Dm]), bf16_round(k[:, :Dm]), bf16_round(v[:, :Dm]), N,
                         N, heads, d, np.float32(scale))
    err = np.linalg.norm(got - want) / np.linalg.norm(want)
    assert err <= 1e-2, err
    dev.close()
