# SPDX-License-Identifier: Unlicense
"""CPU restatement of the reference's Efficient LoFTR device stage (TEST
INFRASTRUCTURE: the checker of the CUDA path, never the product).

Follows i.coregistration.opencl's eloftr.c (folding :103-230, RoPE table
:262-291, backbone :369-394, aggregated attention :407-449, transformer
:451-463, coarse matching :473-571, fusion :575-604) and eloftr_kernels.cl
(dual softmax :12-140, fine matching :146-295) in float64: torch for the
convolutions, oracle/ops_ref.py's pinned LayerNorm, attention, RoPE and
resize for the rest. The reference's own model-level compare script runs
against transformers' EfficientLoFTRForKeypointMatching; this restatement
is pinned to that model by tests/test_eloftr_oracle.py against the fixture
of tests/golden/make_eloftr_golden.py: the coarse stage (backbone,
aggregated attention with RoPE, coarse matches), the fine features (the
model's refinement layer), and the two fine stages, which follow the
authors' FineMatching as eloftr_kernels.cl does (the fixture restates it in
torch on the model's own fine windows, since transformers' version
departs from it). The dual softmax and the fine matching are also pinned
to the reference's own eloftr_kernels.cl, compiled as C and run on the CPU
(tests/test_eloftr_disk_kernels_ref.py), and the whole stage to the
reference's own eloftr.c, ops.c and kernels run on the CPU: its debug dumps
of the backbone, transformer and fusion features, and its matches
(tests/test_eloftr_ref_cpu.py).
"""

import math

import numpy as np
import torch
import torch.nn.functional as F

from . import ops_ref

STAGE_BLOCKS, STAGE_OUT, STAGE_STRIDE = (1, 2, 4, 14), (64, 64, 128, 256), (2, 1, 2, 2)
D, HEADS, MLP = 256, 8, 512
EPS_BN, EPS_LN, LEAKY = 1e-5, 1e-5, 0.01
COARSE_T, COARSE_THR, BORDER, FINE_T = 0.1, 0.2, 2, 10.0
ROPE_BASE, ROPE_DIM = 10000.0, 128
FW, FW1, FC, FS = 8, 10, 64, 8


def _t(x):
    return torch.from_numpy(np.asarray(x, np.float64))


def _fold(w, sd, pre, c):
    """BatchNorm <pre> folded into (w, b): w (c, ...) scaled per output
    channel, b = (0 - mean) * s + beta (ops.c:612-626)."""
    s = np.asarray(sd[pre + ".weight"], np.float64) / np.sqrt(
        np.asarray(sd[pre + ".running_var"], np.float64) + EPS_BN)
    w = np.asarray(w, np.float64) * s.reshape(-1, *([1] * (np.ndim(w) - 1)))
    b = -np.asarray(sd[pre + ".running_mean"], np.float64) * s + np.asarray(sd[pre + ".bias"],
                                                                             np.float64)
    return w, b


class Model:
    def __init__(self, sd, pos_scale=1.0):
        self.sd = sd
        self.pos_scale = pos_scale
        self.blocks = []
        cin = 1
        for s, (nb, co, st) in enumerate(zip(STAGE_BLOCKS, STAGE_OUT, STAGE_STRIDE)):
            for b in range(nb):
                stride = st if b == 0 else 1
                pre = f"efficientloftr.backbone.stages.{s}.blocks.{b}"
                w, bias = _fold(sd[pre + ".conv1.conv.weight"], sd, pre + ".conv1.norm", co)
                w1, b1 = _fold(sd[pre + ".conv2.conv.weight"], sd, pre + ".conv2.norm", co)
                w = w.copy()
                w[:, :, 1, 1] += w1[:, :, 0, 0]
                bias = bias + b1
                if pre + ".identity.weight" in sd:
                    wi, bi = _fold(np.eye(co)[:, :, None, None], sd, pre + ".identity", co)
                    w[:, :, 1, 1] += wi[:, :, 0, 0]
                    bias = bias + bi
                self.blocks.append((_t(w), _t(bias), stride))
                cin = co

    def attn(self, layer, kind):
        """Accessor of one attention block's weights, float64."""
        pre = f"efficientloftr.local_feature_transformer.layers.{layer}.{kind}."
        return lambda k: np.asarray(self.sd[pre + k], np.float64)

    def backbone(self, grey):
        x = _t(grey)[None, None]
        feats = []
        i = 0
        for s, nb in enumerate(STAGE_BLOCKS):
            for b in range(nb):
                w, bias, st = self.blocks[i]
                x = F.relu(F.conv2d(x, w, bias, stride=st, padding=1))
                i += 1
            feats.append(x)
        return feats[1][0].numpy(), feats[2][0].numpy(), feats[3][0].numpy()

    def rope_table(self, ah, aw):
        np_ = D // 2
        t = np.zeros((ah * aw, np_, 2))
        for i in range(ah):
            for j in range(aw):
                for p in range(np_):
                    f = np.float32(1.0 / ROPE_BASE ** (2 * (p // 2) / ROPE_DIM))
                    a = np.float32((j + 1) if p % 2 else (i + 1)) * np.float32(self.pos_scale) * f
                    t[i * aw + j, p] = (np.cos(np.float32(a)), np.sin(np.float32(a)))
        return t.reshape(-1)

    def agg_attn(self, a, X, Y, rope):
        """X (256, h, w) attends to Y; returns the updated X."""
        h, w = X.shape[1:]
        ah, aw = h // 4, w // 4
        na, n = ah * aw, h * w
        q = F.conv2d(_t(X)[None], _t(a("aggregation.q_aggregation.weight")), stride=4,
                     groups=D)[0].numpy()
        kv = F.max_pool2d(_t(Y)[None], 4, 4)[0].numpy()
        qn = ops_ref.layernorm(q.reshape(D, na).T, na, D, a("aggregation.norm.weight"),
                               a("aggregation.norm.bias"), EPS_LN)
        kvn = ops_ref.layernorm(kv.reshape(D, na).T, na, D, a("aggregation.norm.weight"),
                                a("aggregation.norm.bias"), EPS_LN)
        Q = qn @ a("attention.q_proj.weight").T
        K = kvn @ a("attention.k_proj.weight").T
        V = kvn @ a("attention.v_proj.weight").T
        if rope is not None:
            Q = ops_ref.rope(Q.reshape(-1), 0, D, na, 1, D, na, rope, 1).reshape(na, D)
            K = ops_ref.rope(K.reshape(-1), 0, D, na, 1, D, na, rope, 1).reshape(na, D)
        O = ops_ref.attention(Q, K, V, na, na, HEADS, D // HEADS, 1.0 / math.sqrt(D // HEADS))
        O = O @ a("attention.o_proj.weight").T
        up = ops_ref.resize(O.T.reshape(D, ah, aw), D, ah, aw, h, w, 0, 4.0)
        tok = np.concatenate([X, up], 0).reshape(2 * D, n).T
        hid = ops_ref.act(tok @ a("mlp.fc1.weight").T, ops_ref.ACT_LEAKY, LEAKY)
        out = ops_ref.layernorm(hid @ a("mlp.fc2.weight").T, n, D, a("mlp.layer_norm.weight"),
                                a("mlp.layer_norm.bias"), EPS_LN)
        return X + out.T.reshape(D, h, w)

    def transformer(self, x0, x1):
        h, w = x0.shape[1:]
        rope = self.rope_table(h // 4, w // 4)
        for l in range(4):
            sa, ca = self.attn(l, "self_attention"), self.attn(l, "cross_attention")
            x0 = self.agg_attn(sa, x0, x0, rope)
            x1 = self.agg_attn(sa, x1, x1, rope)
            x0 = self.agg_attn(ca, x0, x1, None)
            x1 = self.agg_attn(ca, x1, x0, None)
        return x0, x1

    def fusion(self, x, f2, f1, H, W):
        sd = self.sd
        t = lambda k: _t(sd[k])
        h, w = x.shape[1:]
        a = F.conv2d(_t(x)[None], t("refinement_layer.out_conv.weight") / 16.0)
        feat = _t(ops_ref.resize(a[0].numpy(), 256, h, w, 2 * h, 2 * w, 0, 2.0))[None]
        skips = [f2, f1]
        for i, (hid, inter) in enumerate(((128, 256), (64, 128))):
            pre = f"refinement_layer.out_conv_layers.{i}."
            c = F.conv2d(_t(skips[i])[None], t(pre + "out_conv1.weight")) + feat
            w2, b2 = _fold(sd[pre + "out_conv2.weight"], sd, pre + "batch_norm", inter)
            c = F.leaky_relu(F.conv2d(c, _t(w2), _t(b2), padding=1), LEAKY)
            c = F.conv2d(c, t(pre + "out_conv3.weight"), padding=1)
            hh, ww = c.shape[2:]
            feat = _t(ops_ref.resize(c[0].numpy(), hid, hh, ww, 2 * hh, 2 * ww, 0, 2.0))[None]
        return feat[0].numpy()

    def run(self, grey0, grey1):
        H, W = grey0.shape
        f = [self.backbone(g) for g in (grey0, grey1)]
        dumps = {"backbone_0": f[0][2], "backbone_1": f[1][2]}
        x0, x1 = self.transformer(f[0][2], f[1][2])
        dumps["coarse_0"], dumps["coarse_1"] = x0, x1
        mi, mj, mconf = coarse_match(x0, x1)
        fine = [self.fusion(xk, f[k][1], f[k][0], H, W) for k, xk in enumerate((x0, x1))]
        dumps["fine_0"], dumps["fine_1"] = fine
        h, w = x0.shape[1:]
        kp = np.array([fine_one(fine[0], fine[1], i % w, i // w, j % w, j // w)
                       for i, j in zip(mi, mj)]).reshape(-1, 4)
        return mi, mj, mconf, kp, dumps


def dual_softmax_maxima(S):
    """The dual-softmax confidence softmax_row(S) * softmax_col(S) of the
    scores S (n0, n1) (eloftr_kernels.cl:12-144): each row's maximum and
    first argmax, each column's maximum and first argmax."""
    sr = S - S.max(1, keepdims=True)
    pr = np.exp(sr) / np.exp(sr).sum(1, keepdims=True)
    sc = S - S.max(0, keepdims=True)
    pc = np.exp(sc) / np.exp(sc).sum(0, keepdims=True)
    conf = pr * pc
    rarg = conf.argmax(1)
    carg = conf.argmax(0)
    return (conf[np.arange(len(S)), rarg], rarg, conf[carg, np.arange(S.shape[1])], carg)


def coarse_match(x0, x1):
    """Dual softmax of S = f0 f1^T / (256 0.1), mutual first argmaxes above
    0.2, away from the 2-cell border (eloftr.c:473-571); also the margins
    of each decision (row: best - second confidence)."""
    h, w = x0.shape[1:]
    n = h * w
    S = x0.reshape(D, n).T @ x1.reshape(D, n) / (D * COARSE_T)
    rmax, rarg, _, carg = dual_softmax_maxima(S)
    mi, mj, mc = [], [], []
    for i in range(n):
        j = rarg[i]
        xi, yi, xj, yj = i % w, i // w, j % w, j // w
        if not rmax[i] > COARSE_THR or carg[j] != i:
            continue
        if min(xi, yi, xj, yj) < BORDER or max(xi, xj) >= w - BORDER or max(yi, yj) >= h - BORDER:
            continue
        mi.append(i)
        mj.append(j)
        mc.append(rmax[i])
    return np.array(mi, int), np.array(mj, int), np.array(mc)


def fine_one(f0, f1, x0, y0, x1, y1):
    """Both fine stages for one coarse match (eloftr_kernels.cl:146-295)."""
    C, H, W = f0.shape

    def at(f, c, x, y):
        return f[c, y, x] if 0 <= x < W and 0 <= y < H else 0.0

    A = np.array([[at(f0, c, x0 * FW + p % FW, y0 * FW + p // FW) for c in range(FC)]
                  for p in range(FW * FW)])
    B = np.array([[at(f1, c, x1 * FW - 1 + q % FW1, y1 * FW - 1 + q // FW1) for c in range(FC)]
                  for q in range(FW1 * FW1)])
    sc = A[:, :FC - FS] @ B[:, :FC - FS].T / FC
    e0 = np.exp(sc - sc.max(0, keepdims=True))
    p0 = e0 / e0.sum(0, keepdims=True)
    e1 = np.exp(sc - sc.max(1, keepdims=True))
    p1 = e1 / e1.sum(1, keepdims=True)
    conf = p0 * p1
    inner = conf.reshape(FW * FW, FW1, FW1)[:, 1:FW + 1, 1:FW + 1].reshape(-1)
    e = int(np.argmax(inner))
    bp, bq = e // (FW * FW), e % (FW * FW)
    qi, qj = bq // FW, bq % FW
    ax, ay = x0 * FW + bp % FW, y0 * FW + bp // FW
    s2 = []
    for t in range(9):
        ii = (qi + t // 3 - 1 + FW1) % FW1
        jj = (qj + t % 3 - 1 + FW1) % FW1
        bx, by = x1 * FW - 1 + jj, y1 * FW - 1 + ii
        d = sum(at(f0, c, ax, ay) * at(f1, c, bx, by) for c in range(FC - FS, FC))
        s2.append(d / math.sqrt(FS) / FINE_T)
    s2 = np.array(s2)
    wgt = np.exp(s2 - s2.max())
    wgt /= wgt.sum()
    ex = float((wgt * (np.arange(9) % 3 - 1)).sum())
    ey = float((wgt * (np.arange(9) // 3 - 1)).sum())
    off = FW / 2 - 0.5
    return (x0 * FW + bp % FW - off, y0 * FW + bp // FW - off, x1 * FW + qj - off + ex,
            y1 * FW + qi - off + ey)
