# SPDX-License-Identifier: Unlicense
"""CPU restatement of the reference's generic tensor kernels (TEST
INFRASTRUCTURE: the checker of the CUDA ops, never the thing measured).

Each function restates one kernel of i.coregistration.opencl's ops.cl in
numpy float64, following the cited lines: the same indexing, padding,
clamping and masking rules. Pinned against the reference's own checker
(tests/ops_compare.py, torch float64) by tests/test_oracle_ops.py through
tests/golden/ops_golden.npz.
"""

import numpy as np
from scipy.special import erf

ACT_NONE, ACT_GELU, ACT_RELU, ACT_LEAKY, ACT_GELU_TANH = range(5)


def act(v, a, slope=0.0):
    """apply_act, ops.cl:23-37."""
    v = np.asarray(v, np.float64)
    if a == ACT_GELU:
        return 0.5 * v * (1.0 + erf(v / np.sqrt(2.0)))
    if a == ACT_RELU:
        return np.maximum(v, 0.0)
    if a == ACT_LEAKY:
        return np.where(v >= 0.0, v, slope * v)
    if a == ACT_GELU_TANH:
        return 0.5 * v * (1.0 + np.tanh(np.sqrt(2.0 / np.pi) * (v + 0.044715 * v ** 3)))
    return v


def gemm(A, B, transb, M, N, K, nb=1, bias=None, biasrow=0, R=None, alpha=1.0,
         a=ACT_NONE, slope=0.0):
    """gemm / gemm_big, ops.cl:39-284: per product b, C = act(alpha A op(B)
    + bias) + R. A (nb, M, K); B (nb, N, K) if transb else (nb, K, N); R
    (nb, M, N)."""
    A = np.asarray(A, np.float64).reshape(nb, M, K)
    if transb:
        Bm = np.asarray(B, np.float64).reshape(nb, N, K).transpose(0, 2, 1)
    else:
        Bm = np.asarray(B, np.float64).reshape(nb, K, N)
    v = alpha * (A @ Bm)
    if bias is not None:
        bias = np.asarray(bias, np.float64)
        v = v + (bias[None, :M, None] if biasrow else bias[None, None, :N])
    v = act(v, a, slope)
    if R is not None:
        v = v + np.asarray(R, np.float64).reshape(nb, M, N)
    return v


def conv2d(x, C, H, W, w, bias, K, kh, kw, sy, sx, py, px, dy=1, dx=1, groups=1,
           mean=None, rstd=None, alpha=None, a=ACT_NONE, slope=0.0):
    """conv2d / conv5x5, ops.cl:323-448: the input normalized and gated,
    prelu((x - mean) rstd, alpha) (alpha None: gate slope 1), before the
    zero padding; weights (K, C / groups, kh, kw); activation after the
    bias."""
    x = np.asarray(x, np.float64).reshape(C, H, W)
    if mean is not None:
        x = (x - np.asarray(mean, np.float64)[:, None, None]) * np.asarray(rstd, np.float64)[:, None, None]
        al = np.ones(C) if alpha is None else np.asarray(alpha, np.float64)
        x = np.where(x >= 0, x, al[:, None, None] * x)
    Ho = (H + 2 * py - dy * (kh - 1) - 1) // sy + 1
    Wo = (W + 2 * px - dx * (kw - 1) - 1) // sx + 1
    xp = np.zeros((C, H + 2 * py, W + 2 * px))
    xp[:, py:py + H, px:px + W] = x
    cg, kg = C // groups, K // groups
    w = np.asarray(w, np.float64).reshape(K, cg, kh, kw)
    out = np.zeros((K, Ho, Wo))
    for gi in range(groups):
        cols = np.empty((cg, kh, kw, Ho, Wo))
        for i in range(kh):
            for j in range(kw):
                cols[:, i, j] = xp[gi * cg:(gi + 1) * cg,
                                   i * dy: i * dy + sy * (Ho - 1) + 1: sy,
                                   j * dx: j * dx + sx * (Wo - 1) + 1: sx]
        wg = w[gi * kg:(gi + 1) * kg].reshape(kg, -1)
        out[gi * kg:(gi + 1) * kg] = (wg @ cols.reshape(cg * kh * kw, -1)).reshape(kg, Ho, Wo)
    if bias is not None:
        out += np.asarray(bias, np.float64)[:, None, None]
    return act(out, a, slope)


def chan_stats(x, C, HW, eps):
    """chan_stats, ops.cl:453-492: mean and 1 / sqrt(biased var + eps)."""
    x = np.asarray(x, np.float64).reshape(C, HW)
    m = x.mean(1)
    v = ((x - m[:, None]) ** 2).mean(1)
    return m, 1.0 / np.sqrt(v + eps)


def chan_affine(x, C, HW, mean=None, rstd=None, g=None, b=None, a=ACT_NONE, slope=0.0):
    """chan_affine, ops.cl:499-519."""
    v = np.asarray(x, np.float64).reshape(C, HW)
    if mean is not None:
        v = (v - np.asarray(mean, np.float64)[:, None]) * np.asarray(rstd, np.float64)[:, None]
    if g is not None:
        v = v * np.asarray(g, np.float64)[:, None]
    if b is not None:
        v = v + np.asarray(b, np.float64)[:, None]
    return act(v, a, slope)


def prelu(x, C, HW, alpha):
    """prelu, ops.cl:522-532."""
    v = np.asarray(x, np.float64).reshape(C, HW)
    return np.where(v >= 0, v, np.asarray(alpha, np.float64)[:, None] * v)


def layernorm(x, rows, C, g, b, eps, a=ACT_NONE, slope=0.0):
    """layernorm, ops.cl:547-578."""
    x = np.asarray(x, np.float64).reshape(rows, C)
    m = x.mean(1, keepdims=True)
    v = ((x - m) ** 2).mean(1, keepdims=True)
    y = (x - m) / np.sqrt(v + eps)
    if g is not None:
        y = y * np.asarray(g, np.float64) + np.asarray(b, np.float64)
    return act(y, a, slope)


def softmax_rows(x, rows, L, scale):
    """softmax_rows, ops.cl:583-602."""
    s = np.asarray(x, np.float64).reshape(rows, L) * scale
    e = np.exp(s - s.max(1, keepdims=True))
    return e / e.sum(1, keepdims=True)


def attention(Q, K, V, Nq, Nk, nh, d, scale, kmask=None):
    """attention, ops.cl:607-687: per head h (columns h d ..), softmax of
    scale Q K^T over the unmasked keys times V; a query with no key left
    gets zeros. Q (Nq, nh d), K and V (Nk, nh d)."""
    out = np.zeros((Nq, nh * d))
    keep = np.ones(Nk, bool) if kmask is None else np.asarray(kmask) != 0
    if not keep.any():
        return out
    for h in range(nh):
        q = np.asarray(Q, np.float64)[:, h * d:(h + 1) * d]
        k = np.asarray(K, np.float64)[keep, h * d:(h + 1) * d]
        v = np.asarray(V, np.float64)[keep, h * d:(h + 1) * d]
        s = (q * scale) @ k.T
        e = np.exp(s - s.max(1, keepdims=True))
        out[:, h * d:(h + 1) * d] = (e / e.sum(1, keepdims=True)) @ v
    return out


def rope(x, off, ld, rows, nh, d, npos, cs, interleaved):
    """rope, ops.cl:695-716, in place on a copy of the flat buffer x; cs
    holds (cos, sin) pairs, npos x d / 2."""
    out = np.asarray(x, np.float64).copy()
    cs = np.asarray(cs, np.float64).reshape(npos, d // 2, 2)
    nf = d // 2
    for r in range(rows):
        c, s = cs[r % npos, :, 0], cs[r % npos, :, 1]
        for h in range(nh):
            base = off + r * ld + h * d
            i0 = base + (2 * np.arange(nf) if interleaved else np.arange(nf))
            i1 = base + (2 * np.arange(nf) + 1 if interleaved else np.arange(nf) + nf)
            a, b = out[i0].copy(), out[i1].copy()
            out[i0] = a * c - b * s
            out[i1] = a * s + b * c
    return out


def resize(x, C, h, w, H, W, align, scale):
    """resize_bilinear, ops.cl:723-754 with ops.c:496-516's steps: source
    step 1 / scale when scale > 0, else the size ratio; without
    align_corners the source coordinate is clamped at 0 and the upper
    neighbour at the last row / column."""
    x = np.asarray(x, np.float64).reshape(C, h, w)
    if align:
        ux = np.arange(W) * ((w - 1) / (W - 1)) if W > 1 else np.zeros(W)
        uy = np.arange(H) * ((h - 1) / (H - 1)) if H > 1 else np.zeros(H)
    else:
        sy = 1.0 / scale if scale > 0 else h / H
        sx = 1.0 / scale if scale > 0 else w / W
        ux = np.maximum((np.arange(W) + 0.5) * sx - 0.5, 0.0)
        uy = np.maximum((np.arange(H) + 0.5) * sy - 0.5, 0.0)
    x0 = ux.astype(int)
    y0 = uy.astype(int)
    x1 = np.minimum(x0 + 1, w - 1)
    y1 = np.minimum(y0 + 1, h - 1)
    fx = (ux - x0)[None, None, :]
    fy = (uy - y0)[None, :, None]
    v00 = x[:, y0][:, :, x0]
    v01 = x[:, y0][:, :, x1]
    v10 = x[:, y1][:, :, x0]
    v11 = x[:, y1][:, :, x1]
    return (1 - fy) * ((1 - fx) * v00 + fx * v01) + fy * ((1 - fx) * v10 + fx * v11)


def bilinear_zero(p, H, W, gx, gy, align=0):
    """Bilinear value of planes p (C, H, W) at normalized points (gx, gy),
    zero padding, non-finite points 0 (grid_sample ops.cl:759-793,
    bilinear0 roma_kernels.cl:106-128). Returns (C, n)."""
    p = np.asarray(p, np.float64).reshape(-1, H, W)
    gx = np.asarray(gx, np.float64)
    gy = np.asarray(gy, np.float64)
    if align:
        ix = (gx + 1.0) * 0.5 * (W - 1)
        iy = (gy + 1.0) * 0.5 * (H - 1)
    else:
        ix = ((gx + 1.0) * W - 1.0) * 0.5
        iy = ((gy + 1.0) * H - 1.0) * 0.5
    ok = np.isfinite(ix) & np.isfinite(iy)
    ix = np.where(ok, ix, 0.0)
    iy = np.where(ok, iy, 0.0)
    x0 = np.floor(ix).astype(np.int64)
    y0 = np.floor(iy).astype(np.int64)
    fx = ix - x0
    fy = iy - y0

    def at(yy, xx):
        inside = (xx >= 0) & (xx < W) & (yy >= 0) & (yy < H)
        v = p[:, np.clip(yy, 0, H - 1), np.clip(xx, 0, W - 1)]
        return np.where(inside[None, :], v, 0.0)

    v = (1 - fy) * ((1 - fx) * at(y0, x0) + fx * at(y0, x0 + 1)) + \
        fy * ((1 - fx) * at(y0 + 1, x0) + fx * at(y0 + 1, x0 + 1))
    return np.where(ok[None, :], v, 0.0)


def grid_sample(x, C, H, W, grid, n, align):
    g = np.asarray(grid, np.float64).reshape(n, 2)
    return bilinear_zero(np.asarray(x).reshape(C, H, W), H, W, g[:, 0], g[:, 1], align)


def unfold(x, C, H, W, k, s, p):
    """unfold, ops.cl:799-816: (C k k, Ho Wo)."""
    Ho = (H + 2 * p - k) // s + 1
    Wo = (W + 2 * p - k) // s + 1
    xp = np.zeros((C, H + 2 * p, W + 2 * p))
    xp[:, p:p + H, p:p + W] = np.asarray(x, np.float64).reshape(C, H, W)
    out = np.empty((C, k, k, Ho, Wo))
    for i in range(k):
        for j in range(k):
            out[:, i, j] = xp[:, i:i + s * (Ho - 1) + 1:s, j:j + s * (Wo - 1) + 1:s]
    return out.reshape(C * k * k, Ho * Wo)


def pool2d(x, C, H, W, k, s, p, mx):
    """avgpool2 / pool2d, ops.cl:819-860: max ignores the padding, the
    average counts it (divides by k k)."""
    x = np.asarray(x, np.float64).reshape(C, H, W)
    Ho = (H + 2 * p - k) // s + 1
    Wo = (W + 2 * p - k) // s + 1
    fill = -np.inf if mx else 0.0
    xp = np.full((C, H + 2 * p, W + 2 * p), fill)
    xp[:, p:p + H, p:p + W] = x
    win = np.stack([xp[:, i:i + s * (Ho - 1) + 1:s, j:j + s * (Wo - 1) + 1:s]
                    for i in range(k) for j in range(k)])
    return win.max(0) if mx else win.sum(0) / (k * k)


def transpose(x, B, R, C):
    """transpose2d, ops.cl:864-880."""
    return np.asarray(x, np.float64).reshape(B, R, C).transpose(0, 2, 1)


def axpby(a, alpha, b, beta, n, bmod):
    """axpby, ops.cl:884-893."""
    a = np.asarray(a, np.float64).reshape(-1)[:n]
    if b is None:
        return alpha * a
    b = np.asarray(b, np.float64)
    return alpha * a + beta * b[np.arange(n) % bmod]


def fold_bn(w, b, K, per, gamma, beta, mean, var, eps):
    """ops_fold_bn, ops.c:612-626 (double arithmetic, float results)."""
    w = np.asarray(w, np.float32).reshape(K, per).astype(np.float64)
    s = np.asarray(gamma, np.float64) / np.sqrt(np.asarray(var, np.float64) + np.float64(np.float32(eps)))
    wf = (w * s[:, None]).astype(np.float32)
    bf = ((np.asarray(b, np.float64) - np.asarray(mean, np.float64)) * s +
          np.asarray(beta, np.float64)).astype(np.float32)
    return wf.reshape(-1), bf


# ---------------------------------------------------------------- cases

def run_case(c):
    """Oracle outputs of one ops_cases.Case: {output name: float64 array}."""
    p, x = c.p, c.inputs
    op = c.op
    if op == "gemm":
        M, N, K, nb = p["M"], p["N"], p["K"], p["nb"]
        return {"out": gemm(x["a"], x["b"], p["transb"], M, N, K, nb, bias=x["bias"],
                            R=x.get("r"), alpha=p["alpha"], a=p["act"], slope=p["slope"])}
    if op == "conv1x1":
        C, HW, K = p["C"], p["HW"], p["K"]
        return {"out": gemm(x["w"], x["x"], 0, K, HW, C, 1, bias=x["bias"], biasrow=1,
                            a=p["act"])}
    if op == "conv2d":
        return {"out": conv2d(x["x"], p["C"], p["H"], p["W"], x["w"], x["bias"], p["K"],
                              p["k"], p["k"], p["s"], p["s"], p["p"], p["p"], p["d"], p["d"],
                              p["groups"], x.get("mean"), x.get("rstd"), x.get("alpha"),
                              p["act"], p["slope"])}
    if op == "instnorm":
        m, r = chan_stats(x["x"], p["C"], p["HW"], p["eps"])
        return {"out": chan_affine(x["x"], p["C"], p["HW"], m, r, x["g"], x["bias"],
                                   p["act"], p["slope"])}
    if op == "layernorm":
        return {"out": layernorm(x["x"], p["rows"], p["C"], x["g"], x["bias"], p["eps"], p["act"])}
    if op == "softmax":
        return {"out": softmax_rows(x["x"], p["rows"], p["L"], p["scale"])}
    if op == "attention":
        Nq, Nk, nh, d = p["Nq"], p["Nk"], p["nh"], p["d"]
        E = nh * d
        qkv = np.asarray(x["qkv"], np.float64).reshape(Nk, 3 * E)
        return {"out": attention(qkv[:Nq, :E], qkv[:, E:2 * E], qkv[:, 2 * E:], Nq, Nk, nh, d,
                                 np.float32(p["scale"]), x.get("mask"))}
    if op == "rope":
        from .ops_cases import rope_table
        return {"out": rope(x["x"], p["off"], p["ld"], p["rows"], p["nh"], p["d"], p["npos"],
                            rope_table(x["angles"]), p["interleaved"])}
    if op == "resize":
        C, H, W, coff = p["C"], p["H"], p["W"], p["coff"]
        out = np.zeros((C + coff, H, W))
        out[coff:] = resize(x["x"], C, p["h"], p["w"], H, W, p["align"], p["scale"])
        return {"out": out}
    if op == "grid_sample":
        return {"out": grid_sample(x["x"], p["C"], p["H"], p["W"], x["grid"], p["n"], p["align"])}
    if op == "unfold":
        return {"out": unfold(x["x"], p["C"], p["H"], p["W"], p["k"], p["s"], p["p"])}
    if op == "pool":
        return {"out": pool2d(x["x"], p["C"], p["H"], p["W"], p["k"], p["s"], p["p"], p["max"])}
    if op == "transpose":
        return {"out": transpose(x["x"], p["B"], p["R"], p["C"])}
    if op == "elementwise":
        C, HW = p["C"], p["HW"]
        r = {"prelu": prelu(x["x"], C, HW, x["alpha"])}
        for a in (ACT_GELU, ACT_RELU, ACT_LEAKY, ACT_GELU_TANH):
            r[f"act{a}"] = act(x["x"], a, p["slope"])
        r["axpby"] = axpby(x["x"], p["a"], x["b"], p["b"], C * HW, HW)
        return r
    if op == "fold_bn":
        C, H, W, K = p["C"], p["H"], p["W"], p["K"]
        wf, bf = fold_bn(x["w"], x["bias"], K, C * 9, x["gamma"], x["beta"], x["mean"],
                         x["var"], p["eps"])
        return {"out": conv2d(x["x"], C, H, W, wf, bf, K, 3, 3, 1, 1, 1, 1)}
    raise ValueError(op)


def vit_block(x, w, heads, eps=1e-6):
    """One pre-norm DINOv2 block as the reference runs it (roma.c:679-713:
    LayerNorm, fused qkv linear, attention with the full score matrix,
    output projection, LayerNorm, GELU MLP; LayerScale folded into the
    output projection and fc2, roma.c:191-201), float64. w holds the
    transformers Dinov2Layer names. Returns every intermediate: ln1, q, k,
    v, ctx, attn (output projection before LayerScale), ln2, fc1 (before
    GELU), mlp (fc2 output before LayerScale), out."""
    x = np.asarray(x, np.float64)
    N, D = x.shape
    d = D // heads
    f = lambda k: np.asarray(w[k], np.float64)
    lin = lambda a, W, b: a @ f(W).T + f(b)
    r = {}
    r["ln1"] = layernorm(x, N, D, f("norm1.weight"), f("norm1.bias"), eps)
    pre = "attention.attention."
    r["q"] = lin(r["ln1"], pre + "query.weight", pre + "query.bias")
    r["k"] = lin(r["ln1"], pre + "key.weight", pre + "key.bias")
    r["v"] = lin(r["ln1"], pre + "value.weight", pre + "value.bias")
    r["ctx"] = attention(r["q"], r["k"], r["v"], N, N, heads, d, 1.0 / np.sqrt(d))
    r["attn"] = lin(r["ctx"], "attention.output.dense.weight", "attention.output.dense.bias")
    h = x + f("layer_scale1.lambda1") * r["attn"]
    r["ln2"] = layernorm(h, N, D, f("norm2.weight"), f("norm2.bias"), eps)
    r["fc1"] = lin(r["ln2"], "mlp.fc1.weight", "mlp.fc1.bias")
    r["mlp"] = lin(act(r["fc1"], ACT_GELU), "mlp.fc2.weight", "mlp.fc2.bias")
    r["out"] = h + f("layer_scale2.lambda1") * r["mlp"]
    return r
