# SPDX-License-Identifier: Unlicense
"""The reference's developer op check as data (TEST INFRASTRUCTURE).

Restates tests/ops_check.c of i.coregistration.opencl: its xorshift64
generator (ops_check.c:33-52, seed 88172645463325252) and its 41 cases in
the same order (ops_check.c:448-487), so that every case draws the same
inputs, in the same order, as the reference's producer. A case is
(name, op, params, inputs); the checker (oracle.ops_ref) and the CUDA
drivers (tests) compute the outputs. Nothing here is part of the product.
"""

import math

import numpy as np

SEED = 88172645463325252
MASK = (1 << 64) - 1
ACT_NONE, ACT_GELU, ACT_RELU, ACT_LEAKY, ACT_GELU_TANH = range(5)


class XorShift:
    """urand() of ops_check.c:37-43: uniform in lo..hi in float32
    arithmetic from a 53-bit draw."""

    def __init__(self, seed=SEED):
        self.s = seed

    def draws(self, n):
        s = self.s
        u = np.empty(n, np.float64)
        for i in range(n):
            s ^= (s << 13) & MASK
            s ^= s >> 7
            s ^= (s << 17) & MASK
            u[i] = (s >> 11) * (1.0 / 9007199254740992.0)
        self.s = s
        return u

    def rand(self, n, lo, hi):
        f = self.draws(n).astype(np.float32)
        lo32, hi32 = np.float32(lo), np.float32(hi)
        return (lo32 + (hi32 - lo32) * f).astype(np.float32)


class Case:
    def __init__(self, name, op, params):
        self.name = name
        self.op = op
        self.p = dict(params)
        self.inputs = {}

    def __getitem__(self, k):
        return self.p[k]

    def __repr__(self):
        return f"Case({self.name}, {self.op}, {self.p})"


def build_cases():
    """The 41 cases of ops_check.c:448-487 with their inputs."""
    rng = XorShift()
    cases = []

    def inp(c, name, n, lo, hi):
        c.inputs[name] = rng.rand(n, lo, hi)

    def gemm(name, M, N, K, transb, nb, act, residual):
        c = Case(name, "gemm", dict(M=M, N=N, K=K, transb=transb, nb=nb, act=act,
                                   residual=residual, alpha=0.5, slope=0.1))
        inp(c, "a", nb * M * K, -1, 1)
        inp(c, "b", nb * N * K, -1, 1)
        inp(c, "bias", N, -1, 1)
        if residual:
            inp(c, "r", nb * M * N, -1, 1)
        cases.append(c)

    def conv1x1(name, C, HW, K):
        c = Case(name, "conv1x1", dict(C=C, HW=HW, K=K, act=ACT_RELU))
        inp(c, "x", C * HW, -1, 1)
        inp(c, "w", K * C, -1, 1)
        inp(c, "bias", K, -1, 1)
        cases.append(c)

    def conv(name, C, H, W, K, k, s, p, d, groups, act, norm, im2col_bytes=None):
        c = Case(name, "conv2d", dict(C=C, H=H, W=W, K=K, k=k, s=s, p=p, d=d,
                                     groups=groups, act=act, slope=0.2, norm=norm))
        if im2col_bytes:
            c.p["im2col_bytes"] = im2col_bytes
        inp(c, "x", C * H * W, -1, 1)
        inp(c, "w", K * (C // groups) * k * k, -0.3, 0.3)
        inp(c, "bias", K, -1, 1)
        if norm:
            inp(c, "mean", C, -0.5, 0.5)
            inp(c, "rstd", C, 0.5, 2.0)
            inp(c, "alpha", C, 0.0, 0.5)
        cases.append(c)

    def instnorm(name, C, HW):
        c = Case(name, "instnorm", dict(C=C, HW=HW, eps=1e-5, act=ACT_LEAKY, slope=0.01))
        inp(c, "x", C * HW, -2, 3)
        inp(c, "g", C, 0.5, 1.5)
        inp(c, "bias", C, -1, 1)
        cases.append(c)

    def layernorm(name, rows, C):
        c = Case(name, "layernorm", dict(rows=rows, C=C, eps=1e-6, act=ACT_GELU))
        inp(c, "x", rows * C, -2, 3)
        inp(c, "g", C, 0.5, 1.5)
        inp(c, "bias", C, -1, 1)
        cases.append(c)

    def softmax(name, rows, L, scale):
        c = Case(name, "softmax", dict(rows=rows, L=L, scale=float(np.float32(scale))))
        inp(c, "x", rows * L, -20, 20)
        cases.append(c)

    def attention(name, Nq, Nk, nh, d, masked):
        E = nh * d
        scale = float(np.float32(1.0) / np.sqrt(np.float32(d)))
        c = Case(name, "attention", dict(Nq=Nq, Nk=Nk, nh=nh, d=d, scale=scale, masked=masked))
        inp(c, "qkv", Nk * 3 * E, -2, 2)
        if masked:
            u = rng.rand(Nk, 0, 1)
            c.inputs["mask"] = (u > np.float32(0.3)).astype(np.float32)
        cases.append(c)

    def rope(name, rows, nh, d, npos, interleaved):
        ld = nh * d + 6
        c = Case(name, "rope", dict(rows=rows, nh=nh, d=d, npos=npos, ld=ld, off=3,
                                   interleaved=interleaved))
        inp(c, "x", rows * ld + 3, -1, 1)
        c.inputs["angles"] = rng.rand(npos * d // 2, -3.2, 3.2)
        cases.append(c)

    def resize(name, C, h, w, H, W, align, scale):
        c = Case(name, "resize", dict(C=C, h=h, w=w, H=H, W=W, coff=2, align=align,
                                     scale=float(scale)))
        inp(c, "x", C * h * w, -1, 1)
        cases.append(c)

    def grid_sample(name, C, H, W, n, align):
        c = Case(name, "grid_sample", dict(C=C, H=H, W=W, n=n, align=align))
        inp(c, "x", C * H * W, -1, 1)
        inp(c, "grid", 2 * n, -1.2, 1.2)
        cases.append(c)

    def unfold(name, C, H, W, k, s, p):
        c = Case(name, "unfold", dict(C=C, H=H, W=W, k=k, s=s, p=p))
        inp(c, "x", C * H * W, -1, 1)
        cases.append(c)

    def pool(name, C, H, W, k, s, p, mx):
        c = Case(name, "pool", dict(C=C, H=H, W=W, k=k, s=s, p=p, max=mx))
        inp(c, "x", C * H * W, -1, 1)
        cases.append(c)

    def transpose(name, B, R, C_):
        c = Case(name, "transpose", dict(B=B, R=R, C=C_))
        inp(c, "x", B * R * C_, -1, 1)
        cases.append(c)

    def elementwise(name, C_, HW):
        c = Case(name, "elementwise", dict(C=C_, HW=HW, slope=0.05, a=0.5, b=-2.0))
        inp(c, "x", C_ * HW, -3, 3)
        inp(c, "alpha", C_, 0, 0.5)
        inp(c, "b", HW, -1, 1)
        cases.append(c)

    def fold_bn(name, C_, H, W, K):
        per = C_ * 9
        c = Case(name, "fold_bn", dict(C=C_, H=H, W=W, K=K, eps=1e-5))
        c.inputs["w"] = rng.rand(K * per, -0.3, 0.3)
        c.inputs["bias"] = rng.rand(K, -1, 1)
        c.inputs["gamma"] = rng.rand(K, 0.5, 1.5)
        c.inputs["beta"] = rng.rand(K, -1, 1)
        c.inputs["mean"] = rng.rand(K, -1, 1)
        c.inputs["var"] = rng.rand(K, 0.2, 2.0)
        inp(c, "x", C_ * H * W, -1, 1)
        cases.append(c)

    gemm("gemm_small_nt", 37, 29, 21, 0, 1, ACT_GELU, 0)
    gemm("gemm_small_t", 70, 65, 33, 1, 3, ACT_LEAKY, 1)
    gemm("gemm_big_t", 300, 200, 96, 1, 2, ACT_RELU, 1)
    gemm("gemm_big_nt", 256, 130, 64, 0, 1, ACT_NONE, 0)
    conv1x1("conv1x1", 48, 300, 40)
    conv("conv5x5_norm", 12, 37, 45, 10, 5, 1, 2, 1, 1, ACT_NONE, 1)
    conv("conv5x5_first", 3, 33, 20, 16, 5, 1, 2, 1, 1, ACT_NONE, 0)
    conv("conv3x3_s2_g2", 6, 37, 29, 8, 3, 2, 1, 1, 2, ACT_RELU, 0)
    conv("conv3x3_dil2", 5, 21, 26, 7, 3, 1, 2, 2, 1, ACT_LEAKY, 0)
    conv("conv_dw4_s4", 8, 32, 40, 8, 4, 4, 0, 1, 8, ACT_NONE, 0)
    conv("conv5x5_norm_relu", 6, 19, 23, 5, 5, 1, 2, 1, 1, ACT_RELU, 1)
    conv("conv3x3_im2col", 24, 37, 29, 20, 3, 1, 1, 1, 1, ACT_RELU, 0)
    # Three im2col blocks of at most 128 output positions.
    conv("conv3x3_s2_im2col_blocks", 16, 33, 41, 12, 3, 2, 1, 1, 1, ACT_LEAKY, 0,
         im2col_bytes=16 * 9 * 128 * 4)
    instnorm("instnorm", 7, 1000)
    layernorm("layernorm_96", 50, 96)
    layernorm("layernorm_1030", 9, 1030)
    softmax("softmax", 7, 300, 0.1)
    softmax("softmax_short", 5, 20, 10.0)
    attention("attention_d40", 50, 77, 3, 40, 0)
    attention("attention_d128_mask", 33, 300, 2, 128, 1)
    attention("attention_d32", 260, 260, 8, 32, 0)
    rope("rope_interleaved", 20, 2, 16, 10, 1)
    rope("rope_half", 20, 2, 16, 10, 0)
    resize("resize_x2", 3, 16, 24, 32, 48, 0, 2.0)
    resize("resize_size", 2, 13, 17, 29, 31, 0, 0)
    resize("resize_align", 2, 13, 17, 29, 31, 1, 0)
    grid_sample("grid_sample", 3, 20, 25, 500, 0)
    grid_sample("grid_sample_align", 3, 20, 25, 500, 1)
    unfold("unfold", 4, 12, 10, 3, 2, 1)
    unfold("unfold_8", 2, 16, 16, 8, 8, 0)
    pool("avgpool2", 3, 16, 22, 2, 2, 0, 0)
    pool("maxpool4", 3, 16, 24, 4, 4, 0, 1)
    pool("avgpool3_pad", 2, 15, 17, 3, 2, 1, 0)
    transpose("transpose", 2, 37, 50)
    elementwise("elementwise", 5, 77)
    fold_bn("fold_bn", 4, 11, 13, 6)
    return cases


def conv_out(n, k, s, p, d=1):
    return (n + 2 * p - d * (k - 1) - 1) // s + 1


def rope_table(angles):
    """(cos, sin) float32 pairs as ops_check.c:286-291 builds them."""
    a = angles.astype(np.float32)
    cs = np.empty(a.size * 2, np.float32)
    cs[0::2] = np.cos(a)
    cs[1::2] = np.sin(a)
    return cs
