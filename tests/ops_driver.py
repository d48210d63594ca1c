# SPDX-License-Identifier: Unlicense
"""Runs one oracle/ops_cases.py case through the C-ABI (ops.h), making the
same calls as the reference's tests/ops_check.c case functions
(ops_check.c:113-430), and returns the device outputs."""

import ctypes as C

import numpy as np

import coreg
from coreg import handle
from oracle.ops_cases import conv_out, rope_table


def run_case_dev(dev, c):
    lib, o = dev.lib, dev.ops_p
    p, x = c.p, c.inputs
    up = {k: dev.upload(v.astype(np.float32)) for k, v in x.items()}
    out = {}
    op = c.op

    def mat(b, off, ld):
        return coreg.Opnd(handle(b), off, ld, 0, 0)

    def bmat(b, off, ld, s0, s1):
        return coreg.Opnd(handle(b), off, ld, s0, s1)

    if op == "gemm":
        M, N, K, nb = p["M"], p["N"], p["K"], p["nb"]
        Cb = up["r"] if p["residual"] else dev.zeros(nb * M * N)
        lib.ops_gemm(o, M, N, K, bmat(up["a"], 0, K, M * K, 0),
                     bmat(up["b"], 0, K if p["transb"] else N, N * K, 0), p["transb"],
                     bmat(Cb, 0, N, M * N, 0), nb, 1, handle(up["bias"]), 0,
                     handle(Cb) if p["residual"] else None, 0, p["alpha"], p["act"], p["slope"])
        out["out"] = Cb.read(count=nb * M * N)
    elif op == "conv1x1":
        C_, HW, K = p["C"], p["HW"], p["K"]
        Y = dev.zeros(K * HW)
        lib.ops_conv1x1(o, handle(up["x"]), 0, C_, HW, handle(up["w"]), handle(up["bias"]), K,
                        handle(Y), 0, p["act"], 0.0)
        out["out"] = Y.read(count=K * HW)
    elif op == "conv2d":
        k, s, pd, d = p["k"], p["s"], p["p"], p["d"]
        g = coreg.ConvGeom(k, k, s, s, pd, pd, d, d, p["groups"])
        Ho, Wo = conv_out(p["H"], k, s, pd, d), conv_out(p["W"], k, s, pd, d)
        Y = dev.zeros(p["K"] * Ho * Wo)
        old = dev.ops.im2col_bytes
        if "im2col_bytes" in p:
            dev.ops.im2col_bytes = p["im2col_bytes"]
        lib.ops_conv2d(o, handle(up["x"]), p["C"], p["H"], p["W"], handle(up["w"]),
                       handle(up["bias"]), p["K"], C.byref(g), handle(up.get("mean")),
                       handle(up.get("rstd")), handle(up.get("alpha")), p["act"], p["slope"],
                       handle(Y))
        dev.ops.im2col_bytes = old
        out["out"] = Y.read(count=p["K"] * Ho * Wo)
    elif op == "instnorm":
        C_, HW = p["C"], p["HW"]
        mean, rstd, Y = dev.zeros(C_), dev.zeros(C_), dev.zeros(C_ * HW)
        lib.ops_chan_stats(o, handle(up["x"]), C_, HW, p["eps"], handle(mean), handle(rstd))
        lib.ops_chan_affine(o, handle(up["x"]), handle(Y), C_, HW, handle(mean), handle(rstd),
                            handle(up["g"]), handle(up["bias"]), p["act"], p["slope"])
        out["out"] = Y.read(count=C_ * HW)
    elif op == "layernorm":
        rows, C_ = p["rows"], p["C"]
        Y = dev.zeros(rows * C_)
        lib.ops_layernorm(o, rows, C_, handle(up["x"]), handle(Y), handle(up["g"]),
                          handle(up["bias"]), p["eps"], p["act"], 0.0)
        out["out"] = Y.read(count=rows * C_)
    elif op == "softmax":
        lib.ops_softmax_rows(o, handle(up["x"]), p["rows"], p["L"], p["scale"])
        out["out"] = up["x"].read(count=p["rows"] * p["L"])
    elif op == "attention":
        Nq, Nk, nh, d = p["Nq"], p["Nk"], p["nh"], p["d"]
        E = nh * d
        Ob = dev.zeros(Nq * E)
        mask = None
        if p["masked"]:
            mask = dev.upload(x["mask"].astype(np.uint8))
        X = up["qkv"]
        lib.ops_attention(o, mat(X, 0, 3 * E), mat(X, E, 3 * E), mat(X, 2 * E, 3 * E),
                          mat(Ob, 0, E), Nq, Nk, nh, d, p["scale"], handle(mask))
        out["out"] = Ob.read(count=Nq * E)
    elif op == "rope":
        T = dev.upload(rope_table(x["angles"]))
        lib.ops_rope(o, handle(up["x"]), p["off"], p["ld"], p["rows"], p["nh"], p["d"],
                     p["npos"], handle(T), p["interleaved"])
        out["out"] = up["x"].read(count=x["x"].size)
    elif op == "resize":
        C_, H, W = p["C"], p["H"], p["W"]
        Y = dev.zeros((C_ + 2) * H * W)
        lib.ops_resize(o, handle(up["x"]), C_, p["h"], p["w"], handle(Y), H, W, 2, p["align"],
                       p["scale"])
        out["out"] = Y.read(count=(C_ + 2) * H * W)
    elif op == "grid_sample":
        C_, n = p["C"], p["n"]
        Y = dev.zeros(C_ * n)
        lib.ops_grid_sample(o, handle(up["x"]), C_, p["H"], p["W"], handle(up["grid"]), n,
                            p["align"], handle(Y))
        out["out"] = Y.read(count=C_ * n)
    elif op == "unfold":
        k, s, pd = p["k"], p["s"], p["p"]
        g = coreg.ConvGeom(k, k, s, s, pd, pd, 1, 1, 1)
        Ho, Wo = conv_out(p["H"], k, s, pd), conv_out(p["W"], k, s, pd)
        n = p["C"] * k * k * Ho * Wo
        Y = dev.zeros(n)
        lib.ops_unfold(o, handle(up["x"]), p["C"], p["H"], p["W"], C.byref(g), handle(Y))
        out["out"] = Y.read(count=n)
    elif op == "pool":
        k, s, pd = p["k"], p["s"], p["p"]
        Ho, Wo = conv_out(p["H"], k, s, pd), conv_out(p["W"], k, s, pd)
        n = p["C"] * Ho * Wo
        Y = dev.zeros(n)
        if k == 2 and s == 2 and pd == 0 and not p["max"]:
            lib.ops_avgpool2(o, handle(up["x"]), p["C"], p["H"], p["W"], handle(Y))
        else:
            lib.ops_pool2d(o, handle(up["x"]), p["C"], p["H"], p["W"], k, s, pd, p["max"],
                           handle(Y))
        out["out"] = Y.read(count=n)
    elif op == "transpose":
        n = p["B"] * p["R"] * p["C"]
        Y = dev.zeros(n)
        lib.ops_transpose(o, handle(up["x"]), handle(Y), p["B"], p["R"], p["C"])
        out["out"] = Y.read(count=n)
    elif op == "elementwise":
        C_, HW = p["C"], p["HW"]
        n = C_ * HW
        Y = dev.zeros(n)
        lib.ops_prelu(o, handle(up["x"]), handle(Y), C_, HW, handle(up["alpha"]))
        out["prelu"] = Y.read(count=n)
        for a in range(1, 5):
            lib.ops_act(o, handle(up["x"]), handle(Y), n, a, p["slope"])
            out[f"act{a}"] = Y.read(count=n)
        lib.ops_axpby(o, handle(Y), handle(up["x"]), p["a"], handle(up["b"]), p["b"], n, HW)
        out["axpby"] = Y.read(count=n)
    elif op == "fold_bn":
        C_, H, W, K = p["C"], p["H"], p["W"], p["K"]
        per = C_ * 9
        w = x["w"].astype(np.float32).copy()
        b = x["bias"].astype(np.float32).copy()
        f32 = [x[k].astype(np.float32) for k in ("gamma", "beta", "mean", "var")]
        lib.ops_fold_bn(w.ctypes.data, b.ctypes.data, K, per, *[a.ctypes.data for a in f32],
                        p["eps"])
        Wd, Bd = dev.upload(w), dev.upload(b)
        g = coreg.ConvGeom(3, 3, 1, 1, 1, 1, 1, 1, 1)
        Y = dev.zeros(K * H * W)
        lib.ops_conv2d(o, handle(up["x"]), C_, H, W, handle(Wd), handle(Bd), K, C.byref(g),
                       None, None, None, 0, 0.0, handle(Y))
        out["out"] = Y.read(count=K * H * W)
    else:
        raise ValueError(op)
    coreg.check(lib)
    return out
