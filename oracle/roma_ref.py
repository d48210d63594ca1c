# SPDX-License-Identifier: Unlicense
"""CPU restatement of the reference's RoMa device stage (TEST
INFRASTRUCTURE: the checker of the CUDA path, and the CPU baseline of
bench.py; never the product).

Follows i.coregistration.opencl's roma.c (load and fold :101-544, the
tile :679-1435) and roma_kernels.cl in torch on the CPU, channel-major
like the reference, float32 by default (float64 on request), the
Gaussian-process solve in float64 as the reference's host code. Each
function cites the lines it restates. The coarse-pass side is a parameter
(roma.c fixes it at ROMA_COARSE = 560) so that the parity tests can run
small.

Parity pinned for the whole tile: tests/test_roma_ref_pin.py checks this
restatement against the reference's own roma_match (roma.c:1357-1435), run
unchanged on the CPU over an OpenCL emulation for roma_v2ref and RoMa v1 at
its fixed 560 coarse side (the fixture tests/golden/roma_ref_golden.npz and
the script that made it), stage by stage: the warps within relative L2
2.2e-6, the final warp within 0.0003 px at p99. RoMa v2's second pass (vgg2 and refiners2, roma.c:1000-1306) is
pinned to the reference's own code run on the CPU over an OpenCL
emulation (tests/test_roma_v2_ref_cpu.py). The two encoders are pinned to the libraries RoMa builds them
from, on the same seeded weights (tests/test_roma_oracle_pins.py): the
DINOv2 encoder with its position interpolation to transformers' Dinov2Model
and DINOv2's original interpolation call, the VGG19-BN pyramid to
torchvision's vgg19_bn. The Gaussian-process solve (gp_solve), prepare and
interp_pos are pinned to the reference's own host functions, compiled from
its roma.c by oracle/Makefile. The decoder's transformer blocks are pinned to
transformers' Dinov2Layer configured as RoMa's decoder block, the input
resampling bit-exact to Pillow's own resize of float bands, and the
refiners' local correlation to its sampling form through torch's
grid_sample. Its kernel-level steps (the Gaussian-process kernel
matrices, cls_to_flow, warp sampling, local correlation, displacement,
updates, depthwise convolution) are pinned to the reference's own
roma_kernels.cl, compiled as C and run on the CPU through oracle/cl_emul.h.
The rest is checked
through the generic ops they share with oracle/ops_ref.py (pinned to the
reference's ops_compare.py) and by reading the cited lines.
"""

import math

import numpy as np
import torch
import torch.nn.functional as F

VIT_DIM, VIT_DEPTH, DEC_DEPTH, VIT_HEADS, DEC_HEADS = 1024, 24, 5, 16, 8
EPS_BN, EPS_LN_VIT, EPS_LN_DEC = 1e-5, 1e-6, 1e-5
GP_DIM, GP_T, GP_NOISE, COS_EPS = 512, 0.2, 0.1, 1e-6
VIT_GRID, CLS_RES = 37, 64
NCLS = CLS_RES * CLS_RES
REF_SCALE = (16, 8, 4, 2, 1)
REF_FEAT = (512, 512, 256, 64, 9)
REF_EMB = (128, 64, 32, 16, 6)
REF_RADIUS = (7, 3, 2, 0, 0)
PROJ_IN = (1024, 512, 256, 128, 64)
REF2_SCALE = (4, 2, 1)
REF2_IN = (256, 128, 64)
REF2_FEAT = (192, 48, 12)
REF2_EMB = (79, 23, 8)
REF2_RADIUS = (3, 1, 0)
VGG_BLOCKS = (2, 2, 4, 4)
VGG_WIDTH = (64, 128, 256, 512)
IM_MEAN = np.array([0.485, 0.456, 0.406], np.float32)
IM_STD = np.array([0.229, 0.224, 0.225], np.float32)


# ------------------------------------------------------------------ load

def fold_bn(w, b, gamma, beta, mean, var, eps=EPS_BN):
    """ops_fold_bn (ops.c:612-626): per output channel, double scale, float
    results."""
    K = w.shape[0]
    w64 = w.reshape(K, -1).astype(np.float64)
    s = gamma.astype(np.float64) / np.sqrt(var.astype(np.float64) + np.float64(np.float32(eps)))
    wf = (w64 * s[:, None]).astype(np.float32).reshape(w.shape)
    bf = ((b.astype(np.float64) - mean) * s + beta).astype(np.float32)
    return wf, bf


def conv_bn(sd, conv, bn, co):
    """load_conv_bn (roma.c:127-150)."""
    w = sd[f"{conv}.weight"]
    b = sd.get(f"{conv}.bias", np.zeros(co, np.float32))
    return fold_bn(w, b, sd[f"{bn}.weight"], sd[f"{bn}.bias"], sd[f"{bn}.running_mean"],
                   sd[f"{bn}.running_var"])


def cubic_weights(t):
    """PyTorch's bicubic weights, A = -0.75 (roma.c:242-255)."""
    A = -0.75
    x = t + 1
    w0 = ((A * x - 5 * A) * x + 8 * A) * x - 4 * A
    x = t
    w1 = ((A + 2) * x - (A + 3)) * x * x + 1
    x = 1 - t
    w2 = ((A + 2) * x - (A + 3)) * x * x + 1
    x = 2 - t
    w3 = ((A * x - 5 * A) * x + 8 * A) * x - 4 * A
    return np.array([w0, w1, w2, w3])


def interp_pos(pos, c16):
    """DINOv2's interpolate_pos_encoding with scale_factor semantics
    (roma.c:257-298), in double; returns (1 + c16^2, 1024) float32."""
    pos = pos.reshape(-1, VIT_DIM).astype(np.float64)
    grid = pos[1:].reshape(VIT_GRID, VIT_GRID, VIT_DIM)
    inv = VIT_GRID / (c16 + 0.1)
    out = np.empty((1 + c16 * c16, VIT_DIM))
    out[0] = pos[0]
    r = inv * (np.arange(c16) + 0.5) - 0.5
    i0 = np.floor(r).astype(int)
    wts = np.stack([cubic_weights(t) for t in r - i0])  # (c16, 4)
    idx = np.clip(i0[:, None] - 1 + np.arange(4)[None, :], 0, VIT_GRID - 1)  # (c16, 4)
    # out[oy, ox] = sum_ij wy[i] wx[j] grid[idx_y[i], idx_x[j]]
    tmp = np.einsum("yi,yixc->yxc", wts, grid[idx])            # rows
    res = np.einsum("xj,yxjc->yxc", wts, tmp[:, idx])          # columns
    out[1:] = res.reshape(-1, VIT_DIM)
    return out.astype(np.float32)


def gp_basis(w, b, c16):
    """cos(8 pi pos_conv(x, y)) at the c16^2 cell centres, float32 as
    roma.c:328-350."""
    i = np.arange(c16 * c16)
    f32 = np.float32
    x = (f32(-1) + f32(1) / f32(c16) + (i % c16).astype(f32) * (f32(2) - f32(2) / f32(c16)) / f32(c16 - 1)).astype(f32)
    y = (f32(-1) + f32(1) / f32(c16) + (i // c16).astype(f32) * (f32(2) - f32(2) / f32(c16)) / f32(c16 - 1)).astype(f32)
    w = w.reshape(GP_DIM, 2)
    v = (w[None, :, 0] * x[:, None] + w[None, :, 1] * y[:, None]).astype(f32) + b[None, :]
    return np.cos(f32(8.0 * math.pi) * v.astype(f32)).astype(f32)


class Model:
    """Folded weights of RoMa (+ v2), as the reference holds them after
    roma_load / roma_load_v2."""

    def __init__(self, main, dino, v2=None, imagenet=True):
        self.imagenet = imagenet
        self.v2 = v2 is not None
        main = {k[len("matcher.model."):] if k.startswith("matcher.model.") else k: v
                for k, v in main.items()}
        self.vgg = self._vgg(main, "encoder.cnn.layers", 4)
        self.patch_w = dino["patch_embed.proj.weight"]
        self.patch_b = dino["patch_embed.proj.bias"]
        self.cls = dino["cls_token"].reshape(-1)
        self.pos_raw = dino["pos_embed"]
        self.vit = [self._block(dino, f"blocks.{i}", True, True) for i in range(VIT_DEPTH)]
        self.norm_g, self.norm_b = dino["norm.weight"], dino["norm.bias"]
        self.proj = [conv_bn(main, f"decoder.proj.{REF_SCALE[s]}.0", f"decoder.proj.{REF_SCALE[s]}.1",
                             REF_FEAT[s]) for s in range(5)]
        self.gp_w = main["decoder.gps.16.pos_conv.weight"]
        self.gp_b = main["decoder.gps.16.pos_conv.bias"]
        self.dec = [self._block(main, f"decoder.embedding_decoder.blocks.{i}", False, False)
                    for i in range(DEC_DEPTH)]
        self.to_out_w = main["decoder.embedding_decoder.to_out.weight"]
        self.to_out_b = main["decoder.embedding_decoder.to_out.bias"]
        self.ref = [self._refiner(main, s) for s in range(5)]
        if v2 is not None:
            self.vgg2 = self._vgg(v2, "refiner_features.layers", 3)
            self.ref2 = [self._refiner2(v2, j) for j in range(3)]

    @staticmethod
    def _vgg(sd, pre, nblk):
        """load_vgg (roma.c:217-239)."""
        out, idx, cin = [], 0, 3
        for blk in range(nblk):
            for _ in range(VGG_BLOCKS[blk]):
                co = VGG_WIDTH[blk]
                out.append(conv_bn(sd, f"{pre}.{idx}", f"{pre}.{idx + 1}", co))
                cin = co
                idx += 3
            idx += 1
        return out

    @staticmethod
    def _block(sd, pre, qkv_bias, ls):
        """load_block (roma.c:155-214): LayerScales folded into proj and
        fc2 (float products, as the reference's float loop)."""
        b = {k: sd[f"{pre}.{n}"] for k, n in (
            ("n1g", "norm1.weight"), ("n1b", "norm1.bias"), ("qkv_w", "attn.qkv.weight"),
            ("n2g", "norm2.weight"), ("n2b", "norm2.bias"), ("fc1_w", "mlp.fc1.weight"),
            ("fc1_b", "mlp.fc1.bias"))}
        b["qkv_b"] = sd[f"{pre}.attn.qkv.bias"] if qkv_bias else None
        for j, wn in enumerate(("attn.proj", "mlp.fc2")):
            w = sd[f"{pre}.{wn}.weight"].copy()
            bias = sd[f"{pre}.{wn}.bias"].copy()
            if ls:
                g = sd[f"{pre}.ls{j + 1}.gamma"]
                w = (w * g[:, None]).astype(np.float32)
                bias = (bias * g).astype(np.float32)
            b["fc2_w" if j else "proj_w"] = w
            b["fc2_b" if j else "proj_b"] = bias
        return b

    @staticmethod
    def _ref_blocks(sd, pre, cin, v2):
        blocks = []
        for b in range(9):
            blk = f"{pre}.block1" if b == 0 else f"{pre}.hidden_blocks.{b - 1}"
            dw, bn, pw = ((f"{blk}.conv_depthwise", f"{blk}.norm", f"{blk}.conv_pointwise") if v2
                          else (f"{blk}.0", f"{blk}.1", f"{blk}.3"))
            w, bias = conv_bn(sd, dw, bn, cin)
            blocks.append((w, bias, sd[f"{pw}.weight"].reshape(cin, cin), sd[f"{pw}.bias"]))
        return blocks

    def _refiner(self, sd, s):
        """load_refiner (roma.c:352-396)."""
        f, e, r = REF_FEAT[s], REF_EMB[s], REF_RADIUS[s]
        cin = 2 * f + e + ((2 * r + 1) ** 2 if r else 0)
        pre = f"decoder.conv_refiner.{REF_SCALE[s]}"
        return dict(scale=REF_SCALE[s], feat=f, emb=e, radius=r, cin=cin, nout=3,
                    blocks=self._ref_blocks(sd, pre, cin, False),
                    out_w=sd[f"{pre}.out_conv.weight"].reshape(3, cin),
                    out_b=sd[f"{pre}.out_conv.bias"],
                    emb_w=sd[f"{pre}.disp_emb.weight"].reshape(e, 2),
                    emb_b=sd[f"{pre}.disp_emb.bias"])

    def _refiner2(self, sd, j):
        """load_refiner2 (roma.c:460-531): heads concatenated."""
        f, e, r = REF2_FEAT[j], REF2_EMB[j], REF2_RADIUS[j]
        cin = 2 * f + e + ((2 * r + 1) ** 2 if r else 0)
        pre = f"refiners.{REF2_SCALE[j]}"
        return dict(scale=REF2_SCALE[j], feat=f, emb=e, radius=r, cin=cin, nout=6,
                    proj_w=sd[f"{pre}.proj.weight"], proj_b=sd[f"{pre}.proj.bias"],
                    blocks=self._ref_blocks(sd, pre, cin, True),
                    out_w=np.concatenate([sd[f"{pre}.warp_head.weight"].reshape(2, cin),
                                          sd[f"{pre}.confidence_head.weight"].reshape(4, cin)]),
                    out_b=np.concatenate([sd[f"{pre}.warp_head.bias"],
                                          sd[f"{pre}.confidence_head.bias"]]),
                    emb_w=sd[f"{pre}.disp_emb.weight"].reshape(e, 2),
                    emb_b=sd[f"{pre}.disp_emb.bias"])


# ------------------------------------------------------------- the tile

def cos_exp(S, nx, ny):
    """roma_cos_exp (roma_kernels.cl:27-38) on the dot products S (N, M)
    with the row norms nx (N) and ny (M)."""
    return torch.exp((S / (nx[:, None] * ny[None, :] + COS_EPS) - 1.0) / GP_T)


def disp(flow, gx, gy, fx, fy):
    """roma_disp (roma_kernels.cl:196-208): (fx, fy) (warp - cell centre)."""
    return torch.stack([fx * (flow[0] - gx), fy * (flow[1] - gy)])


def update(flow, cert, d, scale, Wf, Hf):
    """roma_update (roma_kernels.cl:213-224)."""
    flow = flow + torch.stack([scale * (d[0] / (4.0 * Wf)), scale * (d[1] / (4.0 * Hf))])
    return flow, cert + d[2]


def update2(flow, conf, d, W, H):
    """roma2_update (roma_kernels.cl:230-250): warp += d / (4 W, 4 H),
    confidence += overlap logit and the precision terms of the softplus
    Cholesky factor (threshold 20, + 1e-6)."""
    flow = flow + torch.stack([d[0] / (4.0 * W), d[1] / (4.0 * H)])
    sp = lambda x: torch.where(x > 20, x, torch.log1p(torch.exp(x)))
    l00 = sp(d[3]) + 1e-6
    l10 = d[4]
    l11 = sp(d[5]) + 1e-6
    return flow, conf + torch.stack([d[2], l00 * l00, l00 * l10, l10 * l10 + l11 * l11])


def gp_solve(K, F):
    """gp_solve (roma.c:772-836): (K + 0.1 I)^-1 F in float64 through the
    Cholesky factor, K (n, n) and F (n, d) as given (float32 in the
    reference), the result in float64."""
    n = K.shape[0]
    A = K.double() + GP_NOISE * torch.eye(n, dtype=torch.float64)
    return torch.cholesky_solve(F.double(), torch.linalg.cholesky(A))


def pil_cubic(x):
    a = -0.5
    x = abs(x)
    if x < 1:
        return ((a + 2) * x - (a + 3)) * x * x + 1
    if x < 2:
        return (((x - 5) * x + 8) * x - 4) * a
    return 0.0


def pil_matrix(n_in, n_out):
    """Pillow's antialiased bicubic resampling as an (n_out, n_in) double
    matrix (resize_axis, roma.c:1120-1155)."""
    scale = n_in / n_out
    fs = max(scale, 1.0)
    support = 2 * fs
    M = np.zeros((n_out, n_in))
    for o in range(n_out):
        center = (o + 0.5) * scale
        xmin = max(int(center - support + 0.5), 0)
        xmax = min(int(center + support + 0.5), n_in) - xmin
        k = np.array([pil_cubic((x + xmin - center + 0.5) / fs) for x in range(xmax)])
        ww = k.sum()
        M[o, xmin:xmin + xmax] = k / ww if ww != 0 else 0
    return M


def prepare(img, h, w, imagenet):
    """prepare (roma.c:1159-1186): (3, H, W) float32 in 0..1 resized to
    (3, h, w) (rows first, float between the passes), normalized."""
    img = np.asarray(img, np.float32)
    _, H, W = img.shape
    if (H, W) == (h, w):
        out = img.copy()
    else:
        mx, my = pil_matrix(W, w), pil_matrix(H, h)
        tmp = np.einsum("chw,ow->cho", img.astype(np.float64), mx).astype(np.float32)
        out = np.einsum("oh,chw->cow", my, tmp.astype(np.float64)).astype(np.float32)
    if imagenet:
        out = ((out - IM_MEAN[:, None, None]) / IM_STD[:, None, None]).astype(np.float32)
    return out


class Runner:
    """roma_match of the reference on the CPU, keeping every intermediate
    the reference dumps (roma.c:1188-1227) in `dumps`."""

    def __init__(self, model, coarse=560, dtype=torch.float32):
        self.m = model
        self.Cs = coarse
        self.c16 = coarse // 14
        self.n16 = self.c16 ** 2
        self.dt = dtype
        self.pos = self.t(interp_pos(model.pos_raw, self.c16))
        self.basis = gp_basis(model.gp_w, model.gp_b, self.c16)
        self.dumps = {}
        self.force_mode = None

    def t(self, a):
        return torch.as_tensor(np.asarray(a)).to(self.dt)

    # -- layers -------------------------------------------------------

    def conv(self, x, w, b, stride=1, pad=0, act=None, groups=1):
        y = F.conv2d(x[None], self.t(w), self.t(b), stride=stride, padding=pad, groups=groups)[0]
        return F.relu(y) if act == "relu" else y

    def vgg(self, img, k, P, need, weights):
        """vgg (roma.c:742-768) / vgg2 (roma.c:1000-1027) on one image."""
        x, l = img, 0
        nblk = len(need)
        for blk in range(nblk):
            for _ in range(VGG_BLOCKS[blk]):
                w, b = weights[l]
                x = self.conv(x, w, b, pad=1, act="relu")
                l += 1
            need[blk](x, k)
            if blk < nblk - 1:
                x = F.max_pool2d(x[None], 2, 2)[0]
        return P

    def block(self, x, b, heads, eps):
        """block + attention (roma.c:675-713): pre-norm, full softmax."""
        N, D = x.shape
        hd = D // heads
        h = F.layer_norm(x, (D,), self.t(b["n1g"]), self.t(b["n1b"]), eps)
        qkv = h @ self.t(b["qkv_w"]).T
        if b["qkv_b"] is not None:
            qkv = qkv + self.t(b["qkv_b"])
        q, kk, v = (qkv[:, i * D:(i + 1) * D].reshape(N, heads, hd).transpose(0, 1) for i in range(3))
        s = torch.softmax((q @ kk.transpose(1, 2)) * (1.0 / math.sqrt(hd)), -1)
        o = (s @ v).transpose(0, 1).reshape(N, D)
        x = x + (o @ self.t(b["proj_w"]).T + self.t(b["proj_b"]))
        h = F.layer_norm(x, (D,), self.t(b["n2g"]), self.t(b["n2b"]), eps)
        h = F.gelu(h @ self.t(b["fc1_w"]).T + self.t(b["fc1_b"]))
        return x + (h @ self.t(b["fc2_w"]).T + self.t(b["fc2_b"]))

    def dino(self, img, k):
        """dino (roma.c:717-738): tokens, 24 blocks, LayerNorm, proj.16;
        returns P[0] (512, n16) and dumps the normalized tokens (1024, n16)."""
        m = self.m
        p = self.conv(img, m.patch_w, m.patch_b, stride=14)  # (1024, c16, c16)
        tok = p.reshape(VIT_DIM, -1).T
        x = torch.cat([self.t(m.cls)[None], tok], 0) + self.pos
        for b in m.vit:
            x = self.block(x, b, VIT_HEADS, EPS_LN_VIT)
        x = F.layer_norm(x, (VIT_DIM,), self.t(m.norm_g), self.t(m.norm_b), EPS_LN_VIT)
        feat = x[1:].T.contiguous()  # (1024, n16)
        self.dumps[f"dino_{k}"] = feat
        w, b = m.proj[0]
        return self.t(w.reshape(GP_DIM, VIT_DIM)) @ feat + self.t(b)[:, None]

    def gp(self, fa, fb):
        """gp + cos_kernel + gp_solve (roma.c:772-896): the decoder's input
        tokens (n16, 1024)."""
        ya, yb = fa.T, fb.T  # (n16, 512)
        na, nb = ya.norm(dim=1), yb.norm(dim=1)

        def cosk(a, an, b, bn):
            return cos_exp(a @ b.T, an, bn)

        kyy = cosk(yb, nb, yb, nb)
        kxy = cosk(ya, na, yb, nb)
        X = gp_solve(kyy, torch.from_numpy(self.basis)).to(self.dt)
        mu = kxy @ X
        self.dumps["gp"] = mu
        return torch.cat([mu, ya], 1)

    def cls_to_flow(self, L):
        """roma_cls_to_flow (roma_kernels.cl:46-102): first-index argmax,
        clamped neighbours (a clamped one counts twice).

        With `force_mode` set (one anchor index per token), those anchors
        replace the argmax and the expectation is taken around them: a
        check uses it to start the refiners of this restatement from the
        anchors another run chose at its near-ties."""
        n = L.shape[0]
        logits = L[:, :NCLS]
        m, _ = logits.max(1)
        # First index of the maximum.
        idx = torch.arange(NCLS)[None, :].expand(n, NCLS)
        mode = torch.where(logits == m[:, None], idx, NCLS).min(1).values
        if getattr(self, "force_mode", None) is not None:
            mode = torch.as_tensor(np.asarray(self.force_mode), dtype=torch.long)
            m = torch.gather(logits, 1, mode[:, None])[:, 0]
        s = torch.exp(logits - m[:, None]).sum(1)
        nb = torch.stack([mode - 1, mode, mode + 1, mode - CLS_RES, mode + CLS_RES], 1).clamp(0, NCLS - 1)
        pr = torch.exp(torch.gather(logits, 1, nb) - m[:, None]) / s[:, None]
        cx = -1.0 + (2 * (nb % CLS_RES) + 1).to(self.dt) / CLS_RES
        cy = -1.0 + (2 * (nb // CLS_RES) + 1).to(self.dt) / CLS_RES
        tot = pr.sum(1)
        flow = torch.stack([(pr * cx).sum(1) / tot, (pr * cy).sum(1) / tot])
        return flow, L[:, NCLS].clone()

    def decoder(self, x):
        """decoder (roma.c:900-919)."""
        for b in self.m.dec:
            x = self.block(x, b, DEC_HEADS, EPS_LN_DEC)
        L = x @ self.t(self.m.to_out_w).T + self.t(self.m.to_out_b)
        self.dumps["cls_logits"] = L
        return self.cls_to_flow(L)

    # -- refiners -----------------------------------------------------

    @staticmethod
    def grid(H, W, dt):
        """Cell centres, align_corners False (roma_disp, roma_kernels.cl:196-208)."""
        i = torch.arange(H * W)
        f32 = dt
        gx = -1.0 + 1.0 / W + (i % W).to(f32) * (2.0 - 2.0 / W) / (W - 1)
        gy = -1.0 + 1.0 / H + (i // W).to(f32) * (2.0 - 2.0 / H) / (H - 1)
        return gx, gy

    def sample(self, f, H, W, flow):
        """roma_warp_sample (roma_kernels.cl:130-141): (C, n); zero where
        the warp is not finite (bilinear0, roma_kernels.cl:106-128)."""
        ok = torch.isfinite(flow).all(0)
        g = torch.where(ok[None], flow, 0).T.reshape(1, 1, H * W, 2)
        out = F.grid_sample(f.reshape(1, -1, H, W), g, mode="bilinear", padding_mode="zeros",
                            align_corners=False)[0, :, 0]
        return torch.where(ok[None], out, 0)

    def local_corr(self, f1, f2, H, W, r, flow):
        """roma_local_corr (roma_kernels.cl:153-192): whole-cell dot
        products at the (2r + 2)^2 cells around the warp, combined with the
        shared bilinear weights."""
        C, n = f1.shape
        side, ps = 2 * r + 1, 2 * r + 2
        a1 = f1 * (1.0 / math.sqrt(C))
        ix = ((flow[0] + 1.0) * W - 1.0) * 0.5
        iy = ((flow[1] + 1.0) * H - 1.0) * 0.5
        ok = torch.isfinite(ix) & torch.isfinite(iy)
        x0 = torch.where(ok, torch.floor(torch.where(ok, ix, 0)), 0).long()
        y0 = torch.where(ok, torch.floor(torch.where(ok, iy, 0)), 0).long()
        fx = torch.where(ok, ix - x0, 0).to(self.dt)
        fy = torch.where(ok, iy - y0, 0).to(self.dt)
        out = torch.empty(side * side, n, dtype=self.dt)
        f2f = f2.reshape(C, H * W)
        step = max(1, (1 << 24) // (C * ps * ps))
        for a in range(0, n, step):
            sl = slice(a, a + step)
            e = torch.arange(ps * ps)
            yy = y0[sl, None] - r + e[None] // ps
            xx = x0[sl, None] - r + e[None] % ps
            inb = ok[sl, None] & (xx >= 0) & (xx < W) & (yy >= 0) & (yy < H)
            cell = (yy.clamp(0, H - 1) * W + xx.clamp(0, W - 1))
            v = f2f[:, cell]  # (C, m, ps^2)
            S = torch.einsum("cm,cme->me", a1[:, sl], v) * inb
            S = S.reshape(-1, ps, ps)
            fxs, fys = fx[sl, None, None], fy[sl, None, None]
            comb = (1 - fys) * ((1 - fxs) * S[:, :side, :side] + fxs * S[:, :side, 1:]) + \
                fys * ((1 - fxs) * S[:, 1:, :side] + fxs * S[:, 1:, 1:])
            out[:, sl] = comb.reshape(-1, side * side).T
        return out

    def refine_body(self, r, fa, fb, H, W, dfx, dfy, flow):
        """refine / refine2 (roma.c:923-995, 1033-1104) up to the out conv:
        d = (f_A, f_B at the warp, displacement embedding, correlation),
        9 blocks of depthwise 5 x 5 (+ ReLU) and 1 x 1."""
        n = H * W
        gx, gy = self.grid(H, W, self.dt)
        emb = self.t(r["emb_w"]) @ disp(flow, gx, gy, dfx, dfy) + self.t(r["emb_b"])[:, None]
        parts = [fa, self.sample(fb, H, W, flow), emb]
        if r["radius"]:
            parts.append(self.local_corr(fa, fb, H, W, r["radius"], flow))
        d = torch.cat(parts, 0)
        for dw_w, dw_b, pw_w, pw_b in r["blocks"]:
            d = self.conv(d.reshape(-1, H, W), dw_w, dw_b, pad=2, act="relu",
                          groups=r["cin"]).reshape(r["cin"], n)
            d = self.t(pw_w) @ d + self.t(pw_b)[:, None]
        return self.t(r["out_w"]) @ d + self.t(r["out_b"])[:, None]

    def refine(self, s, P, H, W, Hf, Wf, sf, flow, cert):
        """refine + roma_update (roma.c:923-995, roma_kernels.cl:213-224)."""
        r = self.m.ref[s]
        fac = 40.0 / 32.0 * sf
        d = self.refine_body(r, P[s][0], P[s][1], H, W, fac, fac, flow)
        return update(flow, cert, d, r["scale"], Wf, Hf)

    def refine2(self, j, P2, H, W, Hp, Wp, flow, conf):
        """refine2 + roma2_update (roma.c:1033-1104, roma_kernels.cl:230-250)."""
        r = self.m.ref2[j]
        d = self.refine_body(r, P2[j][0], P2[j][1], H, W, Wp / 512.0, Hp / 512.0, flow)
        return update2(flow, conf, d, W, H)

    def refiners2(self, p, Hp, Wp, h, w, flow, conf, zero_prec, Pp):
        """refiners2 (roma.c:1272-1306): RoMa v2's refiners of pass p (size
        Hp x Wp) from the warp and confidence on an h x w grid; with
        zero_prec the precision is cleared first."""
        for j in range(3):
            hs, ws = Hp // REF2_SCALE[j], Wp // REF2_SCALE[j]
            if zero_prec and j == 0:
                conf = conf.clone()
                conf[1:] = 0
            flow = self.resize(flow, 2, h, w, hs, ws)
            conf = self.resize(conf, 4, h, w, hs, ws)
            flow, conf = self.refine2(j, Pp, hs, ws, Hp, Wp, flow, conf)
            self.dumps[f"p{p}_v2s{REF2_SCALE[j]}_flow"] = flow
            self.dumps[f"p{p}_v2s{REF2_SCALE[j]}_conf"] = conf
            h, w = hs, ws
        return flow, conf, h, w

    @staticmethod
    def resize(x, C, h, w, H, W):
        """ops_resize with size semantics (ops.cl:723-754)."""
        return F.interpolate(x.reshape(1, C, h, w), size=(H, W), mode="bilinear",
                             align_corners=False)[0].reshape(C, H * W)

    def side(self, n, s):
        return n // 14 if s == 0 else n // REF_SCALE[s]

    # -- roma_match -----------------------------------------------------

    def run(self, imgA, imgB):
        """roma_match (roma.c:1357-1435): returns flow (2, H, W), cert (H,
        W) and, with v2, sd (H, W), all float32 numpy."""
        m, Cs = self.m, self.Cs
        H, W = imgA.shape[1:]
        P = [[None, None] for _ in range(5)]
        P2 = [[None, None] for _ in range(3)]
        ins = (imgA, imgB)

        def keep(P_, s, proj):
            def f(x, k):
                w, b = proj[s] if isinstance(proj[s], tuple) else proj[s]
                C = x.shape[0]
                P_[s][k] = (self.t(w.reshape(w.shape[0], -1)) @ x.reshape(C, -1) +
                            self.t(b)[:, None])
            return f

        for k in range(2):
            img = self.t(prepare(ins[k], Cs, Cs, m.imagenet))
            self.dumps[f"in_c_{k}"] = img
            self.vgg(img, k, P, [keep(P, 4 - blk, m.proj) for blk in range(4)], m.vgg)
            if m.v2:
                proj2 = [(r["proj_w"], r["proj_b"]) for r in m.ref2]
                self.vgg(img, k, P2, [keep(P2, 2 - blk, proj2) for blk in range(3)], m.vgg2)
            P[0][k] = self.dino(img, k)
        x = self.gp(P[0][0], P[0][1])
        flow, cert = self.decoder(x)
        self.dumps["cls_flow"], self.dumps["cls_cert"] = flow, cert

        def refiners(p, s0, s1, Hp, Wp, sf, flow, cert, Pp):
            for s in range(s0, s1):
                hs, ws = self.side(Hp, s), self.side(Wp, s)
                flow, cert = self.refine(s, Pp, hs, ws, Hp, Wp, sf, flow, cert)
                if p == 0 and s == 0:
                    self.cert16 = cert.clone()
                self.dumps[f"p{p}_s{REF_SCALE[s]}_flow"] = flow
                self.dumps[f"p{p}_s{REF_SCALE[s]}_cert"] = cert
                if s < s1 - 1:
                    hn, wn = self.side(Hp, s + 1), self.side(Wp, s + 1)
                    flow = self.resize(flow, 2, hs, ws, hn, wn)
                    cert = self.resize(cert, 1, hs, ws, hn, wn)[0]
            return flow, cert

        flow, cert = refiners(0, 0, 2 if m.v2 else 5, Cs, Cs, 1.0, flow, cert, P)
        if m.v2:
            h = w = self.side(Cs, 1)
            conf = torch.zeros(4, h * w, dtype=self.dt)
            conf[0] = cert

            flow, conf, h, w = self.refiners2(0, Cs, Cs, h, w, flow, conf, False, P2)
            proj2 = [(r["proj_w"], r["proj_b"]) for r in m.ref2]
            for k in range(2):
                img = self.t(prepare(ins[k], H, W, m.imagenet))
                self.dumps[f"in_f_{k}"] = img
                self.vgg(img, k, P2, [keep(P2, 2 - blk, proj2) for blk in range(3)], m.vgg2)
            flow, conf, h, w = self.refiners2(1, H, W, h, w, flow, conf, True, P2)
            flow = flow.double().numpy()
            c = conf[0].double().numpy()
            prec = conf[1:].float().double().numpy()
            det = prec[0] * prec[2] - prec[1] * prec[1]
            with np.errstate(invalid="ignore", divide="ignore"):
                sd = np.where(det > 0, np.power(np.where(det > 0, det, 1.0), -0.25), np.nan)
            return self._finish(flow, c, None, H, W) + (sd.reshape(H, W).astype(np.float32),)
        for k in range(2):
            img = self.t(prepare(ins[k], H, W, m.imagenet))
            self.dumps[f"in_f_{k}"] = img
            self.vgg(img, k, P, [keep(P, 4 - blk, m.proj) for blk in range(4)], m.vgg)
        flow = self.resize(flow, 2, Cs, Cs, self.side(H, 1), self.side(W, 1))
        cert = self.resize(cert, 1, Cs, Cs, self.side(H, 1), self.side(W, 1))[0]
        flow, cert = refiners(1, 1, 5, H, W, math.sqrt(H * W) / Cs, flow, cert, P)
        low = self.resize(self.cert16, 1, self.c16, self.c16, H, W)[0]
        return self._finish(flow.double().numpy(), cert.double().numpy(), low.double().numpy(), H, W)

    @staticmethod
    def _finish(flow, c, low, H, W):
        """Host post-processing (roma.c:1340-1349 v2, 1419-1429 v1)."""
        if low is not None:
            c = c - np.where(low < 0, 0.5 * low, 0.0)
        c = 1.0 / (1.0 + np.exp(-c))
        out = (np.abs(flow[0]) > 1) | (np.abs(flow[1]) > 1)
        c = np.where(out, 0.0, c)
        flow = np.clip(flow, -1, 1)
        return flow.reshape(2, H, W).astype(np.float32), c.reshape(H, W).astype(np.float32)
