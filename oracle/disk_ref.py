# SPDX-License-Identifier: Unlicense
"""CPU restatement of the reference's DISK device stage and its
descriptor-distance step (TEST INFRASTRUCTURE: the checker of the CUDA
path, never the product).

Follows i.coregistration.opencl's disk.c (U-Net :23-31 and :163-214,
candidate selection :236-266), disk_kernels.cl (nms5x5 :10-35, gather_desc
:39-60) and adalam.c (nearest :38-98), in float64 (torch for the
convolutions). The upstream kornia DISK is not available here; the
reference's own DISK stage is the checker instead. The whole detect
(network, NMS, selection, descriptors) is pinned to the reference's disk.c,
ops.c and kernels, unchanged, run on the CPU over the OpenCL emulation of
oracle/cl_backend_emul.c (tests/test_disk_ref_cpu.py). Its pieces are
pinned as well: the keypoint selection (select) is pinned to the reference's own disk_detect
host code, compiled by oracle/Makefile (tests/test_disk_select_ref.py), and
nms_mask and gather to its disk_kernels.cl, compiled as C and run on the
CPU (tests/test_eloftr_disk_kernels_ref.py).
"""

import numpy as np
import torch
import torch.nn.functional as F

CIN = (3, 16, 32, 64, 64, 128, 128, 96, 80)
COUT = (16, 32, 64, 64, 64, 64, 64, 64, 129)
DESC = 128


def _layer(w, l):
    pre = f"unet.path_down.{l}.1" if l < 5 else f"unet.path_up.{l - 5}.conv"
    t = lambda k: torch.from_numpy(np.asarray(w[k], np.float64))
    alpha = t(f"{pre}.1.weight") if l > 0 else None
    return t(f"{pre}.3.weight"), t(f"{pre}.3.bias"), alpha


def _conv(x, w, l, gate):
    """Layer l on x (1, C, H, W): for l > 0 the input normalized by its
    per-channel statistics (biased variance, eps 1e-5) and PReLU-gated
    before the zero padding (ops_conv2d with mean / rstd / alpha, ops.cl
    conv2d; disk.c:133-147)."""
    W_, b, alpha = _layer(w, l)
    if gate:
        m = x.mean((2, 3), keepdim=True)
        v = ((x - m) ** 2).mean((2, 3), keepdim=True)
        x = (x - m) / torch.sqrt(v + 1e-5)
        x = torch.where(x >= 0, x, alpha[None, :, None, None] * x)
    return F.conv2d(x, W_, b, padding=2)


def unet(img, w):
    """(3, H, W) image -> (129, H, W) network output, float64."""
    x = torch.from_numpy(np.asarray(img, np.float64))[None]
    f = [_conv(x, w, 0, False)]
    for lev in range(1, 5):
        t = F.avg_pool2d(f[lev - 1], 2)
        f.append(_conv(t, w, lev, True))
    u = f[4]
    for j in range(4):
        lvl = 3 - j
        up = F.interpolate(u, scale_factor=2.0, mode="bilinear", align_corners=False)
        u = _conv(torch.cat([up, f[lvl]], 1), w, 5 + j, True)
    return u[0].numpy()


def nms_mask(heat, h, w, thresh):
    """nms5x5 (disk_kernels.cl:10-35) on the h x w crop of heat (H, W)."""
    hv = heat[:h, :w]
    mask = np.zeros((h, w), bool)
    for y in range(2, h - 2):
        for x in range(2, w - 2):
            v = hv[y, x]
            win = hv[y - 2:y + 3, x - 2:x + 3].copy()
            win[2, 2] = -np.inf
            mask[y, x] = v > thresh and np.all(v > win)
    return mask


def select(heat, mask, n, valid=None):
    """The n highest candidates in raster order (disk.c:236-266): those
    above the (n + 1)-th highest score (with n or fewer candidates, the
    lowest is the threshold and is dropped)."""
    h, w = mask.shape
    ok = mask if valid is None else mask & (np.asarray(valid) != 0)
    cand = np.sort(heat[:h, :w][ok])[::-1]
    cut = -np.inf
    if cand.size:
        cut = cand[min(n, cand.size - 1)]
    xy, score = [], []
    for y in range(h):
        for x in range(w):
            if len(xy) >= n:
                break
            if ok[y, x] and heat[y, x] > cut:
                xy.append((x, y))
                score.append(heat[y, x])
    return np.array(xy, np.int64).reshape(-1, 2), np.array(score)


def gather(out, xy):
    """gather_desc (disk_kernels.cl:39-60): L2-normalized descriptors."""
    d = out[:DESC, xy[:, 1], xy[:, 0]].T
    return d / np.maximum(np.linalg.norm(d, axis=1, keepdims=True), 1e-12)


def detect(img, w, h, wd, n, thresh=0.0, valid=None):
    out = unet(img, w)
    mask = nms_mask(out[DESC], h, wd, thresh)
    xy, score = select(out[DESC], mask, n, valid)
    return out, xy, score, gather(out, xy) if len(xy) else np.zeros((0, DESC))


def nearest(d1, d2):
    """adalam.c:38-98 in float64: nn12, Lowe ratio score (second clamped
    at 1e-3), nn21, and the per-row gap between the two smallest distances
    (to tell near-ties apart)."""
    d1 = np.asarray(d1, np.float64)
    d2 = np.asarray(d2, np.float64)
    dm = (d1 ** 2).sum(1)[:, None] + (d2 ** 2).sum(1)[None] - 2.0 * d1 @ d2.T
    order = np.argsort(dm, axis=1, kind="stable")
    nn12 = order[:, 0]
    best = dm[np.arange(len(d1)), nn12]
    second = dm[np.arange(len(d1)), order[:, 1]] if d2.shape[0] > 1 else np.full(len(d1), np.inf)
    score = best / np.maximum(second, 1e-3)
    nn21 = np.argmin(dm, axis=0)
    col_gap = np.sort(dm, axis=0)[1] - np.sort(dm, axis=0)[0] if d1.shape[0] > 1 else None
    return nn12, score, nn21, second - best, col_gap
