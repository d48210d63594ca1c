# SPDX-License-Identifier: Unlicense
"""CPU restatement of the reference's matcher glue (TEST INFRASTRUCTURE):
the RoMa sampling of the dense warp into matches (matcher_roma.c:103-145),
its dense field (:150-178) and cycle error (:61-90), and the Efficient
LoFTR keypoint offsets and validity filter (matcher_eloftr.c:66-96).
Pinned to the reference's own glue, compiled into oracle/_ref/libglue_ref.so
by oracle/Makefile (tests/test_matcher_host_stage.py)."""

import math

import numpy as np


def _valid_at(v, h, w, x, y):
    ix, iy = int(math.floor(x + 0.5)) if x >= 0 else -int(math.floor(-x + 0.5)), \
        int(math.floor(y + 0.5)) if y >= 0 else -int(math.floor(-y + 0.5))
    return 0 <= ix < w and 0 <= iy < h and (v is None or v[iy, ix] != 0)


def cycle_error(bflow, H, W, h, w, x, y, xr, yr):
    if w == 1 or h == 1:
        return float("nan")
    xr = min(max(xr, 0.0), w - 1)
    yr = min(max(yr, 0.0), h - 1)
    x0 = min(int(xr), w - 1)
    y0 = min(int(yr), h - 1)
    if x0 == w - 1:
        x0 -= 1
    if y0 == h - 1:
        y0 -= 1
    fx, fy = xr - x0, yr - y0
    bx = by = 0.0
    for j in range(2):
        for i in range(2):
            wgt = (fx if i else 1 - fx) * (fy if j else 1 - fy)
            bx += wgt * ((float(bflow[0, y0 + j, x0 + i]) + 1.0) * 0.5 * W - 0.5)
            by += wgt * ((float(bflow[1, y0 + j, x0 + i]) + 1.0) * 0.5 * H - 0.5)
    return math.hypot(bx - x, by - y)


def roma_matches(flow, cert, sd, h, w, spacing, min_cert, valid1=None, valid2=None,
                 bflow=None):
    """Matches (x1, y1, x2, y2, cost, sd, cycle) of a (2, H, W) warp and
    (H, W) certainty: per spacing x spacing block of the h x w tile the cell
    of highest certainty among valid1 cells (the first on ties), kept when
    its certainty reaches min_cert and its target is a valid2 cell."""
    _, H, W = flow.shape
    out = []
    for by in range(0, h, spacing):
        for bx in range(0, w, spacing):
            best = None
            for y in range(by, min(by + spacing, h)):
                for x in range(bx, min(bx + spacing, w)):
                    if valid1 is not None and not valid1[y, x]:
                        continue
                    if best is None or cert[y, x] > cert[best]:
                        best = (y, x)
            if best is None or not cert[best] >= min_cert:
                continue
            y, x = best
            x2 = (float(flow[0, y, x]) + 1.0) * 0.5 * W - 0.5
            y2 = (float(flow[1, y, x]) + 1.0) * 0.5 * H - 0.5
            if not _valid_at(valid2, h, w, x2, y2):
                continue
            cyc = cycle_error(bflow, H, W, h, w, x, y, x2, y2) if bflow is not None else float("nan")
            out.append((x, y, x2, y2, np.float32(1.0) - cert[y, x],
                        sd[y, x] if sd is not None else float("nan"), cyc))
    return out


def roma_field(flow, cert, sd, h, w, valid1=None, valid2=None):
    """The dense shift (dx, dy) in cells, certainty and sd per cell of the
    h x w tile; NaN shifts and certainty 0 where the cell or its target is
    not valid."""
    _, H, W = flow.shape
    dx = np.full((h, w), np.nan, np.float32)
    dy = np.full((h, w), np.nan, np.float32)
    c = np.zeros((h, w), np.float32)
    s = np.full((h, w), np.nan, np.float32)
    for y in range(h):
        for x in range(w):
            xr = (float(flow[0, y, x]) + 1.0) * 0.5 * W - 0.5
            yr = (float(flow[1, y, x]) + 1.0) * 0.5 * H - 0.5
            if (valid1 is not None and not valid1[y, x]) or not _valid_at(valid2, h, w, xr, yr):
                continue
            dx[y, x], dy[y, x], c[y, x] = xr - x, yr - y, cert[y, x]
            if sd is not None:
                s[y, x] = sd[y, x]
    return dx, dy, c, s


def eloftr_matches(kp, mconf, h, w, valid1=None, valid2=None):
    """Keypoints (x0, y0, x1, y1) in the network's convention, + 3.5 px,
    cost 1 - confidence, kept when both ends round to valid cells."""
    out = []
    for k, c in zip(kp, mconf):
        x1, y1, x2, y2 = (float(v) + 3.5 for v in k)
        if _valid_at(valid1, h, w, x1, y1) and _valid_at(valid2, h, w, x2, y2):
            out.append((x1, y1, x2, y2, np.float32(1.0) - np.float32(c)))
    return out
