# SPDX-License-Identifier: Unlicense
"""The Efficient LoFTR and DISK kernels of the oracle (oracle/eloftr_ref.py,
oracle/disk_ref.py) against the reference's own OpenCL kernels
(eloftr_kernels.cl, disk_kernels.cl), compiled as C through
oracle/cl_emul.h and run on the CPU with the reference's work-group sizes
(oracle/_ref/libeloftr_cl_ref.so, libdisk_cl_ref.so, built by
oracle/Makefile; the tests skip when they have not been built). CPU only.

* The blockwise dual softmax (eloftr_row_lse, eloftr_col_lse,
  eloftr_conf_row, eloftr_conf_col), driven in two passes over row blocks
  as eloftr.c does, in one block and in blocks of 16 rows, with a tie in a
  column: the same first argmaxes, maxima within 1e-6.
* The two-stage fine matching (eloftr_fine) for 40 cell pairs, windows at
  the borders included: keypoints within 1e-5 px.
* nms5x5 (same mask, a ragged crop of a wider heatmap plane) and
  gather_desc (descriptors within 1e-6)."""

import ctypes as C
from pathlib import Path

import numpy as np
import pytest

from oracle import disk_ref
from oracle import eloftr_ref as E

REF = Path(__file__).resolve().parents[1] / "oracle" / "_ref"
P, I, FL = C.c_void_p, C.c_int, C.c_float


def load(name, sig):
    path = REF / name
    if not path.exists():
        pytest.skip(f"oracle/_ref/{name} not built (make -C oracle)")
    lib = C.CDLL(str(path))
    for fn, args in sig.items():
        getattr(lib, fn).restype = None
        getattr(lib, fn).argtypes = args
    return lib


@pytest.fixture(scope="module")
def el():
    return load("libeloftr_cl_ref.so", {
        "ref_row_lse": [P, I, I, I, P], "ref_col_lse": [P, I, I, P, P],
        "ref_conf_row": [P, I, I, I, P, P, P, P, P], "ref_conf_col": [P, I, I, I, P, P, P, P, P],
        "ref_fine": [P, P, I, I, P, I, FL, P]})


@pytest.fixture(scope="module")
def dk():
    return load("libdisk_cl_ref.so", {"ref_nms5x5": [P, C.c_ulong, I, I, I, FL, P],
                                      "ref_gather_desc": [P, I, I, I, P, I, P]})


def ref_dual_softmax(el, S, R):
    """The reference's two passes over blocks of R rows (eloftr.c
    coarse_match): row lse and running column lse, then the row and
    running column maxima of the confidence."""
    n0, n1 = S.shape
    lse = np.zeros(n0, np.float32)
    cm, cs = np.full(n1, -np.inf, np.float32), np.zeros(n1, np.float32)
    blocks = [(r0, np.ascontiguousarray(S[r0:r0 + R])) for r0 in range(0, n0, R)]
    for r0, b in blocks:
        el.ref_row_lse(b.ctypes.data, len(b), n1, r0, lse.ctypes.data)
        el.ref_col_lse(b.ctypes.data, len(b), n1, cm.ctypes.data, cs.ctypes.data)
    rmax, rarg = np.zeros(n0, np.float32), np.zeros(n0, np.int32)
    cmax, carg = np.full(n1, -1, np.float32), np.full(n1, -1, np.int32)
    for r0, b in blocks:
        el.ref_conf_row(b.ctypes.data, len(b), n1, r0, lse.ctypes.data, cm.ctypes.data,
                        cs.ctypes.data, rmax.ctypes.data, rarg.ctypes.data)
        el.ref_conf_col(b.ctypes.data, len(b), n1, r0, lse.ctypes.data, cm.ctypes.data,
                        cs.ctypes.data, cmax.ctypes.data, carg.ctypes.data)
    return rmax, rarg, cmax, carg


@pytest.mark.parametrize("R", [150, 16])
def test_dual_softmax(el, R):
    rng = np.random.default_rng(0)
    S = (rng.standard_normal((150, 130)) * 4).astype(np.float32)
    S[5, 7] = S[9, 7] = 30  # two rows tie in column 7: the first wins
    rmax, rarg, cmax, carg = ref_dual_softmax(el, S, R)
    wr, wra, wc, wca = E.dual_softmax_maxima(S.astype(np.float64))
    assert np.array_equal(rarg, wra) and np.array_equal(carg, wca)
    assert np.abs(rmax - wr).max() <= 1e-6 and np.abs(cmax - wc).max() <= 1e-6


def test_fine_matching(el):
    rng = np.random.default_rng(1)
    H, W = 64, 80
    f0 = rng.standard_normal((E.FC, H, W)).astype(np.float32)
    f1 = rng.standard_normal((E.FC, H, W)).astype(np.float32)
    c0 = np.stack([rng.integers(0, W // 8, 40), rng.integers(0, H // 8, 40)], 1)
    c1 = np.clip(c0 + rng.integers(-1, 2, (40, 2)), 0, [W // 8 - 1, H // 8 - 1])
    cells = np.ascontiguousarray(np.concatenate([c0, c1], 1), np.int32)
    cells[0] = (0, 0, 0, 0)
    cells[1] = (W // 8 - 1, H // 8 - 1, W // 8 - 1, H // 8 - 1)
    got = np.zeros((len(cells), 4), np.float32)
    el.ref_fine(f0.ctypes.data, f1.ctypes.data, H, W, cells.ctypes.data, len(cells), E.FINE_T,
                got.ctypes.data)
    want = np.array([E.fine_one(f0.astype(np.float64), f1.astype(np.float64), *c) for c in cells])
    assert np.abs(got - want).max() <= 1e-5


def test_nms_and_gather(dk):
    rng = np.random.default_rng(2)
    H, W, h, w = 40, 50, 37, 45
    out = rng.standard_normal((disk_ref.DESC + 1, H, W)).astype(np.float32)
    mask = np.zeros((h, w), np.uint8)
    dk.ref_nms5x5(out.ctypes.data, disk_ref.DESC * H * W, W, h, w, 0.0, mask.ctypes.data)
    want = disk_ref.nms_mask(out[disk_ref.DESC], h, w, 0.0)
    assert np.array_equal(mask.astype(bool), want) and want.sum() > 10
    xy = np.ascontiguousarray(np.argwhere(want)[:, ::-1], np.int32)
    desc = np.zeros((len(xy), disk_ref.DESC), np.float32)
    dk.ref_gather_desc(out.ctypes.data, H, W, disk_ref.DESC, xy.ctypes.data, len(xy),
                       desc.ctypes.data)
    assert np.abs(desc - disk_ref.gather(out.astype(np.float64), xy)).max() <= 1e-6
