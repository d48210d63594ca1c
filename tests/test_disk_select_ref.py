# SPDX-License-Identifier: Unlicense
"""DISK's keypoint selection in the oracle (oracle/disk_ref.py select:
the NMS candidates of the h x w crop above the (n + 1)-th highest score,
in raster order, valid cells only) against the reference's own disk.c,
compiled where it lies behind the harness oracle/disk_select_ref.c into
oracle/_ref/libdisk_select_ref.so by oracle/Makefile (the test skips when
it has not been built): disk_detect runs with its device stage replaced
by stand-ins that return the given NMS mask and heatmap. The same
keypoints and scores, bit for bit, with ties at the cut (which drop
keypoints), fewer candidates than n (the lowest is dropped), ragged
crops and validity masks. CPU only."""

import ctypes as C
from pathlib import Path

import numpy as np
import pytest

from oracle import disk_ref

LIB = Path(__file__).resolve().parents[1] / "oracle" / "_ref" / "libdisk_select_ref.so"


@pytest.fixture(scope="module")
def ref():
    if not LIB.exists():
        pytest.skip("oracle/_ref/libdisk_select_ref.so not built (make -C oracle)")
    lib = C.CDLL(str(LIB))
    P, I = C.c_void_p, C.c_int
    lib.ref_disk_select.restype = I
    lib.ref_disk_select.argtypes = [P, P, I, I, I, I, I, P, P, P]
    return lib


@pytest.mark.parametrize("H,W,h,w,n,ties,masked", [
    (64, 64, 60, 60, 40, False, False), (64, 80, 64, 72, 500, False, True),
    (48, 48, 45, 47, 30, True, True), (32, 32, 32, 32, 5, True, False),
    (40, 40, 40, 40, 12, True, False),
    (128, 128, 125, 120, 2048, False, True)])
def test_selection_matches_reference(ref, H, W, h, w, n, ties, masked):
    rng = np.random.default_rng(H + n)
    heat = rng.standard_normal((H, W)).astype(np.float32)
    if ties:
        heat = (np.round(heat * 2) / 2).astype(np.float32)
        mask = rng.random((h, w)) > 0.7
    else:
        mask = disk_ref.nms_mask(heat, h, w, 0.0)
    mask8 = np.ascontiguousarray(mask, np.uint8)
    valid = (rng.random((h, w)) > 0.2).astype(np.uint8) if masked else None
    xy = np.zeros((n, 2), np.int32)
    score = np.zeros(n, np.float32)
    k = ref.ref_disk_select(mask8.ctypes.data, heat.ctypes.data, H, W, h, w, n,
                            None if valid is None else valid.ctypes.data, xy.ctypes.data,
                            score.ctypes.data)
    want_xy, want_score = disk_ref.select(heat, mask, n, valid)
    assert k == len(want_xy)
    assert k > 0 or ties  # with ties at the cut, every candidate can drop
    assert np.array_equal(xy[:k], want_xy)
    assert np.array_equal(score[:k], want_score.astype(np.float32))
