# SPDX-License-Identifier: Unlicense
"""The matchers' host stages against the restated glue of
oracle/matcher_ref.py (CPU; the library's host code only): RoMa's
(roma_sample_matches, roma_dense_field of include/matcher_roma.h;
matcher_roma.c:61-178) on seeded warps, certainties and masks, and
ELoFTR's (eloftr_sample_matches of include/matcher_eloftr.h;
matcher_eloftr.c:66-96) on seeded keypoint pairs. The rules are exact: the same matches in the
same order, the same positions, costs, sd and cycle distances (float to
double conversions aside), and the same dense field bit for bit.

Both are also checked against the reference's own glue: oracle/Makefile
compiles the reference's matcher.c, matcher_roma.c and matcher_eloftr.c
where they lie into oracle/_ref/libglue_ref.so (those tests skip when it
has not been built), and the library's results equal theirs bit for bit,
as do the restated glue's.

Cases: ragged tiles (h, w not multiples of the spacing, smaller than the
padded H x W), warps that leave the tile, NaN certainties, blocks with no
valid cell, a reverse warp for the cycle distance (including a
single-column tile, where it is NaN), spacing 1 and a large spacing."""

import ctypes as C
from pathlib import Path

import numpy as np
import pytest

import coreg
from coreg.roma import MatchList
from oracle import matcher_ref

LIBC = C.CDLL(None)
LIBC.free.argtypes = [C.c_void_p]


def case(seed, H, W, h, w, nan_cert=False, masks=True):
    rng = np.random.default_rng(seed)
    flow = rng.uniform(-1.15, 1.15, (2, H, W)).astype(np.float32)
    cert = rng.uniform(0, 1, (H, W)).astype(np.float32)
    if nan_cert:
        cert[rng.random((H, W)) < 0.05] = np.nan
    sd = rng.uniform(0.1, 3, (H, W)).astype(np.float32)
    bflow = rng.uniform(-1, 1, (2, H, W)).astype(np.float32)
    v1 = v2 = None
    if masks:
        v1 = (rng.random((h, w)) > 0.2).astype(np.uint8)
        v1[: min(h, 9), : min(w, 9)] = 0  # a block with no valid cell
        v2 = (rng.random((h, w)) > 0.1).astype(np.uint8)
    return flow, cert, sd, bflow, v1, v2


def ptr(a):
    return None if a is None else np.ascontiguousarray(a).ctypes.data


def sample(lib, flow, cert, sd, bflow, h, w, spacing, min_cert, v1, v2):
    ml = MatchList()
    H, W = cert.shape
    n = lib.roma_sample_matches(ptr(flow), ptr(cert), ptr(sd), ptr(bflow), H, W, h, w, spacing,
                                min_cert, ptr(v1), ptr(v2), C.byref(ml))
    coreg.check(lib)
    out = [(m.x1, m.y1, m.x2, m.y2, m.cost, m.sd, m.cycle) for m in ml.v[:ml.n]]
    if ml.v:
        LIBC.free(C.cast(ml.v, C.c_void_p))
    assert n == len(out)
    return out


def same(a, b):
    return (a == b) or (np.isnan(a) and np.isnan(b))


@pytest.fixture(scope="module")
def lib():
    lib = coreg.load()
    lib.coreg_set_error_mode(coreg.ERRORS_RECORD)
    yield lib
    lib.coreg_set_error_mode(coreg.ERRORS_FATAL)


@pytest.mark.parametrize("seed,H,W,h,w,spacing,min_cert,nan_cert,masks,cycle", [
    (0, 64, 64, 60, 57, 8, 0.0, False, True, True),
    (1, 64, 80, 64, 80, 8, 0.5, True, True, False),
    (2, 48, 48, 41, 45, 5, 0.2, False, False, True),
    (3, 32, 32, 32, 1, 4, 0.0, False, True, True),
    (4, 40, 40, 33, 39, 1, 0.3, True, True, True),
    (5, 64, 64, 64, 64, 64, 0.0, False, True, True),
])
def test_sampling_matches_oracle(lib, seed, H, W, h, w, spacing, min_cert, nan_cert, masks,
                                 cycle):
    flow, cert, sd, bflow, v1, v2 = case(seed, H, W, h, w, nan_cert, masks)
    if w == 1:
        flow[0] = np.float32(1.0 / W - 1.0)  # every warp lands in the one column
    got = sample(lib, flow, cert, sd, bflow if cycle else None, h, w, spacing, min_cert, v1, v2)
    want = matcher_ref.roma_matches(flow, cert, sd, h, w, spacing, min_cert, v1, v2,
                                    bflow if cycle else None)
    assert len(got) == len(want) > 0
    for g, r in zip(got, want):
        assert g[:4] == tuple(float(v) for v in r[:4])
        assert np.float32(g[4]) == np.float32(r[4]) and same(g[5], float(r[5]))
        assert same(g[6], float(np.float32(r[6])))


@pytest.mark.parametrize("seed,H,W,h,w,masks,with_sd", [
    (0, 64, 64, 60, 57, True, True), (1, 40, 48, 40, 48, False, False), (2, 32, 32, 1, 32, True, True)])
def test_dense_field_matches_oracle(lib, seed, H, W, h, w, masks, with_sd):
    flow, cert, sd, _, v1, v2 = case(seed, H, W, h, w, False, masks)
    dx, dy, c, s = (np.empty((h, w), np.float32) for _ in range(4))
    lib.roma_dense_field(ptr(flow), ptr(cert), ptr(sd) if with_sd else None, H, W, h, w, ptr(v1),
                         ptr(v2), dx.ctypes.data, dy.ctypes.data, c.ctypes.data, s.ctypes.data)
    coreg.check(lib)
    wdx, wdy, wc, ws = matcher_ref.roma_field(flow, cert, sd if with_sd else None, h, w, v1, v2)
    for a, b in ((dx, wdx), (dy, wdy), (c, wc), (s, ws)):
        assert np.array_equal(a, b, equal_nan=True)


def test_bad_spacing_is_an_error(lib):
    flow, cert, sd, _, v1, v2 = case(0, 16, 16, 16, 16)
    ml = MatchList()
    n = lib.roma_sample_matches(ptr(flow), ptr(cert), None, None, 16, 16, 16, 16, 0, 0.0, None,
                                None, C.byref(ml))
    assert n == 0
    with pytest.raises(coreg.CoregError):
        coreg.check(lib)


@pytest.mark.parametrize("seed,h,w,masks", [(0, 120, 120, True), (1, 64, 80, False),
                                            (2, 50, 61, True)])
def test_eloftr_sampling_matches_oracle(lib, seed, h, w, masks):
    rng = np.random.default_rng(seed)
    nm = 300
    # Keypoints around and past the tile, half-cell positions included.
    kp = (rng.uniform(-6, max(h, w) + 2, (nm, 4)) - 3.5).astype(np.float32)
    kp[:20] = np.round(kp[:20]) + np.float32(0.5) - np.float32(3.5)
    mconf = rng.uniform(0, 1, nm).astype(np.float32)
    v1 = v2 = None
    if masks:
        v1 = (rng.random((h, w)) > 0.2).astype(np.uint8)
        v2 = (rng.random((h, w)) > 0.2).astype(np.uint8)
    ml = MatchList()
    n = lib.eloftr_sample_matches(ptr(kp), ptr(mconf), nm, h, w, ptr(v1), ptr(v2), C.byref(ml))
    coreg.check(lib)
    got = [(m.x1, m.y1, m.x2, m.y2, m.cost, m.sd, m.cycle) for m in ml.v[:ml.n]]
    if ml.v:
        LIBC.free(C.cast(ml.v, C.c_void_p))
    want = matcher_ref.eloftr_matches(kp, mconf, h, w, v1, v2)
    assert n == len(got) == len(want) > 0
    for g, r in zip(got, want):
        assert g[:4] == tuple(float(v) for v in r[:4])
        assert np.float32(g[4]) == np.float32(r[4])
        assert np.isnan(g[5]) and np.isnan(g[6])


GLUE = Path(__file__).resolve().parents[1] / "oracle" / "_ref" / "libglue_ref.so"


@pytest.fixture(scope="module")
def glue():
    if not GLUE.exists():
        pytest.skip("oracle/_ref/libglue_ref.so not built (make -C oracle)")
    g = C.CDLL(str(GLUE))
    P, I, F = C.c_void_p, C.c_int, C.c_float
    g.ref_roma_sample.restype = I
    g.ref_roma_sample.argtypes = [P, P, P, P, I, I, I, I, I, F, P, P, P, I]
    g.ref_roma_field.restype = None
    g.ref_roma_field.argtypes = [P, P, P, I, I, I, I, P, P, P, P, P, P]
    g.ref_eloftr_sample.restype = I
    g.ref_eloftr_sample.argtypes = [P, P, I, I, I, P, P, P, I]
    return g


def rows_equal(got, rows):
    assert len(got) == len(rows)
    for g, r in zip(got, rows):
        assert all(same(a, b) for a, b in zip(g, r)), (g, r)


@pytest.mark.parametrize("seed,H,W,h,w,spacing,min_cert,nan_cert,masks,cycle", [
    (0, 64, 64, 60, 57, 8, 0.0, False, True, True),
    (1, 64, 80, 64, 80, 8, 0.5, True, True, False),
    (3, 32, 32, 32, 1, 4, 0.0, False, True, True),
    (4, 40, 40, 33, 39, 1, 0.3, True, True, True),
])
def test_roma_sampling_matches_reference_glue(lib, glue, seed, H, W, h, w, spacing, min_cert,
                                              nan_cert, masks, cycle):
    flow, cert, sd, bflow, v1, v2 = case(seed, H, W, h, w, nan_cert, masks)
    if w == 1:
        flow[0] = np.float32(1.0 / W - 1.0)
    bf = bflow if cycle else None
    rows = np.zeros((h * w, 7))
    n = glue.ref_roma_sample(ptr(flow), ptr(cert), ptr(sd), ptr(bf), H, W, h, w, spacing,
                             min_cert, ptr(v1), ptr(v2), rows.ctypes.data, len(rows))
    assert n > 0
    ref = [tuple(r) for r in rows[:n]]
    rows_equal(sample(lib, flow, cert, sd, bf, h, w, spacing, min_cert, v1, v2), ref)
    # The restated glue of the oracle agrees with the reference as well.
    want = matcher_ref.roma_matches(flow, cert, sd, h, w, spacing, min_cert, v1, v2, bf)
    assert len(want) == n
    for r, o in zip(ref, want):
        assert r[:4] == tuple(float(v) for v in o[:4]) and np.float32(r[4]) == np.float32(o[4])
        assert same(r[6], float(np.float32(o[6])))


def test_roma_field_matches_reference_glue(lib, glue):
    H, W, h, w = 64, 64, 60, 57
    flow, cert, sd, _, v1, v2 = case(7, H, W, h, w, True, True)
    mine = [np.empty((h, w), np.float32) for _ in range(4)]
    ref = [np.empty((h, w), np.float32) for _ in range(4)]
    lib.roma_dense_field(ptr(flow), ptr(cert), ptr(sd), H, W, h, w, ptr(v1), ptr(v2),
                         *[a.ctypes.data for a in mine])
    coreg.check(lib)
    glue.ref_roma_field(ptr(flow), ptr(cert), ptr(sd), H, W, h, w, ptr(v1), ptr(v2),
                        *[a.ctypes.data for a in ref])
    for a, b in zip(mine, ref):
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


def test_eloftr_sampling_matches_reference_glue(lib, glue):
    rng = np.random.default_rng(11)
    h, w, nm = 90, 70, 400
    kp = (rng.uniform(-6, 100, (nm, 4)) - 3.5).astype(np.float32)
    kp[:30] = np.round(kp[:30]) + np.float32(0.5) - np.float32(3.5)
    mconf = rng.uniform(0, 1, nm).astype(np.float32)
    v1 = (rng.random((h, w)) > 0.2).astype(np.uint8)
    v2 = (rng.random((h, w)) > 0.2).astype(np.uint8)
    rows = np.zeros((nm, 7))
    n = glue.ref_eloftr_sample(ptr(kp), ptr(mconf), nm, h, w, ptr(v1), ptr(v2),
                               rows.ctypes.data, nm)
    assert n > 0
    ml = MatchList()
    k = lib.eloftr_sample_matches(ptr(kp), ptr(mconf), nm, h, w, ptr(v1), ptr(v2), C.byref(ml))
    coreg.check(lib)
    got = [(m.x1, m.y1, m.x2, m.y2, m.cost, m.sd, m.cycle) for m in ml.v[:ml.n]]
    if ml.v:
        LIBC.free(C.cast(ml.v, C.c_void_p))
    assert k == n
    rows_equal(got, [tuple(r) for r in rows[:n]])
