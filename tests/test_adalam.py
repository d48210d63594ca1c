# SPDX-License-Identifier: Unlicense
"""AdaLAM (include/adalam.h) against the reference's own adalam.c,
compiled where it lies into oracle/_ref/libadalam_ref.so by oracle/Makefile
(test infrastructure; the tests skip when it has not been built). The
CPU tests run adalam_filter's host path; the GPU tests run its device
passes on the same scenes, and adalam_match with its nearest neighbours on
the device too.

The reference's adalam_match computes its nearest neighbours on the host;
this build's adalam_filter takes them as input. The scenes use descriptors
on a 1/16 grid with small entries, so that every squared norm, dot product
and distance is exact in float32 whatever the summation order: the
nearest neighbours and ratios computed here in numpy are then the
reference's own, and both sides filter the same matches. Keypoints are
integer cells, as DISK's. The bar is bit-exact: the same pairs in the
same order with the same inverse confidences.

Scenes: one affine motion with outliers, two motions, repeated keypoint
positions (equal residuals, so the half-precision duplicate weights take
effect), too few keypoints for a neighbourhood (the ratio-test fallback),
a single keypoint (no match), mutual-nearest-neighbour seeds, and
non-default settings; each over several seeds."""

import ctypes as C
from pathlib import Path

import numpy as np
import pytest

from coreg import disk as D

ROOT = Path(__file__).resolve().parents[1]
REF_LIB = ROOT / "oracle" / "_ref" / "libadalam_ref.so"
DIM = 128


@pytest.fixture(scope="module")
def ref():
    if not REF_LIB.exists():
        pytest.skip("oracle/_ref/libadalam_ref.so not built (make -C oracle)")
    lib = C.CDLL(str(REF_LIB))
    IP, FP = C.POINTER(C.c_int), C.POINTER(C.c_float)
    lib.adalam_defaults.argtypes = [C.POINTER(D.AdalamConfig)]
    lib.adalam_match.restype = C.c_int
    lib.adalam_match.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_void_p, C.c_void_p,
                                 C.c_int, C.c_int, C.POINTER(D.AdalamConfig), C.POINTER(IP),
                                 C.POINTER(FP)]
    return lib


def ref_match(lib, k1, d1, k2, d2, cfg):
    k1, k2, d1, d2 = (np.ascontiguousarray(a, np.float32) for a in (k1, k2, d1, d2))
    pairs, dist = C.POINTER(C.c_int)(), C.POINTER(C.c_float)()
    n = lib.adalam_match(k1.ctypes.data, d1.ctypes.data, len(d1), k2.ctypes.data,
                         d2.ctypes.data, len(d2), d1.shape[1], C.byref(cfg), C.byref(pairs),
                         C.byref(dist))
    if not pairs:
        return np.zeros((0, 2), np.int32), np.zeros(0, np.float32)
    return D.take_matches(n, pairs, dist)


def nearest_exact(d1, d2):
    """The reference's nearest neighbours (adalam.c:38-98) for descriptors
    whose arithmetic is exact: first minimum, ratio with the second
    clamped below at 1e-3, and the nearest d1 of each d2."""
    q1 = (d1 * d1).sum(1)
    q2 = (d2 * d2).sum(1)
    dm = q1[:, None] + q2[None, :] - np.float32(2) * (d1 @ d2.T)
    nn12 = dm.argmin(1).astype(np.int32)
    best = dm[np.arange(len(d1)), nn12]
    rest = dm.copy()
    rest[np.arange(len(d1)), nn12] = np.inf
    second = np.maximum(rest.min(1), np.float32(1e-3)) if dm.shape[1] > 1 else \
        np.full(len(d1), np.float32(3.4028235e38))
    score = (best / second).astype(np.float32)
    nn21 = dm.argmin(0).astype(np.int32)
    return nn12, score, nn21


def grid_desc(rng, n):
    """Descriptors with entries in {-4..4}/16 on 24 random dimensions."""
    d = np.zeros((n, DIM), np.float32)
    for i in range(n):
        idx = rng.choice(DIM, 24, replace=False)
        d[i, idx] = rng.integers(-4, 5, 24) / np.float32(16)
    return d


def scene(seed, n=400, outliers=0.3, motions=1, repeats=0, side=640):
    """Keypoints and descriptors of two images related by `motions` affine
    maps (each on its own part of the image), with a share of outliers."""
    rng = np.random.default_rng(seed)
    k1 = rng.integers(0, side, (n, 2)).astype(np.float32)
    if repeats:
        k1[n - repeats:] = k1[:repeats]
    d2 = grid_desc(rng, n)
    perm = rng.permutation(n)
    k2 = np.zeros_like(k1)
    part = np.minimum((k1[:, 0] * motions / side).astype(int), motions - 1)
    for m in range(motions):
        ang = rng.uniform(-0.3, 0.3)
        sc = rng.uniform(0.8, 1.25)
        A = sc * np.array([[np.cos(ang), -np.sin(ang)], [np.sin(ang), np.cos(ang)]])
        t = rng.uniform(-60, 60, 2)
        sel = part == m
        k2[perm[sel]] = k1[sel] @ A.T + t + rng.normal(0, 0.7, (sel.sum(), 2))
    k2 = np.round(k2).astype(np.float32)
    d1 = d2[perm].copy()
    # A small exact perturbation keeps each inlier's nearest neighbour.
    for i in range(n):
        j = rng.integers(0, DIM)
        d1[i, j] += np.float32(rng.integers(-1, 2) / 16)
    bad = rng.random(n) < outliers
    d1[bad] = grid_desc(rng, int(bad.sum()))
    return k1, d1, k2, d2


def check_same(lib, k1, d1, k2, d2, cfg):
    want_p, want_d = ref_match(lib, k1, d1, k2, d2, cfg)
    nn12, score, nn21 = nearest_exact(d1, d2)
    got_p, got_d = D.adalam_filter(k1, k2, nn12, score, nn21 if cfg.force_seed_mnn else None,
                                   cfg)
    assert got_p.shape == want_p.shape
    assert np.array_equal(got_p, want_p)
    assert np.array_equal(got_d.view(np.uint32), want_d.view(np.uint32))
    return len(want_p)


@pytest.mark.parametrize("seed", [0, 1, 2])
def test_one_motion_with_outliers(ref, seed):
    assert check_same(ref, *scene(seed), D.adalam_config()) > 50


@pytest.mark.parametrize("seed", [3, 4])
def test_two_motions(ref, seed):
    assert check_same(ref, *scene(seed, n=500, outliers=0.2, motions=2), D.adalam_config()) > 50


def test_repeated_keypoints(ref):
    assert check_same(ref, *scene(5, n=300, repeats=60), D.adalam_config()) > 0


def test_mutual_seeds(ref):
    assert check_same(ref, *scene(6), D.adalam_config(force_seed_mnn=1)) > 0


@pytest.mark.parametrize("seed", [7, 8])
def test_other_settings(ref, seed):
    cfg = D.adalam_config(search_expansion=4.0, ransac_iters=64, min_inliers=4, det_thr=2.0,
                          min_confidence=50.0, area_ratio=60.0)
    check_same(ref, *scene(seed, n=350, outliers=0.4), cfg)


def test_fallback_without_neighbourhood(ref):
    k1, d1, k2, d2 = scene(9, n=5, outliers=0.0)
    cfg = D.adalam_config()
    n = check_same(ref, k1, d1, k2, d2, cfg)
    assert n > 0  # every match with a ratio up to 0.95


def test_single_keypoint_gives_nothing(ref):
    k1, d1, k2, d2 = scene(10, n=6)
    want_p, _ = ref_match(ref, k1[:1], d1[:1], k2, d2, D.adalam_config())
    nn12, score, _ = nearest_exact(d1[:1], d2)
    got_p, got_d = D.adalam_filter(k1[:1], k2, nn12, score)
    assert len(want_p) == len(got_p) == 0 and len(got_d) == 0


@pytest.fixture(scope="module")
def device():
    import coreg

    dev = coreg.Device(0)
    yield dev
    dev.close()


@pytest.mark.gpu
@pytest.mark.parametrize("case", ["one", "two", "repeats", "mnn", "settings", "fallback"])
def test_device_passes_match_reference(ref, device, case):
    """adalam_filter with its RANSAC passes on the device, given the same
    nearest neighbours as the host path: the reference's result."""
    cfg = D.adalam_config()
    if case == "one":
        sc = scene(0)
    elif case == "two":
        sc = scene(3, n=500, outliers=0.2, motions=2)
    elif case == "repeats":
        sc = scene(5, n=300, repeats=60)
    elif case == "mnn":
        sc, cfg = scene(6), D.adalam_config(force_seed_mnn=1)
    elif case == "settings":
        sc = scene(7, n=350, outliers=0.4)
        cfg = D.adalam_config(search_expansion=4.0, ransac_iters=64, min_inliers=4,
                              det_thr=2.0, min_confidence=50.0, area_ratio=60.0)
    else:
        sc = scene(9, n=5, outliers=0.0)
    k1, d1, k2, d2 = sc
    want_p, want_d = ref_match(ref, k1, d1, k2, d2, cfg)
    nn12, score, nn21 = nearest_exact(d1, d2)
    got_p, got_d = D.adalam_filter(k1, k2, nn12, score, nn21 if cfg.force_seed_mnn else None,
                                   cfg, dev=device)
    assert np.array_equal(got_p, want_p)
    assert np.array_equal(got_d.view(np.uint32), want_d.view(np.uint32))


@pytest.mark.gpu
@pytest.mark.parametrize("seed,mnn", [(12, 0), (13, 1)])
def test_adalam_match_on_device_matches_reference(ref, seed, mnn):
    """adalam_match: nearest neighbours on the device (float32 products,
    exact on these descriptors), then the filter; the reference's result
    bit for bit."""
    import coreg

    dev = coreg.Device(0)
    try:
        k1, d1, k2, d2 = scene(seed, n=700, outliers=0.25, motions=2)
        cfg = D.adalam_config(force_seed_mnn=mnn)
        got_p, got_d = D.adalam_match(dev, k1, d1, k2, d2, cfg)
    finally:
        dev.close()
    want_p, want_d = ref_match(ref, k1, d1, k2, d2, cfg)
    assert len(want_p) > 50
    assert np.array_equal(got_p, want_p)
    assert np.array_equal(got_d.view(np.uint32), want_d.view(np.uint32))
