# SPDX-License-Identifier: Unlicense
"""The matcher.h device stage through the C-ABI (matcher_roma_create,
matcher_eloftr_create, matcher_disk_create; GPU): the struct matcher's
alloc / run / match / field / destroy against the same model run directly
plus the restated glue of the reference (oracle/matcher_ref.py:
matcher_roma.c:61-178, matcher_eloftr.c:66-96; the DISK matcher's glue,
matcher_disk.c:62-92, is the keypoints of each AdaLAM pair at their cells
with the inverse confidence as cost). The model results of both routes
come from the same kernels, so cell positions, costs and fields must agree
exactly (float to double conversions aside)."""

import ctypes as C
import os
import tempfile
from pathlib import Path

import numpy as np
import pytest

import coreg
from coreg import synth
from oracle import matcher_ref

CACHE = Path(os.environ.get("COREG_CACHE", Path(tempfile.gettempdir()) / "coreg_cache"))
libc = C.CDLL("libc.so.6")
libc.free.argtypes = [C.c_void_p]


def tile_struct(img1, img2, v1, v2, h, w):
    from coreg.roma import MatcherTile

    fp = lambda a: a.ctypes.data_as(C.POINTER(C.c_float))
    return MatcherTile(img1=fp(img1), img2=fp(img2), valid1=v1.ctypes.data, valid2=v2.ctypes.data,
                       H=img1.shape[1], W=img1.shape[2], h=h, w=w, x0=0, y0=0, index=1)


def read_list(ml):
    out = [(m.x1, m.y1, m.x2, m.y2, m.cost, m.sd, m.cycle) for m in ml.v[:ml.n]]
    if ml.v:
        libc.free(C.cast(ml.v, C.c_void_p))
    return out


def masks(h, w):
    v1 = np.ones((h, w), np.uint8)
    v1[:, :10] = 0
    v2 = np.ones((h, w), np.uint8)
    v2[-12:, :] = 0
    return v1, v2


@pytest.mark.gpu
def test_roma_matcher_matches_direct_model():
    from coreg.roma import Matcher, MatchList, Roma, open_pth
    from roma_fixtures import tile_pair, weight_paths

    H = W = 128
    h = w = 120
    dev = coreg.Device(0, precision=coreg.OPS_FP32)
    lib = dev.lib
    main, dino, v2 = weight_paths()
    pfs = [open_pth(lib, p) for p in (main, dino, v2)]
    m = Matcher()
    lib.matcher_roma_create(C.byref(m), dev.ops_p, *(C.byref(p) for p in pfs), b"roma_v2ref", 1,
                            8, 0.0)
    coreg.check(lib)
    for p in pfs:
        lib.pth_close(C.byref(p))
    m.cycle = 1
    m.alloc(C.byref(m), H, W)
    coreg.check(lib)
    img1, img2, _ = tile_pair(6, H, W)
    img1 = np.ascontiguousarray(img1, np.float32)
    img2 = np.ascontiguousarray(img2, np.float32)
    v1, v2m = masks(h, w)
    t = tile_struct(img1, img2, v1, v2m, h, w)
    m.run(C.byref(m), C.byref(t))
    coreg.check(lib)
    ml = MatchList()
    n = m.match(C.byref(m), C.byref(t), C.byref(ml))
    coreg.check(lib)
    got = read_list(ml)
    fx, fy, fc, fs = (np.zeros(h * w, np.float32) for _ in range(4))
    fp = lambda a: a.ctypes.data_as(C.POINTER(C.c_float))
    m.field(C.byref(m), C.byref(t), fp(fx), fp(fy), fp(fc), fp(fs))
    coreg.check(lib)
    m.destroy(C.byref(m))

    net = Roma(dev, main, dino, v2, H=H, W=W)
    try:
        bflow = net.match(img2, img1)[0]
        flow, cert, sd = net.match(img1, img2)
    finally:
        net.close()
        dev.close()
    want = matcher_ref.roma_matches(flow, cert, sd, h, w, 8, 0.0, v1, v2m, bflow)
    assert n == len(got) == len(want) > 0
    for a, b in zip(got, want):
        assert a[:2] == b[:2]
        assert abs(a[2] - b[2]) < 1e-9 and abs(a[3] - b[3]) < 1e-9
        assert a[4] == pytest.approx(float(b[4]), abs=1e-7)
        assert a[5] == pytest.approx(float(b[5]), rel=1e-6, nan_ok=True)
        assert a[6] == pytest.approx(b[6], abs=1e-5, nan_ok=True)
    wdx, wdy, wc, ws = matcher_ref.roma_field(flow, cert, sd, h, w, v1, v2m)
    for g, e in ((fx, wdx), (fy, wdy), (fc, wc), (fs, ws)):
        g = g.reshape(h, w)
        assert np.array_equal(np.isnan(g), np.isnan(e))
        ok = ~np.isnan(e)
        assert np.max(np.abs(g[ok] - e[ok])) <= 1e-5


@pytest.mark.gpu
def test_eloftr_matcher_matches_direct_model():
    from coreg.eloftr import Eloftr
    from coreg.roma import Matcher, MatchList, open_pth

    H = W = 128
    h = w = 120
    dev = coreg.Device(0, precision=coreg.OPS_FP32)
    lib = dev.lib
    wpath = synth.write_eloftr_weights(CACHE / "weights", 0)
    pf = open_pth(lib, wpath)
    m = Matcher()
    lib.matcher_eloftr_create(C.byref(m), dev.ops_p, C.byref(pf), b"eloftr", 1)
    coreg.check(lib)
    lib.pth_close(C.byref(pf))
    m.alloc(C.byref(m), H, W)
    coreg.check(lib)
    rng = np.random.default_rng(7)
    base = np.stack([synth.band_limited(rng, H, W, 3.0) for _ in range(3)]) / 255.0
    img1 = np.ascontiguousarray(base, np.float32)
    img2 = np.ascontiguousarray(np.roll(base, (8, 8), (1, 2)), np.float32)
    v1, v2m = masks(h, w)
    t = tile_struct(img1, img2, v1, v2m, h, w)
    m.run(C.byref(m), C.byref(t))
    coreg.check(lib)
    ml = MatchList()
    n = m.match(C.byref(m), C.byref(t), C.byref(ml))
    coreg.check(lib)
    got = read_list(ml)
    m.destroy(C.byref(m))

    grey = lambda im: (np.float32(0.2989) * im[0] + np.float32(0.5870) * im[1] +
                       np.float32(0.1140) * im[2]).astype(np.float32)
    net = Eloftr(dev, wpath, H, W, pos_scale=832.0 / 128)
    try:
        mi, mj, mconf, kp = net.match(grey(img1), grey(img2))
    finally:
        net.close()
        dev.close()
    want = matcher_ref.eloftr_matches(kp, mconf, h, w, v1, v2m)
    assert n == len(got) == len(want)
    for a, b in zip(got, want):
        assert np.allclose(a[:4], b[:4], atol=1e-3)
        assert a[4] == pytest.approx(float(b[4]), abs=1e-5)


@pytest.mark.gpu
def test_disk_matcher_matches_direct_stages():
    from coreg import disk as D
    from coreg.roma import Matcher, MatchList, open_pth

    H = W = 128
    h = w = 120
    n = 256
    dev = coreg.Device(0, precision=coreg.OPS_FP32)
    lib = dev.lib
    wpath = synth.write_disk_weights(CACHE / "weights", 0)
    pf = open_pth(lib, wpath)
    cfg = D.DiskMatcherConfig(features=n, threshold=0.0, adalam=D.adalam_config())
    m = Matcher()
    lib.matcher_disk_create(C.byref(m), dev.ops_p, C.byref(pf), C.byref(cfg))
    coreg.check(lib)
    lib.pth_close(C.byref(pf))
    assert m.name == b"disk" and m.multiple == D.DISK_MULTIPLE and not m.field
    m.alloc(C.byref(m), H, W)
    coreg.check(lib)
    rng = np.random.default_rng(9)
    base = np.stack([synth.band_limited(rng, H, W, 2.0) for _ in range(3)]) / 255.0
    img1 = np.ascontiguousarray(base, np.float32)
    img2 = np.ascontiguousarray(np.roll(base, (6, 4), (1, 2)), np.float32)
    v1, v2m = masks(h, w)
    t = tile_struct(img1, img2, v1, v2m, h, w)
    m.run(C.byref(m), C.byref(t))
    coreg.check(lib)
    ml = MatchList()
    got_n = m.match(C.byref(m), C.byref(t), C.byref(ml))
    coreg.check(lib)
    got = read_list(ml)
    m.destroy(C.byref(m))

    net = D.Disk(dev, wpath, H, W, nmax=n)
    try:
        xy1, _, d1 = net.detect(img1, h=h, w=w, n=n, thresh=0.0, valid=v1)
        xy2, _, d2 = net.detect(img2, h=h, w=w, n=n, thresh=0.0, valid=v2m)
        pairs, dist = D.adalam_match(dev, xy1, d1, xy2, d2, D.adalam_config())
    finally:
        net.close()
        dev.close()
    assert got_n == len(got) == len(pairs)
    for g, (a, b), c in zip(got, pairs, dist):
        assert g[:4] == (xy1[a, 0], xy1[a, 1], xy2[b, 0], xy2[b, 1])
        assert np.float32(g[4]) == c
        assert np.isnan(g[5]) and np.isnan(g[6])
