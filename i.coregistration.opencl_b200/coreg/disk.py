# SPDX-License-Identifier: Unlicense
"""DISK keypoints (include/disk.h), the device descriptor-distance stage,
AdaLAM (include/adalam.h) and the DISK matcher (include/matcher_disk.h)
through the C-ABI."""

import ctypes as C

import numpy as np

from . import EXTRA_SIGNATURES, OclBackend, Ops, check, load
from .roma import PthFile

DISK_DESC, DISK_LAYERS, DISK_MULTIPLE = 128, 9, 16

I, F, P = C.c_int, C.c_float, C.c_void_p


class DiskModel(C.Structure):
    _fields_ = [
        ("ocl", C.POINTER(OclBackend)),
        ("ops", C.POINTER(Ops)),
        ("cin", C.c_int * DISK_LAYERS),
        ("cout", C.c_int * DISK_LAYERS),
        ("H", C.c_int),
        ("W", C.c_int),
        ("nmax", C.c_int),
        ("impl", C.c_void_p),
    ]


class AdalamConfig(C.Structure):
    _fields_ = [
        ("area_ratio", C.c_double),
        ("search_expansion", C.c_double),
        ("ransac_iters", I),
        ("min_inliers", I),
        ("min_confidence", C.c_double),
        ("det_thr", C.c_double),
        ("force_seed_mnn", I),
    ]


class DiskMatcherConfig(C.Structure):
    _fields_ = [("features", I), ("threshold", F), ("adalam", AdalamConfig)]


IP, FP = C.POINTER(C.c_int), C.POINTER(C.c_float)

EXTRA_SIGNATURES.update({
    "adalam_defaults": (None, [C.POINTER(AdalamConfig)]),
    "adalam_filter": (I, [C.POINTER(Ops), P, I, P, I, P, P, P, C.POINTER(AdalamConfig),
                          C.POINTER(IP), C.POINTER(FP)]),
    "adalam_match": (I, [C.POINTER(Ops), P, P, I, P, P, I, I, C.POINTER(AdalamConfig),
                         C.POINTER(IP), C.POINTER(FP)]),
    "disk_load": (None, [C.POINTER(DiskModel), C.POINTER(Ops), C.POINTER(PthFile)]),
    "disk_alloc": (None, [C.POINTER(DiskModel), I, I, I]),
    "disk_detect": (I, [C.POINTER(DiskModel), P, I, I, I, I, I, F, P, P, P, P]),
    "disk_free": (None, [C.POINTER(DiskModel)]),
    "disk_output_dev": (P, [C.POINTER(DiskModel)]),
    "desc_nearest": (None, [C.POINTER(Ops), P, I, P, I, I, P, P, P]),
})


class Disk:
    """One DISK model on a coreg.Device."""

    def __init__(self, dev, weights, H, W, nmax=2048):
        self.dev, self.lib = dev, load()
        pf = PthFile()
        self.lib.pth_open(C.byref(pf), str(weights).encode())
        check(self.lib)
        self.m = DiskModel()
        self.mp = C.pointer(self.m)
        try:
            self.lib.disk_load(self.mp, dev.ops_p, C.byref(pf))
            check(self.lib)
        finally:
            self.lib.pth_close(C.byref(pf))
        self.lib.disk_alloc(self.mp, H, W, nmax)
        check(self.lib)
        self.H, self.W, self.nmax = H, W, nmax

    def detect(self, img, h=None, w=None, n=None, thresh=0.0, valid=None):
        """img (3, H, W) float32 in 0..1 -> xy (k, 2) int32, score (k,),
        desc (k, 128)."""
        H, W = img.shape[1:]
        h, w = h or H, w or W
        n = n or self.nmax
        img = np.ascontiguousarray(img, np.float32)
        xy = np.zeros((n, 2), np.int32)
        score = np.zeros(n, np.float32)
        desc = np.zeros((n, DISK_DESC), np.float32)
        v = None if valid is None else np.ascontiguousarray(valid, np.uint8)
        k = self.lib.disk_detect(self.mp, img.ctypes.data, H, W, h, w, n, thresh,
                                 None if v is None else v.ctypes.data, xy.ctypes.data,
                                 score.ctypes.data, desc.ctypes.data)
        check(self.lib)
        return xy[:k], score[:k], desc[:k]

    def output(self, H, W):
        """The last detect's network output (129, H, W), read back."""
        ptr = self.lib.disk_output_dev(self.mp)
        n = (DISK_DESC + 1) * H * W
        h = self.lib.ocl_wrap(ptr, n * 4)
        out = np.empty(n, np.float32)
        self.lib.ocl_read(self.dev.ocl_p, h, 0, out.ctypes.data, out.nbytes)
        hh = C.c_void_p(h)
        self.lib.ocl_release(C.byref(hh))
        check(self.lib)
        return out.reshape(DISK_DESC + 1, H, W)

    def close(self):
        if self.mp is not None:
            self.lib.disk_free(self.mp)
            self.mp = None


def nearest(dev, d1, d2, both=True):
    """desc_nearest: (nn12, score, nn21 or None)."""
    lib = load()
    d1 = np.ascontiguousarray(d1, np.float32)
    d2 = np.ascontiguousarray(d2, np.float32)
    n1, dim = d1.shape
    n2 = d2.shape[0]
    nn12 = np.zeros(n1, np.int32)
    score = np.zeros(n1, np.float32)
    nn21 = np.zeros(n2, np.int32) if both else None
    lib.desc_nearest(dev.ops_p, d1.ctypes.data, n1, d2.ctypes.data, n2, dim, nn12.ctypes.data,
                     score.ctypes.data, None if nn21 is None else nn21.ctypes.data)
    check(lib)
    return nn12, score, nn21


_LIBC = C.CDLL(None)
_LIBC.free.argtypes = [C.c_void_p]


def adalam_config(**kw):
    """adalam_defaults, then the given fields."""
    cfg = AdalamConfig()
    load().adalam_defaults(C.byref(cfg))
    for k, v in kw.items():
        setattr(cfg, k, v)
    return cfg


def take_matches(n, pairs, dist):
    """(pairs (n, 2) int32, dist (n,) float32) copied out of the library's
    malloc'd arrays, which are freed."""
    out = (np.ctypeslib.as_array(pairs, (2 * n,)).reshape(n, 2).copy() if n else
           np.zeros((0, 2), np.int32),
           np.ctypeslib.as_array(dist, (n,)).copy() if n else np.zeros(0, np.float32))
    _LIBC.free(C.cast(pairs, C.c_void_p))
    _LIBC.free(C.cast(dist, C.c_void_p))
    return out


def adalam_filter(k1, k2, nn12, score, nn21=None, cfg=None, dev=None):
    """adalam_filter on host arrays, its passes on dev (a coreg.Device) or,
    with dev None, on host threads: (pairs, dist)."""
    lib = load()
    cfg = cfg or adalam_config()
    k1 = np.ascontiguousarray(k1, np.float32)
    k2 = np.ascontiguousarray(k2, np.float32)
    nn12 = np.ascontiguousarray(nn12, np.int32)
    score = np.ascontiguousarray(score, np.float32)
    nn21 = None if nn21 is None else np.ascontiguousarray(nn21, np.int32)
    pairs, dist = IP(), FP()
    n = lib.adalam_filter(None if dev is None else dev.ops_p, k1.ctypes.data, len(k1),
                          k2.ctypes.data, len(k2), nn12.ctypes.data,
                          score.ctypes.data, None if nn21 is None else nn21.ctypes.data,
                          C.byref(cfg), C.byref(pairs), C.byref(dist))
    check(lib)
    return take_matches(n, pairs, dist)


def adalam_match(dev, k1, d1, k2, d2, cfg=None):
    """adalam_match (nearest neighbours on dev, then AdaLAM): (pairs, dist)."""
    lib = load()
    cfg = cfg or adalam_config()
    k1, k2 = (np.ascontiguousarray(k, np.float32) for k in (k1, k2))
    d1, d2 = (np.ascontiguousarray(d, np.float32) for d in (d1, d2))
    pairs, dist = IP(), FP()
    n = lib.adalam_match(dev.ops_p, k1.ctypes.data, d1.ctypes.data, len(d1), k2.ctypes.data,
                         d2.ctypes.data, len(d2), d1.shape[1], C.byref(cfg), C.byref(pairs),
                         C.byref(dist))
    check(lib)
    return take_matches(n, pairs, dist)
