# SPDX-License-Identifier: Unlicense
"""DISK keypoints (include/disk.h) and the device descriptor-distance stage
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


EXTRA_SIGNATURES.update({
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
