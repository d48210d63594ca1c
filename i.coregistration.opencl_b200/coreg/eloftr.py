# SPDX-License-Identifier: Unlicense
"""Efficient LoFTR (include/eloftr.h) through the C-ABI."""

import ctypes as C

import numpy as np

from . import EXTRA_SIGNATURES, OclBackend, Ops, check, load
from .roma import Matcher, PthFile

ELOFTR_MULTIPLE, ELOFTR_DIM, ELOFTR_FINE_DIM = 32, 256, 64


class EloftrModel(C.Structure):
    _fields_ = [
        ("ops", C.POINTER(Ops)),
        ("ocl", C.POINTER(OclBackend)),
        ("pos_scale", C.c_float),
        ("H", C.c_int), ("W", C.c_int), ("h", C.c_int), ("w", C.c_int),
        ("ah", C.c_int), ("aw", C.c_int), ("nmax", C.c_int),
        ("nm", C.c_int),
        ("mi", C.POINTER(C.c_int)), ("mj", C.POINTER(C.c_int)),
        ("mconf", C.POINTER(C.c_float)), ("kp", C.POINTER(C.c_float)),
        ("impl", C.c_void_p),
    ]


EXTRA_SIGNATURES.update({
    "eloftr_load": (None, [C.POINTER(EloftrModel), C.POINTER(Ops), C.POINTER(PthFile)]),
    "eloftr_alloc": (None, [C.POINTER(EloftrModel), C.c_int, C.c_int]),
    "eloftr_match": (None, [C.POINTER(EloftrModel), C.c_void_p, C.c_void_p, C.c_char_p,
                            C.c_int]),
    "eloftr_free": (None, [C.POINTER(EloftrModel)]),
    "matcher_eloftr_create": (None, [C.POINTER(Matcher), C.POINTER(Ops), C.POINTER(PthFile),
                                     C.c_char_p, C.c_int]),
})


class Eloftr:
    """One Efficient LoFTR model on a coreg.Device."""

    def __init__(self, dev, weights, H, W, pos_scale=1.0):
        self.dev, self.lib = dev, load()
        pf = PthFile()
        self.lib.pth_open(C.byref(pf), str(weights).encode())
        check(self.lib)
        self.m = EloftrModel()
        self.mp = C.pointer(self.m)
        try:
            self.lib.eloftr_load(self.mp, dev.ops_p, C.byref(pf))
            check(self.lib)
        finally:
            self.lib.pth_close(C.byref(pf))
        self.m.pos_scale = pos_scale
        self.lib.eloftr_alloc(self.mp, H, W)
        check(self.lib)

    def match(self, grey0, grey1, dump=None, tile=1):
        """Grey (H, W) float32 images -> (mi, mj, mconf, kp (nm, 4))."""
        a = np.ascontiguousarray(grey0, np.float32)
        b = np.ascontiguousarray(grey1, np.float32)
        self.lib.eloftr_match(self.mp, a.ctypes.data, b.ctypes.data,
                              str(dump).encode() if dump else None, tile)
        check(self.lib)
        nm = self.m.nm
        if nm == 0:
            return (np.zeros(0, np.int32), np.zeros(0, np.int32), np.zeros(0, np.float32),
                    np.zeros((0, 4), np.float32))
        return (np.ctypeslib.as_array(self.m.mi, (nm,)).copy(),
                np.ctypeslib.as_array(self.m.mj, (nm,)).copy(),
                np.ctypeslib.as_array(self.m.mconf, (nm,)).copy(),
                np.ctypeslib.as_array(self.m.kp, (nm * 4,)).reshape(nm, 4).copy())

    def close(self):
        if self.mp is not None:
            self.lib.eloftr_free(self.mp)
            self.mp = None
