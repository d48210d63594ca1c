# SPDX-License-Identifier: Unlicense
"""ctypes binding of include/roma.h, include/pth_loader.h and
include/matcher*.h (see coreg/__init__.py)."""

import ctypes as C

import numpy as np

from . import EXTRA_SIGNATURES, OclBackend, Ops, check, load

P, I, F, L = C.c_void_p, C.c_int, C.c_float, C.c_long


PTH_F32, PTH_F16, PTH_BF16, PTH_OTHER = range(4)
PTH_MAX_DIMS = 8


class PthTensor(C.Structure):
    _fields_ = [
        ("name", C.c_char_p),
        ("ndim", I),
        ("shape", L * PTH_MAX_DIMS),
        ("stride", L * PTH_MAX_DIMS),
        ("storage_offset", L),
        ("dtype", I),
        ("data_offset", C.c_int64),
        ("storage_bytes", C.c_size_t),
    ]


class PthFile(C.Structure):
    _fields_ = [("fp", P), ("path", C.c_char_p), ("ntensors", I),
                ("tensors", C.POINTER(PthTensor))]


class RomaModel(C.Structure):
    _fields_ = [
        ("ops", C.POINTER(Ops)),
        ("ocl", C.POINTER(OclBackend)),
        ("imagenet", I),
        ("v2", I),
        ("precision", I),
        ("coarse", I),
        ("H", I),
        ("W", I),
        ("flow", C.POINTER(C.c_float)),
        ("cert", C.POINTER(C.c_float)),
        ("sd", C.POINTER(C.c_float)),
        ("impl", P),
    ]


class MatcherTile(C.Structure):
    _fields_ = [
        ("img1", C.POINTER(C.c_float)), ("img2", C.POINTER(C.c_float)),
        ("valid1", P), ("valid2", P),
        ("H", I), ("W", I), ("h", I), ("w", I), ("x0", I), ("y0", I), ("index", I),
    ]


class Match(C.Structure):
    _fields_ = [("x1", C.c_double), ("y1", C.c_double), ("x2", C.c_double),
                ("y2", C.c_double), ("cost", F), ("sd", F), ("cycle", F)]


class MatchList(C.Structure):
    _fields_ = [("n", I), ("cap", I), ("v", C.POINTER(Match))]


class Matcher(C.Structure):
    pass


Matcher._fields_ = [
    ("name", C.c_char_p), ("multiple", I), ("ops", C.POINTER(Ops)), ("state", P),
    ("dump_dir", C.c_char_p),
    ("alloc", C.CFUNCTYPE(None, C.POINTER(Matcher), I, I)),
    ("run", C.CFUNCTYPE(None, C.POINTER(Matcher), C.POINTER(MatcherTile))),
    ("match", C.CFUNCTYPE(I, C.POINTER(Matcher), C.POINTER(MatcherTile), C.POINTER(MatchList))),
    ("dump", C.CFUNCTYPE(None, C.POINTER(Matcher), C.POINTER(MatcherTile), C.c_char_p)),
    ("field", C.CFUNCTYPE(None, C.POINTER(Matcher), C.POINTER(MatcherTile), C.POINTER(F),
                          C.POINTER(F), C.POINTER(F), C.POINTER(F))),
    ("has_sd", I), ("cycle", I),
    ("destroy", C.CFUNCTYPE(None, C.POINTER(Matcher))),
]

EXTRA_SIGNATURES.update({
    "pth_open": (None, [C.POINTER(PthFile), C.c_char_p]),
    "pth_close": (None, [C.POINTER(PthFile)]),
    "pth_find": (P, [C.POINTER(PthFile), C.c_char_p]),
    "pth_strip_prefix": (I, [C.POINTER(PthFile), C.c_char_p]),
    "pth_bytes": (C.c_double, [C.POINTER(PthFile), C.c_char_p]),
    "pth_require": (C.POINTER(PthTensor), [C.POINTER(PthFile), C.c_char_p, I, C.POINTER(L)]),
    "pth_numel": (L, [C.POINTER(PthTensor)]),
    "pth_read_f32": (C.POINTER(C.c_float), [C.POINTER(PthFile), C.POINTER(PthTensor)]),
    "roma_load": (None, [C.POINTER(RomaModel), C.POINTER(Ops), C.POINTER(PthFile),
                         C.POINTER(PthFile)]),
    "roma_load_v2": (None, [C.POINTER(RomaModel), C.POINTER(PthFile)]),
    "roma_set_coarse": (None, [C.POINTER(RomaModel), I]),
    "roma_alloc": (None, [C.POINTER(RomaModel), I, I]),
    "roma_match": (None, [C.POINTER(RomaModel), P, P, C.c_char_p, I]),
    "roma_match_dev": (None, [C.POINTER(RomaModel), P, P]),
    "roma_results_dev": (None, [C.POINTER(RomaModel), C.POINTER(P), C.POINTER(P), C.POINTER(P)]),
    "roma_sync": (I, [C.POINTER(RomaModel)]),
    "roma_graph_build": (I, [C.POINTER(RomaModel), P, P]),
    "roma_graph_launch": (None, [C.POINTER(RomaModel)]),
    "coreg_host_alloc": (P, [C.c_size_t]),
    "coreg_host_free": (None, [P]),
    "roma_free": (None, [C.POINTER(RomaModel)]),
    "matcher_roma_create": (None, [C.POINTER(Matcher), C.POINTER(Ops), C.POINTER(PthFile),
                                   C.POINTER(PthFile), C.POINTER(PthFile), C.c_char_p, I, I, F]),
    "match_add": (None, [C.POINTER(MatchList), C.POINTER(Match)]),
    "roma_sample_matches": (I, [P, P, P, P, I, I, I, I, I, F, P, P, C.POINTER(MatchList)]),
    "roma_dense_field": (None, [P, P, P, I, I, I, I, P, P, P, P, P, P]),
    "roma_sample_matches_dev": (I, [C.POINTER(Ops), P, P, P, P, I, I, I, I, I, F, P, P,
                                    C.POINTER(MatchList)]),
    "roma_dense_field_dev": (None, [C.POINTER(Ops), P, P, P, I, I, I, I, P, P, P, P, P, P]),
    "eloftr_sample_matches": (I, [P, P, I, I, I, P, P, C.POINTER(MatchList)]),
    "roma_tiles_create": (P, [C.POINTER(C.c_int), I, I, I, C.c_char_p, C.c_char_p, C.c_char_p,
                              I, I, I, I]),
    "roma_tiles_run": (I, [P, I, P, P, P]),
    "roma_tiles_pipelines": (I, [P]),
    "roma_tiles_free": (None, [P]),
})

TILE_GET = C.CFUNCTYPE(None, P, I, C.POINTER(F), C.POINTER(F))
TILE_PUT = C.CFUNCTYPE(None, P, I, C.POINTER(F), C.POINTER(F), C.POINTER(F))


def open_pth(lib, path):
    pf = PthFile()
    lib.pth_open(C.byref(pf), str(path).encode())
    check(lib)
    return pf


class Roma:
    """roma_load (+ roma_load_v2), roma_set_coarse, roma_alloc on a Device."""

    def __init__(self, dev, main, dino, v2=None, H=864, W=864, coarse=560, imagenet=True):
        self.dev = dev
        self.lib = lib = load()
        self.m = RomaModel()
        self.mp = C.pointer(self.m)
        pfs = [open_pth(lib, main), open_pth(lib, dino)]
        lib.roma_load(self.mp, dev.ops_p, C.byref(pfs[0]), C.byref(pfs[1]))
        check(lib)
        if v2 is not None:
            pfs.append(open_pth(lib, v2))
            lib.roma_load_v2(self.mp, C.byref(pfs[2]))
            check(lib)
        for pf in pfs:
            lib.pth_close(C.byref(pf))
        self.m.imagenet = int(imagenet)
        if coarse != 560:
            lib.roma_set_coarse(self.mp, coarse)
            check(lib)
        lib.roma_alloc(self.mp, H, W)
        check(lib)
        self.H, self.W = H, W

    def match(self, imgA, imgB, dump=None, tile=1):
        """Host (3, H, W) float32 images -> (flow (2, H, W), cert (H, W),
        sd (H, W) or None), copies of the model's host results."""
        a = np.ascontiguousarray(imgA, np.float32)
        b = np.ascontiguousarray(imgB, np.float32)
        self.lib.roma_match(self.mp, a.ctypes.data, b.ctypes.data,
                            str(dump).encode() if dump else None, tile)
        check(self.lib)
        return self.results()

    def results(self):
        H, W = self.H, self.W
        flow = np.ctypeslib.as_array(self.m.flow, (2 * H * W,)).reshape(2, H, W).copy()
        cert = np.ctypeslib.as_array(self.m.cert, (H * W,)).reshape(H, W).copy()
        sd = None
        if self.m.v2:
            sd = np.ctypeslib.as_array(self.m.sd, (H * W,)).reshape(H, W).copy()
        return flow, cert, sd

    def match_dev(self, ptrA, ptrB):
        self.lib.roma_match_dev(self.mp, ptrA, ptrB)

    def results_dev(self):
        f, c, s = P(), P(), P()
        self.lib.roma_results_dev(self.mp, C.byref(f), C.byref(c), C.byref(s))
        return f.value, c.value, s.value

    def sync(self):
        r = self.lib.roma_sync(self.mp)
        check(self.lib)
        return r

    def graph_build(self, ptrA, ptrB):
        n = self.lib.roma_graph_build(self.mp, ptrA, ptrB)
        check(self.lib)
        return n

    def graph_launch(self):
        self.lib.roma_graph_launch(self.mp)

    def close(self):
        if self.mp is not None:
            self.lib.roma_free(self.mp)
            self.mp = None


class RomaTiles:
    """roma_tiles.h: pipelines of RoMa models on several devices (or
    several per device), tiles dealt to free pipelines, results in tile
    order."""

    def __init__(self, devices, per_device, precision, main, dino, v2=None, H=864, W=864,
                 coarse=560, imagenet=True):
        self.lib = lib = load()
        devs = (C.c_int * len(devices))(*devices)
        self.h = lib.roma_tiles_create(devs, len(devices), per_device, precision,
                                       str(main).encode(), str(dino).encode(),
                                       str(v2).encode() if v2 else None, H, W, coarse,
                                       int(imagenet))
        check(lib)
        self.H, self.W = H, W

    @property
    def pipelines(self):
        return self.lib.roma_tiles_pipelines(self.h)

    def run(self, ntiles, get, put):
        """get(index, imgA, imgB) fills two (3, H, W) float32 numpy views of
        the pipeline's pinned inputs; put(index, flow, cert, sd) receives
        numpy views (valid during the call; sd None without v2), in
        index order. Returns the number of tiles delivered."""
        H, W = self.H, self.W
        errors = []

        def c_get(_ctx, idx, a, b):
            try:
                get(idx, np.ctypeslib.as_array(a, (3, H, W)), np.ctypeslib.as_array(b, (3, H, W)))
            except Exception as e:  # re-raised on the calling thread
                errors.append(e)

        def c_put(_ctx, idx, flow, cert, sd):
            try:
                put(idx, np.ctypeslib.as_array(flow, (2, H, W)),
                    np.ctypeslib.as_array(cert, (H, W)),
                    np.ctypeslib.as_array(sd, (H, W)) if sd else None)
            except Exception as e:
                errors.append(e)

        g, p = TILE_GET(c_get), TILE_PUT(c_put)
        n = self.lib.roma_tiles_run(self.h, ntiles, C.cast(g, P), C.cast(p, P), None)
        check(self.lib)
        if errors:
            raise errors[0]
        return n

    def close(self):
        if self.h:
            self.lib.roma_tiles_free(self.h)
            self.h = None
