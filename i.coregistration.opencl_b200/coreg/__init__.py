# SPDX-License-Identifier: Unlicense
"""ctypes binding of libcoreg_b200.so, the C-ABI library of this build.

This is the stub a Python caller of the reference's C API would write
(the reference itself is C and has no Python binding): the structs and
entry points of include/ocl_backend.h, include/ops.h, include/roma.h and
include/matcher.h, declared with their C signatures. Tests and bench.py
use it; it holds no arithmetic.

The library is loaded from the package directory. Loading fails loudly
(OSError) when it has not been built: there is no fallback.
"""

import ctypes as C
import os
from pathlib import Path

import numpy as np

PKG_DIR = Path(__file__).resolve().parent.parent
LIB_PATH = PKG_DIR / "libcoreg_b200.so"

ACT_NONE, ACT_GELU, ACT_RELU, ACT_LEAKY, ACT_GELU_TANH = range(5)
OPS_FP32, OPS_BF16 = 0, 1
ERRORS_FATAL, ERRORS_RECORD = 0, 1


class OclBackend(C.Structure):
    _fields_ = [
        ("device", C.c_int),
        ("queue", C.c_void_p),
        ("device_name", C.c_char * 256),
        ("platform_name", C.c_char * 256),
        ("max_alloc", C.c_uint64),
        ("global_mem", C.c_uint64),
        ("is_gpu", C.c_int),
        ("profile", C.c_int),
        ("sm_count", C.c_int),
        ("cc_major", C.c_int),
        ("cc_minor", C.c_int),
        ("pinned", C.c_void_p),
        ("pinned_bytes", C.c_size_t),
    ]


class Ops(C.Structure):
    _fields_ = [
        ("ocl", C.POINTER(OclBackend)),
        ("precision", C.c_int),
        ("scratch", C.c_void_p),
        ("scratch_bytes", C.c_size_t),
        ("im2col_bytes", C.c_size_t),
        ("scratch16", C.c_void_p),
        ("scratch16_bytes", C.c_size_t),
    ]


class Opnd(C.Structure):
    _fields_ = [
        ("buf", C.c_void_p),
        ("off", C.c_int64),
        ("ld", C.c_int32),
        ("s0", C.c_int64),
        ("s1", C.c_int64),
    ]


class ConvGeom(C.Structure):
    _fields_ = [(n, C.c_int) for n in ("kh", "kw", "sy", "sx", "py", "px", "dy", "dx", "groups")]


P = C.c_void_p
I = C.c_int
L = C.c_long
F = C.c_float
SZ = C.c_size_t

# name: (restype, argtypes)
SIGNATURES = {
    "coreg_set_error_mode": (None, [I]),
    "coreg_last_error": (C.c_char_p, []),
    "coreg_clear_error": (None, []),
    "ocl_init": (None, [C.POINTER(OclBackend), C.c_char_p, C.c_char_p]),
    "ocl_free": (None, [C.POINTER(OclBackend)]),
    "ocl_errstr": (C.c_char_p, [C.c_int32]),
    "ocl_check": (None, [C.c_int32, C.c_char_p]),
    "ocl_alloc": (P, [C.POINTER(OclBackend), SZ, C.c_char_p]),
    "ocl_upload": (P, [C.POINTER(OclBackend), P, SZ, C.c_char_p]),
    "ocl_write": (None, [C.POINTER(OclBackend), P, SZ, P, SZ]),
    "ocl_read": (None, [C.POINTER(OclBackend), P, SZ, P, SZ]),
    "ocl_release": (None, [C.POINTER(P)]),
    "ocl_wrap": (P, [P, SZ]),
    "ocl_ptr": (P, [P]),
    "ocl_bytes": (SZ, [P]),
    "ocl_copy": (None, [C.POINTER(OclBackend), P, SZ, P, SZ, SZ]),
    "ocl_zero": (None, [C.POINTER(OclBackend), P, SZ, SZ]),
    "ocl_finish": (None, [C.POINTER(OclBackend)]),
    "ocl_join": (None, [C.POINTER(OclBackend), C.POINTER(OclBackend)]),
    "ocl_timer_start": (None, [C.POINTER(OclBackend)]),
    "ocl_timer_stop": (C.c_double, [C.POINTER(OclBackend)]),
    "ops_init": (None, [C.POINTER(Ops), C.POINTER(OclBackend)]),
    "ops_free": (None, [C.POINTER(Ops)]),
    "ops_report": (None, []),
    "ops_report_reset": (None, []),
    "ops_report_text": (SZ, [C.c_char_p, SZ]),
    "ops_mat": (Opnd, [P, L, I]),
    "ops_bmat": (Opnd, [P, L, I, L, L]),
    "ops_gemm": (None, [C.POINTER(Ops), I, I, I, Opnd, Opnd, I, Opnd, I, I, P, I, P, L, F, I, F]),
    "ops_linear": (None, [C.POINTER(Ops), I, I, I, P, L, P, P, P, L, I, F, I]),
    "ops_conv1x1": (None, [C.POINTER(Ops), P, L, I, I, P, P, I, P, L, I, F]),
    "ops_geom": (ConvGeom, [I, I, I]),
    "ops_conv_out": (I, [I, I, I, I, I]),
    "ops_conv2d": (None, [C.POINTER(Ops), P, I, I, I, P, P, I, C.POINTER(ConvGeom), P, P, P, I, F, P]),
    "ops_chan_stats": (None, [C.POINTER(Ops), P, I, I, F, P, P]),
    "ops_chan_affine": (None, [C.POINTER(Ops), P, P, I, I, P, P, P, P, I, F]),
    "ops_prelu": (None, [C.POINTER(Ops), P, P, I, I, P]),
    "ops_act": (None, [C.POINTER(Ops), P, P, L, I, F]),
    "ops_layernorm": (None, [C.POINTER(Ops), L, I, P, P, P, P, F, I, F]),
    "ops_softmax_rows": (None, [C.POINTER(Ops), P, L, I, F]),
    "ops_attention": (None, [C.POINTER(Ops), Opnd, Opnd, Opnd, Opnd, I, I, I, I, F, P]),
    "ops_rope": (None, [C.POINTER(Ops), P, L, I, L, I, I, I, P, I]),
    "ops_resize": (None, [C.POINTER(Ops), P, I, I, I, P, I, I, I, I, F]),
    "ops_grid_sample": (None, [C.POINTER(Ops), P, I, I, I, P, I, I, P]),
    "ops_unfold": (None, [C.POINTER(Ops), P, I, I, I, C.POINTER(ConvGeom), P]),
    "ops_avgpool2": (None, [C.POINTER(Ops), P, I, I, I, P]),
    "ops_pool2d": (None, [C.POINTER(Ops), P, I, I, I, I, I, I, I, P]),
    "ops_transpose": (None, [C.POINTER(Ops), P, P, I, I, I]),
    "ops_axpby": (None, [C.POINTER(Ops), P, P, F, P, F, L, L]),
    "ops_fold_bn": (None, [P, P, I, L, P, P, P, P, F]),
    "coreg_tc_status": (I, []),
    "ops_conv3x3_cl": (None, [C.POINTER(Ops), P, I, I, I, P, P, I, I, F, P]),
    "roma_dwconv5_cl": (None, [C.POINTER(Ops), P, I, I, I, P, P, P]),
    "roma_refiner_block_cl": (None, [C.POINTER(Ops), P, I, I, I, P, P, P, P, P]),
    "roma_local_corr_cl": (None, [C.POINTER(Ops), P, P, I, I, I, I, P, P]),
    "ops_gemm_noalloc": (None, [C.POINTER(Ops), I, I, I, Opnd, Opnd, I, Opnd, I, I, P, I, P, L, F, I, F]),
    "ops_gemm_noalloc_max_bytes": (C.c_size_t, []),
    "ops_attention_qkv": (None, [C.POINTER(Ops), P, I, I, I, F, P]),
    "roma_gp_solve": (I, [C.POINTER(Ops), P, I, P, I, C.c_double, P]),
}

_lib = None


def load(path=None):
    """Load the library (once) and declare every entry point; raises
    OSError if it is missing and AttributeError if a declared symbol is
    not exported."""
    global _lib
    if _lib is not None and path is None:
        lib = _lib
    else:
        lib = C.CDLL(str(path or LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
    # Model modules add their entry points to EXTRA_SIGNATURES on import.
    for name, (res, args) in EXTRA_SIGNATURES.items():
        fn = getattr(lib, name, None)
        if fn is not None:
            fn.restype = res
            fn.argtypes = args
    if path is None:
        _lib = lib
    return lib


# Entry points of the model headers, declared by the modules that use them.
EXTRA_SIGNATURES = {}


class CoregError(RuntimeError):
    pass


def check(lib=None):
    """Raise CoregError with the recorded library error, if any."""
    lib = lib or load()
    msg = lib.coreg_last_error()
    if msg:
        lib.coreg_clear_error()
        raise CoregError(msg.decode())


class Buffer:
    """A device buffer (cl_mem) of the library."""

    def __init__(self, dev, handle, nbytes):
        self.dev = dev
        self.handle = handle
        self.nbytes = nbytes

    @property
    def ptr(self):
        return self.dev.lib.ocl_ptr(self.handle)

    def write(self, arr, off=0):
        arr = np.ascontiguousarray(arr)
        self.dev.lib.ocl_write(self.dev.ocl_p, self.handle, off, arr.ctypes.data, arr.nbytes)
        check(self.dev.lib)

    def read(self, dtype=np.float32, count=None, off=0):
        dtype = np.dtype(dtype)
        if count is None:
            count = (self.nbytes - off) // dtype.itemsize
        out = np.empty(count, dtype)
        self.dev.lib.ocl_read(self.dev.ocl_p, self.handle, off, out.ctypes.data, out.nbytes)
        check(self.dev.lib)
        return out

    def release(self):
        if self.handle:
            h = C.c_void_p(self.handle)
            self.dev.lib.ocl_release(C.byref(h))
            self.handle = None

    def __del__(self):
        try:
            self.release()
        except Exception:
            pass


class Device:
    """One ocl_backend + ops pair on CUDA device `index`."""

    def __init__(self, index=0, precision=OPS_FP32, record_errors=True):
        self.lib = load()
        if record_errors:
            self.lib.coreg_set_error_mode(ERRORS_RECORD)
        self.ocl = OclBackend()
        self.ocl_p = C.pointer(self.ocl)
        self.lib.ocl_init(self.ocl_p, str(index).encode(), None)
        check(self.lib)
        self.ops = Ops()
        self.ops_p = C.pointer(self.ops)
        self.lib.ops_init(self.ops_p, self.ocl_p)
        self.ops.precision = precision
        self.buffers = []

    def alloc(self, nbytes, what=b"buffer"):
        h = self.lib.ocl_alloc(self.ocl_p, nbytes, what)
        check(self.lib)
        return Buffer(self, h, nbytes)

    def upload(self, arr):
        arr = np.ascontiguousarray(arr)
        b = self.alloc(max(arr.nbytes, 4))
        if arr.nbytes:
            b.write(arr)
        return b

    def zeros(self, count, dtype=np.float32):
        return self.upload(np.zeros(count, dtype))

    def finish(self):
        self.lib.ocl_finish(self.ocl_p)
        check(self.lib)

    def close(self):
        if self.ops_p is not None:
            self.lib.ops_free(self.ops_p)
            self.lib.ocl_free(self.ocl_p)
            self.ops_p = None


def handle(b):
    """cl_mem of a Buffer, or NULL for None."""
    return None if b is None else b.handle
