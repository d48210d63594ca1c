# SPDX-License-Identifier: Unlicense
"""Efficient LoFTR's RoPE table in the oracle (oracle/eloftr_ref.py
Model.rope_table) against the reference's own eloftr.c rope_table
(eloftr.c:267-291), compiled where it lies behind the harness
oracle/eloftr_host_ref.c into oracle/_ref/libeloftr_host_ref.so by
oracle/Makefile (the test skips when it has not been built). This pins
the position scale of the authors' "npe" (832 over the tile's long side),
which transformers' model lacks, beside position scale 1. The angles are
the same float32 products; their cosines and sines come from different
math libraries (numpy here, the C library's cosf / sinf there) and agree
to one unit in the last place. CPU only."""

import ctypes as C
from pathlib import Path

import numpy as np
import pytest

from coreg import synth
from oracle import eloftr_ref

LIB = Path(__file__).resolve().parents[1] / "oracle" / "_ref" / "libeloftr_host_ref.so"


@pytest.fixture(scope="module")
def ref():
    if not LIB.exists():
        pytest.skip("oracle/_ref/libeloftr_host_ref.so not built (make -C oracle)")
    lib = C.CDLL(str(LIB))
    lib.ref_rope_table.restype = None
    lib.ref_rope_table.argtypes = [C.c_int, C.c_int, C.c_float, C.c_void_p]
    return lib


@pytest.fixture(scope="module")
def model():
    return eloftr_ref.Model(synth.eloftr_weights(0), pos_scale=1.0)


@pytest.mark.parametrize("ah,aw,pos_scale", [(4, 5, 1.0), (20, 20, 832 / 640),
                                             (8, 13, 832 / 1040), (40, 30, 832 / 1280)])
def test_rope_table_matches_reference(ref, model, ah, aw, pos_scale):
    want = np.zeros(ah * aw * eloftr_ref.D, np.float32)
    ref.ref_rope_table(ah, aw, pos_scale, want.ctypes.data)
    model.pos_scale = np.float32(pos_scale)
    got = model.rope_table(ah, aw)
    assert got.shape == want.shape
    assert np.abs(got - want.astype(np.float64)).max() <= 2.0 ** -23
