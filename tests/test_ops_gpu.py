# SPDX-License-Identifier: Unlicense
"""Per-op parity of the CUDA kernels (through the C-ABI) against the
oracle, on the reference's ops_check cases (GPU).

Tolerance: the reference's own, max |diff| / max |ref| <= 2e-5
(tests/ops_compare.py:25-26), and a relative L2 error <= 1e-5 (the FP32
mode bound of the build's contract)."""

import numpy as np
import pytest

import coreg
from oracle.ops_cases import build_cases
from oracle.ops_ref import run_case
from ops_driver import run_case_dev

CASES = build_cases()
TOL_MAX = 2e-5
TOL_L2 = 1e-5


def compare(got, want):
    got = np.asarray(got, np.float64).reshape(-1)
    want = np.asarray(want, np.float64).reshape(-1)
    assert got.shape == want.shape
    assert np.isfinite(got).all()
    scale = max(np.abs(want).max(), 1e-30)
    err = np.abs(got - want).max() / scale
    l2 = np.linalg.norm(got - want) / max(np.linalg.norm(want), 1e-30)
    return err, l2


@pytest.mark.gpu
@pytest.mark.parametrize("case", CASES, ids=[c.name for c in CASES])
def test_op_parity_fp32(dev, case):
    got = run_case_dev(dev, case)
    ref = run_case(case)
    assert set(got) == set(ref)
    for name in ref:
        err, l2 = compare(got[name], ref[name])
        assert err <= TOL_MAX and l2 <= TOL_L2, (name, err, l2)


@pytest.mark.gpu
def test_error_is_recorded_not_fatal(dev):
    """A head dimension above OPS_MAX_HEAD_DIM is refused with an error
    (the reference: G_fatal_error at ops.c:453-455), recorded here."""
    X = dev.zeros(16 * 3 * 256)
    O = dev.zeros(16 * 256)
    m = coreg.Opnd(X.handle, 0, 3 * 256, 0, 0)
    dev.lib.ops_attention(dev.ops_p, m, m, m, coreg.Opnd(O.handle, 0, 256, 0, 0), 16, 16, 1,
                          256, 1.0, None)
    with pytest.raises(coreg.CoregError, match="head dimension"):
        coreg.check(dev.lib)
