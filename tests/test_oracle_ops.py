# SPDX-License-Identifier: Unlicense
"""The ops oracle against the reference's own checker (CPU).

tests/golden/ops_golden.npz holds the outputs of the reference's
tests/ops_compare.py (torch float64, rounded to float32) on the inputs of
the reference's tests/ops_check.c cases; oracle/ops_ref.py restates the
kernels independently in numpy. Agreement to float32 rounding pins the
oracle used by the GPU parity tests.
"""

from pathlib import Path

import numpy as np
import pytest

from oracle.ops_cases import build_cases
from oracle.ops_ref import run_case

GOLDEN = Path(__file__).resolve().parent / "golden" / "ops_golden.npz"
CASES = build_cases()


@pytest.fixture(scope="module")
def golden():
    return np.load(GOLDEN)


def test_case_list_matches_reference_producer():
    # ops_check.c:448-487: 36 cases, 41 outputs (elementwise has 6).
    assert len(CASES) == 36
    names = [c.name for c in CASES]
    assert names[0] == "gemm_small_nt" and names[-1] == "fold_bn"
    assert len(set(names)) == len(names)


def test_generator_is_ops_check_xorshift():
    # First draw of xorshift64 from seed 88172645463325252, mapped to
    # -1..1 in float32 arithmetic (ops_check.c:37-43).
    from oracle.ops_cases import XorShift

    s = 88172645463325252
    M = (1 << 64) - 1
    s ^= (s << 13) & M
    s ^= s >> 7
    s ^= (s << 17) & M
    u = np.float32((s >> 11) * (1.0 / 9007199254740992.0))
    want = np.float32(-1) + np.float32(2) * u
    assert XorShift().rand(1, -1, 1)[0] == want


@pytest.mark.parametrize("case", CASES, ids=[c.name for c in CASES])
def test_oracle_matches_reference_checker(case, golden):
    for name, ref in run_case(case).items():
        want = golden[f"{case.name}/{name}"].astype(np.float64)
        got = np.asarray(ref, np.float64).reshape(-1)
        assert got.shape == want.shape
        scale = max(np.abs(want).max(), 1e-30)
        assert np.abs(got - want).max() / scale <= 1e-6, name
