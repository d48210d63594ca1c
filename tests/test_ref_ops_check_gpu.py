# SPDX-License-Identifier: Unlicense
"""The reference's own generic-op checker, run on this build (GPU).

oracle/_ref/ops_check is the reference's tests/ops_check.c compiled
unchanged against include/ops.h and libcoreg_b200.so (oracle/Makefile). It
writes every case's inputs and the library's outputs in its folder format.
The inputs must be bit-identical to the oracle's generator
(oracle/ops_cases.py), and the outputs must pass the reference's own rule
(tests/ops_compare.py:26 and 257-276: max |diff| / max |ref| <= 2e-5, all
finite) against the outputs of the reference's checker functions committed
in tests/golden/ops_golden.npz."""

import subprocess
from pathlib import Path

import numpy as np
import pytest

from oracle.ops_cases import build_cases

ROOT = Path(__file__).resolve().parents[1]
BIN = ROOT / "oracle" / "_ref" / "ops_check"
GOLDEN = ROOT / "tests" / "golden" / "ops_golden.npz"
TOL = 2e-5


@pytest.fixture(scope="module")
def folder(tmp_path_factory):
    if not BIN.exists():
        pytest.skip("oracle/_ref/ops_check not built (needs the reference checkout)")
    d = tmp_path_factory.mktemp("ops_check")
    r = subprocess.run([str(BIN), str(d), "0"], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    return d


@pytest.mark.gpu
def test_inputs_match_the_oracle_generator(folder):
    for c in build_cases():
        for k, v in c.inputs.items():
            got = np.fromfile(folder / f"{c.name}_{k}.f32", dtype=np.float32)
            assert np.array_equal(got, v.astype(np.float32).reshape(-1)), (c.name, k)


@pytest.mark.gpu
def test_outputs_pass_the_reference_rule(folder):
    golden = np.load(GOLDEN)
    cases = (folder / "cases.txt").read_text().split()
    assert cases
    worst = {}
    for key in golden.files:
        case, out = key.split("/")
        got = np.fromfile(folder / f"{case}_{out}.f32", dtype=np.float32)
        ref = golden[key]
        assert got.shape == ref.shape, (key, got.size, ref.size)
        assert np.isfinite(got).all(), key
        err = float(np.abs(got - ref).max() / max(float(np.abs(ref).max()), 1e-30))
        worst[key] = err
    bad = {k: v for k, v in worst.items() if v > TOL}
    assert not bad, bad
