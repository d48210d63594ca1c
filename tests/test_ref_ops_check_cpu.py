# SPDX-License-Identifier: Unlicense
"""The reference itself, run here: its own generic-op checker
(tests/ops_check.c) with its own ops.c and ops.cl, unchanged, compiled by
oracle/Makefile into oracle/_ref/ops_check_cpu over oracle/cl_backend_emul.c
(its OpenCL runtime over host memory, the kernels compiled as C and run on
the CPU). The test skips when the binary has not been built. CPU only.

The binary writes every case's inputs and the reference's outputs in its
folder format. The inputs must be bit-identical to the oracle's generator
(oracle/ops_cases.py), and the reference's outputs must pass its own rule
(tests/ops_compare.py:26, 257-276: max |diff| / max |ref| <= 2e-5, all
finite) against its torch restatement (tests/golden/ops_golden.npz) and
against the oracle (oracle/ops_ref.py), which the CUDA path is checked
against on the GPU."""

import subprocess
from pathlib import Path

import numpy as np
import pytest

from oracle.ops_cases import build_cases
from oracle.ops_ref import run_case

ROOT = Path(__file__).resolve().parents[1]
BIN = ROOT / "oracle" / "_ref" / "ops_check_cpu"
GOLDEN = ROOT / "tests" / "golden" / "ops_golden.npz"
TOL = 2e-5


@pytest.fixture(scope="module")
def folder(tmp_path_factory):
    if not BIN.exists():
        pytest.skip("oracle/_ref/ops_check_cpu not built (make -C oracle)")
    d = tmp_path_factory.mktemp("ops_check_cpu")
    r = subprocess.run([str(BIN), str(d), "auto"], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    return d


def rule(got, ref):
    assert got.shape == ref.shape and np.isfinite(got).all()
    return float(np.abs(got - ref).max() / max(float(np.abs(ref).max()), 1e-30))


def test_inputs_match_the_oracle_generator(folder):
    for c in build_cases():
        for k, v in c.inputs.items():
            got = np.fromfile(folder / f"{c.name}_{k}.f32", dtype=np.float32)
            assert np.array_equal(got, v.astype(np.float32).reshape(-1)), (c.name, k)


def test_reference_outputs_pass_its_rule_against_its_restatement(folder):
    golden = np.load(GOLDEN)
    assert len(golden.files) == 41
    worst = {}
    for key in golden.files:
        case, out = key.split("/")
        got = np.fromfile(folder / f"{case}_{out}.f32", dtype=np.float32)
        worst[key] = rule(got, golden[key])
    bad = {k: v for k, v in worst.items() if v > TOL}
    assert not bad, bad


def test_oracle_passes_the_rule_against_the_reference(folder):
    worst = {}
    for c in build_cases():
        for name, out in run_case(c).items():
            ref = np.fromfile(folder / f"{c.name}_{name}.f32", dtype=np.float32)
            worst[f"{c.name}/{name}"] = rule(np.asarray(out, np.float64).reshape(-1),
                                             ref.astype(np.float64))
    assert len(worst) == 41
    bad = {k: v for k, v in worst.items() if v > TOL}
    assert not bad, bad
