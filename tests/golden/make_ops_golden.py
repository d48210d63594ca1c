# SPDX-License-Identifier: Unlicense
"""Generate tests/golden/ops_golden.npz from the reference's own checker.

Writes the inputs of every case of oracle/ops_cases.py (the reference's
tests/ops_check.c cases and generator) in the folder format that
ops_check.c produces, then runs the reference's tests/ops_compare.py
reference functions (torch float64) on them and stores their outputs as
float32. Needs the reference checkout ($COREG_REFERENCE, else `reference` beside
this repository's folder) and torch; run from the repository root:

    python tests/golden/make_ops_golden.py
"""

import importlib.util
import os
import sys
import tempfile
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

from oracle.ops_cases import build_cases, rope_table  # noqa: E402


def main():
    ref = Path(os.environ.get("COREG_REFERENCE", ROOT.parent / "reference"))
    spec = importlib.util.spec_from_file_location("ops_compare", ref / "tests" / "ops_compare.py")
    oc = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(oc)
    out = {}
    with tempfile.TemporaryDirectory() as d:
        d = Path(d)
        lines = []
        for c in build_cases():
            for k, v in c.inputs.items():
                v.astype(np.float32).tofile(d / f"{c.name}_{k}.f32")
            params = " ".join(f"{k}={v!r}" for k, v in c.p.items())
            lines.append(f"{c.name} op={c.op} {params}")
        for line in lines:
            case = oc.Case(d, line)
            for name, val in oc.REFS[case["op"]](case).items():
                out[f"{case.name}/{name}"] = val.reshape(-1).numpy().astype(np.float32)
    dst = ROOT / "tests" / "golden" / "ops_golden.npz"
    np.savez_compressed(dst, **out)
    print(f"{len(out)} outputs -> {dst} ({dst.stat().st_size} bytes)")


if __name__ == "__main__":
    main()
