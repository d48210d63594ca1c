# SPDX-License-Identifier: Unlicense
"""Every public header of the C-ABI (include/*.h) compiles as plain C11 on
its own, as the reference's C callers include it (CPU; gcc only)."""

import shutil
import subprocess
from pathlib import Path

import pytest

INCLUDE = Path(__file__).resolve().parents[1] / "include"
HEADERS = sorted(p.name for p in INCLUDE.glob("*.h"))


@pytest.mark.parametrize("header", HEADERS)
def test_header_compiles_as_c(header):
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    src = f'#include "{header}"\n#include "{header}"\nint main(void) {{ return 0; }}\n'
    r = subprocess.run([cc, "-std=gnu11", "-Wall", "-Werror", "-fsyntax-only",
                        f"-I{INCLUDE}", "-x", "c", "-"], input=src, text=True,
                       capture_output=True)
    assert r.returncode == 0, r.stderr
