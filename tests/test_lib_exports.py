# SPDX-License-Identifier: Unlicense
"""The C-ABI library loads without a GPU and exports every function that
include/*.h declares (CPU; no compute call)."""

import ctypes
import re
from pathlib import Path

import coreg

INCLUDE = Path(__file__).resolve().parents[1] / "include"
DECL = re.compile(r"^[A-Za-z_][\w \*]*?\b(\w+)\s*\(", re.M)


def declared():
    names = set()
    for h in INCLUDE.glob("*.h"):
        text = h.read_text()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        text = re.sub(r"^\s*#.*$", "", text, flags=re.M)
        for m in DECL.finditer(text):
            line = text[m.start():text.find(";", m.start()) + 1]
            if "(" in line and line.rstrip().endswith(");") and "typedef" not in line \
                    and "(*" not in line and not line.lstrip().startswith(("struct", "union")):
                names.add(m.group(1))
    return names


def test_library_loads():
    lib = coreg.load()
    assert lib is not None


def test_every_declared_symbol_is_exported():
    lib = ctypes.CDLL(str(coreg.LIB_PATH))
    names = declared()
    assert "ops_gemm" in names and "ocl_init" in names
    missing = [n for n in sorted(names) if not hasattr(lib, n)]
    assert not missing, missing


def test_binding_declares_only_exported_symbols():
    lib = ctypes.CDLL(str(coreg.LIB_PATH))
    for name in coreg.SIGNATURES:
        assert hasattr(lib, name), name
