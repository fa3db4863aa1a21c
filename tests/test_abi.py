"""The C-ABI library loads without a GPU and exports every function that
include/*.h declares (no compute calls here)."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def declared_functions() -> set[str]:
    names = set()
    for h in (ROOT / "include").glob("*.h"):
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        for m in re.finditer(r"\b(voom_[a-z0-9_]+)\s*\(", text):
            names.add(m.group(1))
    return names


def test_library_exports_every_declared_symbol(built_lib):
    declared = declared_functions()
    assert declared, "no declarations found"
    lib = ctypes.CDLL(str(ROOT / "voom_b200" / "libvoom_b200.so"))
    missing = [n for n in sorted(declared) if not hasattr(lib, n)]
    assert not missing, missing


def test_python_binding_covers_header(built_lib):
    from voom_b200 import _lib

    assert declared_functions() == set(_lib.exported_symbols())


def test_build_entry_compiles_for_sm100a():
    from voom_b200 import build

    assert "arch=compute_100a,code=sm_100a" in " ".join(build.ARCH_FLAGS)
