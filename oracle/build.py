"""Builds the oracle's C restatements into oracle/liboracle.so with gcc.

Test infrastructure only (see oracle/__init__.py).
"""

from __future__ import annotations

import shutil
import subprocess
from pathlib import Path

HERE = Path(__file__).resolve().parent
SOURCES = sorted(HERE.glob("*.c"))
LIB = HERE / "liboracle.so"


def build(force: bool = False) -> Path:
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        raise RuntimeError("gcc is required to build the oracle")
    if not force and LIB.exists() and all(LIB.stat().st_mtime >= s.stat().st_mtime for s in SOURCES):
        return LIB
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [cc, "-O2", "-std=c11", "-fPIC", "-shared", "-Wall", "-o", str(tmp), *map(str, SOURCES)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"oracle build failed:\n{res.stderr}")
    tmp.replace(LIB)
    return LIB


if __name__ == "__main__":
    print(build(force=True))
