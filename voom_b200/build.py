"""Builds libvoom_b200.so (every CUDA/C++ source under csrc/) for sm_100a.

The library is built in-tree next to this file so it travels with the
repository snapshot; nothing is installed into site-packages.  Objects are
compiled in parallel and only when a source or header is newer than the
library.
"""

from __future__ import annotations

import os
import shutil
import subprocess
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = ROOT / "include"
BUILD_DIR = PKG / "_build"
LIB_PATH = PKG / "libvoom_b200.so"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-fvisibility=hidden,-O3",
                "-I", str(INCLUDE), "--expt-relaxed-constexpr"]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: the CUDA toolkit is required to build voom_b200")


def _sources() -> list[Path]:
    return sorted(list(CSRC.glob("*.cu")) + list(CSRC.glob("*.cpp")))


def _headers() -> list[Path]:
    return sorted(list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list(INCLUDE.glob("*.h")))


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def build_hostbuf(verbose: bool = False, force: bool = False) -> Path:
    """The small CPython extension of pyext/hostbuf.c (buffer addresses for
    the KV page gather), built with the host C compiler next to this file."""
    import sysconfig

    src = PKG / "pyext" / "hostbuf.c"
    out = PKG / ("_hostbuf" + sysconfig.get_config_var("EXT_SUFFIX"))
    if force or _stale(out, [src]):
        cc = os.environ.get("CC") or shutil.which("gcc") or "cc"
        cmd = [cc, "-O2", "-shared", "-fPIC", "-I", sysconfig.get_paths()["include"], str(src), "-o", str(out)]
        if verbose:
            print(" ".join(cmd), flush=True)
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"building _hostbuf failed:\n{res.stdout}\n{res.stderr}")
    return out


def build(verbose: bool = False, force: bool = False, extra_flags: list[str] | None = None) -> Path:
    """Compile every source under csrc/ and link libvoom_b200.so (and the
    _hostbuf extension); return the library's path."""
    build_hostbuf(verbose, force)
    nvcc = _nvcc()
    BUILD_DIR.mkdir(exist_ok=True)
    srcs = _sources()
    headers = _headers()
    extra = list(extra_flags or [])

    def compile_one(src: Path) -> Path:
        obj = BUILD_DIR / (src.name + ".o")
        if force or _stale(obj, [src, *headers]):
            cmd = [nvcc, *ARCH_FLAGS, *COMMON_FLAGS, *extra, "-c", str(src), "-o", str(obj)]
            if verbose:
                print(" ".join(cmd), flush=True)
            res = subprocess.run(cmd, capture_output=True, text=True)
            if res.returncode != 0:
                raise RuntimeError(f"nvcc failed on {src.name}:\n{res.stdout}\n{res.stderr}")
            if verbose and res.stderr.strip():
                print(res.stderr, flush=True)
        return obj

    with ThreadPoolExecutor(max_workers=min(8, len(srcs))) as pool:
        objs = list(pool.map(compile_one, srcs))
    if force or _stale(LIB_PATH, objs):
        tmp = LIB_PATH.with_suffix(".so.tmp")
        cmd = [nvcc, *ARCH_FLAGS, "-shared", "-o", str(tmp), *map(str, objs), "-lpthread"]
        if verbose:
            print(" ".join(cmd), flush=True)
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
        os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    import sys

    print(build(verbose=True, force="--force" in sys.argv))
