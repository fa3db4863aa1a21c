"""Oracle wrapper around oracle/zstd_oracle.c -- TEST INFRASTRUCTURE ONLY.

`decompress` is the C restatement of the RFC 8878 decoder; `libzstd_decompress`
calls the system libzstd (the library behind the reference's
`compression.zstd`), used to pin the restatement.
"""

from __future__ import annotations

import ctypes
import ctypes.util
import functools

import numpy as np

from .build import build


class ZstdError(Exception):
    """Decoding failed (mirrors compression.zstd.ZstdError)."""


@functools.lru_cache(maxsize=1)
def _lib() -> ctypes.CDLL:
    lib = ctypes.CDLL(str(build()))
    vp, sz = ctypes.c_void_p, ctypes.c_size_t
    lib.oracle_zstd_decompress.restype = ctypes.c_int
    lib.oracle_zstd_decompress.argtypes = [vp, sz, vp, sz, ctypes.POINTER(sz)]
    lib.oracle_xxh64.restype = ctypes.c_uint64
    lib.oracle_xxh64.argtypes = [vp, sz, ctypes.c_uint64]
    return lib


@functools.lru_cache(maxsize=1)
def _zstd() -> ctypes.CDLL:
    name = ctypes.util.find_library("zstd") or "libzstd.so.1"
    lib = ctypes.CDLL(name)
    vp, sz = ctypes.c_void_p, ctypes.c_size_t
    lib.ZSTD_decompress.restype = sz
    lib.ZSTD_decompress.argtypes = [vp, sz, vp, sz]
    lib.ZSTD_isError.restype = ctypes.c_uint
    lib.ZSTD_isError.argtypes = [sz]
    lib.ZSTD_getFrameContentSize.restype = ctypes.c_ulonglong
    lib.ZSTD_getFrameContentSize.argtypes = [vp, sz]
    lib.ZSTD_versionNumber.restype = ctypes.c_uint
    return lib


def libzstd_version() -> str:
    v = _zstd().ZSTD_versionNumber()
    return f"{v // 10000}.{v // 100 % 100}.{v % 100}"


def _u8(b) -> np.ndarray:
    return np.ascontiguousarray(np.frombuffer(b, np.uint8) if not isinstance(b, np.ndarray) else b.view(np.uint8).reshape(-1))


def decompress(data, capacity: int | None = None) -> bytes:
    a = _u8(data)
    cap = capacity if capacity is not None else max(1 << 20, 64 * a.size + 4096)
    out = np.empty(max(cap, 1), np.uint8)
    n = ctypes.c_size_t(0)
    if _lib().oracle_zstd_decompress(a.ctypes.data, a.size, out.ctypes.data, cap, ctypes.byref(n)):
        raise ZstdError("zstd frame decode failed")
    return out[: n.value].tobytes()


def libzstd_decompress(data, capacity: int) -> bytes:
    a = _u8(data)
    out = np.empty(max(capacity, 1), np.uint8)
    r = _zstd().ZSTD_decompress(out.ctypes.data, capacity, a.ctypes.data, a.size)
    if _zstd().ZSTD_isError(r):
        raise ZstdError("libzstd decode failed")
    return out[:r].tobytes()


def xxh64(data, seed: int = 0) -> int:
    a = _u8(data)
    return int(_lib().oracle_xxh64(a.ctypes.data, a.size, seed))
