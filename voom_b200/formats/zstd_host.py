"""Pack-side zstd compression through the system libzstd (ctypes).

The reference compresses vpack hi planes and kv_paged pages with
`compression.zstd` (libzstd): `compress(data, level)` (formats/packed.py:48,
278; runtime/kv_paged.py:82-83) and a streaming `ZstdCompressor` for tensors
above 256 MiB (formats/packed.py:63-81).  This module provides the same two
calls for the pack side.  Decompression is never done here: every decode goes
through the GPU path.
"""

from __future__ import annotations

import ctypes
import ctypes.util
import functools

import numpy as np

ZSTD_e_continue = 0
ZSTD_e_flush = 1
ZSTD_e_end = 2
ZSTD_c_compressionLevel = 100
ZSTD_c_checksumFlag = 201


class ZstdError(Exception):
    pass


class _InBuf(ctypes.Structure):
    _fields_ = [("src", ctypes.c_void_p), ("size", ctypes.c_size_t), ("pos", ctypes.c_size_t)]


class _OutBuf(ctypes.Structure):
    _fields_ = [("dst", ctypes.c_void_p), ("size", ctypes.c_size_t), ("pos", ctypes.c_size_t)]


@functools.lru_cache(maxsize=1)
def _lib() -> ctypes.CDLL:
    name = ctypes.util.find_library("zstd") or "libzstd.so.1"
    lib = ctypes.CDLL(name)
    vp, sz = ctypes.c_void_p, ctypes.c_size_t
    lib.ZSTD_compress.restype = sz
    lib.ZSTD_compress.argtypes = [vp, sz, vp, sz, ctypes.c_int]
    lib.ZSTD_compressBound.restype = sz
    lib.ZSTD_compressBound.argtypes = [sz]
    lib.ZSTD_isError.restype = ctypes.c_uint
    lib.ZSTD_isError.argtypes = [sz]
    lib.ZSTD_createCCtx.restype = vp
    lib.ZSTD_freeCCtx.argtypes = [vp]
    lib.ZSTD_CCtx_setParameter.restype = sz
    lib.ZSTD_CCtx_setParameter.argtypes = [vp, ctypes.c_int, ctypes.c_int]
    lib.ZSTD_compressStream2.restype = sz
    lib.ZSTD_compressStream2.argtypes = [vp, ctypes.POINTER(_OutBuf), ctypes.POINTER(_InBuf), ctypes.c_int]
    lib.ZSTD_CStreamOutSize.restype = sz
    return lib


def _u8(b) -> np.ndarray:
    return np.ascontiguousarray(np.frombuffer(b, np.uint8) if not isinstance(b, np.ndarray) else b.view(np.uint8).reshape(-1))


def compress(data, level: int = 1) -> bytes:
    """One-shot frame (content size recorded, no checksum): compression.zstd.compress."""
    lib = _lib()
    a = _u8(data)
    cap = lib.ZSTD_compressBound(a.size)
    out = np.empty(max(cap, 1), np.uint8)
    r = lib.ZSTD_compress(out.ctypes.data, cap, a.ctypes.data, a.size, int(level))
    if lib.ZSTD_isError(r):
        raise ZstdError("ZSTD_compress failed")
    return out[:r].tobytes()


class ZstdCompressor:
    """Streaming compressor: compress() chunks then flush() ends the frame
    (the content size is not recorded, as in the reference's streamed pack)."""

    def __init__(self, level: int = 1, checksum: bool = False):
        self._lib = _lib()
        self._cctx = self._lib.ZSTD_createCCtx()
        self._lib.ZSTD_CCtx_setParameter(self._cctx, ZSTD_c_compressionLevel, int(level))
        if checksum:
            self._lib.ZSTD_CCtx_setParameter(self._cctx, ZSTD_c_checksumFlag, 1)
        self._outsz = self._lib.ZSTD_CStreamOutSize()

    def _run(self, data, mode: int) -> bytes:
        a = _u8(data)
        inb = _InBuf(a.ctypes.data if a.size else None, a.size, 0)
        out = np.empty(self._outsz, np.uint8)
        parts = []
        while True:
            ob = _OutBuf(out.ctypes.data, self._outsz, 0)
            r = self._lib.ZSTD_compressStream2(self._cctx, ctypes.byref(ob), ctypes.byref(inb), mode)
            if self._lib.ZSTD_isError(r):
                raise ZstdError("ZSTD_compressStream2 failed")
            parts.append(out[: ob.pos].tobytes())
            if mode == ZSTD_e_continue and inb.pos == inb.size:
                break
            if mode == ZSTD_e_end and r == 0:
                break
        return b"".join(parts)

    def compress(self, data) -> bytes:
        return self._run(data, ZSTD_e_continue)

    def flush(self) -> bytes:
        return self._run(b"", ZSTD_e_end)

    def __del__(self):
        try:
            self._lib.ZSTD_freeCCtx(self._cctx)
        except Exception:
            pass
