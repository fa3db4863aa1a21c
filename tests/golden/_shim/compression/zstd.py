"""compress / decompress / ZstdCompressor / ZstdDecompressor over libzstd
(ctypes) -- only for running the reference in make_golden.py."""

import ctypes
import ctypes.util

_lib = ctypes.CDLL(ctypes.util.find_library("zstd") or "libzstd.so.1")
_sz, _vp = ctypes.c_size_t, ctypes.c_void_p
_lib.ZSTD_compressBound.restype = _sz
_lib.ZSTD_compressBound.argtypes = [_sz]
_lib.ZSTD_compress.restype = _sz
_lib.ZSTD_compress.argtypes = [_vp, _sz, _vp, _sz, ctypes.c_int]
_lib.ZSTD_isError.restype = ctypes.c_uint
_lib.ZSTD_isError.argtypes = [_sz]
_lib.ZSTD_createCCtx.restype = _vp
_lib.ZSTD_CCtx_setParameter.argtypes = [_vp, ctypes.c_int, ctypes.c_int]
_lib.ZSTD_createDCtx.restype = _vp


class _In(ctypes.Structure):
    _fields_ = [("src", _vp), ("size", _sz), ("pos", _sz)]


class _Out(ctypes.Structure):
    _fields_ = [("dst", _vp), ("size", _sz), ("pos", _sz)]


_lib.ZSTD_compressStream2.restype = _sz
_lib.ZSTD_compressStream2.argtypes = [_vp, ctypes.POINTER(_Out), ctypes.POINTER(_In), ctypes.c_int]
_lib.ZSTD_decompressStream.restype = _sz
_lib.ZSTD_decompressStream.argtypes = [_vp, ctypes.POINTER(_Out), ctypes.POINTER(_In)]


class ZstdError(Exception):
    pass


def compress(data, level=3):
    data = bytes(data)
    cap = _lib.ZSTD_compressBound(len(data))
    out = ctypes.create_string_buffer(max(cap, 1))
    r = _lib.ZSTD_compress(out, cap, data, len(data), level)
    if _lib.ZSTD_isError(r):
        raise ZstdError("compress")
    return out.raw[:r]


def _stream(ctx, fn, data, mode=None):
    data = bytes(data)
    src = ctypes.create_string_buffer(data, len(data)) if data else None
    inb = _In(ctypes.cast(src, _vp) if src is not None else None, len(data), 0)
    chunk = 1 << 17
    buf = ctypes.create_string_buffer(chunk)
    parts = []
    while True:
        ob = _Out(ctypes.cast(buf, _vp), chunk, 0)
        r = fn(ctx, ctypes.byref(ob), ctypes.byref(inb)) if mode is None else fn(ctx, ctypes.byref(ob), ctypes.byref(inb), mode)
        if _lib.ZSTD_isError(r):
            raise ZstdError("stream")
        parts.append(buf.raw[: ob.pos])
        if mode == 2:
            if r == 0:
                break
        elif inb.pos == inb.size and ob.pos < chunk:
            break
    return b"".join(parts)


def decompress(data):
    return ZstdDecompressor().decompress(data)


class ZstdCompressor:
    def __init__(self, level=3):
        self.ctx = _lib.ZSTD_createCCtx()
        _lib.ZSTD_CCtx_setParameter(self.ctx, 100, level)

    def compress(self, data):
        return _stream(self.ctx, _lib.ZSTD_compressStream2, data, 0)

    def flush(self):
        return _stream(self.ctx, _lib.ZSTD_compressStream2, b"", 2)


class ZstdDecompressor:
    def __init__(self):
        self.ctx = _lib.ZSTD_createDCtx()

    def decompress(self, data):
        return _stream(self.ctx, _lib.ZSTD_decompressStream, data)
