"""Oracle for vpack / vpack2 body decode -- TEST INFRASTRUCTURE ONLY.

Restates formats/packed2.py:178-191 (decode_body) and formats/packed.py:
361-379 (read_tensor_bytes): `hi = zstd.decompress(...)` through libzstd (the
library behind the reference's compression.zstd), `raw[0::2] = lo`,
`raw[1::2] = hi` with numpy.  Also the kv_paged compressed page codec
(runtime/kv_paged.py:56-61, 77-113): pickle of {"shape", "k", "v"} with
zstd level-1 frames of the raw BF16 bytes.
"""

from __future__ import annotations

import ctypes
import ctypes.util
import functools
import pickle

import numpy as np

from .zstd import ZstdError, libzstd_decompress


@functools.lru_cache(maxsize=1)
def _zlib():
    lib = ctypes.CDLL(ctypes.util.find_library("zstd") or "libzstd.so.1")
    lib.ZSTD_compress.restype = ctypes.c_size_t
    lib.ZSTD_compress.argtypes = [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int]
    lib.ZSTD_compressBound.restype = ctypes.c_size_t
    lib.ZSTD_compressBound.argtypes = [ctypes.c_size_t]
    lib.ZSTD_isError.restype = ctypes.c_uint
    lib.ZSTD_isError.argtypes = [ctypes.c_size_t]
    return lib


def zstd_compress(data, level: int = 1) -> bytes:
    a = np.ascontiguousarray(np.frombuffer(data, np.uint8))
    lib = _zlib()
    cap = lib.ZSTD_compressBound(a.size)
    out = np.empty(max(cap, 1), np.uint8)
    r = lib.ZSTD_compress(out.ctypes.data, cap, a.ctypes.data, a.size, level)
    if lib.ZSTD_isError(r):
        raise ZstdError("compress failed")
    return out[:r].tobytes()


def decode_body(head: dict, body) -> np.ndarray:
    """formats/packed2.py:178-191 restated: uint8 array of the original bytes."""
    body = memoryview(body)
    if "raw" in head:
        return np.frombuffer(body, np.uint8)
    if head.get("streamed"):
        lo = body[: head["lo"]]
        hi = libzstd_decompress(body[head["lo"]:], head["lo"])
    else:
        hi = libzstd_decompress(body[: head["hi_z"]], head["lo"])
        lo = body[head["hi_z"]:]
    raw = np.empty(len(hi) * 2, dtype=np.uint8)
    raw[0::2] = np.frombuffer(lo, dtype=np.uint8)
    raw[1::2] = np.frombuffer(hi, dtype=np.uint8)
    return raw


def kv_spill(k_bits: np.ndarray, v_bits: np.ndarray) -> bytes:
    """runtime/kv_paged.py:77-91 restated: the bytes of a compressed .kvz page."""
    shape = tuple(int(x) for x in k_bits.shape)
    return pickle.dumps({"shape": shape, "k": zstd_compress(np.ascontiguousarray(k_bits).tobytes(), 1),
                         "v": zstd_compress(np.ascontiguousarray(v_bits).tobytes(), 1)})


def kv_load(blob: bytes) -> tuple[np.ndarray, np.ndarray]:
    """runtime/kv_paged.py:98-113 restated: (K, V) as uint16 BF16 bit arrays."""
    d = pickle.loads(blob)
    n = int(np.prod(d["shape"])) * 2
    k = np.frombuffer(libzstd_decompress(d["k"], n), np.uint16).reshape(d["shape"])
    v = np.frombuffer(libzstd_decompress(d["v"], n), np.uint16).reshape(d["shape"])
    return k, v
