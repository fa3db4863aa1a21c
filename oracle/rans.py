"""Oracle wrapper around oracle/rans_oracle.c -- TEST INFRASTRUCTURE ONLY.

Python face of the C restatement of formats/bf16_rans.py (encode :148-177,
decode :180-222), raising the reference's ValueError messages.
"""

from __future__ import annotations

import ctypes
import functools

import numpy as np

from .build import build

_MESSAGES = {
    101: "truncated rANS frame",
    102: "not a vOOM rANS frame",
    103: "truncated rANS tile header",
    104: "truncated rANS tile payload",
    105: "raw rANS tile size mismatch",
    106: "truncated rANS plane header",
    107: "truncated rANS plane payload",
    108: "invalid rANS frequency total",
    109: "rANS plane has trailing renormalization bytes",
    110: "compressed rANS tile has trailing bytes",
    111: "unknown rANS tile mode {mode}",
    112: "rANS tile checksum mismatch",
    113: "rANS frame length mismatch",
}


@functools.lru_cache(maxsize=1)
def _lib() -> ctypes.CDLL:
    lib = ctypes.CDLL(str(build()))
    vp, u64, u32 = ctypes.c_void_p, ctypes.c_uint64, ctypes.c_uint32
    lib.oracle_rans_encode.restype = u64
    lib.oracle_rans_encode.argtypes = [vp, u64, u32, vp, u64, vp]
    lib.oracle_rans_decode.restype = ctypes.c_int
    lib.oracle_rans_decode.argtypes = [vp, u64, vp, u64, ctypes.POINTER(u64), ctypes.POINTER(u32),
                                       ctypes.POINTER(u32)]
    lib.oracle_rans_capacity.restype = u64
    lib.oracle_rans_capacity.argtypes = [vp, u64]
    lib.oracle_crc32.restype = u32
    lib.oracle_crc32.argtypes = [vp, u64]
    return lib


def _u8(buf) -> np.ndarray:
    return np.ascontiguousarray(np.frombuffer(buf, dtype=np.uint8) if not isinstance(buf, np.ndarray)
                                else buf.reshape(-1).view(np.uint8))


def crc32(data) -> int:
    a = _u8(data)
    return int(_lib().oracle_crc32(a.ctypes.data, a.size))


def encode(data, *, tile_bytes: int = 1 << 20) -> tuple[bytes, dict]:
    if tile_bytes <= 0:
        raise ValueError("rANS tile_bytes must be positive")
    a = _u8(data)
    tiles = (a.size + tile_bytes - 1) // tile_bytes
    cap = 16 + 13 * tiles + a.size + 2 * 1040 + 64
    out = np.empty(cap, dtype=np.uint8)
    stats = np.zeros(2, dtype=np.uint64)
    n = _lib().oracle_rans_encode(a.ctypes.data, a.size, tile_bytes, out.ctypes.data, cap, stats.ctypes.data)
    if n == 0:
        raise RuntimeError("oracle rANS encode failed")
    return out[:n].tobytes(), {"tiles": int(stats[0]), "compressed_tiles": int(stats[1])}


def decode_status(frame) -> tuple[int, bytes, int, int]:
    """(status, decoded bytes, failing tile, bad mode) without raising."""
    a = _u8(frame)
    lib = _lib()
    cap = int(lib.oracle_rans_capacity(a.ctypes.data, a.size))
    out = np.empty(max(cap, 1), dtype=np.uint8)
    n = ctypes.c_uint64(0)
    tile = ctypes.c_uint32(0)
    mode = ctypes.c_uint32(0)
    rc = lib.oracle_rans_decode(a.ctypes.data, a.size, out.ctypes.data, cap, ctypes.byref(n),
                                ctypes.byref(tile), ctypes.byref(mode))
    return rc, out[: n.value].tobytes(), tile.value, mode.value


def decode(frame) -> bytes:
    rc, data, _tile, mode = decode_status(frame)
    if rc:
        raise ValueError(_MESSAGES.get(rc, f"status {rc}").format(mode=mode))
    return data


def message(rc: int, mode: int = 0) -> str:
    return _MESSAGES[rc].format(mode=mode)
