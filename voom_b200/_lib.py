"""ctypes binding of libvoom_b200.so (the C ABI declared in include/voom_b200.h).

The library is the only compute path: if it is missing or CUDA is not
available the callers raise; there is no CPU fallback.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

import numpy as np

LIB_PATH = Path(__file__).resolve().with_name("libvoom_b200.so")

# ---------------------------------------------------------------- status codes
VOOM_OK = 0
VOOM_E_INVALID_ARG = -1
VOOM_E_CUDA = -2
VOOM_E_CAPACITY = -3
VOOM_E_UNSUPPORTED = -4

RANS_MESSAGES = {
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

# ------------------------------------------------------------------ structs
# voom_rans_tile (56 bytes, no padding)
RANS_TILE_DTYPE = np.dtype([
    ("src", "<u8"), ("dst", "<u8"), ("low_freq", "<u8"), ("high_freq", "<u8"),
    ("low_payload", "<u4"), ("high_payload", "<u4"), ("raw_len", "<u4"),
    ("crc32", "<u4"), ("mode", "<u4"), ("flags", "<u4"),
])
assert RANS_TILE_DTYPE.itemsize == 56

RANS_CHUNK_DTYPE = np.dtype([("tile", "<u4"), ("seg_begin", "<u4"), ("seg_end", "<u4"), ("n_in_tile", "<u4")])


# MoE families (VOOM_MOE_*) and voom_moe_variant
MOE_FAMILIES = {"generic": 0, "qwen35": 1, "glm": 2}


class MoeVariant(ctypes.Structure):
    _fields_ = [
        ("family", ctypes.c_uint32),
        ("norm_topk", ctypes.c_uint32),
        ("routed_scale", ctypes.c_float),
        ("shared_expert", ctypes.c_int32),
        ("d_shared_gate_w", ctypes.c_void_p),
        ("d_router_bias", ctypes.c_void_p),
    ]


class MoeEp(ctypes.Structure):
    _fields_ = [
        ("d_holders", ctypes.c_void_p),
        ("rank", ctypes.c_uint32),
        ("world", ctypes.c_uint32),
        ("t_pad", ctypes.c_uint32),
    ]


class RansPlanInfo(ctypes.Structure):
    _fields_ = [
        ("raw_size", ctypes.c_uint64),
        ("out_bytes", ctypes.c_uint64),
        ("tile_bytes", ctypes.c_uint32),
        ("tile_count", ctypes.c_uint32),
        ("n_tiles", ctypes.c_uint32),
        ("struct_error", ctypes.c_int32),
        ("struct_tile", ctypes.c_uint32),
        ("struct_ordinal", ctypes.c_uint32),
        ("bad_mode", ctypes.c_uint32),
        ("frame_end", ctypes.c_uint32),
    ]


_c_u8p = ctypes.c_void_p
_u64 = ctypes.c_uint64
_u32 = ctypes.c_uint32
_i32 = ctypes.c_int
_vp = ctypes.c_void_p

# name -> (restype, argtypes)
SIGNATURES: dict[str, tuple] = {
    "voom_rans_plan": (_i32, [_vp, _u64, _u64, _u64, _vp, _u32, ctypes.POINTER(RansPlanInfo)]),
    "voom_rans_decode": (_i32, [_vp, _vp, _u32, _vp, _vp, _vp, _vp, _u32, _vp]),
    "voom_rans_decode_indexed": (_i32, [_vp, _vp, _vp, _u32, _vp, _vp, _vp, _vp, _u32, _vp, _vp]),
    "voom_rans_chunks": (_i32, [_vp, _u32, _u32, _vp, _u32, ctypes.POINTER(_u32)]),
    "voom_rans_ckpt_words": (_u64, [_u32, _u32]),
    "voom_rans_resolve": (_i32, [ctypes.POINTER(RansPlanInfo), _vp, _u32, ctypes.POINTER(_u32)]),
    "voom_rans_encode": (_i32, [_vp, _u64, _u32, _vp, _u64, ctypes.POINTER(_u64), _vp, _i32]),
    "voom_zstd_plan_create": (_vp, [_vp, _u64, _vp, _u32, _i32]),
    "voom_zstd_plan_info_get": (_i32, [_vp, _vp]),
    "voom_zstd_plan_image": (_i32, [_vp, _vp, _u64]),
    "voom_zstd_plan_job_status": (_i32, [_vp, _vp]),
    "voom_zstd_plan_destroy": (None, [_vp]),
    "voom_zstd_decode": (_i32, [_vp, _vp, _vp, _vp, _vp, _vp, _vp]),
    "voom_kvz_gather": (_i32, [_vp, _vp, _vp, _u32, _vp, _vp, _i32]),
    "voom_zstd_set_timing": (_i32, [_i32]),
    "voom_copy_from_host": (_i32, [_vp, _vp, _u64, _vp]),
    "voom_zstd_encode_slot_bytes": (_u64, []),
    "voom_zstd_encode_block_bytes": (_u32, []),
    "voom_zstd_encode": (_i32, [_vp, _vp, _u32, _vp, _vp, _vp]),
    "voom_zstd_encode_pack": (_i32, [_vp, _vp, _vp, _u32, _vp, _vp]),
    "voom_zstd_kernel_times": (_i32, [_vp, _vp, _i32]),
    "voom_moe_scratch_bytes": (_u64, [_u32, _u32, _u32, _u32]),
    "voom_moe_layer": (_i32, [_vp, _u32, _vp, _vp, ctypes.c_float, _vp, _vp, _u32, _u32, _u32, _u32, _u32, _u32,
                              _u32, _u32, _vp, _u64, _vp, _vp]),
    "voom_moe_experts": (_i32, [_vp, _u32, _vp, _vp, _vp, ctypes.c_float, _vp, _u32, _u32, _u32, _u32, _u32, _u32,
                                _u32, _vp, _vp, _u64, _vp, _vp]),
    "voom_moe_combine": (_i32, [_vp, _vp, _vp, _vp, _u32, _u32, _u32, _vp]),
    "voom_moe_scratch_bytes_v": (_u64, [_vp, _u32, _u32, _u32, _u32]),
    "voom_moe_layer_v": (_i32, [_vp, _vp, _u32, _vp, _vp, ctypes.c_float, _vp, _vp, _u32, _u32, _u32, _u32, _u32,
                                _u32, _u32, _vp, _u64, _vp, _vp]),
    "voom_moe_experts_v": (_i32, [_vp, _vp, _u32, _vp, _vp, ctypes.c_float, _vp, _u32, _u32, _u32, _u32, _u32,
                                  _u32, _vp, _vp, _u64, _vp, _vp]),
    "voom_moe_experts_ep": (_i32, [_vp, _vp, _vp, _u32, _vp, _vp, ctypes.c_float, _vp, _u32, _u32, _u32, _u32,
                                   _u32, _u32, _vp, _vp, _u64, _vp, _vp]),
    "voom_moe_combine_tm": (_i32, [_vp, _vp, _vp, _vp, _u32, _u32, _u32, _u32, _vp]),
    "voom_moe_layer_noalloc": (_i32, [_vp, _u32, _vp, _vp, ctypes.c_float, _vp, _vp, _u32, _u32, _u32, _u32, _u32,
                                      _u32, _u32, _u32, _vp, _vp]),
    "voom_nf12_decode": (_i32, [_vp, _u64, _u64, _u32, _u32, _u64, _vp, _u64, _vp, _vp]),
    "voom_nf12_linear_scratch_bytes": (_u64, [_u32, _u32, _u32]),
    "voom_nf12_linear": (_i32, [_vp, _u32, _u32, _u32, _vp, _u64, _u64, _u32, _vp, _u64, _vp, _vp, _vp]),
    "voom_nf12_linear_batch_scratch_bytes": (_u64, [_vp, _u32, _u32]),
    "voom_nf12_linear_batch": (_i32, [_vp, _u32, _u32, _vp, _u64, _u64, _vp, _u64, _vp, _vp]),
    "voom_expert_swiglu": (_i32, [_vp, _vp, _u32, _vp, _vp, _u32, _u32, _vp, _u32, _u32, _u32, _u32, _vp, _vp,
                                  _u64, _vp, _vp]),
}

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


class VoomError(RuntimeError):
    """A C-ABI call failed for a reason that is not a format error."""


def load() -> ctypes.CDLL:
    """Load libvoom_b200.so once; raise if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise VoomError(
                    f"{LIB_PATH.name} is not built; run `python -m voom_b200.build` "
                    "(or __graft_entry__.build()) first")
            lib = ctypes.CDLL(str(LIB_PATH))
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


def check(rc: int, what: str) -> None:
    if rc == VOOM_OK:
        return
    names = {VOOM_E_INVALID_ARG: "invalid argument", VOOM_E_CUDA: "CUDA launch/runtime failure",
             VOOM_E_CAPACITY: "capacity exceeded", VOOM_E_UNSUPPORTED: "unsupported input"}
    raise VoomError(f"{what} failed: {names.get(rc, rc)}")


def exported_symbols() -> list[str]:
    return list(SIGNATURES)
