"""GPU drop-in for vOOM's exact tile-local BF16 rANS codec (formats/bf16_rans.py).

Same frame format, same API (`encode`, `decode`, the `_FRAME`/`_TILE`/`_PLANE`/
`_FREQUENCIES` structs, `RANSFrameStats`) and the same ValueError messages, in
the order the reference raises them.  `decode` runs on the GPU through
libvoom_b200 (header walk on the host, symbol decode + plane interleave +
CRC-32 on the device); `decode_device` returns the decoded bytes as a CUDA
uint8 tensor without the device->host copy.  `RansPage` keeps a frame
resident in HBM with a checkpoint index so every later decode runs all
checkpoint segments in parallel.

Reference interface replaced: formats/bf16_rans.py:148-222.
"""

from __future__ import annotations

import ctypes
import struct
from dataclasses import dataclass

import numpy as np
import torch

from .. import _device
from .._lib import RANS_CHUNK_DTYPE, RANS_MESSAGES, RANS_TILE_DTYPE, RansPlanInfo, VoomError, check, load

_MAGIC = b"VRN1"
_SCALE_BITS = 12
_TOTAL = 1 << _SCALE_BITS
_RANS_L = 1 << 23
_FRAME = struct.Struct("<4sIII")
_TILE = struct.Struct("<BIII")
_PLANE = struct.Struct("<I")
_FREQUENCIES = struct.Struct("<256H")

DEFAULT_CKPT_EVERY = 256


@dataclass(frozen=True)
class RANSFrameStats:
    raw_bytes: int
    encoded_bytes: int
    tiles: int
    compressed_tiles: int

    @property
    def ratio(self) -> float:
        return self.raw_bytes / self.encoded_bytes if self.encoded_bytes else 1.0


def encode(data, *, tile_bytes: int = 1 << 20, threads: int = 0) -> tuple[bytes, RANSFrameStats]:
    """Pack side (host, multi-threaded C++): byte-identical to the reference encode."""
    if tile_bytes <= 0:
        raise ValueError("rANS tile_bytes must be positive")
    lib = load()
    arr = np.ascontiguousarray(_device.as_u8(data))
    cap = ctypes.c_uint64(0)
    check(lib.voom_rans_encode(arr.ctypes.data, arr.size, tile_bytes, None, 0, ctypes.byref(cap), None, 0),
          "voom_rans_encode(size)")
    out = np.empty(cap.value, dtype=np.uint8)
    n = ctypes.c_uint64(0)
    stats = np.zeros(2, dtype=np.uint64)
    check(lib.voom_rans_encode(arr.ctypes.data, arr.size, tile_bytes, out.ctypes.data, out.size,
                               ctypes.byref(n), stats.ctypes.data, int(threads)), "voom_rans_encode")
    frame = out[: n.value].tobytes()
    return frame, RANSFrameStats(raw_bytes=arr.size, encoded_bytes=len(frame), tiles=int(stats[0]),
                                 compressed_tiles=int(stats[1]))


class RansPlan:
    """Host-side walk of one frame: tile descriptors + structural error."""

    __slots__ = ("tiles", "info")

    def __init__(self, tiles: np.ndarray, info: RansPlanInfo):
        self.tiles = tiles
        self.info = info

    @property
    def raw_size(self) -> int:
        return int(self.info.raw_size)

    @property
    def out_bytes(self) -> int:
        return int(self.info.out_bytes)


def plan(frame, *, src_base: int = 0, dst_base: int = 0) -> RansPlan:
    lib = load()
    arr = np.ascontiguousarray(_device.as_u8(frame))
    info = RansPlanInfo()
    check(lib.voom_rans_plan(arr.ctypes.data, arr.size, src_base, dst_base, None, 0, ctypes.byref(info)),
          "voom_rans_plan(size)")
    tiles = np.zeros(info.n_tiles, dtype=RANS_TILE_DTYPE)
    if info.n_tiles:
        check(lib.voom_rans_plan(arr.ctypes.data, arr.size, src_base, dst_base, tiles.ctypes.data,
                                 tiles.size, ctypes.byref(info)), "voom_rans_plan")
    return RansPlan(tiles, info)


def _raise(code: int, info: RansPlanInfo) -> None:
    msg = RANS_MESSAGES.get(code)
    if msg is None:
        raise VoomError(f"rANS decode failed with status {code}")
    raise ValueError(msg.format(mode=info.bad_mode))


def resolve(p: RansPlan, status: np.ndarray) -> int:
    lib = load()
    st = np.ascontiguousarray(status, dtype=np.uint32)
    tile = ctypes.c_uint32(0)
    return lib.voom_rans_resolve(ctypes.byref(p.info), st.ctypes.data if st.size else None, st.size,
                                 ctypes.byref(tile))


def _frame_level_error(p: RansPlan) -> int:
    if p.info.struct_error and p.info.n_tiles == 0 and p.info.struct_error in (101, 102):
        return p.info.struct_error
    return 0


def decode_device(frame, *, device=None, stream: torch.cuda.Stream | None = None,
                  check_errors: bool = True) -> torch.Tensor:
    """Decode one frame on the GPU; return the bytes as a CUDA uint8 tensor."""
    dev = _device.require_cuda(device)
    p = plan(frame)
    early = _frame_level_error(p)
    if early:
        _raise(early, p.info)
    lib = load()
    sptr = _device.stream_ptr(dev, stream)
    with torch.cuda.device(dev):
        src = _device.upload(frame, dev, stream=stream)
        out = torch.empty(max(p.out_bytes, 1), dtype=torch.uint8, device=dev)
        n = int(p.info.n_tiles)
        status = torch.zeros(max(n, 1), dtype=torch.int32, device=dev)
        if n:
            tiles = _device.tensor_from_numpy(p.tiles, dev)
            check(lib.voom_rans_decode(src.data_ptr(), tiles.data_ptr(), n, out.data_ptr(),
                                       status.data_ptr(), None, None, 0, sptr), "voom_rans_decode")
        if check_errors:
            st = status[:n].cpu().numpy().view(np.uint32) if n else np.zeros(0, np.uint32)
            code = resolve(p, st)
            if code:
                _raise(code, p.info)
    return out[: p.raw_size] if p.out_bytes >= p.raw_size else out[: p.out_bytes]


def decode(frame: bytes) -> bytes:
    """Drop-in for formats/bf16_rans.py decode(): bytes in, bytes out, same errors."""
    return decode_device(frame).cpu().numpy().tobytes()


class RansPage:
    """A VRN1 frame resident in HBM with its tile plan and checkpoint index.

    Built once (cold decode that also records a (state, cursor) checkpoint
    every `every` symbols of each plane); afterwards `decode_into` runs every
    checkpoint segment of every tile in parallel and verifies that each
    segment ends exactly on the next checkpoint and that every tile matches
    its CRC-32.  This is how expert pages that stay compressed in HBM are
    decoded on every use.
    """

    def __init__(self, frame, *, device=None, every: int = DEFAULT_CKPT_EVERY,
                 stream: torch.cuda.Stream | None = None):
        self.device = _device.require_cuda(device)
        self.every = int(every)
        self.plan = plan(frame)
        early = _frame_level_error(self.plan)
        if early:
            _raise(early, self.plan.info)
        if self.plan.info.struct_error:
            code = self.plan.info.struct_error
            _raise(code, self.plan.info)
        lib = load()
        n = int(self.plan.info.n_tiles)
        self.n_tiles = n
        words = [int(lib.voom_rans_ckpt_words(int(t["raw_len"]), self.every)) for t in self.plan.tiles]
        base = np.zeros(max(n, 1), dtype=np.uint32)
        if n:
            base[:n] = np.cumsum([0] + words[:-1])
        with torch.cuda.device(self.device):
            self.src = _device.upload(frame, self.device, stream=stream)
            self.tiles = _device.tensor_from_numpy(self.plan.tiles, self.device)
            self.ckpt_base = _device.tensor_from_numpy(base, self.device)
            self.ckpt = torch.zeros(max(sum(words), 1), dtype=torch.int32, device=self.device)
            out = torch.empty(max(self.plan.out_bytes, 1), dtype=torch.uint8, device=self.device)
            status = torch.zeros(max(n, 1), dtype=torch.int32, device=self.device)
            sptr = _device.stream_ptr(self.device, stream)
            if n:
                check(lib.voom_rans_decode(self.src.data_ptr(), self.tiles.data_ptr(), n, out.data_ptr(),
                                           status.data_ptr(), self.ckpt.data_ptr(),
                                           self.ckpt_base.data_ptr(), self.every, sptr),
                      "voom_rans_decode(index)")
            st = status[:n].cpu().numpy().view(np.uint32)
            code = resolve(self.plan, st)
            if code:
                _raise(code, self.plan.info)
            nch = ctypes.c_uint32(0)
            tiles_h = np.ascontiguousarray(self.plan.tiles)
            check(lib.voom_rans_chunks(tiles_h.ctypes.data if n else None, n, self.every, None, 0,
                                       ctypes.byref(nch)), "voom_rans_chunks(size)")
            chunks = np.zeros(max(nch.value, 1), dtype=RANS_CHUNK_DTYPE)
            check(lib.voom_rans_chunks(tiles_h.ctypes.data if n else None, n, self.every, chunks.ctypes.data,
                                       chunks.size, ctypes.byref(nch)), "voom_rans_chunks")
            self.n_chunks = int(nch.value)
            self.chunks = _device.tensor_from_numpy(chunks, self.device)
            self.tile_scratch = torch.zeros(4 * max(n, 1), dtype=torch.int32, device=self.device)
        self.raw_size = self.plan.raw_size
        self.compressed_bytes = int(self.src.numel() - _device.PAD)

    def decode_into(self, out: torch.Tensor, status: torch.Tensor,
                    stream: torch.cuda.Stream | None = None) -> None:
        """Enqueue an indexed decode into `out` (>= raw_size bytes); status gets
        one u32 per tile (0 = exact).  No host synchronisation."""
        lib = load()
        if self.n_tiles:
            check(lib.voom_rans_decode_indexed(self.src.data_ptr(), self.tiles.data_ptr(), self.chunks.data_ptr(),
                                               self.n_chunks, out.data_ptr(), status.data_ptr(),
                                               self.ckpt.data_ptr(), self.ckpt_base.data_ptr(), self.every,
                                               self.tile_scratch.data_ptr(),
                                               _device.stream_ptr(self.device, stream)),
                  "voom_rans_decode_indexed")

    def decode(self) -> torch.Tensor:
        out = torch.empty(max(self.raw_size, 1), dtype=torch.uint8, device=self.device)
        status = torch.zeros(max(self.n_tiles, 1), dtype=torch.int32, device=self.device)
        self.decode_into(out, status)
        st = status[: self.n_tiles].cpu().numpy().view(np.uint32)
        code = resolve(self.plan, st)
        if code:
            _raise(code, self.plan.info)
        return out[: self.raw_size]
