"""GPU Zstandard decompression (RFC 8878) through libvoom_b200.

`decompress(data)` is the drop-in for `compression.zstd.decompress` as the
reference uses it (formats/packed.py:376-378, formats/packed2.py:182-191,
runtime/kv_paged.py:102-103) but returns a CUDA uint8 tensor.  `ZstdBatch`
decodes many independent jobs (frames, optionally interleaved with a raw lo
plane as vpack bodies are) in one set of launches: the host plans frame and
block headers, the GPU decodes the entropy-coded payloads, executes the
sequences and writes the output.
"""

from __future__ import annotations

import ctypes

import numpy as np
import torch

from .. import _device
from .._lib import VoomError, check, load

JOB_DTYPE = np.dtype([("src", "<u8"), ("src_len", "<u8"), ("dst", "<u8"), ("dst_len", "<u8"),
                      ("lo_src", "<u8"), ("flags", "<u4"), ("pad", "<u4")])
assert JOB_DTYPE.itemsize == 48

INTERLEAVE = 1
ST_FORMAT, ST_LITERALS, ST_SEQUENCES, ST_OFFSET, ST_SIZE, ST_CHECKSUM, ST_UNRESOLVED = 1, 2, 4, 8, 16, 32, 64
ST_TOO_LARGE = 128
_ST_NAMES = {ST_FORMAT: "malformed frame", ST_LITERALS: "corrupt literals", ST_SEQUENCES: "corrupt sequences",
             ST_OFFSET: "offset out of range", ST_SIZE: "content size mismatch",
             ST_CHECKSUM: "content checksum mismatch", ST_UNRESOLVED: "unresolved match chain",
             ST_TOO_LARGE: "job too large for one decode (more than 2 GiB - 1 MiB with matches)"}


class ZstdError(Exception):
    """A job failed to decode (mirrors compression.zstd.ZstdError)."""


def describe(status: int) -> str:
    return ", ".join(n for b, n in _ST_NAMES.items() if status & b) or "ok"


class PlanInfo(ctypes.Structure):
    _fields_ = [("n_jobs", ctypes.c_uint32), ("n_frames", ctypes.c_uint32), ("n_blocks", ctypes.c_uint32),
                ("n_huf", ctypes.c_uint32), ("n_fse", ctypes.c_uint32), ("n_bad_jobs", ctypes.c_uint32),
                ("lit_bytes", ctypes.c_uint64), ("n_seq", ctypes.c_uint64), ("decoded_bytes", ctypes.c_uint64),
                ("scratch_bytes", ctypes.c_uint64), ("plan_bytes", ctypes.c_uint64),
                ("n_segments", ctypes.c_uint32), ("n_direct_jobs", ctypes.c_uint32)]


def frame_content_size(data) -> int | None:
    """Sum of Frame_Content_Size over the frames in `data` (skippable frames
    skipped); None when a frame does not record its size."""
    b = memoryview(_device.as_u8(data))
    pos, total = 0, 0
    n = len(b)
    while pos < n:
        if n - pos < 5:
            return None
        magic = int.from_bytes(b[pos:pos + 4], "little")
        if (magic & 0xFFFFFFF0) == 0x184D2A50:
            pos += 8 + int.from_bytes(b[pos + 4:pos + 8], "little")
            continue
        if magic != 0xFD2FB528:
            return None
        fhd = b[pos + 4]
        single = (fhd >> 5) & 1
        fcs_flag = fhd >> 6
        did = (0, 1, 2, 4)[fhd & 3]
        q = pos + 5 + (0 if single else 1) + did
        fcs_sz = (1 if single else 0) if fcs_flag == 0 else (2, 4, 8)[fcs_flag - 1]
        if fcs_sz == 0:
            return None
        v = int.from_bytes(b[q:q + fcs_sz], "little") + (256 if fcs_sz == 2 else 0)
        total += v
        # walk blocks to find the next frame
        q += fcs_sz
        while True:
            if q + 3 > n:
                return None
            bh = int.from_bytes(b[q:q + 3], "little")
            q += 3
            btype, bsize = (bh >> 1) & 3, bh >> 3
            q += 1 if btype == 1 else bsize
            if bh & 1:
                break
        if (fhd >> 2) & 1:
            q += 4
        pos = q
    return total


class ZstdPlan:
    """Host plan of a batch of jobs; owns the native plan handle."""

    def __init__(self, src_host: np.ndarray, jobs: np.ndarray, threads: int = 0):
        self._lib = load()
        self.jobs = np.ascontiguousarray(jobs, dtype=JOB_DTYPE)
        src = np.ascontiguousarray(src_host).reshape(-1).view(np.uint8)
        self.handle = self._lib.voom_zstd_plan_create(src.ctypes.data if src.size else None, src.size,
                                                      self.jobs.ctypes.data if self.jobs.size else None,
                                                      self.jobs.size, int(threads))
        if not self.handle:
            raise VoomError("voom_zstd_plan_create failed")
        self.info = PlanInfo()
        check(self._lib.voom_zstd_plan_info_get(self.handle, ctypes.byref(self.info)), "voom_zstd_plan_info_get")
        self.image = np.empty(max(self.info.plan_bytes, 1), dtype=np.uint8)  # every byte is written below
        check(self._lib.voom_zstd_plan_image(self.handle, self.image.ctypes.data, self.image.size),
              "voom_zstd_plan_image")
        self.plan_status = np.zeros(max(self.jobs.size, 1), dtype=np.uint32)
        check(self._lib.voom_zstd_plan_job_status(self.handle, self.plan_status.ctypes.data),
              "voom_zstd_plan_job_status")

    def __del__(self):
        h = getattr(self, "handle", None)
        if h:
            self._lib.voom_zstd_plan_destroy(h)
            self.handle = None


class ZstdBatch:
    """A planned batch resident on one device: plan image + scratch."""

    def __init__(self, plan: ZstdPlan, device, scratch: torch.Tensor | None = None,
                 stream: torch.cuda.Stream | None = None):
        """`stream` given: the plan image goes up from a pinned copy on that
        stream without the host waiting for the stream's earlier work (as a
        pageable upload would), read by a kernel from the mapped pinned copy
        so that it does not queue behind uploads already on a copy engine."""
        self.plan = plan
        self.device = device
        if stream is None:
            self.d_plan = _device.tensor_from_numpy(plan.image, device)
        else:
            n = plan.image.nbytes
            self._h_plan = _device.pinned_empty(n)  # held until the batch is dropped
            self._h_plan.numpy()[:] = plan.image.reshape(-1).view(np.uint8)
            self.d_plan = torch.empty(n, dtype=torch.uint8, device=device)
            rc = load().voom_copy_from_host(self.d_plan.data_ptr(), self._h_plan.data_ptr(), n,
                                            _device.stream_ptr(device, stream))
            if rc != 0:  # not mapped pinned memory: an ordinary asynchronous copy
                with torch.cuda.stream(stream):
                    self.d_plan.copy_(self._h_plan, non_blocking=True)
        need = int(plan.info.scratch_bytes)
        if scratch is None or scratch.numel() < need:
            scratch = torch.empty(max(need, 1), dtype=torch.uint8, device=device)
        self.scratch = scratch
        self.status = torch.zeros(max(plan.jobs.size, 1), dtype=torch.int32, device=device)

    def run(self, d_src: torch.Tensor, d_out: torch.Tensor, stream: torch.cuda.Stream | None = None) -> None:
        """Enqueue the decode; statuses accumulate into self.status (cleared here)."""
        self.status.zero_()
        check(load().voom_zstd_decode(d_src.data_ptr(), self.d_plan.data_ptr(), self.plan.handle,
                                      self.scratch.data_ptr(), d_out.data_ptr(), self.status.data_ptr(),
                                      _device.stream_ptr(self.device, stream)), "voom_zstd_decode")

    def job_status(self) -> np.ndarray:
        n = self.plan.jobs.size
        st = self.status[:n].cpu().numpy().view(np.uint32) if n else np.zeros(0, np.uint32)
        return st | self.plan.plan_status[:n]


def decompress_device(data, size: int | None = None, *, device=None,
                      stream: torch.cuda.Stream | None = None) -> torch.Tensor:
    """GPU zstd.decompress(data) -> CUDA uint8 tensor of the decoded bytes."""
    dev = _device.require_cuda(device)
    arr = _device.as_u8(data)
    if size is None:
        size = frame_content_size(arr)
        if size is None:
            raise ZstdError("frame content size unknown; pass size=")
    jobs = np.zeros(1, dtype=JOB_DTYPE)
    jobs[0] = (0, arr.size, 0, size, 0, 0, 0)
    plan = ZstdPlan(arr, jobs)
    if plan.plan_status[0]:
        raise ZstdError(describe(int(plan.plan_status[0])))
    with torch.cuda.device(dev):
        d_src = _device.upload(arr, dev, stream=stream)
        out = torch.empty(max(size, 1), dtype=torch.uint8, device=dev)
        batch = ZstdBatch(plan, dev)
        batch.run(d_src, out, stream)
        st = batch.job_status()
    if st[0]:
        raise ZstdError(describe(int(st[0])))
    return out[:size]


def decompress_many(frames: list, sizes: list[int] | None = None, *, device=None, align: int = 256,
                    stream: torch.cuda.Stream | None = None) -> tuple[torch.Tensor, list[tuple[int, int]]]:
    """Many independent zstd frames in ONE batched GPU decode: returns the
    device buffer and each frame's (offset, length) in it (offsets aligned to
    `align` bytes).  Raises ZstdError naming the first failing frame's fault."""
    dev = _device.require_cuda(device)
    arrs = [_device.as_u8(f) for f in frames]
    if sizes is None:
        sizes = []
        for a in arrs:
            n = frame_content_size(a)
            if n is None:
                raise ZstdError("frame content size unknown; pass sizes=")
            sizes.append(n)
    if len(sizes) != len(arrs):
        raise ValueError("one size per frame")
    jobs = np.zeros(len(arrs), dtype=JOB_DTYPE)
    spans, src, dst = [], 0, 0
    for i, (a, n) in enumerate(zip(arrs, sizes)):
        jobs[i] = (src, a.size, dst, n, 0, 0, 0)
        spans.append((dst, int(n)))
        src += a.size
        dst += (int(n) + align - 1) // align * align
    host = np.concatenate(arrs) if arrs else np.zeros(0, np.uint8)
    with torch.cuda.device(dev):
        out = torch.empty(max(dst, 1), dtype=torch.uint8, device=dev)
        if not arrs:
            return out, spans
        plan = ZstdPlan(host, jobs)
        d_src = _device.upload(host, dev, stream=stream)
        batch = ZstdBatch(plan, dev)
        batch.run(d_src, out, stream)
        st = batch.job_status()
    if st.any():
        raise ZstdError(describe(int(st[np.nonzero(st)[0][0]])))
    return out, spans


def decompress(data, size: int | None = None) -> bytes:
    """Drop-in for compression.zstd.decompress(data) (bytes in, bytes out)."""
    return decompress_device(data, size).cpu().numpy().tobytes()


ZENC_BLOCK_DTYPE = np.dtype([("src", "<u8"), ("frame_len", "<u8"), ("len", "<u4"), ("flags", "<u4")])
assert ZENC_BLOCK_DTYPE.itemsize == 24
ZENC_FIRST, ZENC_LAST = 1, 2


class EncodePlan:
    """The block table of many frames for the GPU encoder, built once (frames
    of more than voom_zstd_encode_block_bytes() are split into blocks) and
    resident on `device`; run() encodes the byte ranges of a device buffer."""

    def __init__(self, offsets, lengths, device):
        lib = load()
        self.block = int(lib.voom_zstd_encode_block_bytes())
        self.slot = int(lib.voom_zstd_encode_slot_bytes())
        offs = np.asarray(offsets, np.int64).reshape(-1)
        lens = np.asarray(lengths, np.int64).reshape(-1)
        nb = np.maximum(1, (lens + self.block - 1) // self.block)
        first = np.zeros(nb.size, np.int64)
        if nb.size > 1:
            np.cumsum(nb[:-1], out=first[1:])
        n_blocks = int(nb.sum())
        fr = np.repeat(np.arange(nb.size), nb)
        k = np.arange(n_blocks, dtype=np.int64) - first[fr]
        blocks = np.zeros(n_blocks, dtype=ZENC_BLOCK_DTYPE)
        blocks["src"] = offs[fr] + k * self.block
        blocks["frame_len"] = lens[fr]
        blocks["len"] = np.minimum(self.block, lens[fr] - k * self.block)
        blocks["flags"] = np.where(k == 0, ZENC_FIRST, 0) | np.where(k == nb[fr] - 1, ZENC_LAST, 0)
        self.n_blocks = n_blocks
        self.frames = list(zip(first.tolist(), nb.tolist()))
        self.first, self.nb = first, nb
        self.device = device
        self.d_blocks = _device.tensor_from_numpy(blocks.view(np.uint8), device) if n_blocks else None
        self.slots = torch.empty(max(n_blocks, 1) * self.slot, dtype=torch.uint8, device=device)
        self.sizes = torch.empty(max(2 * n_blocks, 2), dtype=torch.int32, device=device)

    def run(self, d_src: torch.Tensor, stream: torch.cuda.Stream | None = None) -> None:
        """Enqueue the encode of every block (no host synchronisation)."""
        if self.n_blocks:
            check(load().voom_zstd_encode(d_src.data_ptr(), self.d_blocks.data_ptr(), self.n_blocks,
                                          self.slots.data_ptr(), self.sizes.data_ptr(),
                                          _device.stream_ptr(self.device, stream)), "voom_zstd_encode")

    def block_sizes(self) -> np.ndarray:
        """(slot offset within the slot buffer, length) of every block (waits for the encode)."""
        sz = self.sizes[:2 * self.n_blocks].cpu().numpy().view(np.uint32).reshape(-1, 2).astype(np.int64)
        sz[:, 0] += np.arange(self.n_blocks, dtype=np.int64) * self.slot
        return sz


def pack_blocks(plan: EncodePlan, sz: np.ndarray, frame_dst, out: torch.Tensor,
                stream: torch.cuda.Stream | None = None) -> np.ndarray:
    """Packs every frame's encoded blocks (after plan.run; `sz` =
    plan.block_sizes()) into the device buffer `out`, frame i starting at byte
    frame_dst[i].  Returns the frames' lengths."""
    n = plan.n_blocks
    flen = np.add.reduceat(sz[:, 1], plan.first) if n else np.zeros(0, np.int64)
    if n == 0:
        return flen
    fr = np.repeat(np.arange(len(plan.first)), plan.nb)
    cs = np.cumsum(sz[:, 1]) - sz[:, 1]
    dst = (np.asarray(frame_dst, np.int64)[fr] + cs - cs[plan.first[fr]]).astype(np.uint64)
    rel = sz.copy()
    rel[:, 0] -= np.arange(n, dtype=np.int64) * plan.slot
    dev = out.device
    d_sizes = _device.tensor_from_numpy(rel.astype(np.uint32), dev)
    d_dst = _device.tensor_from_numpy(dst, dev)
    check(load().voom_zstd_encode_pack(plan.slots.data_ptr(), d_sizes.data_ptr(), d_dst.data_ptr(), n,
                                       out.data_ptr(), _device.stream_ptr(dev, stream)), "voom_zstd_encode_pack")
    return flen


def compress_device(d_src: torch.Tensor, offsets, lengths, *, stream: torch.cuda.Stream | None = None
                    ) -> tuple[torch.Tensor, np.ndarray, list[tuple[int, int]]]:
    """Compress many byte ranges of one device buffer, each into its own zstd
    frame, in ONE launch of the GPU encoder (voom_zstd_encode).  Returns the
    device slots, the (slot offset, length) of every block (host array, n x 2)
    and each frame's (first block, block count).  The frames are valid
    RFC 8878 frames that zstd.decompress / compression.zstd accept; they are
    not libzstd's bytes."""
    plan = EncodePlan(offsets, lengths, d_src.device)
    with torch.cuda.device(d_src.device):
        plan.run(d_src, stream)
        sz = plan.block_sizes()
    return plan.slots, sz, plan.frames


def compress_many(d_src: torch.Tensor, offsets, lengths, *, stream: torch.cuda.Stream | None = None,
                  pinned: torch.Tensor | None = None, plan: EncodePlan | None = None) -> list[bytes]:
    """Every byte range compressed into a zstd frame on the GPU, returned as
    host bytes: the blocks are packed on the device and cross to the host in
    one copy (into `pinned` when it is a large enough pinned buffer).  A plan
    built once for the same ranges may be passed."""
    plan = plan or EncodePlan(offsets, lengths, d_src.device)
    dev = d_src.device
    with torch.cuda.device(dev):
        plan.run(d_src, stream)
        sz = plan.block_sizes()
    n_blocks = sz.shape[0]
    if n_blocks == 0:
        return [b"" for _ in plan.frames]
    dst = np.zeros(n_blocks, np.uint64)
    np.cumsum(sz[:-1, 1], out=dst[1:])
    total = int(dst[-1] + sz[-1, 1])
    rel = sz.copy()
    rel[:, 0] -= np.arange(n_blocks, dtype=np.int64) * plan.slot
    d_sizes = _device.tensor_from_numpy(rel.astype(np.uint32), dev)
    d_dst = _device.tensor_from_numpy(dst, dev)
    packed = torch.empty(max(total, 1), dtype=torch.uint8, device=dev)
    check(load().voom_zstd_encode_pack(plan.slots.data_ptr(), d_sizes.data_ptr(), d_dst.data_ptr(), n_blocks,
                                       packed.data_ptr(), _device.stream_ptr(dev, stream)), "voom_zstd_encode_pack")
    if pinned is not None and pinned.numel() >= total:
        pinned[:total].copy_(packed[:total])
        host = pinned.numpy()
    else:
        host = packed[:total].cpu().numpy()
    starts = dst[plan.first].astype(np.int64)
    last = plan.first + plan.nb - 1
    ends = (dst[last] + sz[last, 1].astype(np.uint64)).astype(np.int64)
    mv = memoryview(host)
    return [bytes(mv[a:e]) for a, e in zip(starts.tolist(), ends.tolist())]


def compress(data, level: int = 1) -> bytes:
    """compression.zstd.compress(data) on the GPU (level is accepted for the
    signature; the encoder has one setting)."""
    arr = _device.as_u8(data)
    dev = _device.require_cuda(None)
    d = _device.upload(arr, dev) if arr.size else torch.zeros(16, dtype=torch.uint8, device=dev)
    return compress_many(d, [0], [arr.size])[0]
