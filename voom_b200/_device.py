"""Device plumbing shared by the host-side mirrors: CUDA checks, streams and
host<->device staging.  torch supplies device memory and streams only."""

from __future__ import annotations

import threading

import numpy as np
import torch

from ._lib import VoomError

PAD = 16  # every device source buffer carries this many readable bytes past its end


def require_cuda(device: torch.device | str | int | None = None) -> torch.device:
    if not torch.cuda.is_available():
        raise VoomError("voom_b200 decodes on a CUDA device and no CUDA device is available")
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    if dev.type != "cuda":
        raise VoomError(f"voom_b200 needs a CUDA device, got {dev}")
    if dev.index is None:
        dev = torch.device("cuda", torch.cuda.current_device())
    return dev


def stream_ptr(device: torch.device, stream: torch.cuda.Stream | None = None) -> int:
    s = stream if stream is not None else torch.cuda.current_stream(device)
    return int(s.cuda_stream)


def as_u8(buf) -> np.ndarray:
    """bytes / bytearray / memoryview / numpy / CPU tensor -> flat uint8 numpy view."""
    if isinstance(buf, np.ndarray):
        return buf.reshape(-1).view(np.uint8)
    if isinstance(buf, torch.Tensor):
        if buf.device.type != "cpu":
            raise TypeError("expected a host buffer")
        return buf.reshape(-1).view(torch.uint8).numpy()
    return np.frombuffer(buf, dtype=np.uint8)


def pinned_empty(n: int) -> torch.Tensor:
    return torch.empty(int(n), dtype=torch.uint8, pin_memory=True)


class PinnedArena:
    """A growing pinned host buffer reused across calls (pinning memory costs
    milliseconds per hundred MB).  Hold `lock` from `get` until every copy
    out of the buffer has completed."""

    def __init__(self):
        self._buf: torch.Tensor | None = None
        self.lock = threading.Lock()

    def get(self, n: int) -> torch.Tensor:
        if self._buf is None or self._buf.numel() < n:
            self._buf = None
            self._buf = pinned_empty(max(int(n), 1) * 5 // 4 + 4096)
        return self._buf


_STAGE_CHUNK = 8 << 20  # bytes per staging half
_stage: dict = {}         # device index -> (pinned staging tensor, [event, event], lock)
_stage_lock = threading.Lock()


def _staging(device: torch.device):
    """A reusable pinned staging buffer of two halves per device (allocating
    pinned memory per call costs milliseconds per hundred MB)."""
    with _stage_lock:
        st = _stage.get(device.index)
        if st is None:
            buf = pinned_empty(2 * _STAGE_CHUNK)
            st = (buf, [None, None], threading.Lock())
            _stage[device.index] = st
    return st


def upload(host, device: torch.device, *, pad: int = PAD, stream: torch.cuda.Stream | None = None,
           out: torch.Tensor | None = None) -> torch.Tensor:
    """Copy a host buffer into a new (or given) device uint8 tensor with `pad`
    zero bytes after it.  Pinned CPU tensors are copied asynchronously in one
    DMA; pageable buffers go through a cached two-half pinned staging buffer,
    the memcpy of one half overlapping the DMA of the other."""
    if isinstance(host, torch.Tensor) and host.device.type == "cuda":
        src = host.reshape(-1).view(torch.uint8)
        n = src.numel()
        dev = out if out is not None else torch.empty(n + pad, dtype=torch.uint8, device=device)
        dev[:n].copy_(src)
        if pad:
            dev[n:n + pad].zero_()
        return dev
    s = stream if stream is not None else torch.cuda.current_stream(device)
    if isinstance(host, torch.Tensor) and host.is_pinned():
        src = host.reshape(-1).view(torch.uint8)
        n = src.numel()
        dev = out if out is not None else torch.empty(n + pad, dtype=torch.uint8, device=device)
        with torch.cuda.stream(s):
            dev[:n].copy_(src, non_blocking=True)
            if pad:
                dev[n:n + pad].zero_()
        return dev
    arr = as_u8(host)
    n = arr.size
    dev = out if out is not None else torch.empty(n + pad, dtype=torch.uint8, device=device)
    buf, events, lock = _staging(device)
    stage = buf.numpy()
    with lock, torch.cuda.stream(s):
        for i, off in enumerate(range(0, n, _STAGE_CHUNK)):
            half = i & 1
            if events[half] is not None:
                events[half].synchronize()  # that half's previous DMA is done
            m = min(_STAGE_CHUNK, n - off)
            base = half * _STAGE_CHUNK
            stage[base:base + m] = arr[off:off + m]
            dev[off:off + m].copy_(buf[base:base + m], non_blocking=True)
            ev = torch.cuda.Event()
            ev.record(s)
            events[half] = ev
        if pad:
            dev[n:n + pad].zero_()
    return dev


def tensor_from_numpy(arr: np.ndarray, device: torch.device) -> torch.Tensor:
    """Small control arrays (plans, descriptors) -> device uint8 tensor."""
    raw = np.ascontiguousarray(arr).view(np.uint8).reshape(-1)
    # a synchronous copy: the array is read before this returns, so a
    # writable one is wrapped as it is (large plan images are tens of MB)
    host = torch.from_numpy(raw if raw.flags.writeable else raw.copy())
    return host.to(device, non_blocking=False)
