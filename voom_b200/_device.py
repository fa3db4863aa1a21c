"""Device plumbing shared by the host-side mirrors: CUDA checks, streams and
host<->device staging.  torch supplies device memory and streams only."""

from __future__ import annotations

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


def upload(host, device: torch.device, *, pad: int = PAD, stream: torch.cuda.Stream | None = None,
           out: torch.Tensor | None = None) -> torch.Tensor:
    """Copy a host buffer into a new (or given) device uint8 tensor with `pad`
    zero bytes after it.  Pinned CPU tensors are copied asynchronously; other
    buffers are staged through a pinned buffer first."""
    if isinstance(host, torch.Tensor) and host.device.type == "cuda":
        src = host.reshape(-1).view(torch.uint8)
        n = src.numel()
        dev = out if out is not None else torch.empty(n + pad, dtype=torch.uint8, device=device)
        dev[:n].copy_(src)
        if pad:
            dev[n:n + pad].zero_()
        return dev
    if isinstance(host, torch.Tensor) and host.is_pinned():
        src = host.reshape(-1).view(torch.uint8)
    else:
        arr = as_u8(host)
        src = pinned_empty(arr.size)
        src.numpy()[:] = arr
    n = src.numel()
    dev = out if out is not None else torch.empty(n + pad, dtype=torch.uint8, device=device)
    with torch.cuda.stream(stream) if stream is not None else _null():
        dev[:n].copy_(src, non_blocking=True)
        if pad:
            dev[n:n + pad].zero_()
    return dev


class _null:
    def __enter__(self):
        return None

    def __exit__(self, *a):
        return False


def tensor_from_numpy(arr: np.ndarray, device: torch.device) -> torch.Tensor:
    """Small control arrays (plans, descriptors) -> device uint8 tensor."""
    raw = np.ascontiguousarray(arr).view(np.uint8).reshape(-1)
    host = torch.from_numpy(raw.copy())
    return host.to(device, non_blocking=False)
