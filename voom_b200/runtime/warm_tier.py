"""WarmTier: compressed host-RAM tier between the device weight cache and
storage (runtime/warm_tier.py:55-103 of the reference).

Pages evicted from the weight cache are admitted as zstd level-1 frames of
each tensor's raw bytes (BF16, U8 and F32 tensors; a page with any other
tensor type is rejected, runtime/warm_tier.py:22-38), unless the page
compresses by less than MIN_RATIO (runtime/warm_tier.py:56,74-83).  The heap
is bounded by `max_bytes` of compressed bytes and drops its oldest admissions
first (runtime/warm_tier.py:84-91).  `take(key)` removes the page and returns
its tensors (runtime/warm_tier.py:92-99).

B200 layout: admission copies the page to the host once and compresses its
tensors on a host thread pool with libzstd level 1 (the codec call the
reference makes, so the frames are the same bytes); `take` uploads all of a
page's frames and decodes them in ONE batched GPU zstd decode into a single
device buffer, and the returned tensors are views into it.  `take_many`
decodes several pages in one batch.
"""

from __future__ import annotations

import threading
from concurrent.futures import ThreadPoolExecutor
from typing import NamedTuple

import numpy as np
import torch

from .. import _device
from ..formats import zstd_host
from ..formats.zstd_gpu import decompress_many

_KINDS = {torch.bfloat16: "bf16", torch.uint8: "u8", torch.float32: "f32"}
_DTYPES = {"bf16": torch.bfloat16, "u8": torch.uint8, "f32": torch.float32}


def _page_to_blobs(tensors: dict) -> list[tuple[str, str, tuple, np.ndarray]] | None:
    """(name, kind, shape, raw bytes) per tensor, or None when a tensor has a
    type the tier does not hold (runtime/warm_tier.py:22-38)."""
    out = []
    for name, t in tensors.items():
        if not isinstance(t, torch.Tensor) or t.dtype not in _KINDS:
            return None
        raw = t.detach().contiguous().reshape(-1).view(torch.uint8).cpu().numpy()
        out.append((name, _KINDS[t.dtype], tuple(t.shape), raw))
    return out


class _Held(NamedTuple):
    """One admitted page: its (name, kind, shape, zstd frame) entries and the
    compressed bytes they hold."""
    frames: list
    nbytes: int


class WarmTier:
    MIN_RATIO = 1.15  # pages that barely compress are not admitted

    def __init__(self, max_bytes: int, device=None, threads: int = 8):
        self.max_bytes = max_bytes
        self.device = device
        self.threads = max(1, int(threads))
        self._held: dict[str, _Held] = {}  # insertion order is admission order
        self._held_bytes = 0
        self._lock = threading.Lock()
        self.hits = 0
        self.admits = 0
        self.rejects = 0

    def _compress(self, raws: list[np.ndarray]) -> list[bytes]:
        if len(raws) == 1 or self.threads == 1:
            return [zstd_host.compress(r, 1) for r in raws]
        with ThreadPoolExecutor(max_workers=min(self.threads, len(raws))) as pool:
            return list(pool.map(lambda r: zstd_host.compress(r, 1), raws))

    def admit(self, key: str, tensors: dict) -> None:
        """Compress a page evicted from the device cache and hold it.  The page is
        refused (counted in `rejects`) when a tensor has a type the tier does not
        hold or the page shrinks by less than MIN_RATIO; a key already held is
        left as it is."""
        blobs = _page_to_blobs(tensors)
        if blobs is None:
            self.rejects += 1
            return
        if self.device is None:
            self.device = next((t.device for t in tensors.values() if t.is_cuda), None)
        frames = self._compress([raw for *_, raw in blobs])
        held = _Held([(name, kind, shape, f) for (name, kind, shape, _), f in zip(blobs, frames)],
                     sum(len(f) for f in frames))
        raw_bytes = sum(raw.size for *_, raw in blobs)
        if raw_bytes < self.MIN_RATIO * max(held.nbytes, 1):
            self.rejects += 1
            return
        with self._lock:
            if key not in self._held:
                self._held[key] = held
                self._held_bytes += held.nbytes
                self.admits += 1
                self._trim_locked()

    def _trim_locked(self) -> None:
        """Drops the oldest admissions until the held bytes fit `max_bytes`
        (the page just admitted too, when it alone does not fit)."""
        excess = self._held_bytes - self.max_bytes
        if excess <= 0:
            return
        victims = []
        for k, h in self._held.items():
            if excess <= 0:
                break
            victims.append(k)
            excess -= h.nbytes
        for k in victims:
            self._held_bytes -= self._held.pop(k).nbytes

    def _pop(self, key: str) -> list | None:
        with self._lock:
            held = self._held.pop(key, None)
            if held is None:
                return None
            self._held_bytes -= held.nbytes
        return held.frames

    def take(self, key: str) -> dict | None:
        return self.take_many([key])[key]

    def take_many(self, keys: list[str]) -> dict[str, dict | None]:
        """Remove and decode several pages in one batched GPU decode; a key the
        tier does not hold maps to None."""
        pages = {k: self._pop(k) for k in keys}
        held = [(k, c) for k, c in pages.items() if c is not None]
        out: dict[str, dict | None] = {k: None for k in keys}
        if not held:
            return out
        self.hits += len(held)
        frames, sizes, meta = [], [], []
        for k, comp in held:
            for name, kind, shape, c in comp:
                n = int(np.prod(shape, dtype=np.int64)) * torch.empty(0, dtype=_DTYPES[kind]).element_size()
                frames.append(c)
                sizes.append(n)
                meta.append((k, name, kind, shape))
        dev = _device.require_cuda(self.device)
        buf, spans = decompress_many(frames, sizes, device=dev)
        for (k, name, kind, shape), (off, n) in zip(meta, spans):
            if out[k] is None:
                out[k] = {}
            out[k][name] = buf[off:off + n].view(_DTYPES[kind]).reshape(shape)
        return out

    def __contains__(self, key: str) -> bool:
        with self._lock:
            return key in self._held

    def keys(self) -> list[str]:
        """Held page keys, oldest admission first."""
        with self._lock:
            return list(self._held)

    @property
    def resident_bytes(self) -> int:
        return self._held_bytes

    def summary(self) -> str:
        return (f"warm tier: {self.hits} hits, {self.admits} admits, {self.rejects} rejects, "
                f"{self._held_bytes / 1e6:.0f}MB resident")
