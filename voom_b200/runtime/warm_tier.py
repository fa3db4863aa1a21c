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
from collections import OrderedDict
from concurrent.futures import ThreadPoolExecutor

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


class WarmTier:
    MIN_RATIO = 1.15  # pages that barely compress are not admitted

    def __init__(self, max_bytes: int, device=None, threads: int = 8):
        self.max_bytes = max_bytes
        self.device = device
        self.threads = max(1, int(threads))
        self._store: OrderedDict[str, list] = OrderedDict()  # key -> [(name, kind, shape, frame)]
        self._bytes = 0
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
        blobs = _page_to_blobs(tensors)
        if blobs is None:
            self.rejects += 1
            return
        if self.device is None:
            for t in tensors.values():
                if t.is_cuda:
                    self.device = t.device
                    break
        frames = self._compress([raw for *_, raw in blobs])
        raw_total = sum(raw.size for *_, raw in blobs)
        comp_total = sum(len(c) for c in frames)
        if raw_total / max(comp_total, 1) < self.MIN_RATIO:
            self.rejects += 1
            return
        comp = [(name, kind, shape, c) for (name, kind, shape, _), c in zip(blobs, frames)]
        with self._lock:
            if key in self._store:
                return
            self._store[key] = comp
            self._bytes += comp_total
            self.admits += 1
            while self._bytes > self.max_bytes and self._store:
                _, old = self._store.popitem(last=False)
                self._bytes -= sum(len(c) for *_, c in old)

    def _pop(self, key: str) -> list | None:
        with self._lock:
            comp = self._store.pop(key, None)
            if comp is not None:
                self._bytes -= sum(len(c) for *_, c in comp)
        return comp

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
            return key in self._store

    @property
    def resident_bytes(self) -> int:
        return self._bytes

    def summary(self) -> str:
        return (f"warm tier: {self.hits} hits, {self.admits} admits, {self.rejects} rejects, "
                f"{self._bytes / 1e6:.0f}MB resident")
