"""Packed-archive weight store: the vpack2 leg of vOOM's `WeightStore.fetch`
(runtime/model_loader.py:1464, :1498-1617 of the reference).

`fetch(names)` expands the requested logical names into physical archive
names (deduplicated, request order kept), translates them through the
`real_name` map at the archive boundary (wrapper models expose canonical
names that the archive index stores differently), decodes every body in one
batched GPU decode (`Vpack2Reader.fetch`) and returns `(tensors keyed by
logical name, wall seconds, store-accounted bytes)`.  I/O errors retry the
whole transaction up to four times, reopening the reader after each failure
with exponential backoff, as the reference does for remounted network
storage.  Quantized sidecars and the fast overlay tier are not part of the
BF16 page path and are not mirrored.
"""

from __future__ import annotations

import time
from pathlib import Path

import torch


class PackedWeightStore:
    def __init__(self, model_dir: str | Path, *, real_name: dict[str, str] | None = None,
                 require_hashes: bool = False, device=None, attempts: int = 4, backoff_s: float = 5.0,
                 reader_factory=None, sleep=time.sleep, recover=None):
        from ..formats.packed2 import Vpack2Reader

        self.dir = Path(model_dir)
        self.real_name = dict(real_name or {})
        self.require_hashes = require_hashes
        self.device = device
        self.attempts = int(attempts)
        self.backoff_s = float(backoff_s)
        self._factory = reader_factory or (lambda: Vpack2Reader(self.dir, require_hashes=self.require_hashes,
                                                                 device=self.device))
        self._sleep = sleep
        self._recover = recover
        self.vpack2 = self._factory()
        self.archive_bytes = 0
        self.retries = 0

    def fetch(self, names: list[str]) -> tuple[dict, float, int]:
        t0 = time.perf_counter()
        for attempt in range(self.attempts):
            try:
                physical_names: list[str] = []
                seen: set[str] = set()
                for name in names:
                    if name not in seen:
                        physical_names.append(name)
                        seen.add(name)
                stored = [self.real_name.get(n, n) for n in physical_names]
                fetched, _, nbytes = self.vpack2.fetch(stored)
                self.archive_bytes += nbytes
                out = {logical: fetched[s] for logical, s in zip(physical_names, stored)}
                return out, time.perf_counter() - t0, nbytes
            except (OSError, RuntimeError, EOFError):
                if torch.cuda.is_available() and torch.cuda.is_initialized():
                    torch.cuda.empty_cache()
                if attempt == self.attempts - 1:
                    raise
                self.retries += 1
                if self._recover is not None:
                    self._recover()
                self.vpack2 = self._factory()
                self._sleep(self.backoff_s * (2 ** attempt))
        raise RuntimeError("unreachable")

    def release_cache_pages(self, names) -> None:
        """WeightCache release hook: device pages are freed with their tensors."""
        return None
