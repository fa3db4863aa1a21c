"""WeightCache: byte-budgeted, pin-aware cache of materialised weight pages.

Same contract as vOOM's runtime/weight_cache.py (:27-476): a page is a dict of
tensors that live and die together (a layer, or one expert's projections);
misses are fetched from the store (warm tier first), concurrent requests for
the same key share one fetch, `get_many` fetches every missing page of a
routed expert set in one store call (sub-batched by max_fetch_batch) and
releases every in-flight key it owns on failure, short pages are refused,
and eviction follows cache_policy.rank_victims (LFU, recency tie-break,
prefetched pages last, pinned never).  Here the tensors are CUDA tensors
decoded by the GPU page decoders; the device-cache release hook calls
torch.cuda.empty_cache().

Reference interface replaced: runtime/weight_cache.py:27-476.
"""

from __future__ import annotations

import threading
from collections import OrderedDict
from dataclasses import dataclass

from .cache_policy import CacheEntry, rank_victims


@dataclass
class WeightPage:
    key: str
    tensors: dict
    nbytes: int
    pinned: bool = False
    origin: str = "demand"  # "demand" | "prefetch" | "pin"
    hits: int = 0


@dataclass
class CacheStats:
    hits: int = 0
    misses: int = 0
    evictions: int = 0
    prefetch_hits: int = 0
    disk_s: float = 0.0
    bytes_read: int = 0
    incomplete_pages: int = 0

    def summary(self) -> str:
        total = self.hits + self.misses
        rate = self.hits / total * 100 if total else 0.0
        short = f", {self.incomplete_pages} INCOMPLETE PAGES" if self.incomplete_pages else ""
        return (f"cache: {self.hits} hits / {self.misses} misses ({rate:.0f}% hit rate, "
                f"{self.prefetch_hits} via prefetch), {self.evictions} evictions, "
                f"store-accounted {self.bytes_read / 1e6:.0f}MB in {self.disk_s:.2f}s{short}")


def _tensor_bytes(t) -> int:
    return int(t.nbytes)


def _clear_device_cache() -> None:
    """Return cached device memory after pages are dropped."""
    import torch

    if torch.cuda.is_available() and torch.cuda.is_initialized():
        torch.cuda.empty_cache()


class WeightCache:
    def __init__(self, store, max_bytes: int, transform=None, warm=None, max_fetch_batch: int = 0):
        self.store = store
        self.max_bytes = max_bytes
        self.transform = transform
        self.warm = warm
        self.max_fetch_batch = max_fetch_batch
        self._pages: OrderedDict[str, WeightPage] = OrderedDict()
        self._total_bytes = 0
        self._reserved_bytes = 0
        self._lock = threading.Lock()
        self._inflight: dict[str, threading.Event] = {}
        self.stats = CacheStats()
        self.freq: dict[str, int] = {}

    # ------------------------------------------------------------- public
    def pin(self, key: str, names: list[str]) -> dict:
        tensors, secs, nbytes = self._fetch(names)
        with self._lock:
            self.stats.disk_s += secs
            self.stats.bytes_read += nbytes
            self._put_page_locked(WeightPage(key, tensors, self._bytes(tensors), pinned=True, origin="pin"))
        return tensors

    def _fetch(self, names: list[str], *, apply_transform: bool = True):
        tensors, secs, nbytes = self.store.fetch(names)
        self._require_complete(names, tensors, "store fetch")
        if self.transform and apply_transform:
            tensors = {n: self.transform(n, a) for n, a in tensors.items()}
            self._require_complete(names, tensors, "cache transform")
        return tensors, secs, nbytes

    def _require_complete(self, names, tensors, source: str) -> None:
        missing = [n for n in names if n not in tensors]
        if missing:
            with self._lock:
                self.stats.incomplete_pages += 1
            raise KeyError(f"{source} returned an incomplete page: {len(missing)} of {len(names)} tensors "
                           f"missing, first {missing[:3]}")

    @staticmethod
    def _bytes(tensors: dict) -> int:
        return sum(_tensor_bytes(t) for t in tensors.values())

    def _hit_locked(self, key: str, page: WeightPage, origin: str) -> None:
        self._pages.move_to_end(key)
        if origin == "demand":
            self.stats.hits += 1
            page.hits += 1
            if page.origin == "prefetch":
                self.stats.prefetch_hits += 1
                self._mark_demand_locked(page)

    def get(self, key: str, names: list[str], origin: str = "demand", *, apply_transform: bool = True) -> dict:
        while True:
            with self._lock:
                if origin == "demand":
                    self.freq[key] = self.freq.get(key, 0) + 1
                page = self._pages.get(key)
                if page is not None:
                    self._hit_locked(key, page, origin)
                    return page.tensors
                waiting = self._inflight.get(key)
                if waiting is None:
                    self._inflight[key] = threading.Event()
                    break
            waiting.wait()  # another thread is loading this key
        try:
            tensors = self.warm.take(key) if self.warm is not None else None
            if tensors is not None:
                self._require_complete(names, tensors, "warm tier")
                secs, nbytes = 0.0, 0
            else:
                tensors, secs, nbytes = self._fetch(names, apply_transform=apply_transform)
            with self._lock:
                if origin == "demand":
                    self.stats.misses += 1
                self.stats.disk_s += secs
                self.stats.bytes_read += nbytes
                self._put_page_locked(WeightPage(key, tensors, self._bytes(tensors), origin=origin))
                self._evict_locked()
            return tensors
        finally:
            with self._lock:
                self._inflight.pop(key).set()

    def get_many(self, items: list[tuple[str, list[str]]], origin: str = "demand") -> dict[str, dict]:
        result: dict[str, dict] = {}
        missing: list[tuple[str, list[str]]] = []
        owned: set[str] = set()
        with self._lock:
            for key, names in items:
                self.freq[key] = self.freq.get(key, 0) + 1
                page = self._pages.get(key)
                if page is not None:
                    self._hit_locked(key, page, "demand")
                    result[key] = page.tensors
                elif key not in self._inflight:
                    missing.append((key, names))
                    self._inflight[key] = threading.Event()
                    owned.add(key)

        def release(keys) -> None:
            with self._lock:
                for key in keys:
                    if key not in owned:
                        continue
                    owned.discard(key)
                    event = self._inflight.pop(key, None)
                    if event is not None:
                        event.set()

        try:
            if missing and self.warm is not None:
                still = []
                for key, names in missing:
                    t = self.warm.take(key)
                    if t is None:
                        still.append((key, names))
                        continue
                    self._require_complete(names, t, "warm tier")
                    with self._lock:
                        self._put_page_locked(WeightPage(key, t, self._bytes(t), origin="demand"))
                        self._evict_locked()
                    result[key] = t
                    release((key,))
                missing = still
            step = self.max_fetch_batch if self.max_fetch_batch > 0 else len(missing)
            for start in range(0, len(missing), max(step, 1)):
                batch = missing[start:start + step]
                try:
                    tensors, secs, nbytes = self._fetch([n for _, names in batch for n in names])
                    with self._lock:
                        self.stats.misses += len(batch)
                        self.stats.disk_s += secs
                        self.stats.bytes_read += nbytes
                        for key, names in batch:
                            page_tensors = {n: tensors[n] for n in names}
                            self._put_page_locked(WeightPage(key, page_tensors, self._bytes(page_tensors),
                                                             origin=origin))
                            result[key] = page_tensors
                        self._evict_locked()
                finally:
                    release([k for k, _ in batch])
            for key, names in items:
                if key not in result:  # was being loaded by another thread
                    result[key] = self.get(key, names, origin=origin)
            return result
        finally:
            release(tuple(owned))

    def contains(self, key: str) -> bool:
        with self._lock:
            return key in self._pages

    def inflight(self, key: str) -> bool:
        with self._lock:
            return key in self._inflight

    @property
    def total_bytes(self) -> int:
        with self._lock:
            return self._total_bytes

    @property
    def resident_keys(self) -> list[str]:
        with self._lock:
            return list(self._pages)

    def clear(self) -> None:
        released: list[str] = []
        with self._lock:
            if self._inflight:
                raise RuntimeError("cannot clear WeightCache while fetches are in flight")
            for page in self._pages.values():
                released.extend(page.tensors)
            self._pages.clear()
            self._total_bytes = 0
            self._reserved_bytes = 0
        _clear_device_cache()
        self._release(released)

    def discard(self, key: str, names=()) -> bool:
        released = list(names)
        removed = False
        with self._lock:
            page = self._pages.get(key)
            if page is not None:
                if page.pinned:
                    return False
                if not released:
                    released.extend(page.tensors)
                self._remove_page_locked(key)
                self.stats.evictions += 1
                removed = True
        _clear_device_cache()
        self._release(released)
        return removed

    def would_fit(self, nbytes: int) -> bool:
        with self._lock:
            return self._reserved_bytes + nbytes <= self.max_bytes

    def prepare_for(self, incoming_bytes: int) -> None:
        with self._lock:
            self._evict_to_locked(max(0, self.max_bytes - max(0, int(incoming_bytes))))

    def trim_to(self, target_bytes: int) -> int:
        with self._lock:
            before = self._total_bytes
            self._evict_to_locked(max(0, int(target_bytes)))
            return before - self._total_bytes

    # ---------------------------------------------------------- internals
    @staticmethod
    def _reserved(page: WeightPage) -> bool:
        return page.pinned or page.origin == "prefetch"

    def _release(self, names) -> None:
        release = getattr(self.store, "release_cache_pages", None)
        if release is not None and names:
            release(tuple(names))

    def _put_page_locked(self, page: WeightPage) -> None:
        old = self._pages.get(page.key)
        if old is not None:
            self._total_bytes -= old.nbytes
            if self._reserved(old):
                self._reserved_bytes -= old.nbytes
        self._pages[page.key] = page
        self._total_bytes += page.nbytes
        if self._reserved(page):
            self._reserved_bytes += page.nbytes

    def _remove_page_locked(self, key: str) -> WeightPage:
        page = self._pages.pop(key)
        self._total_bytes -= page.nbytes
        if self._reserved(page):
            self._reserved_bytes -= page.nbytes
        return page

    def _mark_demand_locked(self, page: WeightPage) -> None:
        was = self._reserved(page)
        page.origin = "demand"
        if was and not self._reserved(page):
            self._reserved_bytes -= page.nbytes

    def _evict_locked(self) -> None:
        self._evict_to_locked(self.max_bytes)

    def _evict_to_locked(self, target: int) -> None:
        target = max(0, int(target))
        if self._total_bytes <= target:
            return
        order = rank_victims((CacheEntry(k, p.pinned, p.origin == "prefetch") for k, p in self._pages.items()),
                             self.freq)
        evicted = False
        released: list[str] = []
        try:
            for key in order:
                if self._total_bytes <= target:
                    break
                page = self._pages[key]
                if self.warm is not None:
                    self.warm.admit(key, page.tensors)
                else:
                    released.extend(page.tensors)
                self._remove_page_locked(key)
                self.stats.evictions += 1
                evicted = True
        finally:
            if evicted:
                _clear_device_cache()
                self._release(released)
