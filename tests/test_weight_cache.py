"""WeightCache / cache policy / expert batching host logic, restating the
reference's tests (tests/test_expert_fetch_batch.py, tests/test_weight_cache_
eviction.py, tests/test_expert_batching.py pure cases) against voom_b200.
Fault injection is on the host: a store that raises once."""

from __future__ import annotations

import gc
import random
import threading
import time
import weakref
from collections import OrderedDict
from concurrent.futures import ThreadPoolExecutor
from dataclasses import dataclass

import pytest

import voom_b200.runtime.weight_cache as cache_module
from voom_b200.runtime.expert_batching import consume_expert_batches
from voom_b200.runtime.weight_cache import WeightCache


@dataclass(frozen=True)
class FakeTensor:
    name: str
    nbytes: int = 10


class FakeStore:
    def __init__(self, *, delay=0.0, nbytes=10):
        self.delay = delay
        self.nbytes = nbytes
        self.calls: list[list[str]] = []
        self.released = []
        self._lock = threading.Lock()

    def fetch(self, names):
        with self._lock:
            self.calls.append(list(names))
        if self.delay:
            time.sleep(self.delay)
        t = {n: FakeTensor(n, self.nbytes) for n in names}
        return t, 0.0, sum(x.nbytes for x in t.values())

    def release_cache_pages(self, names):
        self.released.append(tuple(names))


class FailOnceStore(FakeStore):
    def __init__(self, **kw):
        super().__init__(**kw)
        self.fail = True

    def fetch(self, names):
        if self.fail:
            self.fail = False
            self.calls.append(list(names))
            raise OSError("injected first-batch read failure")
        return super().fetch(names)


class RecordingWarmTier:
    def __init__(self):
        self.admitted = []

    def take(self, _key):
        return None

    def admit(self, key, _tensors):
        self.admitted.append(key)


@pytest.fixture(autouse=True)
def no_device_clear(monkeypatch):
    clears = []
    monkeypatch.setattr(cache_module, "_clear_device_cache", lambda: clears.append(True))
    return clears


def items(n):
    return [(f"expert.{i}", [f"expert.{i}.w"]) for i in range(n)]


def test_zero_batch_size_single_fetch():
    store = FakeStore(nbytes=4096)
    cache = WeightCache(store, max_bytes=10_000_000)
    res = cache.get_many(items(5))
    assert len(store.calls) == 1 and len(store.calls[0]) == 5
    assert set(res) == {k for k, _ in items(5)}


def test_sub_batching_bounds_fetch_size():
    store = FakeStore(nbytes=4096)
    cache = WeightCache(store, max_bytes=10_000_000, max_fetch_batch=2)
    res = cache.get_many(items(5))
    assert len(store.calls) == 3 and all(len(c) <= 2 for c in store.calls)
    assert set(res) == {k for k, _ in items(5)}


def test_sub_batching_evicts_between_fetches():
    store = FakeStore(nbytes=4096)
    cache = WeightCache(store, max_bytes=10_000, max_fetch_batch=2)
    cache.get_many(items(10))
    assert cache.total_bytes <= 10_000 and len(store.calls) == 5


def test_failed_batch_releases_every_owned_inflight_key():
    store = FailOnceStore(nbytes=4096)
    cache = WeightCache(store, max_bytes=10_000_000, max_fetch_batch=2)
    with pytest.raises(OSError, match="injected"):
        cache.get_many(items(7))
    assert not any(cache.inflight(k) for k, _ in items(7))
    assert set(cache.get_many(items(7))) == {k for k, _ in items(7)}


def test_incomplete_page_is_refused():
    class ShortStore(FakeStore):
        def fetch(self, names):
            t, s, n = super().fetch(names)
            t.pop(names[-1])
            return t, s, n

    cache = WeightCache(ShortStore(), max_bytes=1000)
    with pytest.raises(KeyError, match="incomplete page"):
        cache.get("p", ["a", "b"])
    assert cache.stats.incomplete_pages == 1 and not cache.inflight("p")


def test_consumer_releases_batch_before_next():
    class Payload:
        pass

    seen = []

    def batches():
        previous = None
        for i in range(4):
            if previous is not None:
                gc.collect()
                assert previous() is None, f"batch {i - 1} survived into fetch {i}"
            payload = Payload()
            previous = weakref.ref(payload)
            yield [i], {i: payload}
            del payload

    consume_expert_batches(batches(), lambda ids, pages: seen.append(ids[0]))
    assert seen == [0, 1, 2, 3]


def test_consumer_exception_closes_producer():
    class Payload:
        pass

    state = {"closed": False, "payload": None}

    def batches():
        try:
            for i in range(3):
                payload = Payload()
                state["payload"] = weakref.ref(payload)
                yield [i], {i: payload}
                del payload
        finally:
            state["closed"] = True

    def boom(ids, pages):
        raise RuntimeError("injected compute")

    with pytest.raises(RuntimeError, match="injected compute"):
        consume_expert_batches(batches(), boom)
    gc.collect()
    assert state["closed"] and state["payload"]() is None


def test_prepare_for_evicts_before_known_size_fetch():
    cache = WeightCache(FakeStore(nbytes=4096), max_bytes=12_000)
    cache.get("expert.0", ["expert.0.w"])
    cache.get("expert.1", ["expert.1.w"])
    assert cache.total_bytes == 8192
    cache.prepare_for(8000)
    assert cache.total_bytes <= 4000 and cache.stats.evictions == 2


def test_one_pass_eviction_policy_order(no_device_clear):
    warm = RecordingWarmTier()
    cache = WeightCache(FakeStore(), max_bytes=1_000, warm=warm)
    cache.pin("pin", ["pin.weight"])
    cache.get("prefetch-old", ["prefetch-old.weight"], origin="prefetch")
    cache.get("demand-old", ["demand-old.weight"])
    cache.get("demand-new", ["demand-new.weight"])
    cache.get("prefetch-new", ["prefetch-new.weight"], origin="prefetch")
    cache.freq["demand-old"] = 5
    cache.freq["demand-new"] = 1
    cache.max_bytes = 25
    with cache._lock:
        cache._evict_locked()
    assert warm.admitted == ["demand-new", "demand-old", "prefetch-old"]
    assert cache.resident_keys == ["pin", "prefetch-new"]
    assert cache.total_bytes == 20 and cache.stats.evictions == 3
    assert no_device_clear == [True]
    assert cache.would_fit(5) and not cache.would_fit(6)


def _legacy_eviction(pages, frequencies, budget):
    pages = OrderedDict(pages)
    victims = []
    while sum(p.nbytes for p in pages.values()) > budget:
        cands = [(frequencies.get(k, 0), age, k) for age, (k, p) in enumerate(pages.items())
                 if not p.pinned and p.origin != "prefetch"]
        if not cands:
            cands = [(frequencies.get(k, 0), age, k) for age, (k, p) in enumerate(pages.items()) if not p.pinned]
        if not cands:
            break
        v = min(cands)[2]
        victims.append(v)
        del pages[v]
    return list(pages), victims


def test_eviction_matches_legacy_policy_random(no_device_clear):
    for seed in range(100):
        rng = random.Random(seed)
        warm = RecordingWarmTier()
        cache = WeightCache(FakeStore(), max_bytes=rng.randrange(0, 300), warm=warm)
        with cache._lock:
            for index in range(rng.randrange(1, 32)):
                key = f"page-{index}"
                page = cache_module.WeightPage(key, {key: FakeTensor(key, rng.randrange(1, 40))}, 0,
                                               pinned=rng.random() < 0.15,
                                               origin="prefetch" if rng.random() < 0.3 else "demand")
                page.nbytes = next(iter(page.tensors.values())).nbytes
                cache._put_page_locked(page)
                cache.freq[key] = rng.randrange(0, 12)
            keys, victims = _legacy_eviction(cache._pages, cache.freq, cache.max_bytes)
            before = len(no_device_clear)
            cache._evict_locked()
        assert cache.resident_keys == keys and warm.admitted == victims
        assert cache.total_bytes == sum(p.nbytes for p in cache._pages.values())
        assert len(no_device_clear) - before == bool(victims)


def test_trim_to_keeps_budget(no_device_clear):
    store = FakeStore()
    cache = WeightCache(store, max_bytes=100)
    cache.pin("pin", ["pin.weight"])
    cache.get("old", ["old.weight"])
    cache.get("new", ["new.weight"])
    assert cache.trim_to(20) == 10
    assert cache.resident_keys == ["pin", "new"] and cache.max_bytes == 100
    assert store.released == [("old.weight",)] and no_device_clear == [True]


def test_prefetch_hit_reserved_accounting():
    cache = WeightCache(FakeStore(), max_bytes=100)
    t = cache.get("page", ["page.weight"], origin="prefetch")
    assert not cache.would_fit(95) and cache.total_bytes == 10
    assert cache.get("page", ["page.weight"], origin="demand") is t
    assert cache.would_fit(95) and cache.stats.prefetch_hits == 1


def test_replacing_pinned_page_counters():
    cache = WeightCache(FakeStore(), max_bytes=100)
    cache.pin("shared", ["first"])
    cache.pin("shared", ["second", "third"])
    assert cache.total_bytes == 20 and cache.resident_keys == ["shared"]
    assert not cache.would_fit(81) and cache.would_fit(80)


def test_clear_releases_once(no_device_clear):
    cache = WeightCache(FakeStore(), max_bytes=100)
    cache.pin("pinned", ["pinned.weight"])
    cache.get("prefetched", ["prefetched.weight"], origin="prefetch")
    cache.get("demand", ["demand.weight"])
    cache.clear()
    assert cache.total_bytes == 0 and cache.resident_keys == [] and cache.would_fit(100)
    assert no_device_clear == [True]
    assert cache.store.released == [("pinned.weight", "prefetched.weight", "demand.weight")]


def test_clear_refuses_inflight():
    cache = WeightCache(FakeStore(), max_bytes=100)
    with cache._lock:
        cache._inflight["loading"] = threading.Event()
    with pytest.raises(RuntimeError, match="fetches are in flight"):
        cache.clear()


def test_discard_after_budget_eviction(no_device_clear):
    cache = WeightCache(FakeStore(), max_bytes=5)
    assert cache.get("layer.0", ["model.layers.0.weight"])
    assert not cache.contains("layer.0")
    assert cache.discard("layer.0", ["model.layers.0.weight"]) is False
    assert cache.store.released[-1] == ("model.layers.0.weight",)
    assert len(no_device_clear) == 2


def test_concurrent_same_key_single_fetch():
    store = FakeStore(delay=0.02)
    cache = WeightCache(store, max_bytes=100)
    with ThreadPoolExecutor(max_workers=12) as ex:
        results = list(ex.map(lambda _i: cache.get("shared", ["shared.weight"]), range(24)))
    assert len(store.calls) == 1 and all(r is results[0] for r in results)
    assert cache.stats.misses == 1 and cache.stats.hits == 23


def test_rank_victims_and_pinned_prefix():
    from voom_b200.runtime.cache_policy import CacheEntry, plan_pinned_prefix, rank_victims

    ents = [CacheEntry("a"), CacheEntry("b", prefetched=True), CacheEntry("c", pinned=True), CacheEntry("d")]
    assert rank_victims(ents, {"a": 2, "d": 1}) == ["d", "a", "b"]
    assert plan_pinned_prefix([10, 10, 10, 10], 35) == 2
    assert plan_pinned_prefix([10, 10], 5) == 0
