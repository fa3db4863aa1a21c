"""The drop-in seam, exercised with the reference's own host code unmodified.

The reference keeps its WeightCache (runtime/weight_cache.py) and its
consume_expert_batches (runtime/expert_batching.py:13-41); this library
replaces what sits under them: the packed weight store behind
`store.fetch(names) -> (tensors, seconds, bytes)` (the seam at
runtime/weight_cache.py:116-122) and the engine's batch producer.  These
tests import the reference classes from a reference checkout (skipped where
there is none) and drive this library's PackedWeightStore and
iter_expert_batches through them.

The store's device decode needs a GPU; here the store is given a reader that
serves the golden archive's bodies decoded on the CPU (by the test oracle),
so what is tested is the page protocol itself: names, the result tuple,
tensor sizes, errors and the release hook.  The GPU tests cover the same
store with the real batched GPU decode (tests/test_vpack_gpu.py).
"""

from __future__ import annotations

import hashlib
import json
import threading
import time
from concurrent.futures import ThreadPoolExecutor

import numpy as np
import pytest
import torch

from oracle import vpack as ov
from tests.conftest import GOLDEN
from tests.reference_checkout import reference_module


class GoldenReader:
    """Vpack2Reader's fetch contract over the golden archive, decoded on the
    CPU: name -> tensor of the body's dtype and shape, KeyError for a name the
    index does not hold."""

    def __init__(self):
        self.index = json.loads((GOLDEN / "vpack2_tiny.index.json").read_text())
        self.blob = (GOLDEN / "vpack2_tiny.bin").read_bytes()
        self.calls: list[list[str]] = []

    def fetch(self, names, parallel: int = 4):
        self.calls.append(list(names))
        out, nbytes = {}, 0
        for n in names:
            e = self.index[n]  # KeyError for unknown names, as the reader raises
            body = np.frombuffer(self.blob, np.uint8)[e["off"]:e["off"] + e["len"]]
            raw = ov.decode_body(e["head"], body)
            out[n] = torch.from_numpy(raw.copy())
            nbytes += e["len"]
        return out, 0.0, nbytes


@pytest.fixture()
def ref_cache():
    wc = reference_module("runtime.weight_cache")
    cleared = []
    # the one reference-side edit: its device-cache hook calls the CUDA
    # allocator instead of mx.clear_cache (runtime/weight_cache.py:69-73)
    orig = wc._clear_device_cache
    wc._clear_device_cache = lambda: cleared.append(True)
    yield wc, cleared
    wc._clear_device_cache = orig


def _store(tmp_path, reader, **kw):
    from voom_b200.runtime.weight_store import PackedWeightStore

    index = json.loads((GOLDEN / "vpack2_tiny.index.json").read_text())
    names = sorted(index)
    real = {f"model.{n}": n for n in names}
    st = PackedWeightStore(tmp_path, real_name=real, reader_factory=lambda: reader, sleep=lambda s: None, **kw)
    return st, [f"model.{n}" for n in names], real


def test_reference_weight_cache_over_packed_store(tmp_path, ref_cache):
    wc, _ = ref_cache
    decoded = json.loads((GOLDEN / "vpack2_tiny.decoded.json").read_text())["decoded_sha256"]
    reader = GoldenReader()
    store, logical, real = _store(tmp_path, reader)
    cache = wc.WeightCache(store, max_bytes=1 << 30)
    pages = cache.get_many([(f"page{i}", [n]) for i, n in enumerate(logical)])
    for i, n in enumerate(logical):
        t = pages[f"page{i}"][n]
        assert hashlib.sha256(t.numpy().tobytes()).hexdigest() == decoded[real[n]], n
    assert cache.stats.misses == len(logical) and cache.stats.hits == 0
    assert cache.stats.bytes_read == store.archive_bytes > 0
    calls = len(reader.calls)
    again = cache.get("page0", [logical[0]])  # resident: no store call
    assert torch.equal(again[logical[0]], pages["page0"][logical[0]])
    assert len(reader.calls) == calls and cache.stats.hits == 1


def test_reference_cache_eviction_releases_through_the_store_hook(tmp_path, ref_cache):
    wc, cleared = ref_cache
    reader = GoldenReader()
    store, logical, _ = _store(tmp_path, reader)
    released = []
    store.release_cache_pages = lambda names: released.append(tuple(names))
    sizes = {}
    for n in logical[:3]:
        t, _, _ = store.fetch([n])
        sizes[n] = t[n].nbytes
    budget = max(sizes.values()) + 1  # room for one page at a time
    cache = wc.WeightCache(store, max_bytes=budget)
    for i, n in enumerate(logical[:3]):
        cache.get(f"p{i}", [n])
    assert cache.stats.evictions >= 1 and cleared
    assert logical[0] in released[0]  # the oldest page goes first, through the store's hook


def test_reference_cache_refuses_a_short_page(tmp_path, ref_cache):
    wc, _ = ref_cache
    store, logical, _ = _store(tmp_path, GoldenReader())

    class Short:
        def fetch(self, names):
            t, s, b = store.fetch(names[:-1])
            return t, s, b

    cache = wc.WeightCache(Short(), max_bytes=1 << 30)
    with pytest.raises(KeyError, match="incomplete page"):
        cache.get("pair", logical[:2])
    assert cache.stats.incomplete_pages == 1


def test_reference_cache_unknown_name_propagates(tmp_path, ref_cache):
    wc, _ = ref_cache
    store, _, _ = _store(tmp_path, GoldenReader())
    cache = wc.WeightCache(store, max_bytes=1 << 30)
    with pytest.raises(KeyError):
        cache.get("nope", ["model.not.in.the.archive"])
    assert store.retries == 0  # not an I/O failure: no retry


def test_reference_consumer_over_pipelined_producer():
    eb = reference_module("runtime.expert_batching")
    from voom_b200.runtime.expert_batching import BatchStats, iter_expert_batches

    live, peak, lock = [0], [0], threading.Lock()
    alive_pages = []

    def fetch(ids):
        with lock:
            live[0] += 1
            peak[0] = max(peak[0], live[0])
        time.sleep(0.01)
        with lock:
            live[0] -= 1
        return {i: np.zeros(4) for i in ids}

    seen = []
    st = BatchStats()

    def consume(ids, pages):
        seen.append((list(ids), sorted(pages)))
        alive_pages.append(len(pages))

    with ThreadPoolExecutor(max_workers=2) as ex:
        eb.consume_expert_batches(iter_expert_batches(list(range(10)), fetch, fetch_batch=3, compute_batch=2,
                                                      executor=ex, stats=st), consume)
    assert [ids for ids, _ in seen] == [[0, 1], [2], [3, 4], [5], [6, 7], [8], [9]]
    assert seen[0][1] == [0, 1, 2]  # compute chunks share their storage batch's mapping
    assert peak[0] == 1 and st.prefetch_submitted == 4 and st.compute_batches == 7


def test_reference_consumer_error_closes_producer_and_cancels_fetch():
    eb = reference_module("runtime.expert_batching")
    from voom_b200.runtime.expert_batching import iter_expert_batches

    release = threading.Event()
    started = []

    def fetch(ids):
        started.append(list(ids))
        if ids[0] > 0:
            release.wait(2)
        return {i: i for i in ids}

    def boom(ids, pages):
        raise ValueError("compute failed")

    with ThreadPoolExecutor(max_workers=1) as ex:
        with pytest.raises(ValueError, match="compute failed"):
            eb.consume_expert_batches(iter_expert_batches(list(range(6)), fetch, fetch_batch=2, executor=ex), boom)
        release.set()
    assert [0, 1] in started and [4, 5] not in started
