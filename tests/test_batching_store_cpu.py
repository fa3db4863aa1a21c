"""Host logic of the expert batch producer (runtime/engine.py
`_iter_expert_batches`) and the packed weight store's retry / name mapping
(runtime/model_loader.py WeightStore.fetch, packed branch), on CPU."""

from __future__ import annotations

import threading
import time
from concurrent.futures import ThreadPoolExecutor

import pytest

from voom_b200.runtime.expert_batching import BatchStats, iter_expert_batches


def test_batches_and_compute_chunks():
    fetched = []

    def fetch(ids):
        fetched.append(list(ids))
        return {i: f"page{i}" for i in ids}

    out = [(ids, sorted(pages)) for ids, pages in iter_expert_batches(list(range(1, 11)), fetch, fetch_batch=4,
                                                                       compute_batch=2)]
    assert fetched == [[1, 2, 3, 4], [5, 6, 7, 8], [9, 10]]
    assert [ids for ids, _ in out] == [[1, 2], [3, 4], [5, 6], [7, 8], [9, 10]]
    assert out[0][1] == [1, 2, 3, 4]  # chunks share their storage batch's mapping


def test_decode_batch_size_for_single_position():
    fetched = []
    list(iter_expert_batches(list(range(6)), lambda ids: fetched.append(ids) or {}, fetch_batch=6,
                             decode_fetch_batch=2, single_position=True))
    assert fetched == [[0, 1], [2, 3], [4, 5]]


class Governor:
    def __init__(self, admit):
        self.admit = admit
        self.calls = []

    def admissible_units(self, *, unit_bytes, fixed_bytes, max_units, margin):
        self.calls.append((unit_bytes, fixed_bytes, max_units, margin))
        return min(self.admit, max_units)


def test_governor_clamp_keeps_compute_boundaries():
    fetched = []
    st = BatchStats()
    g = Governor(6)
    list(iter_expert_batches(list(range(16)), lambda ids: fetched.append(ids) or {}, fetch_batch=8,
                             compute_batch=4, governor=g, page_bytes=10, fixed_bytes=3, margin=1, stats=st))
    # 6 admitted of 8 -> rounded down to the compute boundary 4 (never 4 + 2)
    assert [len(b) for b in fetched] == [4, 4, 4, 4]
    # the last batch (4 left) is admitted in full: 3 clamps
    assert st.adaptive_clamps == 3 and st.min_adaptive_batch == 4
    assert g.calls[0] == (10, 3, 8, 1)
    fetched.clear()
    list(iter_expert_batches(list(range(5)), lambda ids: fetched.append(ids) or {}, fetch_batch=8,
                             compute_batch=4, governor=Governor(3)))
    assert [len(b) for b in fetched] == [3, 2]  # below one compute batch: taken as admitted


def test_pipelined_one_fetch_in_flight_and_order():
    live, peak, lock = [0], [0], threading.Lock()
    order = []

    def fetch(ids):
        with lock:
            live[0] += 1
            peak[0] = max(peak[0], live[0])
        time.sleep(0.01)
        with lock:
            live[0] -= 1
        order.append(ids)
        return {i: i for i in ids}

    st = BatchStats()
    seen = []
    with ThreadPoolExecutor(max_workers=2) as ex:
        gen = iter_expert_batches(list(range(10)), fetch, fetch_batch=3, executor=ex, stats=st)
        for ids, pages in gen:
            seen.append((ids, sorted(pages)))
            del pages
    assert [ids for ids, _ in seen] == [[0, 1, 2], [3, 4, 5], [6, 7, 8], [9]]
    assert order == [[0, 1, 2], [3, 4, 5], [6, 7, 8], [9]]
    assert peak[0] == 1 and st.prefetch_submitted == 4


def test_pipelined_close_cancels_pending_fetch():
    release = threading.Event()
    started = []

    def fetch(ids):
        started.append(ids)
        if ids[0] > 0:
            release.wait(2)
        return {i: i for i in ids}

    with ThreadPoolExecutor(max_workers=1) as ex:
        gen = iter_expert_batches(list(range(6)), fetch, fetch_batch=2, executor=ex)
        ids, pages = next(gen)  # batch 1 fetch is now submitted
        assert ids == [0, 1]
        # batch 2 is queued behind the running batch-1 fetch; closing cancels it
        gen.close()
        release.set()
    assert [0, 1] in started and [4, 5] not in started


class FakeReader:
    def __init__(self, plan):
        self.plan = plan  # shared list of outcomes

    def fetch(self, names):
        outcome = self.plan.pop(0)
        if isinstance(outcome, Exception):
            raise outcome
        return {n: f"T({n})" for n in names}, 0.0, 10 * len(names)


def test_store_retries_reopen_and_backoff(tmp_path):
    from voom_b200.runtime.weight_store import PackedWeightStore

    plan = [OSError("stale mount"), EOFError("short read"), "ok"]
    opened, sleeps, recovered = [], [], []

    def factory():
        opened.append(True)
        return FakeReader(plan)

    st = PackedWeightStore(tmp_path, real_name={"model.a": "language_model.a"}, reader_factory=factory,
                           sleep=sleeps.append, recover=lambda: recovered.append(True))
    out, secs, nbytes = st.fetch(["model.a", "b", "model.a"])
    assert out == {"model.a": "T(language_model.a)", "b": "T(b)"}  # deduplicated, translated back
    assert nbytes == 20 and st.retries == 2
    assert sleeps == [5.0, 10.0] and len(recovered) == 2 and len(opened) == 3


def test_store_gives_up_after_four_attempts(tmp_path):
    from voom_b200.runtime.weight_store import PackedWeightStore

    plan = [RuntimeError("x")] * 4
    st = PackedWeightStore(tmp_path, reader_factory=lambda: FakeReader(plan), sleep=lambda s: None)
    with pytest.raises(RuntimeError):
        st.fetch(["a"])
    assert st.retries == 3 and plan == []


def test_store_other_errors_are_not_retried(tmp_path):
    from voom_b200.runtime.weight_store import PackedWeightStore

    plan = [KeyError("missing tensor"), "ok"]
    st = PackedWeightStore(tmp_path, reader_factory=lambda: FakeReader(plan), sleep=lambda s: None)
    with pytest.raises(KeyError):
        st.fetch(["a"])
    assert st.retries == 0
