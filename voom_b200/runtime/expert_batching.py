"""Producer of streamed expert compute batches (runtime/engine.py
`_iter_expert_batches`, :3628-3767 of the reference).

The batches feed the reference's own `consume_expert_batches`
(runtime/expert_batching.py:13-41), which stays at its call sites unchanged:
it releases batch N (its page mapping) before asking this producer for batch
N+1, so at most about one batch of expert pages is alive at a time, and a
consumer exception closes the generator so its cleanup runs.
"""

from __future__ import annotations

import time
from collections.abc import Callable


class BatchStats:
    """Counters the reference engine keeps for expert batching."""

    def __init__(self) -> None:
        self.adaptive_clamps = 0
        self.min_adaptive_batch = 0
        self.compute_batches = 0
        self.max_experts_per_compute_batch = 0
        self.prefetch_submitted = 0
        self.prefetch_wait_s = 0.0
        self.prefetch_hidden_s = 0.0


def iter_expert_batches(expert_ids: list[int], fetch: Callable[[list[int]], dict], *,
                        fetch_batch: int = 0, compute_batch: int = 0, decode_fetch_batch: int = 0,
                        single_position: bool = False, governor=None, page_bytes: int = 0,
                        fixed_bytes: int = 0, margin: int = 0, executor=None,
                        stats: BatchStats | None = None):
    """Bounded expert pages for immediate compute and release
    (runtime/engine.py `_iter_expert_batches`, :3628-3767 of the reference).

    The routed union `expert_ids` is cut into storage batches of `fetch_batch`
    experts (`decode_fetch_batch` when every routed expert serves one token
    position); a `governor` with `admissible_units(unit_bytes, fixed_bytes,
    max_units, margin)` may shrink a batch under memory pressure, but a batch
    larger than `compute_batch` only shrinks to a multiple of it, so the
    arithmetic grouping (and with it the floating accumulation order) stays the
    validated one.  Each storage batch is fetched with `fetch(ids)` and yielded
    as `(compute_ids, pages)` chunks of `compute_batch` experts sharing the
    batch's page mapping.  With an `executor`, batch N+1 is fetched while batch
    N computes, with at most one fetch in flight; closing the generator cancels
    it.
    """
    st = stats if stats is not None else BatchStats()
    fetch_size = (decode_fetch_batch if single_position and decode_fetch_batch > 0 else fetch_batch) \
        or len(expert_ids) or 1
    compute_size = compute_batch or fetch_size

    def plan_batch(start: int) -> tuple[list[int], int]:
        remaining = len(expert_ids) - start
        size = min(fetch_size, remaining)
        if governor is not None and size > 1:
            admitted = governor.admissible_units(unit_bytes=page_bytes, fixed_bytes=fixed_bytes,
                                                 max_units=size, margin=margin)
            if admitted < size:
                st.adaptive_clamps += 1
            size = admitted
            if remaining > compute_size and size >= compute_size and fetch_size > compute_size:
                size = max(compute_size, (size // compute_size) * compute_size)
            st.min_adaptive_batch = size if st.min_adaptive_batch == 0 else min(st.min_adaptive_batch, size)
        size = max(1, size)
        return expert_ids[start:start + size], start + size

    def compute_chunks(batch_ids: list[int], pages: dict):
        for off in range(0, len(batch_ids), compute_size):
            ids = batch_ids[off:off + compute_size]
            st.compute_batches += 1
            st.max_experts_per_compute_batch = max(st.max_experts_per_compute_batch, len(ids))
            yield ids, pages

    def timed_fetch(ids: list[int]):
        t0 = time.perf_counter()
        pages = fetch(ids)
        return pages, time.perf_counter() - t0

    if not expert_ids:
        return iter(())
    if executor is None:
        def synchronous():
            start = 0
            while start < len(expert_ids):
                ids, start = plan_batch(start)
                pages = fetch(ids)
                yield from compute_chunks(ids, pages)
                del pages
        return synchronous()

    first_ids, first_start = plan_batch(0)
    first_future = executor.submit(timed_fetch, first_ids)
    st.prefetch_submitted += 1

    def pipelined():
        cur_ids, cur_start, future = first_ids, first_start, first_future
        try:
            t0 = time.perf_counter()
            pages, fetch_s = future.result()
            wait = time.perf_counter() - t0
            st.prefetch_wait_s += wait
            st.prefetch_hidden_s += max(0.0, fetch_s - wait)
            future = None
            while True:
                if cur_start < len(expert_ids):
                    next_ids, next_start = plan_batch(cur_start)
                    future = executor.submit(timed_fetch, next_ids)
                    st.prefetch_submitted += 1
                yield from compute_chunks(cur_ids, pages)
                del pages  # the consumer released its reference before resuming us
                if future is None:
                    return
                t0 = time.perf_counter()
                pages, fetch_s = future.result()
                wait = time.perf_counter() - t0
                st.prefetch_wait_s += wait
                st.prefetch_hidden_s += max(0.0, fetch_s - wait)
                cur_ids, cur_start, future = next_ids, next_start, None
        finally:
            if future is not None:
                future.cancel()

    return pipelined()
