"""Lifetime boundary for streamed expert compute batches
(runtime/expert_batching.py:13-41 of the reference).

The consumer releases batch N (its page mapping) before asking the producer
for batch N+1, so at most about one batch of decoded or compressed expert
pages is alive at a time; a consumer exception closes a generator producer
immediately so its cleanup runs.
"""

from __future__ import annotations

from collections.abc import Callable, Iterable


def consume_expert_batches(batches: Iterable[tuple[list[int], dict]],
                           consume: Callable[[list[int], dict], None]) -> None:
    it = iter(batches)
    try:
        while True:
            try:
                batch_ids, experts = next(it)
            except StopIteration:
                return
            try:
                consume(batch_ids, experts)
            finally:
                # drop this batch before next() runs the producer again
                del experts, batch_ids
    finally:
        close = getattr(it, "close", None)
        if close is not None:
            close()
