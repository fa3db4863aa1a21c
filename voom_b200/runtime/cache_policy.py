"""Eviction order shared by the weight cache and any capacity simulator.

Same policy as runtime/cache_policy.py:42-60 of the reference: pinned pages
are never victims; ordinary pages go first, then pages that were prefetched
and not yet demanded; within each class the lowest cumulative frequency goes
first and recency (position in the LRU order) breaks ties.
"""

from __future__ import annotations

from typing import Hashable, Iterable, Mapping, NamedTuple, Sequence


class CacheEntry(NamedTuple):
    key: Hashable
    pinned: bool = False
    prefetched: bool = False


def rank_victims(entries: Iterable[CacheEntry], frequencies: Mapping[Hashable, int]) -> list[Hashable]:
    """Evictable keys in removal order; `entries` oldest first."""
    ordinary, prefetched = [], []
    for age, entry in enumerate(entries):
        if entry.pinned:
            continue
        (prefetched if entry.prefetched else ordinary).append((int(frequencies.get(entry.key, 0)), age, entry.key))
    ordinary.sort(key=lambda t: (t[0], t[1]))
    prefetched.sort(key=lambda t: (t[0], t[1]))
    return [k for _, _, k in ordinary] + [k for _, _, k in prefetched]


def plan_pinned_prefix(layer_bytes: Sequence[int], budget_bytes: int, *, reserve_bytes: int = 0) -> int:
    """Largest n such that pinning layers [0, n) plus the largest remaining
    layer (streamed through) plus `reserve_bytes` fits in the budget
    (runtime/cache_policy.py:63-99)."""
    sizes = [max(0, int(v)) for v in layer_bytes]
    budget, reserve = max(0, int(budget_bytes)), max(0, int(reserve_bytes))
    best, prefix = 0, 0
    for n in range(1, len(sizes) + 1):
        prefix += sizes[n - 1]
        if prefix + max(sizes[n:], default=0) + reserve <= budget:
            best = n
    return best
