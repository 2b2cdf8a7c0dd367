"""Host-side placement of independent sequences on GPUs (one process per GPU, no collective).

Batched decode of many sequences is bound by each step's KV-cache read, so a rank's step time
grows with the sum of its sequences' contexts; the job's step time is that of the slowest rank.
``balanced_shards`` splits the sequences so that every rank holds the same number of them
(the weight stream and the per-row work of the linears) and close to the same total context.
Every rank computes the same placement from the same lengths, so no exchange is needed.
"""
from __future__ import annotations

import heapq
from typing import Sequence


def balanced_shards(lengths: Sequence[int], world: int) -> list[list[int]]:
    """Indices of ``lengths`` per rank: counts differ by at most one, totals balanced greedily.

    Longest first, each sequence goes to the rank with the smallest total among the ranks that
    still have room for their share of the count (ties: the lower rank).  Within a rank the
    indices are ascending.  Deterministic for given inputs.
    """
    if world <= 0:
        raise ValueError("world must be positive")
    n = len(lengths)
    cap = [n // world + (1 if r < n % world else 0) for r in range(world)]
    order = sorted(range(n), key=lambda i: (-int(lengths[i]), i))
    heap = [(0, r) for r in range(world)]  # (total context, rank)
    parts: list[list[int]] = [[] for _ in range(world)]
    for i in order:
        full = []
        while True:
            total, r = heapq.heappop(heap)
            if len(parts[r]) < cap[r]:
                break
            full.append((total, r))
        parts[r].append(i)
        heapq.heappush(heap, (total + int(lengths[i]), r))
        for item in full:  # ranks at their count stay out of later rounds too, but keep the heap whole
            heapq.heappush(heap, item)
    return [sorted(p) for p in parts]
