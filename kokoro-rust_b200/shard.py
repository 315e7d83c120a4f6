"""Data-parallel sharding of independent lines across GPUs (one engine per GPU, no collectives on
the hot path) and in-order reassembly on the host.

The reference is single-GPU; its in-GPU batching sorts lines by length (src/engine.rs:165-183) and
its writer reassembles per-line audio in line order (src/wav.rs:136-187). Across GPUs the same
two rules apply: lines are length-sorted and assigned longest-first to the least-loaded rank
(LPT), each rank batches its share with ``plan_batches``, and results are merged back by line
index, with a missing or failed line reported at its own position.
"""
from __future__ import annotations

import heapq
from typing import Dict, List, Sequence


def shard_lpt(costs: Sequence[float], world: int) -> List[List[int]]:
    """Longest-processing-time-first assignment of line indices to ``world`` ranks; each rank's
    list is returned in ascending line order. Ties go to the lower rank."""
    if world < 1:
        raise ValueError("world must be >= 1")
    heap = [(0.0, r) for r in range(world)]
    out: List[List[int]] = [[] for _ in range(world)]
    for i in sorted(range(len(costs)), key=lambda i: (-costs[i], i)):
        load, r = heapq.heappop(heap)
        out[r].append(i)
        heapq.heappush(heap, (load + float(costs[i]), r))
    return [sorted(s) for s in out]


class LineError(RuntimeError):
    """A line that failed (or never came back) on its rank."""


def assemble_in_order(n_lines: int, per_rank: Sequence[Dict[int, object]]) -> list:
    """Merge {line index: result} maps from every rank into one list in line order. A result
    that is an exception stays at its position; a line no rank returned becomes a LineError."""
    merged: Dict[int, object] = {}
    for part in per_rank:
        for i, r in part.items():
            if i in merged:
                raise ValueError(f"line {i} returned by two ranks")
            merged[i] = r
    return [merged.get(i, LineError(f"line {i} missing from every rank")) for i in range(n_lines)]
