"""Row sharding of a mixed-adapter batch across the GPUs of one node.

The reference is single-GPU; the B200 build runs one process per GPU with
the adapter pool replicated on each, and splits the batch's rows across
ranks.  No collective is needed on the data path: a row's output depends only
on its own x and its adapter.

Partition (adapter affinity): rows are grouped by slot and each group goes,
whole, to the least-loaded rank (longest-processing-time first), so every
adapter's A and B are streamed by one GPU only and the total HBM bytes stay
those of the unsharded batch.  The load of a group is its algorithmic bytes:
the adapter's A+B bytes plus x and y bytes of its rows.  A group heavier
than one rank's fair share is split into row pieces first (each piece pays
the adapter bytes again).  Rows with slot -1 carry no work and are assigned to
no rank -- their y is, by the op's contract, left untouched.
"""

from __future__ import annotations

import heapq
from typing import List

import numpy as np


def partition_rows(slots: np.ndarray, n_ranks: int, adapter_bytes: int, row_bytes: int) -> List[np.ndarray]:
    """Return, per rank, the sorted row indices it processes."""
    slots = np.asarray(slots)
    if n_ranks <= 0:
        raise ValueError("n_ranks must be positive")
    rows = np.arange(slots.shape[0])
    active = slots >= 0
    if n_ranks == 1:
        return [rows[active]]
    order = np.argsort(slots[active], kind="stable")
    act_rows = rows[active][order]
    act_slots = slots[active][order]
    bounds = np.flatnonzero(np.diff(act_slots)) + 1
    groups = np.split(act_rows, bounds) if act_rows.size else []
    total = sum(adapter_bytes + g.size * row_bytes for g in groups)
    fair = total / n_ranks
    pieces = []
    for g in groups:
        cost = adapter_bytes + g.size * row_bytes
        n_split = max(1, int(np.ceil(cost / fair))) if fair > 0 else 1
        n_split = min(n_split, g.size)
        for part in np.array_split(g, n_split):
            pieces.append((adapter_bytes + part.size * row_bytes, part))
    pieces.sort(key=lambda p: (-p[0], int(p[1][0])))
    heap = [(0, r) for r in range(n_ranks)]
    heapq.heapify(heap)
    assigned: List[List[np.ndarray]] = [[] for _ in range(n_ranks)]
    for cost, part in pieces:
        load, r = heapq.heappop(heap)
        assigned[r].append(part)
        heapq.heappush(heap, (load + cost, r))
    return [np.sort(np.concatenate(a)) if a else np.zeros(0, np.int64) for a in assigned]


def shard_bytes(slots: np.ndarray, rows: np.ndarray, adapter_bytes: int, row_bytes: int) -> int:
    """Algorithmic bytes one rank moves for its rows (distinct adapters once)."""
    s = np.asarray(slots)[rows]
    s = s[s >= 0]
    return int(np.unique(s).size * adapter_bytes + s.size * row_bytes)
