"""Row sharding of a mixed-adapter batch across the GPUs of one node.

The reference is single-GPU; the B200 build runs one process per GPU with
the adapter pool replicated on each, and splits the batch's rows across
ranks.  No collective is needed on the data path: a row's output depends only
on its own x and its adapter.

Partition (adapter affinity): rows are grouped by slot and each group goes
to the least-loaded rank (longest-processing-time first), so an adapter's A
and B are streamed by as few GPUs as possible.  The load of a group is what
the fused kernel streams for it: the kernel takes a group's rows in items of
``rows_per_item`` (16) and reads the adapter's A and B once per item (from
HBM for the first item, from L2 after that, at the same cost per byte), plus
the x and y bytes of its rows.  Launch time follows that load, not the
group's algorithmic bytes: a hot adapter of a Zipf batch (818 of 4096 rows
at 8 GPUs) costs 52 adapter reads.  A group heavier than one rank's fair
share is cut into pieces of whole items (each piece pays one more HBM read
of the adapter, on another GPU).  Rows with slot -1 carry no work and are
assigned to no rank -- their y is, by the op's contract, left untouched.
"""

from __future__ import annotations

import heapq
from typing import List

import numpy as np


def partition_rows(slots: np.ndarray, n_ranks: int, adapter_bytes: int, row_bytes: int,
                   rows_per_item: int = 16) -> List[np.ndarray]:
    """Return, per rank, the sorted row indices it processes."""
    slots = np.asarray(slots)
    if n_ranks <= 0:
        raise ValueError("n_ranks must be positive")
    if rows_per_item <= 0:
        raise ValueError("rows_per_item must be positive")
    rows = np.arange(slots.shape[0])
    active = slots >= 0
    if n_ranks == 1:
        return [rows[active]]
    order = np.argsort(slots[active], kind="stable")
    act_rows = rows[active][order]
    act_slots = slots[active][order]
    bounds = np.flatnonzero(np.diff(act_slots)) + 1
    groups = np.split(act_rows, bounds) if act_rows.size else []

    def load(n_rows: int) -> int:
        return -(-n_rows // rows_per_item) * adapter_bytes + n_rows * row_bytes

    fair = sum(load(g.size) for g in groups) / n_ranks
    pieces = []
    for g in groups:
        items = -(-g.size // rows_per_item)
        n_split = min(items, max(1, int(np.ceil(load(g.size) / fair)))) if fair > 0 else 1
        step = -(-items // n_split) * rows_per_item
        for s in range(0, g.size, step):
            part = g[s:s + step]
            pieces.append((load(part.size), part))
    pieces.sort(key=lambda p: (-p[0], int(p[1][0])))
    heap = [(0, r) for r in range(n_ranks)]
    heapq.heapify(heap)
    assigned: List[List[np.ndarray]] = [[] for _ in range(n_ranks)]
    for cost, part in pieces:
        load_r, r = heapq.heappop(heap)
        assigned[r].append(part)
        heapq.heappush(heap, (load_r + cost, r))
    return [np.sort(np.concatenate(a)) if a else np.zeros(0, np.int64) for a in assigned]


def shard_bytes(slots: np.ndarray, rows: np.ndarray, adapter_bytes: int, row_bytes: int) -> int:
    """Algorithmic bytes one rank moves for its rows (distinct adapters once)."""
    s = np.asarray(slots)[rows]
    s = s[s >= 0]
    return int(np.unique(s).size * adapter_bytes + s.size * row_bytes)
