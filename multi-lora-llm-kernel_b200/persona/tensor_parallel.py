"""Tensor-parallel segmented LoRA for prefill across the GPUs of one node.

A prefill batch (SGMV, rows grouped by adapter) is split by OUTPUT COLUMNS:
rank r owns columns [n0_r, n1_r) of y.  Every rank computes the full rank-R
intermediate v itself (the shrink reads x and A once per rank, a small cost
next to B and y at rank 16), expands into its own column block of y with the
matching rows of B (a view of the pool, no copy), and the ranks then
all-gather the column blocks so that every rank holds the full updated y.
The all-gather is the path's only exchange step.  Two forms:

* ``sgmv_fused_tp_nvlink`` -- one kernel per rank does the math AND the
  exchange: every finished 128 x 128 tile of y goes to the rank's own y and,
  with plain stores over NVLink, into every other rank's y (mapped once with
  CUDA IPC by ``PeerBuffers``), so the transfer overlaps the math tile by
  tile; a one-element all-reduce after the launch is the barrier.
* ``sgmv_fused_tp`` -- the kernel on the column block, then an all-gather on
  the process group's backend (NCCL); the baseline, and the CPU-testable form.

Column blocks are whole multiples of 128 (the tensor-core tile of the SGMV
kernel) whenever N allows it.
"""

from __future__ import annotations

from typing import Callable, List, Optional, Tuple

import torch
import torch.distributed as dist


def column_shards(N: int, world: int, align: int = 128) -> List[Tuple[int, int]]:
    """[n0, n1) of every rank: contiguous, covering [0, N), sizes multiples of
    `align` except possibly the last, as even as that allows."""
    if world <= 0:
        raise ValueError("world must be positive")
    units = (N + align - 1) // align
    base, extra = divmod(units, world)
    out, u = [], 0
    for r in range(world):
        take = base + (1 if r < extra else 0)
        n0, n1 = min(N, u * align), min(N, (u + take) * align)
        out.append((n0, n1))
        u += take
    return out


def sgmv_fused_tp(x: torch.Tensor, a_pool: torch.Tensor, b_pool: torch.Tensor, seg_indptr: torch.Tensor,
                  seg_slots: torch.Tensor, y: torch.Tensor, group: Optional[dist.ProcessGroup] = None,
                  fused: Optional[Callable] = None) -> torch.Tensor:
    """``y += B[s] @ (A[s] @ x)`` for a segmented batch, with the expand split
    by output columns over the ranks of `group` and the column blocks
    all-gathered.  `y` holds the full [T, N] output on every rank before and
    after the call.  `fused` defaults to ``persona.ops.sgmv_fused``."""
    if fused is None:
        from persona import ops

        fused = ops.sgmv_fused
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    T, N = y.shape
    shards = column_shards(N, world)
    n0, n1 = shards[rank]
    if n1 > n0:
        fused(x, a_pool, b_pool[:, n0:n1, :], seg_indptr, seg_slots, y[:, n0:n1])
    width = max(b - a for a, b in shards)
    send = torch.zeros((T, width), dtype=y.dtype, device=y.device)
    send[:, : n1 - n0] = y[:, n0:n1]
    recv = [torch.empty_like(send) for _ in range(world)]
    dist.all_gather(recv, send, group=group)
    for r, (a, b) in enumerate(shards):
        if r != rank and b > a:
            y[:, a:b] = recv[r][:, : b - a]
    return y


class PeerBuffers:
    """Maps the y buffer of every other rank into this process (CUDA IPC),
    once per buffer; pass it to ``sgmv_fused_tp_nvlink`` for every call on
    the same y.  Every rank must build it (it exchanges handles on `group`)."""

    def __init__(self, y: torch.Tensor, group: Optional[dist.ProcessGroup] = None):
        from persona import ops

        ext = ops._load()
        self._ext = ext
        self.device = y.device.index
        handle, offset = ext.ipc_export(y)
        world = dist.get_world_size(group)
        rank = dist.get_rank(group)
        got = [None] * world
        dist.all_gather_object(got, (bytes(handle), int(offset)), group=group)
        self.peers: List[int] = []
        self._bases: List[int] = []
        for r, (h, off) in enumerate(got):
            if r == rank:
                continue
            ptr, base = ext.ipc_import(h, off, self.device)
            self.peers.append(ptr)
            self._bases.append(base)

    def close(self) -> None:
        for b in self._bases:
            self._ext.ipc_close(b, self.device)
        self._bases, self.peers = [], []


def sgmv_fused_tp_nvlink(x: torch.Tensor, a_pool: torch.Tensor, b_pool: torch.Tensor, seg_indptr: torch.Tensor,
                         seg_slots: torch.Tensor, y: torch.Tensor, peers: PeerBuffers,
                         group: Optional[dist.ProcessGroup] = None) -> torch.Tensor:
    """Same result as ``sgmv_fused_tp``, with the all-gather fused into the
    kernel (NVLink stores of each finished tile into the other ranks' y).
    Tensor-core shapes only (rank 16 / 32 / 64, K % 64 == 0, N % 64 == 0)."""
    from persona import ops

    ext = ops._load()
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    n0, n1 = column_shards(y.shape[1], world)[rank]
    flag = torch.zeros(1, dtype=torch.int32, device=y.device)
    # Barriers on the stream.  Before: no rank writes into a peer's y while
    # that peer may still be reading it.  After: when it completes on a rank,
    # every rank's kernel (and so every tile stored into this rank's y) has
    # finished.
    dist.all_reduce(flag, group=group)
    ext.sgmv_fused_tp(x, a_pool, b_pool, seg_indptr, seg_slots, y, peers.peers, n0, n1)
    dist.all_reduce(flag, group=group)
    return y
