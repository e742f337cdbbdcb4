"""The N > 1 host logic on CPU with world_size-2 gloo process groups: row
sharding of a mixed-adapter batch (no collective on the data path; the test
gathers the shards only to check them) and the tensor-parallel expand of a
segmented prefill (column blocks + all-gather).  The oracle stands in for the
CUDA kernels, which need a GPU."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import bgmv_oracle as O
from persona import workloads
from persona.sharding import partition_rows, shard_bytes
from persona.tensor_parallel import column_shards, sgmv_fused_tp

WORLD = 2


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, port):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=WORLD)


def _row_shard_worker(rank, port):
    _init(rank, port)
    try:
        wl = workloads.mixed_batch(seed=6, T=96, R=16, S=24, names=["k_proj"])
        p = wl.projections[0]
        rows = partition_rows(wl.slots, WORLD, adapter_bytes=16 * (4096 + 1024) * 2, row_bytes=(4096 + 2048) * 2)
        mine = rows[rank]
        y = p.y.copy()
        y_mine = y[mine].copy()
        O.bgmv_forward_ref(p.x[mine], p.a_pool, p.b_pool, wl.slots[mine], "f16", y=y_mine)
        # gather (rows, results) on every rank, only to check the partition
        counts = [torch.zeros(1, dtype=torch.int64) for _ in range(WORLD)]
        dist.all_gather(counts, torch.tensor([mine.size], dtype=torch.int64))
        width = int(max(c.item() for c in counts))
        send_rows = torch.full((width,), -1, dtype=torch.int64)
        send_rows[: mine.size] = torch.from_numpy(mine.astype(np.int64))
        send_y = torch.zeros((width, y.shape[1]), dtype=torch.float16)
        send_y[: mine.size] = torch.from_numpy(y_mine)
        all_rows = [torch.empty_like(send_rows) for _ in range(WORLD)]
        all_y = [torch.empty_like(send_y) for _ in range(WORLD)]
        dist.all_gather(all_rows, send_rows)
        dist.all_gather(all_y, send_y)
        got = p.y.copy()
        seen = np.zeros(wl.T, np.int64)
        for r in range(WORLD):
            rr = all_rows[r].numpy()
            rr = rr[rr >= 0]
            seen[rr] += 1
            got[rr] = all_y[r].numpy()[: rr.size]
        active = wl.slots >= 0
        assert np.all(seen[active] == 1) and np.all(seen[~active] == 0)
        want = p.y.copy()
        O.bgmv_forward_ref(p.x, p.a_pool, p.b_pool, wl.slots, "f16", y=want)
        assert np.array_equal(got, want)
        # the shards' bytes add up to at most the unsharded bytes plus one
        # adapter per split group
        b = [shard_bytes(wl.slots, r_, 16 * 5120 * 2, 6144 * 2) for r_ in rows]
        assert sum(b) <= shard_bytes(wl.slots, np.arange(wl.T), 16 * 5120 * 2, 6144 * 2) + WORLD * 16 * 5120 * 2
    finally:
        dist.destroy_process_group()


def _oracle_sgmv_fused(x, a_pool, b_pool, seg_indptr, seg_slots, y):
    """CPU stand-in for ops.sgmv_fused: the oracle on the segments' rows,
    written into the (possibly column-sliced) y view."""
    slots = O.sgmv_slots(seg_indptr.numpy(), seg_slots.numpy(), x.shape[0])
    out = y.numpy().copy()
    O.bgmv_forward_ref(x.numpy(), a_pool.numpy(), b_pool.contiguous().numpy(), slots, "f16", y=out)
    y.copy_(torch.from_numpy(out))
    return y


def _tp_worker(rank, port):
    _init(rank, port)
    try:
        rng = np.random.default_rng(7)
        T, K, N, R, S = 40, 64, 392, 16, 5
        indptr = np.array([0, 12, 12, 31, 40], np.int32)
        seg = np.array([3, 1, -1, 0], np.int32)
        x = rng.standard_normal((T, K)).astype(np.float16)
        a = (rng.uniform(-1, 1, (S, R, K)) / 8).astype(np.float16)
        b = (rng.standard_normal((S, N, R)) * 0.05).astype(np.float16)
        y0 = rng.standard_normal((T, N)).astype(np.float16)
        y = torch.from_numpy(y0.copy())
        sgmv_fused_tp(torch.from_numpy(x), torch.from_numpy(a), torch.from_numpy(b), torch.from_numpy(indptr),
                      torch.from_numpy(seg), y, fused=_oracle_sgmv_fused)
        want = y0.copy()
        O.bgmv_forward_ref(x, a, b, O.sgmv_slots(indptr, seg, T), "f16", y=want)
        assert np.array_equal(y.numpy(), want), f"rank {rank}: tensor-parallel result differs"
    finally:
        dist.destroy_process_group()


def test_column_shards_cover_and_align():
    for N, w in [(14336, 8), (4096, 2), (392, 2), (100, 4), (1024, 8)]:
        sh = column_shards(N, w)
        assert sh[0][0] == 0 and sh[-1][1] == N
        for (a0, a1), (b0, b1) in zip(sh, sh[1:]):
            assert a1 == b0
        assert all(a % 128 == 0 for a, b in sh if b > a)  # empty shards sit at N
        assert all((b - a) % 128 == 0 for a, b in sh if b < N)
    assert column_shards(14336, 8) == [(i * 1792, (i + 1) * 1792) for i in range(8)]


def test_partition_rows_single_rank_and_validation():
    slots = np.array([3, -1, 3, 0, 7], np.int32)
    assert partition_rows(slots, 1, 100, 10)[0].tolist() == [0, 2, 3, 4]
    with pytest.raises(ValueError):
        partition_rows(slots, 0, 100, 10)
    with pytest.raises(ValueError):
        partition_rows(slots, 2, 100, 10, rows_per_item=0)


@pytest.mark.parametrize("world", [2, 4, 8])
def test_partition_rows_balances_item_loads(world):
    """Zipf batch of 512 rows per rank: every active row lands on exactly one
    rank, a split adapter is cut at whole 16-row items (only its last piece
    may be partial), and the per-item load -- one adapter read per 16-row
    item plus the rows' bytes -- is balanced within 10% across ranks."""
    rng = np.random.Generator(np.random.PCG64(2))
    slots = workloads.zipf_slots(rng, 512 * world, 256)
    ab, rb = 64 * 81920 * 2, 124928 * 2  # rank 64, the 7 projections of one layer
    parts = partition_rows(slots, world, ab, rb)
    seen = np.zeros(slots.size, np.int64)
    for p in parts:
        seen[p] += 1
    assert np.array_equal(seen, (slots >= 0).astype(np.int64))
    loads = []
    for p in parts:
        s = slots[p]
        _, c = np.unique(s, return_counts=True)
        loads.append(int(np.sum(-(-c // 16))) * ab + s.size * rb)
    assert max(loads) <= 1.1 * (sum(loads) / world)
    for slot in np.unique(slots[slots >= 0]):
        per_rank = [int(np.sum(slots[p] == slot)) for p in parts]
        split = [n for n in per_rank if n > 0]
        if len(split) > 1:
            assert sum(n % 16 != 0 for n in split) <= 1


@pytest.mark.parametrize("worker", [_row_shard_worker, _tp_worker])
def test_two_rank_gloo(worker):
    mp.spawn(worker, args=(_free_port(),), nprocs=WORLD, join=True)
