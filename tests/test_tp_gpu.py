"""Tensor-parallel segmented LoRA on 2 and 4 GPUs (NCCL): the fused kernel
that stores its column block into every rank's y over NVLink, and the
all-gather baseline, each against a one-GPU sgmv_fused of all columns
(bit-identical: every tile is computed by the same kernel), and that result
against the oracle (atol = rtol = 1e-2, rows without adapter byte for
byte).  Each world size is skipped when the box has fewer GPUs."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, dtype_name, R):
    import datetime

    from persona import ops
    from persona.tensor_parallel import PeerBuffers, sgmv_fused_tp, sgmv_fused_tp_nvlink

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    try:
        dt = torch.bfloat16 if dtype_name == "bf16" else torch.float16
        rng = np.random.default_rng(21)
        lens = [128, 300, 37, 0, 135]  # full and partial 128-row items
        T, K, N, S = sum(lens), 512, 1024, 5
        indptr = torch.tensor(np.concatenate([[0], np.cumsum(lens)]), dtype=torch.int32, device=dev)
        seg = torch.tensor([3, -1, 1, 0, 4], dtype=torch.int32, device=dev)
        x = torch.from_numpy(rng.standard_normal((T, K)).astype(np.float32)).to(dev, dt)
        a = torch.from_numpy((rng.uniform(-1, 1, (S, R, K)) / np.sqrt(K)).astype(np.float32)).to(dev, dt)
        b = torch.from_numpy((rng.standard_normal((S, N, R)) * 0.05).astype(np.float32)).to(dev, dt)
        y0 = torch.from_numpy(rng.standard_normal((T, N)).astype(np.float32)).to(dev, dt)

        y_ref = y0.clone()
        ops.sgmv_fused(x, a, b, indptr, seg, y_ref)
        y_nccl = y0.clone()
        sgmv_fused_tp(x, a, b, indptr, seg, y_nccl)
        y_nv = y0.clone()
        peers = PeerBuffers(y_nv)
        for _ in range(2):  # the mapping is reused across calls
            y_nv.copy_(y0)
            sgmv_fused_tp_nvlink(x, a, b, indptr, seg, y_nv, peers)
            torch.cuda.synchronize()
            assert torch.equal(y_nv, y_ref), f"rank {rank}: NVLink tensor-parallel result differs"
        assert torch.equal(y_nccl, y_ref), f"rank {rank}: all-gather tensor-parallel result differs"
        ops.check_errors(dev)
        if rank == 0:
            from oracle import bgmv_oracle as O

            def n16(t):
                t = t.cpu()
                return t.view(torch.int16).numpy().view(np.uint16) if dtype_name == "bf16" else t.numpy()

            slots = O.sgmv_slots(indptr.cpu().numpy(), seg.cpu().numpy(), T)
            want = n16(y0).copy()
            O.bgmv_forward_ref(n16(x), n16(a), n16(b), slots, dtype_name, y=want)
            got = O.to_f32(n16(y_ref), dtype_name)
            np.testing.assert_allclose(got, O.to_f32(want, dtype_name), rtol=1e-2, atol=1e-2)
            assert np.array_equal(n16(y_ref)[slots < 0], n16(y0)[slots < 0])
            err = float(np.abs(got - O.to_f32(want, dtype_name)).max())
            print(f"tp world={world} {dtype_name} R={R} T={T} K={K} N={N}: bit-identical on every rank; "
                  f"max |y - oracle| = {err:.3g}")
        dist.barrier()
        peers.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("dtype_name,R", [("bf16", 16), ("f16", 32), ("bf16", 64)])
def test_tensor_parallel_sgmv(world, dtype_name, R):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    mp.spawn(_worker, args=(world, _free_port(), dtype_name, R), nprocs=world, join=True)
