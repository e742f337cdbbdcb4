#!/usr/bin/env python
"""Benchmark of the fused multi-LoRA BGMV shrink+expand hot path on B200.

Workload (the large mixed-adapter decode batch): the seven Mistral-7B LoRA
projections of one decoder layer (q/o 4096->4096, k/v 4096->1024, gate/up
4096->14336, down 14336->4096), fp16, rank 64, a pool of 256 adapters
resident in HBM, 512 rows per GPU whose slots are drawn from a truncated
Zipf(1.1) with 5 % of rows without an adapter.  One step = the device-side
row-grouping plan plus one fused shrink->expand launch per projection.

N GPUs (torchrun, one process per GPU): the global batch is 512*N rows,
partitioned across ranks by adapter affinity (persona.sharding) with the pool
replicated -- weak scaling, no collective on the data path.

Metric: algorithmic HBM GB/s of the fused BGMV (distinct adapters' A+B once,
active rows' x once, y read+written once), whole job, max time over ranks.
Per-step traffic (~1.4 GB) is far above the 126 MB L2, so consecutive steps
do not hit in L2.  Synthetic seeded inputs and random-init adapters.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
"""

from __future__ import annotations

import argparse
import datetime
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "multi-lora-llm-kernel_b200"))
sys.path.insert(0, str(ROOT))

import numpy as np  # noqa: E402

METRIC = "fused BGMV shrink+expand GB/s vs HBM peak; mixed-adapter decode tokens/s"
UNIT = "GB/s"
ROWS_PER_GPU = 512
RANK = 64
POOL_SLOTS = 256
SEED = 2


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    return ap.parse_args()


def load_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def projections():
    from persona.workloads import PROJECTIONS

    return [(n, k, nn) for n, (k, nn) in PROJECTIONS.items()]


def adapter_and_row_bytes():
    projs = projections()
    adapter = sum(RANK * (k + n) * 2 for _, k, n in projs)
    row = sum((k + 2 * n) * 2 for _, k, n in projs)
    return adapter, row


def global_slots(world):
    from persona.workloads import zipf_slots

    rng = np.random.Generator(np.random.PCG64(SEED))
    return zipf_slots(rng, ROWS_PER_GPU * world, POOL_SLOTS)


# ------------------------------------------------------------------ clocks --

class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled while the GPU works."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,utilization.gpu,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: str):
        self.index = index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "50"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append((time.monotonic(), line.strip()))

    def stop(self, window=None):
        """Summarise the samples that arrived inside ``window`` (host
        monotonic seconds bracketing the timed region)."""
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.thread.join(timeout=2)
        sm, inside, mx, reasons = [], [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for t, ln in self.lines:
            f = [c.strip() for c in ln.split(",")]
            if len(f) < 10:
                continue
            try:
                mhz, mxv = float(f[1]), float(f[2])
            except ValueError:
                continue
            mx = mxv
            sm.append(mhz)
            if window is None or window[0] <= t <= window[1]:
                inside.append(mhz)
                for nm, val in zip(names, f[6:10]):
                    if val.lower() == "active":
                        reasons.add(nm)
        return {"sm_mhz": statistics.median(inside) if inside else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm), "samples_in_timed_region": len(inside)}


# -------------------------------------------------------------- CPU legs --

class CpuSample:
    """A bounded sample of the workload for the oracle port (the reference's
    fp32 CPU algorithm, persona/ops.py:12-56): the q_proj call (4096->4096,
    rank 64) on `rows` rows of the Zipf batch with a pool of `slots` slots."""

    def __init__(self, rows: int = ROWS_PER_GPU, slots: int = POOL_SLOTS):
        from oracle import bgmv_oracle as O
        from persona.workloads import make_projection, zipf_slots

        self.O = O
        rng = np.random.Generator(np.random.PCG64(SEED))
        self.slots = zipf_slots(rng, rows, slots)
        self.p = make_projection(rng, "q_proj", rows, 4096, 4096, RANK, slots, "f16")
        self.bytes = O.algorithmic_bytes(rows, 4096, 4096, RANK, self.slots)
        self.desc = (f"numpy port of the reference fp32 BGMV: q_proj 4096->4096, {rows} rows, rank 64, "
                     f"{slots}-slot pool widened per call")

    def call(self) -> float:
        y = self.p.y.copy()
        t0 = time.perf_counter()
        self.O.bgmv_forward_ref(self.p.x, self.p.a_pool, self.p.b_pool, self.slots, y=y)
        return time.perf_counter() - t0


def blas_threads() -> int:
    try:
        from threadpoolctl import threadpool_info

        return max([i.get("num_threads", 1) for i in threadpool_info()] or [1])
    except Exception:
        return 1


def cpu_baseline(seconds: float = 12.0, min_reps: int = 2):
    """The oracle port timed on the full q_proj call for ~`seconds`."""
    smp = CpuSample()
    smp.call()  # warm-up
    times = []
    t_end = time.perf_counter() + seconds
    while len(times) < min_reps or time.perf_counter() < t_end:
        times.append(smp.call())
    med = statistics.median(times)
    th = blas_threads()
    return {"value": smp.bytes / med / 1e9, "unit": UNIT, "cores": th, "kind": "port",
            "sample": f"{smp.desc}; {len(times)} reps, median {med * 1e3:.1f} ms; BLAS threads={th} "
                      f"(pool widening single-threaded); host cpus={os.cpu_count()}"}


def workload_config(world: int) -> dict:
    return {
        "workload": "mixed-adapter decode batch: 7 Mistral-7B LoRA projections, 512 rows/GPU, "
                    "rank 64, 256-slot pool, Zipf(1.1) slots + 5% rows without adapter",
        "rows_per_gpu": ROWS_PER_GPU, "global_rows": ROWS_PER_GPU * world, "rank": RANK,
        "pool_slots": POOL_SLOTS, "projections": [n for n, _, _ in projections()],
        "parallelism": f"row-sharded x{world} (adapter affinity), pool replicated",
        "l2": "inputs larger than L2: ~1.4 GB of adapter/x/y traffic per step vs 126 MB L2",
        "launches_per_step": 1 + len(projections()),
    }


def run_reference(args):
    """The reference arm: the reference's CPU implementation of the path (its
    fp32 torch BGMV, restated by the oracle port) on the host cores.  Under
    torchrun only rank 0 works."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    t0 = time.perf_counter()
    # Per-step sample: the largest of these whose warm-up + steps fit in ~2 minutes.
    budget = 120.0
    steps = max(1, args.steps)
    warm = max(0, args.warmup)
    smp = None
    for rows, slots in ((64, 32), (16, 8), (4, 2), (1, 1)):
        smp = CpuSample(rows=rows, slots=slots)
        smp.call()
        t1 = min(smp.call() for _ in range(2))
        if (steps + warm) * t1 <= budget:
            break
    for _ in range(warm):
        smp.call()
    times = [smp.call() for _ in range(steps)]
    med = statistics.median(times)
    value = smp.bytes / med / 1e9
    th = blas_threads()
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
        "steps": steps, "warmup": warm, "ms_per_step": med * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded Zipf slots, random-init rank-64 adapters)",
        "config": workload_config(args.gpus),
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": th, "kind": "port",
                         "sample": f"{smp.desc}; median of {steps} steps; BLAS threads={th}"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "wall_s": time.perf_counter() - t0,
    }
    print(json.dumps(line), flush=True)
    return 0


# --------------------------------------------------------------- GPU leg --

def run_ours(args):
    import torch
    import torch.distributed as dist

    from persona import ops
    from persona.sharding import partition_rows
    from persona.workloads import bgmv_bytes

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=120))
    if not ops.has_cuda_ops():
        raise SystemExit("persona extension missing")

    # ---- workload: global slots, this rank's rows, device-resident pools
    slots_g = global_slots(world)
    adapter_b, row_b = adapter_and_row_bytes()
    rows = partition_rows(slots_g, world, adapter_b, row_b)[rank]
    slots = slots_g[rows].astype(np.int32)
    T = int(slots.size)
    gen = torch.Generator(device=dev)
    gen.manual_seed(SEED * 1000 + 17)
    projs = []
    for name, K, N in projections():
        lim = 1.0 / np.sqrt(K)
        a = (torch.rand(POOL_SLOTS, RANK, K, generator=gen, device=dev) * (2 * lim) - lim).half()
        b = (torch.randn(POOL_SLOTS, N, RANK, generator=gen, device=dev) * 0.04).half()
        x = torch.randn(T, K, generator=gen, device=dev).half()
        y = torch.zeros(T, N, device=dev, dtype=torch.float16)
        projs.append(dict(name=name, K=K, N=N, a=a, b=b, x=x, y=y,
                          bytes=bgmv_bytes(K, N, RANK, slots)))
    slots_d = torch.from_numpy(slots).to(dev)
    step_bytes = sum(p["bytes"] for p in projs)
    stream = torch.cuda.current_stream()

    def step(ev=None):
        plan = ops.bgmv_plan(slots_d, POOL_SLOTS)
        for i, p in enumerate(projs):
            if ev is not None:
                ev[i][0].record(stream)
            ops.bgmv_fused(p["x"], p["a"], p["b"], slots_d, p["y"], plan=plan)
            if ev is not None:
                ev[i][1].record(stream)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])

    def max_over_ranks(v):
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def sum_over_ranks(v):
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.SUM)
        return float(t.item())

    props = torch.cuda.get_device_properties(dev)
    try:
        smi_id = f"{props.pci_domain_id:08X}:{props.pci_bus_id:02X}:{props.pci_device_id:02X}.0"
    except AttributeError:
        smi_id = str(local)
    clocks = ClockSampler(smi_id)
    clocks.start()
    for _ in range(max(3, args.warmup)):
        step()
    torch.cuda.synchronize()
    ops.check_errors(dev)

    # ---- timed region (device time, CUDA events; per-launch events for the roofline)
    K_steps = max(1, args.steps)
    evs = [[(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
            for _ in projs] for _ in range(K_steps)]
    barrier()
    torch.cuda.synchronize()
    t_start, t_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    host_t0 = time.monotonic()
    t_start.record(stream)
    for s in range(K_steps):
        step(evs[s])
    t_end.record(stream)
    torch.cuda.synchronize()
    host_t1 = time.monotonic()
    barrier()
    ms_local = t_start.elapsed_time(t_end) / K_steps
    fused_ms = sum(evs[s][i][0].elapsed_time(evs[s][i][1]) for s in range(K_steps) for i in range(len(projs)))
    fused_ms_per_step = fused_ms / K_steps
    ops.check_errors(dev)

    # ---- end to end through the public API, host buffers in pinned memory
    host = []
    for p in projs:
        host.append(dict(x=p["x"].cpu().pin_memory(), y_in=p["y"].cpu().pin_memory(),
                         y_out=torch.empty_like(p["y"], device="cpu").pin_memory()))
    slots_h = torch.from_numpy(slots).pin_memory()
    h2d = slots_h.numel() * 4 + sum(h["x"].numel() * 2 + h["y_in"].numel() * 2 for h in host)
    d2h = sum(h["y_out"].numel() * 2 for h in host)

    def e2e_step():
        sd = slots_h.to(dev, non_blocking=True)
        plan = ops.bgmv_plan(sd, POOL_SLOTS)
        for p, h in zip(projs, host):
            xd = h["x"].to(dev, non_blocking=True)
            yd = h["y_in"].to(dev, non_blocking=True)
            ops.bgmv_fused(xd, p["a"], p["b"], sd, yd, plan=plan)
            h["y_out"].copy_(yd, non_blocking=True)

    for _ in range(max(3, args.warmup)):
        e2e_step()
    torch.cuda.synchronize()
    barrier()
    e_start, e_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e_steps = max(1, min(K_steps, 50))
    e_start.record(stream)
    for _ in range(e_steps):
        e2e_step()
    e_end.record(stream)
    torch.cuda.synchronize()
    barrier()
    e2e_ms_local = e_start.elapsed_time(e_end) / e_steps
    clk = clocks.stop(window=(host_t0, host_t1))
    ops.check_errors(dev)

    ms = max_over_ranks(ms_local)
    e2e_ms = max_over_ranks(e2e_ms_local)
    total_bytes = sum_over_ranks(step_bytes)
    total_rows = sum_over_ranks(float((slots >= 0).sum()))
    fused_ms_max = max_over_ranks(fused_ms_per_step)
    line = None
    if rank == 0:
        peak, peak_kind = load_peaks()
        achieved = step_bytes / (fused_ms_per_step * 1e-3) / 1e9
        traffic = None
        tf = ROOT / "profiles" / "bgmv_fused_mixed_batch_traffic.json"
        if tf.exists():
            traffic = json.loads(tf.read_text()).get("traffic_bytes_per_launch")
        line = {
            "metric": METRIC,
            "value": total_bytes / (ms * 1e-3) / 1e9,
            "unit": UNIT,
            "n_gpus": world,
            "steps": K_steps,
            "warmup": args.warmup,
            "ms_per_step": ms,
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "f16",
            "data": "synthetic (seeded Zipf slots, random-init rank-64 adapters)",
            "config": workload_config(world),
            "rows_per_s": total_rows / (ms * 1e-3),
            "roofline": {
                "bound": "hbm",
                "kernel": "bgmv_cluster_kernel<half,64,fused>",
                "achieved": achieved,
                "peak": peak,
                "peak_kind": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured" else
                "fallback 6.65 TB/s",
                "unit": "GB/s",
                "frac": achieved / peak,
                "traffic": traffic,
                "algorithmic_bytes_per_launch": step_bytes / len(projs),
                "launch_us_avg": fused_ms_per_step * 1e3 / len(projs),
            },
            "e2e": {"value": total_bytes / (e2e_ms * 1e-3) / 1e9, "unit": UNIT,
                    "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h),
                    "ms_per_step": e2e_ms,
                    "path": "persona.ops.bgmv_plan + bgmv_fused, pinned host x/y/slots copied in, y out"},
            "gpu_launches": K_steps * (1 + len(projs)),
            "clocks": clk,
            "fused_ms_per_step_max_rank": fused_ms_max,
        }
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline()
    if world > 1:
        barrier()
        dist.destroy_process_group()
    if line is not None:
        print(json.dumps(line), flush=True)
    return 0


def main():
    args = parse_args()
    if args.impl == "reference":
        return run_reference(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
