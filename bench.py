#!/usr/bin/env python
"""Benchmark of the fused multi-LoRA BGMV shrink+expand hot path on B200.

Workload (the large mixed-adapter decode batch): the seven Mistral-7B LoRA
projections of one decoder layer (q/o 4096->4096, k/v 4096->1024, gate/up
4096->14336, down 14336->4096), fp16, rank 64, a pool of 256 adapters
resident in HBM, 512 rows per GPU whose slots are drawn from a truncated
Zipf(1.1) with 5 % of rows without an adapter.  One step = the device-side
row-grouping plan plus one fused shrink->expand launch that carries all seven
projections.

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
    ap.add_argument("--no-decode", action="store_true",
                    help="skip the bounded mixed-adapter decode run that the headline line carries")
    ap.add_argument("--workload", choices=["mixed_decode", "sgmv_prefill", "decode_set", "e2e_decode", "nf4_decode",
                                           "decode_kernels"],
                    default="mixed_decode",
                    help="mixed_decode is the headline; the others print their own line")
    ap.add_argument("--batch", type=int, default=None,
                    help="e2e_decode: rows per GPU (default 8 on one GPU, 64 per replica on several); "
                         "nf4_decode: rows of x (default 8)")
    ap.add_argument("--sgmv-rank", type=int, default=16, choices=[16, 32, 64],
                    help="adapter rank of --workload sgmv_prefill on one GPU (16: the segmented prefill config)")
    ap.add_argument("--only", default=None,
                    help="restrict to one projection (e.g. gate_proj), for profiling a small case")
    return ap.parse_args()


def load_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


ONLY = None


def projections():
    from persona.workloads import PROJECTIONS

    return [(n, k, nn) for n, (k, nn) in PROJECTIONS.items() if ONLY is None or n == ONLY]


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
    """SM clock and clock-event (throttle) reasons of one GPU, sampled about
    every millisecond by a thread that makes read-only NVML queries, so that
    even a timed region of a few milliseconds gets samples.  ``mark`` brackets
    the timed region; ``stop`` summarises the samples inside it."""

    # NVML clocks-event reason bits (nvmlClocksEventReason*)
    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown",
               0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown"}

    def __init__(self, pci_bus_id: str, period_s: float = 0.001):
        self.pci = pci_bus_id
        self.period = period_s
        self.samples = []  # (host monotonic s, sm MHz, reasons bitmask)
        self.max_mhz = None
        self.error = None
        self._stop = threading.Event()
        self.thread = None

    def start(self):
        try:
            import pynvml

            pynvml.nvmlInit()
            h = pynvml.nvmlDeviceGetHandleByPciBusId(self.pci)
            self.max_mhz = float(pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM))
            reasons = getattr(pynvml, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                pynvml.nvmlDeviceGetCurrentClocksThrottleReasons
        except Exception as e:  # no NVML: report why, keep benchmarking
            self.error = f"NVML unavailable: {e}"
            return

        def run():
            while not self._stop.is_set():
                try:
                    mhz = pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM)
                    rs = reasons(h)
                    self.samples.append((time.monotonic(), float(mhz), int(rs)))
                except Exception as e:  # pragma: no cover - driver hiccup
                    self.error = str(e)
                    return
                time.sleep(self.period)

        self.thread = threading.Thread(target=run, daemon=True)
        self.thread.start()

    def stop(self, window=None, busy_s=None):
        """Summary of the samples inside ``window`` (host monotonic seconds);
        ``busy_s``: device time of the timed region, for time x clock."""
        self._stop.set()
        if self.thread is not None:
            self.thread.join(timeout=2)
        if self.error and not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [self.error], "samples": 0,
                    "samples_in_timed_region": 0}
        inside = [x for x in self.samples if window is None or window[0] <= x[0] <= window[1]]
        reasons = sorted({name for _, _, rs in inside for bit, name in self.REASONS.items() if rs & bit})
        med = statistics.median([m for _, m, _ in inside]) if inside else None
        out = {"sm_mhz": med, "sm_max_mhz": self.max_mhz, "reasons": reasons, "samples": len(self.samples),
               "samples_in_timed_region": len(inside), "source": "NVML (read-only), ~1 ms period"}
        if med is not None and busy_s is not None:
            out["timed_s_x_median_mhz"] = busy_s * med
        return out


# -------------------------------------------------------------- CPU legs --

def cpu_model() -> str:
    try:
        for ln in Path("/proc/cpuinfo").read_text().splitlines():
            if ln.startswith("model name"):
                return ln.split(":", 1)[1].strip()
    except OSError:
        pass
    import platform

    return platform.processor() or "unknown"


class CpuLayer:
    """The reference's CPU algorithm (its fp32 torch BGMV, persona/ops.py:12-68,
    restated in oracle/bgmv_torch_ref.py) on the headline workload: the seven
    projections of one decoder layer, 512 rows of the Zipf batch, rank 64, a
    256-slot pool, fp16 storage.  ``call(i)`` runs projection i (or all seven
    with i=None) and returns (seconds, algorithmic bytes)."""

    def __init__(self, rows: int = ROWS_PER_GPU, slots: int = POOL_SLOTS):
        import torch

        from oracle import bgmv_oracle as O
        from persona.workloads import zipf_slots

        self.torch = torch
        rng = np.random.Generator(np.random.PCG64(SEED))
        self.slots_np = zipf_slots(rng, rows, slots)
        self.slots = torch.from_numpy(self.slots_np)
        g = torch.Generator().manual_seed(SEED * 1000 + 17)
        self.projs = []
        for name, K, N in projections():
            lim = 1.0 / np.sqrt(K)
            a = (torch.rand(slots, RANK, K, generator=g) * (2 * lim) - lim).half()
            b = (torch.randn(slots, N, RANK, generator=g) * 0.04).half()
            x = torch.randn(rows, K, generator=g).half()
            self.projs.append(dict(name=name, a=a, b=b, x=x, y=torch.zeros(rows, N, dtype=torch.float16),
                                   bytes=O.algorithmic_bytes(rows, K, N, RANK, self.slots_np)))
        self.rows, self.pool = rows, slots

    def call(self, i=None):
        from oracle import bgmv_torch_ref as TR

        ps = self.projs if i is None else [self.projs[i % len(self.projs)]]
        t0 = time.perf_counter()
        for p in ps:
            TR.bgmv_forward_ref(p["x"], p["a"], p["b"], self.slots, p["y"])
        return time.perf_counter() - t0, sum(p["bytes"] for p in ps)

    def describe(self, per_step: str) -> str:
        return (f"the reference's fp32 torch BGMV (persona/ops.py:12-68, restated in oracle/bgmv_torch_ref.py) "
                f"on {per_step} of the headline layer ({self.rows} rows, rank 64, {self.pool}-slot pool, fp16, "
                f"whole pool widened per call as the reference does); torch threads={self.torch.get_num_threads()}, "
                f"host cpus={os.cpu_count()}, cpu={cpu_model()}")


def cpu_baseline(seconds: float = 20.0):
    """The CPU leg of our arm: the seven projections of the headline layer,
    one after another, for about ``seconds`` (at least one full layer)."""
    import torch

    lay = CpuLayer()
    lay.call(0)  # warm-up
    t_tot, b_tot, n = 0.0, 0, 0
    while n < len(lay.projs) or t_tot < seconds:
        t, b = lay.call(n)
        t_tot, b_tot, n = t_tot + t, b_tot + b, n + 1
    return {"value": b_tot / t_tot / 1e9, "unit": UNIT, "cores": torch.get_num_threads(), "kind": "port",
            "cpu_model": cpu_model(), "torch_threads": torch.get_num_threads(), "host_cpus": os.cpu_count(),
            "sample": lay.describe(f"{n} projection calls ({n / len(lay.projs):.1f} layers), "
                                   f"{t_tot:.1f} s in total")}


def workload_config(world: int) -> dict:
    return {
        "workload": "mixed-adapter decode batch: 7 Mistral-7B LoRA projections, 512 rows/GPU, "
                    "rank 64, 256-slot pool, Zipf(1.1) slots + 5% rows without adapter",
        "rows_per_gpu": ROWS_PER_GPU, "global_rows": ROWS_PER_GPU * world, "rank": RANK,
        "pool_slots": POOL_SLOTS, "projections": [n for n, _, _ in projections()],
        "parallelism": f"row-sharded x{world} (adapter affinity), pool replicated",
        "l2": "inputs larger than L2: ~1.4 GB of adapter/x/y traffic per step vs 126 MB L2",
        "launches_per_step": 2,
    }


def run_reference(args):
    """The reference arm: the reference's CPU implementation of the path (its
    fp32 torch BGMV, restated in oracle/bgmv_torch_ref.py) on the host cores,
    on our arm's workload.  One step is the whole 7-projection layer at full
    size when --steps + --warmup of them fit in about two minutes; otherwise
    one full-size projection per step, cycling through the seven (so that
    every seven steps cover the layer).  Under torchrun only rank 0 works."""
    import torch

    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    t0 = time.perf_counter()
    budget = 120.0
    steps = max(1, args.steps)
    warm = max(0, args.warmup)
    lay = CpuLayer()
    t_layer, _ = lay.call(None)
    whole = (steps + warm) * t_layer <= budget
    for k in range(warm):
        lay.call(None if whole else k)
    times, byts = [], []
    for k in range(steps):
        t, b = lay.call(None if whole else k)
        times.append(t)
        byts.append(b)
    value = sum(byts) / sum(times) / 1e9
    per_step = "all seven projections per step" if whole else "one projection per step, cycling through the seven"
    cfg = workload_config(args.gpus)
    cfg["workload"] += f" (CPU arm: {per_step})"
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
        "steps": steps, "warmup": warm, "ms_per_step": statistics.mean(times) * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32 (fp16 storage)",
        "data": "synthetic (seeded Zipf slots, random-init rank-64 adapters)",
        "config": cfg,
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": torch.get_num_threads(), "kind": "port",
                         "cpu_model": cpu_model(), "torch_threads": torch.get_num_threads(),
                         "host_cpus": os.cpu_count(), "sample": lay.describe(per_step)},
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

    xs = [p["x"] for p in projs]
    a_s = [p["a"] for p in projs]
    b_s = [p["b"] for p in projs]
    ys = [p["y"] for p in projs]

    def step(ev=None):
        # one plan for the batch's slots + one launch for all the projections
        plan = ops.bgmv_plan(slots_d, POOL_SLOTS)
        if ev is not None:
            ev[0].record(stream)
        ops.bgmv_fused_multi(xs, a_s, b_s, slots_d, ys, plan=plan)
        if ev is not None:
            ev[1].record(stream)

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
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(K_steps)]
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
    fused_ms = sum(evs[s][0].elapsed_time(evs[s][1]) for s in range(K_steps))
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

    # Steps are pipelined the way a serving loop would run them: three streams
    # (copy in, compute, copy out) and two sets of device buffers, so step
    # k+1's inputs cross PCIe while step k computes and step k-1's outputs
    # come back.  Every step still moves its own inputs in and its y out.
    s_in, s_cmp, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    bufs = []
    for _ in range(2):
        bufs.append(dict(sd=torch.empty(slots_h.shape, dtype=torch.int32, device=dev),
                         xd=[torch.empty_like(p["x"]) for p in projs],
                         yd=[torch.empty_like(p["y"]) for p in projs],
                         h2d=torch.cuda.Event(), cmp=torch.cuda.Event(), d2h=torch.cuda.Event()))
    for b in bufs:
        b["d2h"].record(s_out)

    def e2e_step(k):
        b = bufs[k % 2]
        with torch.cuda.stream(s_in):
            s_in.wait_event(b["d2h"])  # the buffers' previous outputs have left
            b["sd"].copy_(slots_h, non_blocking=True)
            for h, xd, yd in zip(host, b["xd"], b["yd"]):
                xd.copy_(h["x"], non_blocking=True)
                yd.copy_(h["y_in"], non_blocking=True)
            b["h2d"].record(s_in)
        with torch.cuda.stream(s_cmp):
            s_cmp.wait_event(b["h2d"])
            plan = ops.bgmv_plan(b["sd"], POOL_SLOTS)
            ops.bgmv_fused_multi(b["xd"], a_s, b_s, b["sd"], b["yd"], plan=plan)
            b["cmp"].record(s_cmp)
        with torch.cuda.stream(s_out):
            s_out.wait_event(b["cmp"])
            for h, yd in zip(host, b["yd"]):
                h["y_out"].copy_(yd, non_blocking=True)
            b["d2h"].record(s_out)

    for k in range(max(3, args.warmup)):
        e2e_step(k)
    torch.cuda.synchronize()
    barrier()
    e_start, e_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e_steps = max(1, min(K_steps, 50))
    e_start.record(s_in)
    for k in range(e_steps):
        e2e_step(k)
    s_in.wait_stream(s_out)
    e_end.record(s_in)
    torch.cuda.synchronize()
    barrier()
    e2e_ms_local = e_start.elapsed_time(e_end) / e_steps
    clk = clocks.stop(window=(host_t0, host_t1), busy_s=ms_local * K_steps * 1e-3)
    ops.check_errors(dev)

    ms = max_over_ranks(ms_local)
    e2e_ms = max_over_ranks(e2e_ms_local)
    # every rank's launch: rows, algorithmic bytes, mean launch time, fraction of HBM peak
    mine = {"rank": rank, "rows": T, "adapters": int(np.unique(slots[slots >= 0]).size),
            "bytes_per_launch": int(step_bytes), "launch_us": fused_ms_per_step * 1e3,
            "frac": step_bytes / (fused_ms_per_step * 1e-3) / 1e9 / load_peaks()[0]}
    per_rank = [mine]
    if world > 1:
        per_rank = [None] * world
        dist.all_gather_object(per_rank, mine)
    total_bytes = sum_over_ranks(step_bytes)
    total_rows = sum_over_ranks(float((slots >= 0).sum()))
    fused_ms_max = max_over_ranks(fused_ms_per_step)
    line = None
    if rank == 0:
        peak, peak_kind = load_peaks()
        achieved = step_bytes / (fused_ms_per_step * 1e-3) / 1e9
        traffic = None
        tf = ROOT / "profiles" / "bgmv_fused_mixed_batch_traffic.json"
        if tf.exists() and world == 1 and len(projs) == 7:  # captured on the one-GPU 7-projection launch
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
                "kernel": "bgmv_split_kernel<half,64,fused> (7 projections per launch)",
                "achieved": achieved,
                "peak": peak,
                "peak_kind": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured" else
                "fallback 6.65 TB/s",
                "unit": "GB/s",
                "frac": achieved / peak,
                "traffic": traffic,
                "algorithmic_bytes_per_launch": step_bytes,
                "launch_us_avg": fused_ms_per_step * 1e3,
            },
            "e2e": {"value": total_bytes / (e2e_ms * 1e-3) / 1e9, "unit": UNIT,
                    "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h),
                    "ms_per_step": e2e_ms,
                    "path": "persona.ops.bgmv_plan + bgmv_fused_multi per step, pinned host x/y/slots copied "
                            "in and y out every step; copy-in, compute and copy-out on three streams, "
                            "double-buffered across steps"},
            "gpu_launches": K_steps * 2,
            "clocks": clk,
            "fused_ms_per_step_max_rank": fused_ms_max,
            "per_rank": per_rank,
        }
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline()
    if world == 1 and not args.no_decode:
        # the metric's second half: mixed-adapter decode tokens/s (config 5 at
        # batch 8 with 8 adapters), a bounded run after the BGMV measurement
        del projs, xs, a_s, b_s, ys, host, bufs
        torch.cuda.empty_cache()
        dm = decode_measure(dev, 1, 0, 8, 3, 3)
        dl = decode_line(dm, 1, 3, 3)
        line["decode"] = {k: dl[k] for k in ("value", "unit", "ms_per_step", "prefill_ms", "decode_ms",
                                             "decode_ms_per_token_step", "decode_tokens_per_s", "roofline",
                                             "config", "gpu_launches_per_decode_step")}
        line["decode"]["metric"] = "mixed-adapter decode tokens/s (whole generation: prefill + 127 steps)"
        line["decode"]["steps"], line["decode"]["warmup"] = 3, 3
    if world > 1:
        barrier()
        dist.destroy_process_group()
    if line is not None:
        print(json.dumps(line), flush=True)
    return 0


# ------------------------------------------------------ other workloads --

def _timed(fn, steps, stream):
    import torch

    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record(stream)
    for _ in range(steps):
        fn()
    e1.record(stream)
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / steps


def run_extra(args):
    """Single-GPU lines for the segmented prefill (SGMV on the tensor cores)
    and the small decode set (launch-latency bound; eager and CUDA graph)."""
    import torch

    from persona import ops
    from persona.workloads import bgmv_bytes

    if args.gpus != 1:
        raise SystemExit(f"--workload {args.workload} runs on one GPU")
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    stream = torch.cuda.current_stream()
    gen = torch.Generator(device=dev)
    gen.manual_seed(SEED * 1000 + 29)
    steps, warm = max(1, args.steps), max(3, args.warmup)

    def pools(K, N, R, S, dt):
        lim = 1.0 / np.sqrt(K)
        a = (torch.rand(S, R, K, generator=gen, device=dev) * (2 * lim) - lim).to(dt)
        b = (torch.randn(S, N, R, generator=gen, device=dev) * 0.04).to(dt)
        return a, b

    if args.workload == "sgmv_prefill":
        # 32 requests x 512 rows, rank 16 (or --sgmv-rank), 32 adapters, bf16; gate/up/down.
        req, rows, R, S = 32, 512, args.sgmv_rank, 32
        T = req * rows
        rng = np.random.Generator(np.random.PCG64(SEED + 1))
        seg = rng.permutation(req).astype(np.int32)
        indptr = (np.arange(req + 1) * rows).astype(np.int32)
        slots = np.repeat(seg, rows)
        ip, ss = torch.from_numpy(indptr).to(dev), torch.from_numpy(seg).to(dev)
        names = [n for n in ("gate_proj", "up_proj", "down_proj") if ONLY is None or n == ONLY]
        from persona.workloads import PROJECTIONS

        projs = []
        for n in names:
            K, N = PROJECTIONS[n]
            a, b = pools(K, N, R, S, torch.bfloat16)
            x = torch.randn(T, K, generator=gen, device=dev).to(torch.bfloat16)
            y = torch.zeros(T, N, device=dev, dtype=torch.bfloat16)
            projs.append(dict(name=n, K=K, N=N, a=a, b=b, x=x, y=y, bytes=bgmv_bytes(K, N, R, slots),
                              flops=2 * T * R * (K + N)))
        evs = [[(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in projs]
               for _ in range(steps)]

        def step(ev=None):
            for i, p in enumerate(projs):
                if ev is not None:
                    ev[i][0].record(stream)
                ops.sgmv_fused(p["x"], p["a"], p["b"], ip, ss, p["y"])
                if ev is not None:
                    ev[i][1].record(stream)

        for _ in range(warm):
            step()
        torch.cuda.synchronize()
        ops.check_errors(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for k in range(steps):
            step(evs[k])
        e1.record(stream)
        torch.cuda.synchronize()
        ops.check_errors(dev)
        ms = e0.elapsed_time(e1) / steps
        per = {p["name"]: sum(evs[k][i][0].elapsed_time(evs[k][i][1]) for k in range(steps)) / steps
               for i, p in enumerate(projs)}
        tot_b = sum(p["bytes"] for p in projs)
        tot_f = sum(p["flops"] for p in projs)
        peak, _ = load_peaks()
        tpk = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()).get("bf16_tflops") \
            if (ROOT / "MEASURED_PEAKS.json").exists() else 1590.0
        line = {
            "workload": "sgmv_prefill", "metric": "SGMV fused shrink+expand GB/s (algorithmic)",
            "value": tot_b / (ms * 1e-3) / 1e9, "unit": "GB/s", "n_gpus": 1, "steps": steps, "warmup": warm,
            "ms_per_step": ms, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": f"segmented prefill: 32 requests x 512 rows contiguous by adapter, rank {R}, "
                                   "32-slot pool, bf16", "projections": names,
                       "l2": "inputs larger than L2 (~2.9 GB per step)"},
            "per_projection": {n: {"ms": t, "GB/s": p["bytes"] / (t * 1e-3) / 1e9,
                                   "TFLOP/s": p["flops"] / (t * 1e-3) / 1e12,
                                   "hbm_frac": p["bytes"] / (t * 1e-3) / 1e9 / peak}
                               for (n, t), p in zip(per.items(), projs)},
            "tensor": {"TFLOP/s": tot_f / (ms * 1e-3) / 1e12, "peak_bf16_tflops": tpk,
                       "frac": tot_f / (ms * 1e-3) / 1e12 / tpk},
            "roofline": {"bound": "hbm", "achieved": tot_b / (ms * 1e-3) / 1e9, "peak": peak, "unit": "GB/s",
                         "frac": tot_b / (ms * 1e-3) / 1e9 / peak},
            "gpu_launches": steps * len(projs) * 2,
        }
        print(json.dumps(line), flush=True)
        return 0

    # decode_set: 7 projections, T=8, rank 16, 8 adapters (slots = a permutation), fp16.
    from persona.workloads import PROJECTIONS

    T, R, S = 8, 16, 8
    copies = 8  # rotate through 8 independent sets (~184 MB > L2) so no step hits in L2
    rng = np.random.Generator(np.random.PCG64(SEED + 2))
    sets = []
    for c in range(copies):
        slots = rng.permutation(S).astype(np.int32)
        sd = torch.from_numpy(slots).to(dev)
        projs = []
        for n, (K, N) in PROJECTIONS.items():
            if ONLY is not None and n != ONLY:
                continue
            a, b = pools(K, N, R, S, torch.float16)
            projs.append(dict(K=K, N=N, a=a, b=b, x=torch.randn(T, K, generator=gen, device=dev).half(),
                              y=torch.zeros(T, N, device=dev, dtype=torch.float16),
                              bytes=bgmv_bytes(K, N, R, slots)))
        sets.append(dict(slots=sd, projs=projs))
    step_bytes = sum(p["bytes"] for p in sets[0]["projs"])

    def fused_all():
        for st in sets:
            plan = ops.bgmv_plan(st["slots"], S)
            ops.bgmv_fused_multi([p["x"] for p in st["projs"]], [p["a"] for p in st["projs"]],
                                 [p["b"] for p in st["projs"]], st["slots"], [p["y"] for p in st["projs"]],
                                 plan=plan)

    def per_projection_all():
        for st in sets:
            plan = ops.bgmv_plan(st["slots"], S)
            for p in st["projs"]:
                ops.bgmv_fused(p["x"], p["a"], p["b"], st["slots"], p["y"], plan=plan)

    def separate_all():
        for st in sets:
            plan = ops.bgmv_plan(st["slots"], S)
            for p in st["projs"]:
                v = ops.bgmv_shrink(p["x"], p["a"], st["slots"], plan=plan)
                ops.bgmv_expand(v, p["b"], st["slots"], p["y"], plan=plan)

    for _ in range(warm):
        fused_all()
        per_projection_all()
        separate_all()
    ops.check_errors(dev)
    reps = max(1, steps // copies)
    eager_f = _timed(fused_all, reps, stream) / copies
    eager_p = _timed(per_projection_all, reps, stream) / copies
    eager_s = _timed(separate_all, reps, stream) / copies
    g = torch.cuda.CUDAGraph()
    side = torch.cuda.Stream()
    side.wait_stream(stream)
    with torch.cuda.stream(side):
        fused_all()
    stream.wait_stream(side)
    torch.cuda.synchronize()
    with torch.cuda.graph(g):
        fused_all()
    for _ in range(warm):
        g.replay()
    graph_f = _timed(g.replay, reps, stream) / copies
    ops.check_errors(dev)
    peak, _ = load_peaks()
    line = {
        "workload": "decode_set", "metric": "decode step of 7 fused LoRA projections, us per step",
        "value": graph_f * 1e3, "unit": "us", "higher_is_better": False, "n_gpus": 1,
        "steps": reps * copies, "warmup": warm, "dtype": "f16", "data": "synthetic",
        "config": {"workload": "7 Mistral-7B projections, 8 rows, rank 16, 8 adapters (one per row), fp16",
                   "l2": f"{copies} independent input sets rotated (~{copies * step_bytes / 1e6:.0f} MB > L2)"},
        "us_per_step": {"fused_graph": graph_f * 1e3, "fused_eager": eager_f * 1e3,
                        "fused_per_projection_eager": eager_p * 1e3, "separate_eager": eager_s * 1e3},
        "algorithmic_bytes_per_step": step_bytes,
        "GB/s": {"fused_graph": step_bytes / (graph_f * 1e-3) / 1e9,
                 "fused_eager": step_bytes / (eager_f * 1e-3) / 1e9},
        "hbm_frac_fused_graph": step_bytes / (graph_f * 1e-3) / 1e9 / peak,
        "launches_per_step": 2,
    }
    g.reset()
    print(json.dumps(line), flush=True)
    return 0


def run_sgmv_tp(args):
    """Config 4 across N GPUs: the segmented prefill with the expand split by
    output columns and y gathered on every rank, (a) fused: one kernel per rank
    stores each finished tile into every rank's y over NVLink, (b) baseline:
    the same kernel on the column block, then an NCCL all-gather."""
    import datetime

    import torch
    import torch.distributed as dist

    from persona import ops
    from persona.tensor_parallel import PeerBuffers, column_shards, sgmv_fused_tp, sgmv_fused_tp_nvlink
    from persona.workloads import PROJECTIONS, bgmv_bytes

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=120))
    stream = torch.cuda.current_stream()
    req, rows, R, S = 32, 512, 16, 32
    T = req * rows
    rng = np.random.Generator(np.random.PCG64(SEED + 1))
    seg = rng.permutation(req).astype(np.int32)
    indptr = (np.arange(req + 1) * rows).astype(np.int32)
    slots = np.repeat(seg, rows)
    ip, ss = torch.from_numpy(indptr).to(dev), torch.from_numpy(seg).to(dev)
    gen = torch.Generator(device=dev)
    gen.manual_seed(SEED * 1000 + 29)  # same inputs on every rank
    names = [n for n in ("gate_proj", "up_proj", "down_proj") if ONLY is None or n == ONLY]
    projs = []
    for n in names:
        K, N = PROJECTIONS[n]
        lim = 1.0 / np.sqrt(K)
        a = ((torch.rand(S, R, K, generator=gen, device=dev) * 2 - 1) * lim).to(torch.bfloat16)
        b = (torch.randn(S, N, R, generator=gen, device=dev) * 0.04).to(torch.bfloat16)
        x = torch.randn(T, K, generator=gen, device=dev).to(torch.bfloat16)
        y = torch.zeros(T, N, device=dev, dtype=torch.bfloat16)
        projs.append(dict(K=K, N=N, a=a, b=b, x=x, y=y, bytes=bgmv_bytes(K, N, R, slots)))
    peers = [PeerBuffers(p["y"]) for p in projs]
    steps, warm = max(1, args.steps), max(3, args.warmup)

    def fused():
        for p, pb in zip(projs, peers):
            sgmv_fused_tp_nvlink(p["x"], p["a"], p["b"], ip, ss, p["y"], pb)

    def baseline():
        for p in projs:
            sgmv_fused_tp(p["x"], p["a"], p["b"], ip, ss, p["y"])

    def timed(fn):
        for _ in range(warm):
            fn()
        torch.cuda.synchronize()
        dist.barrier(device_ids=[local])
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(steps):
            fn()
        e1.record(stream)
        torch.cuda.synchronize()
        t = torch.tensor([e0.elapsed_time(e1) / steps], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    ms_fused = timed(fused)
    ms_base = timed(baseline)
    ops.check_errors(dev)
    tot = sum(p["bytes"] for p in projs)
    # bytes this rank sends over NVLink per step: its column block of every y, to each peer
    nv = sum(T * (column_shards(p["N"], world)[rank][1] - column_shards(p["N"], world)[rank][0]) * 2
             for p in projs) * (world - 1)
    # per-rank roofline: HBM bytes this rank moves (x and the used A rows
    # whole, its block of B, its block of y read and written, the other
    # blocks of y written by the peers) against the measured copy bandwidth,
    # and the NVLink bytes it sends against the measured 770 GB/s per direction
    used = len(set(int(s_) for s_ in seg if s_ >= 0))
    hbm = 0
    for p in projs:
        n0, n1 = column_shards(p["N"], world)[rank]
        hbm += 2 * (T * p["K"] + used * R * p["K"] + used * (n1 - n0) * R + 2 * T * (n1 - n0)
                    + T * (p["N"] - (n1 - n0)))
    peak, _ = load_peaks()
    t_floor = max(hbm / (peak * 1e9), nv / 770e9)
    if rank == 0:
        print(json.dumps({
            "workload": "sgmv_prefill_tp", "metric": "tensor-parallel SGMV fused shrink+expand GB/s (algorithmic, "
                                                    "whole job, y gathered on every rank)",
            "value": tot / (ms_fused * 1e-3) / 1e9, "unit": "GB/s", "n_gpus": world, "steps": steps, "warmup": warm,
            "ms_per_step": ms_fused, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "segmented prefill: 32 requests x 512 rows, rank 16, 32-slot pool, bf16, "
                                   "expand split by output columns", "projections": names},
            "nvlink_bytes_per_rank_per_step": nv,
            "nvlink_gbs_per_rank": nv / (ms_fused * 1e-3) / 1e9,
            "baseline_nccl_all_gather": {"ms_per_step": ms_base, "GB/s": tot / (ms_base * 1e-3) / 1e9},
            "roofline": {"bound": "hbm+nvlink", "hbm_bytes_per_rank": hbm, "hbm_peak_gbs": peak,
                         "nvlink_peak_gbs": 770.0, "floor_ms": t_floor * 1e3,
                         "frac": t_floor * 1e3 / ms_fused},
            "gpu_launches": steps * len(projs) * 2,
        }), flush=True)
    for pb in peers:
        pb.close()
    dist.barrier(device_ids=[local])
    dist.destroy_process_group()
    return 0


def decode_measure(dev, world: int, rank: int, B: int, warm: int, steps: int) -> dict:
    """Config 5 on this rank: mixed-adapter greedy decode on a random-init
    Mistral-7B architecture (32 layers, NF4 base linears, rank-16 adapters on
    all seven projections), one adapter per row (B rows, B adapters),
    prompts of 128 random token ids, 128 new tokens per row.  A step is one
    whole generation (prefill + 127 graph-replayed decode steps), timed with
    CUDA events; returns this rank's times and the bytes a decode step must
    move."""
    import torch

    from persona import ops
    from persona.adapter_pool import AdapterPool
    from persona.engine import Request, StaticBatchEngine
    from persona.mistral import MistralConfig, MistralLoRAModel

    D, prompt, new = B, 128, 128
    cfg = MistralConfig()
    pool = AdapterPool(max_slots=D, r=16, device=dev)
    g = torch.Generator(device=dev)
    g.manual_seed(SEED * 100 + rank)
    for i in range(D):
        pool.load_random_adapter(f"persona{i}", generator=g)
    model = MistralLoRAModel(cfg, pool, dev, seed=SEED + rank)
    eng = StaticBatchEngine(model, pool, max_batch=B, max_seq_len=prompt + new)
    gen = torch.Generator().manual_seed(SEED * 10 + rank)
    reqs = [Request(f"r{i}", f"persona{i % D}", torch.randint(0, cfg.vocab, (prompt,), generator=gen).tolist(),
                    slot=pool.name_to_slot[f"persona{i % D}"]) for i in range(B)]
    for _ in range(warm):
        eng.run_static_generate(reqs, max_new_tokens=new)
    torch.cuda.synchronize()
    runs = [eng.run_static_generate(reqs, max_new_tokens=new) for _ in range(steps)]
    ops.check_errors(dev)
    # bytes one decode step must stream: the NF4 base weights and the LM head,
    # the adapters the batch uses (all 7 projections, 32 layers) and the KV
    # cache at the mean length
    per_step = model.base_bytes()
    r = 16
    lora_per_adapter = sum(r * (k + n) * 2 for k, n in (
        (cfg.hidden, cfg.q_dim), (cfg.hidden, cfg.kv_dim), (cfg.hidden, cfg.kv_dim), (cfg.q_dim, cfg.hidden),
        (cfg.hidden, cfg.intermediate), (cfg.hidden, cfg.intermediate), (cfg.intermediate, cfg.hidden)))
    per_step += lora_per_adapter * cfg.num_layers * len({q.slot for q in reqs})
    per_step += B * cfg.num_layers * 2 * cfg.kv_dim * 2 * (prompt + new / 2)
    out = {
        "ms": sum(r_["prefill_ms"] + r_["decode_ms"] for r_ in runs) / steps,
        "prefill_ms": sum(r_["prefill_ms"] for r_ in runs) / steps,
        "decode_ms": sum(r_["decode_ms"] for r_ in runs) / steps,
        "bytes_per_decode_step": per_step, "B": B, "D": D, "prompt": prompt, "new": new,
        "launches_per_decode_step": 13 * cfg.num_layers + 5,
    }
    del eng, model, pool
    torch.cuda.empty_cache()
    return out


def decode_line(m: dict, world: int, steps: int, warm: int) -> dict:
    peak, _ = load_peaks()
    step_ms = m["decode_ms"] / (m["new"] - 1)
    return {
        "workload": "e2e_decode", "metric": "mixed-adapter decode tokens/s",
        "value": world * m["B"] * m["new"] / (m["ms"] * 1e-3), "unit": "tokens/s", "n_gpus": world,
        "steps": steps, "warmup": warm, "ms_per_step": m["ms"], "higher_is_better": True, "scaling": "weak",
        "dtype": "f16 (NF4 base weights)", "data": "synthetic: random-init weights and adapters, random ids",
        "config": {"workload": "Mistral-7B architecture, 32 layers, NF4 base, rank-16 adapters on q/k/v/o/"
                               "gate/up/down, greedy", "batch_per_gpu": m["B"], "adapters": m["D"],
                   "prompt_tokens": m["prompt"], "new_tokens": m["new"],
                   "parallelism": f"dp{world} replicas" if world > 1 else "1 GPU"},
        "prefill_ms": m["prefill_ms"], "decode_ms": m["decode_ms"], "decode_ms_per_token_step": step_ms,
        "decode_tokens_per_s": world * m["B"] / (step_ms * 1e-3),
        "roofline": {"bound": "hbm", "bytes_per_decode_step": m["bytes_per_decode_step"],
                     "achieved": m["bytes_per_decode_step"] / (step_ms * 1e-3) / 1e9, "peak": peak, "unit": "GB/s",
                     "frac": m["bytes_per_decode_step"] / (step_ms * 1e-3) / 1e9 / peak},
        "gpu_launches_per_decode_step": m["launches_per_decode_step"],
    }


def run_e2e(args):
    """Config 5 alone (see decode_measure).  One GPU: batch 8 with 8
    adapters; several GPUs: data-parallel replicas (one process per GPU, no
    collective on the data path) with batch 64 and 64 adapters each; value =
    all ranks' new tokens / the max over ranks of the generation time."""
    import datetime

    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=300))
    B = args.batch or (8 if world == 1 else 64)
    # a step is a whole generation (~0.3 s): at most 10 timed, 3 to 20 warm-up
    warm, steps = min(max(3, args.warmup), 20), min(max(1, args.steps), 10)
    if world > 1:
        dist.barrier(device_ids=[local])
    m = decode_measure(dev, world, rank, B, warm, steps)
    t = torch.tensor([m["ms"], m["prefill_ms"], m["decode_ms"]], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    m["ms"], m["prefill_ms"], m["decode_ms"] = (float(v) for v in t.tolist())
    if rank == 0:
        print(json.dumps(decode_line(m, world, steps, warm)), flush=True)
    if world > 1:
        dist.barrier(device_ids=[local])
        dist.destroy_process_group()
    return 0


def run_nf4(args):
    """The seven NF4 base projections of a Mistral-7B decoder layer at decode
    (8 rows of x by default), as the decode step launches them: q / k / v in
    one launch, then o, gate / up, down.  Eight distinct layers (0.9 GB of
    packed weights, more than L2) are cycled through a CUDA graph, so every
    launch streams its weights from HBM.  Metric: packed-weight GB/s."""
    import torch

    from persona import nf4, ops
    from persona.workloads import PROJECTIONS

    if args.gpus != 1:
        raise SystemExit("--workload nf4_decode runs on one GPU")
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    M = args.batch or 8
    g = torch.Generator(device=dev)
    g.manual_seed(SEED * 1000 + 41)
    groups = [["q_proj", "k_proj", "v_proj"], ["o_proj"], ["gate_proj", "up_proj"], ["down_proj"]]
    if ONLY is not None:
        groups = [gr for gr in groups if ONLY in gr or ONLY == "+".join(gr)]
    names = [n for gr in groups for n in gr]
    layers = 8
    qs = [{n: nf4.quantize((torch.randn(PROJECTIONS[n][1], PROJECTIONS[n][0], generator=g, device=dev) * 0.02)
                           .half()) for n in names} for _ in range(layers)]
    xs = {n: torch.randn(M, PROJECTIONS[n][0], generator=g, device=dev).half() for n in names}
    ys = {n: torch.empty(M, PROJECTIONS[n][1], dtype=torch.float16, device=dev) for n in names}

    def body():
        for lq in qs:
            for gr in groups:
                nf4.linear(xs[gr[0]], [lq[n] for n in gr], outs=[ys[n] for n in gr])

    s = torch.cuda.Stream(dev)
    s.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(s):
        body()  # makes the workspace outside the capture
    torch.cuda.current_stream(dev).wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        body()
    warm, steps = max(3, args.warmup), max(1, min(args.steps, 200))
    for _ in range(warm):
        graph.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        graph.replay()
    e1.record()
    torch.cuda.synchronize()
    ops.check_errors(dev)
    ms = e0.elapsed_time(e1) / steps / layers  # one layer's launches
    byts = sum(qs[0][n].nbytes for n in names)
    peak, _ = load_peaks()
    print(json.dumps({
        "workload": "nf4_decode", "metric": "NF4 base linear GB/s (packed weights streamed)",
        "value": byts / (ms * 1e-3) / 1e9, "unit": "GB/s", "n_gpus": 1, "steps": steps, "warmup": warm,
        "ms_per_step": ms, "dtype": "f16 x, NF4 weights", "data": "synthetic",
        "config": {"workload": f"Mistral-7B layer base projections, {M} rows", "groups": ["+".join(gr) for gr in groups],
                   "l2": "8 distinct layers cycled (0.9 GB > L2)"},
        "roofline": {"bound": "hbm", "achieved": byts / (ms * 1e-3) / 1e9, "peak": peak, "unit": "GB/s",
                     "frac": byts / (ms * 1e-3) / 1e9 / peak},
        "gpu_launches": steps * layers * len(groups),
    }), flush=True)
    return 0


def run_decode_kernels(args):
    """Two small kernels of the paths, each timed alone with CUDA events:
    the row-grouping plan of the headline batch (512 Zipf rows, 256-slot
    pool) and the decode step's rotary + cache write + attention launch
    (batch 8, 32 query / 8 KV heads, head dim 128, 255 cached positions,
    the caches of 32 layers cycled so the KV reads come from HBM).  One line
    each."""
    import torch

    from persona import ops

    if args.gpus != 1:
        raise SystemExit("--workload decode_kernels runs on one GPU")
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    steps, warm = max(1, args.steps), max(3, args.warmup)
    stream = torch.cuda.current_stream()
    slots = torch.from_numpy(global_slots(1).astype(np.int32)).to(dev)
    ms = _timed(lambda: ops.bgmv_plan(slots, POOL_SLOTS), warm, stream)
    ms = _timed(lambda: ops.bgmv_plan(slots, POOL_SLOTS), steps, stream)
    print(json.dumps({"workload": "decode_kernels", "kernel": "bgmv_plan_count_kernel<512> (one CTA; pools up to 510 slots)",
                      "metric": "row-grouping plan of the 512-row Zipf batch, us per ops.bgmv_plan call", "value": ms * 1e3,
                      "unit": "us", "higher_is_better": False, "n_gpus": 1, "steps": steps, "warmup": warm,
                      "config": {"rows": ROWS_PER_GPU, "pool_slots": POOL_SLOTS}}), flush=True)
    B, Hq, Hkv, L, D, layers = 8, 32, 8, 256, 128, 32
    g = torch.Generator(device=dev).manual_seed(SEED * 1000 + 53)
    kc = [torch.randn(B, Hkv, L, D, generator=g, device=dev).half() for _ in range(layers)]
    vc = [torch.randn(B, Hkv, L, D, generator=g, device=dev).half() for _ in range(layers)]
    q = torch.randn(B, Hq, D, generator=g, device=dev).half()
    k = torch.randn(B, Hkv, D, generator=g, device=dev).half()
    v = torch.randn(B, Hkv, D, generator=g, device=dev).half()
    out = torch.empty_like(q)
    pos = torch.full((1,), L - 1, dtype=torch.int32, device=dev)
    length = torch.full((1,), L, dtype=torch.int32, device=dev)

    def all_layers():
        for li in range(layers):
            ops.rope_decode_attention(q, k, v, kc[li], vc[li], pos, length, out, 1e6, D ** -0.5)

    _timed(all_layers, warm, stream)
    ms = _timed(all_layers, steps, stream) / layers
    ops.check_errors(dev)
    byts = B * Hkv * L * D * 2 * 2 + B * (Hq + 2 * Hkv) * D * 2 + B * Hq * D * 2  # KV read, q/k/v in, out
    peak, _ = load_peaks()
    print(json.dumps({"workload": "decode_kernels", "kernel": "decode_attention_kernel (rotary + cache write fused)",
                      "metric": "decode attention (rotary + cache write + attention), us per launch",
                      "value": ms * 1e3, "unit": "us", "higher_is_better": False, "n_gpus": 1, "steps": steps,
                      "warmup": warm, "config": {"batch": B, "q_heads": Hq, "kv_heads": Hkv, "positions": L,
                                                 "l2": f"{layers} layers' caches cycled ({layers * 2 * kc[0].numel() * 2 / 1e6:.0f} MB > L2)"},
                      "roofline": {"bound": "hbm", "algorithmic_bytes": byts,
                                   "achieved": byts / (ms * 1e-3) / 1e9, "peak": peak, "unit": "GB/s",
                                   "frac": byts / (ms * 1e-3) / 1e9 / peak},
                      "gpu_launches": steps * layers}), flush=True)
    return 0


def main():
    global ONLY
    args = parse_args()
    ONLY = args.only
    if args.impl == "reference":
        return run_reference(args)
    if args.workload == "e2e_decode":
        return run_e2e(args)
    if args.workload == "nf4_decode":
        return run_nf4(args)
    if args.workload == "decode_kernels":
        return run_decode_kernels(args)
    if args.workload == "sgmv_prefill" and args.gpus > 1:
        return run_sgmv_tp(args)
    if args.workload != "mixed_decode":
        return run_extra(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
