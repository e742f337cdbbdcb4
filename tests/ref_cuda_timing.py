"""Times the reference's own CUDA kernels (rebuilt for sm_100a, separate
shrink + expand through ``tests/ref_cuda_runner.py`` in a process of their own)
against this package's fused and separate ops on the config-2 and config-3
projections; prints JSON.  Needs a GPU and ``oracle/_ref/persona_ref_C.so``.

    python tests/ref_cuda_timing.py
"""
import json
import os
import subprocess
import sys
import tempfile
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parents[1]
sys.path[:0] = [str(ROOT), str(ROOT / "multi-lora-llm-kernel_b200")]
from persona import ops, workloads  # noqa: E402

dev = torch.device("cuda", 0)
res = {}


def ours(wl, p, iters=50):
    """Mean ms of the fused op (plan reused) and of shrink + expand."""
    sd = torch.from_numpy(wl.slots).to(dev)
    x, a, b, y = [torch.from_numpy(np.ascontiguousarray(t)).to(dev) for t in (p.x, p.a_pool, p.b_pool, p.y)]
    plan = ops.bgmv_plan(sd, a.shape[0])
    for _ in range(3): ops.bgmv_fused(x, a, b, sd, y, plan=plan)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(iters): ops.bgmv_fused(x, a, b, sd, y, plan=plan)
    e1.record(); torch.cuda.synchronize()
    f = e0.elapsed_time(e1) / iters
    for _ in range(3):
        v = ops.bgmv_shrink(x, a, sd); ops.bgmv_expand(v, b, sd, y)
    torch.cuda.synchronize()
    e0.record()
    for _ in range(iters):
        v = ops.bgmv_shrink(x, a, sd); ops.bgmv_expand(v, b, sd, y)
    e1.record(); torch.cuda.synchronize()
    return f, e0.elapsed_time(e1) / iters


for tag, wl in (("config2", workloads.decode_set(1)), ("config3", workloads.mixed_batch(2))):
    for p in wl.projections:
        with tempfile.TemporaryDirectory() as td:
            inp, out = os.path.join(td, "i.npz"), os.path.join(td, "o.npz")
            np.savez(inp, x=p.x, a_pool=p.a_pool, b_pool=p.b_pool, slots=wl.slots, y=p.y, dtype=np.array("f16"))
            r = subprocess.run([sys.executable, str(ROOT / "tests" / "ref_cuda_runner.py"), inp, out, "--time", "20"],
                               capture_output=True, text=True)
            assert r.returncode == 0, r.stdout + r.stderr
            ref_ms = float(np.load(out)["ms"])
        f, s = ours(wl, p)
        res[f"{tag}/{p.name}"] = {"reference_cuda_ms": ref_ms, "ours_fused_ms": f, "ours_separate_ms": s,
                                  "speedup_fused": ref_ms / f}
print(json.dumps(res, indent=1))
