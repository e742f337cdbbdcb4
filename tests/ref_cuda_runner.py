"""Runs the reference's own CUDA kernels (``oracle/_ref/persona_ref_C.so``,
built for sm_100a by ``oracle/build_ref_cuda.py``) in a process of their
own, since they register the same ``torch.ops.persona`` namespace as this
package.

    python tests/ref_cuda_runner.py IN.npz OUT.npz [--time ITERS]

IN holds ``x, a_pool, b_pool, slots, y`` (fp16 as uint16 bit patterns under
``*_bits`` when ``dtype`` is bf16); OUT receives ``v`` (fp32) and ``y``
after ``ops.bgmv_shrink`` + ``ops.bgmv_expand`` called the way the
reference's ``persona/ops.py:71-90`` calls them, and, with ``--time``, the
mean device time of one shrink + expand pair in ``ms`` (CUDA events).
"""

import sys
from pathlib import Path

import numpy as np
import torch

LIB = Path(__file__).resolve().parents[1] / "oracle" / "_ref" / "persona_ref_C.so"


def _t(a, dt, dev):
    t = torch.from_numpy(np.ascontiguousarray(a))
    if dt == "bf16":
        return t.view(torch.int16).to(dev).view(torch.bfloat16)
    return t.to(dev)


def main() -> int:
    inp, out = sys.argv[1], sys.argv[2]
    iters = int(sys.argv[4]) if len(sys.argv) > 4 and sys.argv[3] == "--time" else 0
    torch.ops.load_library(str(LIB))
    d = np.load(inp)
    dt = str(d["dtype"])
    dev = torch.device("cuda", 0)
    x, a, b = _t(d["x"], dt, dev), _t(d["a_pool"], dt, dev), _t(d["b_pool"], dt, dev)
    slots = torch.from_numpy(d["slots"]).to(dev)
    y = _t(d["y"], dt, dev)
    T, R = x.shape[0], a.shape[1]
    v = torch.empty(T, R, dtype=torch.float32, device=dev)
    torch.ops.persona.bgmv_shrink(x, a, slots, v)
    torch.ops.persona.bgmv_expand(v, b, slots, y)
    torch.cuda.synchronize()
    res = {"v": v.cpu().numpy()}
    yc = y.cpu()
    res["y"] = yc.view(torch.int16).numpy().view(np.uint16) if dt == "bf16" else yc.numpy()
    if iters:
        ys = _t(d["y"], dt, dev)
        for _ in range(3):
            torch.ops.persona.bgmv_shrink(x, a, slots, v)
            torch.ops.persona.bgmv_expand(v, b, slots, ys)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(iters):
            torch.ops.persona.bgmv_shrink(x, a, slots, v)
            torch.ops.persona.bgmv_expand(v, b, slots, ys)
        e1.record()
        torch.cuda.synchronize()
        res["ms"] = np.float64(e0.elapsed_time(e1) / iters)
    np.savez(out, **res)
    return 0


if __name__ == "__main__":
    sys.exit(main())
