"""Generate the golden BGMV vectors from the reference's own implementation.

Runs ONLY where the reference checkout is present (the build container): it
loads the reference's ``persona/ops.py`` by file path and calls its fp32
torch functions ``bgmv_shrink_ref`` / ``bgmv_expand_ref`` /
``bgmv_forward_ref`` on seeded inputs, and writes inputs + outputs as
``.npz`` fixtures beside this script.  The fixtures are committed; the tests
and the oracle read them without the reference.

    python tests/golden/make_golden.py [--ref /path/to/reference]

bf16 tensors are stored as uint16 bit patterns.
"""

from __future__ import annotations

import argparse
import importlib.util
import os
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parents[1] / "multi-lora-llm-kernel_b200"))

from persona import workloads  # noqa: E402


def load_ref_ops(ref_root: Path):
    spec = importlib.util.spec_from_file_location("reference_persona_ops",
                                                  ref_root / "persona" / "ops.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def t16(a: np.ndarray, dtype: str) -> torch.Tensor:
    if dtype == "f16":
        return torch.from_numpy(np.ascontiguousarray(a, np.float16))
    return torch.from_numpy(np.ascontiguousarray(a, np.uint16).view(np.int16)).view(torch.bfloat16)


def np16(t: torch.Tensor, dtype: str) -> np.ndarray:
    if dtype == "f16":
        return t.contiguous().numpy().astype(np.float16)
    return t.contiguous().view(torch.int16).numpy().view(np.uint16).copy()


def store16(a32: np.ndarray, dtype: str) -> np.ndarray:
    t = torch.from_numpy(np.ascontiguousarray(a32, np.float32))
    return np16(t.to(torch.float16 if dtype == "f16" else torch.bfloat16), dtype)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("PERSONA_REFERENCE_DIR"),
                    required="PERSONA_REFERENCE_DIR" not in os.environ,
                    help="checkout of the reference repository (default: $PERSONA_REFERENCE_DIR)")
    args = ap.parse_args()
    ops = load_ref_ops(Path(args.ref))
    out = {}
    rng = np.random.Generator(np.random.PCG64(1234))
    ref_slots = np.array([0, 1, 2, 3, 0, 1, -1, 2], np.int32)  # tests/test_bgmv_cuda.py:27

    # --- shrink cases, the reference CUDA test's shapes (tests/test_bgmv_cuda.py:19-29)
    for dtype in ("f16", "bf16"):
        for R in (8, 16, 32, 64):
            T, S = 8, 4
            K = 256 if R <= 16 else 64
            x = store16(rng.standard_normal((T, K)).astype(np.float32), dtype)
            a = store16((rng.standard_normal((S, R, K)) * 0.01).astype(np.float32), dtype)
            v = ops.bgmv_shrink_ref(t16(x, dtype), t16(a, dtype), torch.from_numpy(ref_slots))
            key = f"shrink_{dtype}_r{R}"
            out[f"{key}/x"], out[f"{key}/a"], out[f"{key}/slots"] = x, a, ref_slots
            out[f"{key}/v"] = v.numpy()

    # --- expand cases (tests/test_bgmv_cuda.py:32-43), random initial y
    for dtype in ("f16", "bf16"):
        for R in (8, 16, 32, 64):
            T, S = 8, 4
            N = 256 if R <= 16 else 64
            v = rng.standard_normal((T, R)).astype(np.float32)
            b = store16((rng.standard_normal((S, N, R)) * 0.01).astype(np.float32), dtype)
            y = store16(rng.standard_normal((T, N)).astype(np.float32), dtype)
            yt = t16(y, dtype).clone()
            ops.bgmv_expand_ref(torch.from_numpy(v), t16(b, dtype), torch.from_numpy(ref_slots), yt)
            key = f"expand_{dtype}_r{R}"
            out[f"{key}/v"], out[f"{key}/b"], out[f"{key}/slots"] = v, b, ref_slots
            out[f"{key}/y_in"], out[f"{key}/y_out"] = y, np16(yt, dtype)

    # --- forward composition (tests/test_bgmv_reference.py:27-38)
    T, K, N, S, R = 3, 64, 64, 2, 16
    x = store16(rng.standard_normal((T, K)).astype(np.float32), "f16")
    a = store16((rng.standard_normal((S, R, K)) * 0.01).astype(np.float32), "f16")
    b = store16((rng.standard_normal((S, N, R)) * 0.01).astype(np.float32), "f16")
    sl = np.array([0, 1, 0], np.int32)
    y = ops.bgmv_forward_ref(t16(x, "f16"), t16(a, "f16"), t16(b, "f16"), torch.from_numpy(sl))
    for k_, v_ in dict(x=x, a=a, b=b, slots=sl, y=np16(y, "f16")).items():
        out[f"forward_f16/{k_}"] = v_

    # --- all rows without an adapter (tests/test_bgmv_reference.py:9-24)
    T, K, S, R = 8, 128, 4, 16
    x = store16(rng.standard_normal((T, K)).astype(np.float32), "bf16")
    a = store16(rng.standard_normal((S, R, K)).astype(np.float32), "bf16")
    b = store16(rng.standard_normal((S, K, R)).astype(np.float32), "bf16")
    sl = np.full((T,), -1, np.int32)
    v = ops.bgmv_shrink_ref(t16(x, "bf16"), t16(a, "bf16"), torch.from_numpy(sl))
    yt = torch.ones(T, K, dtype=torch.bfloat16)
    ops.bgmv_expand_ref(v, t16(b, "bf16"), torch.from_numpy(sl), yt)
    for k_, v_ in dict(x=x, a=a, b=b, slots=sl, v=v.numpy(), y=np16(yt, "bf16")).items():
        out[f"null_bf16/{k_}"] = v_

    # --- the single-projection benchmark case (8 rows, 4096->4096, rank 16, 4 adapters)
    wl = workloads.single_projection(seed=0)
    p = wl.projections[0]
    v = ops.bgmv_shrink_ref(t16(p.x, "f16"), t16(p.a_pool, "f16"), torch.from_numpy(wl.slots))
    yt = t16(p.y, "f16").clone()
    ops.bgmv_expand_ref(v, t16(p.b_pool, "f16"), torch.from_numpy(wl.slots), yt)
    out["single_projection/checksum"] = np.frombuffer(
        workloads.checksum(p.x, p.a_pool, p.b_pool, wl.slots, p.y).encode(), np.uint8)
    out["single_projection/slots"] = wl.slots
    out["single_projection/v"] = v.numpy()
    out["single_projection/y"] = np16(yt, "f16")

    # --- a small mixed batch: Zipf slots with -1 rows, rank 64, many rows per adapter
    wl = workloads.mixed_batch(seed=5, T=64, R=64, S=16, names=["k_proj"])
    p = wl.projections[0]
    v = ops.bgmv_shrink_ref(t16(p.x, "f16"), t16(p.a_pool, "f16"), torch.from_numpy(wl.slots))
    yt = t16(p.y, "f16").clone()
    ops.bgmv_expand_ref(v, t16(p.b_pool, "f16"), torch.from_numpy(wl.slots), yt)
    out["mixed_small/checksum"] = np.frombuffer(
        workloads.checksum(p.x, p.a_pool, p.b_pool, wl.slots, p.y).encode(), np.uint8)
    out["mixed_small/slots"] = wl.slots
    out["mixed_small/v"] = v.numpy()
    out["mixed_small/y"] = np16(yt, "f16")

    # --- fp32 -> bf16 rounding as torch does it (ties, subnormals, inf, nan)
    vals = np.concatenate([
        rng.standard_normal(4096).astype(np.float32) * 10,
        np.array([1.0 + 2 ** -8, 1.0 + 3 * 2 ** -8, -1.0 - 2 ** -8, 3.3895e38, -3.3895e38,
                  1e-40, -1e-40, 0.0, -0.0, np.inf, -np.inf, np.nan], np.float32)])
    out["bf16_round/f32"] = vals
    out["bf16_round/bits"] = np16(torch.from_numpy(vals).to(torch.bfloat16), "bf16")

    np.savez_compressed(HERE / "golden_bgmv.npz", **out)
    print(f"wrote {HERE / 'golden_bgmv.npz'} ({len(out)} arrays)")


if __name__ == "__main__":
    main()
