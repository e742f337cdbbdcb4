"""BGMV op entry points on B200 (drop-in for the reference's ``persona/ops.py``).

``bgmv_shrink`` / ``bgmv_expand`` keep the reference's signatures and return
conventions (``persona/ops.py:71-90``): shrink allocates and returns the fp32
``v``; expand updates ``y`` in place and returns it.  Both dispatch to the
``torch.ops.persona`` ops registered by the in-tree extension, which this
module loads itself (the reference left that import to the caller, so its
"CUDA" path silently ran the fp32 fallback when nobody imported
``persona._C``).

There is no CPU fallback: CPU tensors, or a missing extension, raise.  The
reference's fp32 functions ``bgmv_*_ref`` are test infrastructure here and
live in the repository's ``oracle`` package.

New in this build:

* ``bgmv_fused`` -- shrink->expand in one launch, rank-R intermediate kept on
  chip (the reference's fused kernel is a stub, ``docs/BENCHMARKS.md:238``).
* ``bgmv_fused_multi`` -- the fused op for up to 8 projections of a layer
  that share the slots, in one launch.
* ``bgmv_plan`` -- groups a batch's rows by adapter slot once on the device;
  pass the result as ``plan=`` to every shrink/expand/fused call that uses
  the same slots (a decode step's 7 projections x 32 layers share one).
* ``check_errors`` -- out-of-range slots are detected on the device (no
  per-row host sync); the next op on that device, or this function, raises.
"""

from __future__ import annotations

from typing import Optional

import torch

_EXT = None


def _load():
    """Import the native extension once; raise loudly if it is unavailable."""
    global _EXT
    if _EXT is None:
        try:
            from persona import _C  # registers torch.ops.persona.*
        except ImportError as e:  # pragma: no cover - depends on the build
            _EXT = e
        else:
            _EXT = _C
    if isinstance(_EXT, Exception):
        raise RuntimeError(
            "persona: the native BGMV extension is not built or cannot be loaded "
            "(run multi-lora-llm-kernel_b200/build.py)") from _EXT
    return _EXT


def has_cuda_ops() -> bool:
    """True when the B200 BGMV ops are registered (reference ``ops.py:8-9``)."""
    try:
        _load()
    except RuntimeError:
        return False
    return hasattr(torch.ops, "persona") and hasattr(torch.ops.persona, "bgmv_shrink")


def _require_cuda(op: str, *tensors: torch.Tensor) -> None:
    _load()
    if not all(t.is_cuda for t in tensors):
        raise RuntimeError(f"{op}: all tensors must be CUDA (this build has no CPU fallback)")


def bgmv_plan(slots: torch.Tensor, num_slots: int) -> torch.Tensor:
    """Device-side row grouping of ``slots`` for a pool of ``num_slots`` slots."""
    _require_cuda("bgmv_plan", slots)
    return torch.ops.persona.bgmv_plan(slots, int(num_slots))


def bgmv_shrink(x: torch.Tensor, a_pool: torch.Tensor, slots: torch.Tensor,
                plan: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``v[t] = A[slots[t]] @ x[t]`` in fp32; rows with slot -1 give zeros."""
    _require_cuda("bgmv_shrink", x, a_pool, slots)
    v = torch.empty((x.shape[0], a_pool.shape[1]), dtype=torch.float32, device=x.device)
    if plan is None:
        torch.ops.persona.bgmv_shrink(x.contiguous(), a_pool, slots, v)
    else:
        torch.ops.persona.bgmv_shrink_with_plan(x.contiguous(), a_pool, slots, plan, v)
    return v


def bgmv_expand(v: torch.Tensor, b_pool: torch.Tensor, slots: torch.Tensor, y: torch.Tensor,
                plan: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``y[t] += B[slots[t]] @ v[t]`` in place (fp32 sum, one rounding)."""
    _require_cuda("bgmv_expand", v, b_pool, slots, y)
    if plan is None:
        torch.ops.persona.bgmv_expand(v, b_pool, slots, y)
    else:
        torch.ops.persona.bgmv_expand_with_plan(v, b_pool, slots, plan, y)
    return y


def bgmv_fused(x: torch.Tensor, a_pool: torch.Tensor, b_pool: torch.Tensor, slots: torch.Tensor,
               y: torch.Tensor, plan: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``y[t] += B[s] @ (A[s] @ x[t])`` in one launch; returns ``y``.

    Equal, within fp32 summation order, to ``bgmv_expand(bgmv_shrink(x))``.
    """
    _require_cuda("bgmv_fused", x, a_pool, b_pool, slots, y)
    if plan is None:
        torch.ops.persona.bgmv_fused(x, a_pool, b_pool, slots, y)
    else:
        torch.ops.persona.bgmv_fused_with_plan(x, a_pool, b_pool, slots, plan, y)
    return y


def bgmv_fused_multi(xs, a_pools, b_pools, slots: torch.Tensor, ys,
                     plan: Optional[torch.Tensor] = None):
    """``ys[i] += B_i[s] @ (A_i[s] @ xs[i])`` for up to 8 projections that
    share ``slots`` (one decoder layer), in one launch; returns ``ys``.

    Each result equals ``bgmv_fused`` on that projection.  All pools share
    the rank and the slot count.
    """
    xs, a_pools, b_pools, ys = list(xs), list(a_pools), list(b_pools), list(ys)
    _require_cuda("bgmv_fused_multi", *xs, *a_pools, *b_pools, slots, *ys)
    torch.ops.persona.bgmv_fused_multi(xs, a_pools, b_pools, slots, ys, plan)
    return ys


def sgmv_shrink(x: torch.Tensor, a_pool: torch.Tensor, seg_indptr: torch.Tensor,
                seg_slots: torch.Tensor) -> torch.Tensor:
    """Segmented shrink: rows ``[seg_indptr[i], seg_indptr[i+1])`` use slot
    ``seg_slots[i]``; rows outside every segment get zeros.  Equals
    ``bgmv_shrink`` on the per-row slots the segments imply."""
    _require_cuda("sgmv_shrink", x, a_pool, seg_indptr, seg_slots)
    v = torch.empty((x.shape[0], a_pool.shape[1]), dtype=torch.float32, device=x.device)
    torch.ops.persona.sgmv_shrink(x.contiguous(), a_pool, seg_indptr, seg_slots, v)
    return v


def sgmv_expand(v: torch.Tensor, b_pool: torch.Tensor, seg_indptr: torch.Tensor,
                seg_slots: torch.Tensor, y: torch.Tensor) -> torch.Tensor:
    """Segmented expand, in place on ``y``; rows outside the segments untouched."""
    _require_cuda("sgmv_expand", v, b_pool, seg_indptr, seg_slots, y)
    torch.ops.persona.sgmv_expand(v, b_pool, seg_indptr, seg_slots, y)
    return y


def sgmv_fused(x: torch.Tensor, a_pool: torch.Tensor, b_pool: torch.Tensor, seg_indptr: torch.Tensor,
               seg_slots: torch.Tensor, y: torch.Tensor) -> torch.Tensor:
    """Segmented shrink->expand in place on ``y``."""
    _require_cuda("sgmv_fused", x, a_pool, b_pool, seg_indptr, seg_slots, y)
    torch.ops.persona.sgmv_fused(x, a_pool, b_pool, seg_indptr, seg_slots, y)
    return y


def gemv_fp16(x: torch.Tensor, W: torch.Tensor, y: torch.Tensor) -> torch.Tensor:
    """Warm-up GEMV kept from the reference (``csrc/gemv_fp16.cu``)."""
    _require_cuda("gemv_fp16", x, W, y)
    torch.ops.persona.gemv_fp16(x, W, y)
    return y


def check_errors(device: Optional[torch.device] = None, synchronize: bool = True) -> None:
    """Raise RuntimeError if a kernel on ``device`` flagged an error.

    With ``synchronize`` the device is synchronised first, so every op
    enqueued before this call has been checked.
    """
    ext = _load()
    if device is None:
        device = torch.device("cuda", torch.cuda.current_device())
    device = torch.device(device)
    if synchronize:
        torch.cuda.synchronize(device)
    bits = ext.take_device_error(device.index or 0)
    if bits:
        what = []
        if bits & 1:
            what.append("slot out of range")
        if bits & 2:
            what.append("device wait timed out")
        if bits & 4:
            what.append("invalid segment table")
        if bits & 8:
            what.append("reused plan does not match the call")
        raise RuntimeError(f"persona: device error 0x{bits:x}: {', '.join(what)}")


# ---- fused steps of the end-to-end decode (persona_add_rmsnorm & co.) ------
def add_rmsnorm(h: torch.Tensor, delta: Optional[torch.Tensor], w: torch.Tensor, out: torch.Tensor,
                eps: float) -> torch.Tensor:
    """``h += delta`` (if given) and ``out = w * fp16(h / rms(h))`` per row."""
    _require_cuda("add_rmsnorm", h, w, out)
    torch.ops.persona.add_rmsnorm(h, delta, w, out, float(eps))
    return out


def rope_cache(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
               start: torch.Tensor, per_seq: int, theta: float) -> None:
    """Rotary embedding of q and k in place and the k / v cache write."""
    _require_cuda("rope_cache", q, k, v, k_cache, v_cache, start)
    torch.ops.persona.rope_cache(q, k, v, k_cache, v_cache, start, int(per_seq), float(theta))


def silu_mul(g: torch.Tensor, u: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
    _require_cuda("silu_mul", g, u, out)
    torch.ops.persona.silu_mul(g, u, out)
    return out


def decode_attention(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, length: torch.Tensor,
                     out: torch.Tensor, scale: float) -> torch.Tensor:
    """One new token per sequence over the first ``length`` cache positions."""
    _require_cuda("decode_attention", q, k_cache, v_cache, length, out)
    torch.ops.persona.decode_attention(q, k_cache, v_cache, length, out, float(scale))
    return out


def rope_decode_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, k_cache: torch.Tensor,
                          v_cache: torch.Tensor, pos: torch.Tensor, length: torch.Tensor, out: torch.Tensor,
                          theta: float, scale: float) -> torch.Tensor:
    """``rope_cache`` (one token per sequence at ``pos``) and
    ``decode_attention`` in one launch, with the same results."""
    _require_cuda("rope_decode_attention", q, k, v, k_cache, v_cache, pos, length, out)
    torch.ops.persona.rope_decode_attention(q, k, v, k_cache, v_cache, pos, length, out, float(theta), float(scale))
    return out


def bgmv_lora_delta_multi(xs, a_pools, b_pools, slots: torch.Tensor, deltas):
    """``deltas[i][t] = B_i[s] @ (A_i[s] @ xs[i][t])`` in fp32 (0 for rows
    without adapter), at most 64 rows: the LoRA term alone, for a base
    projection that adds it (``nf4.linear(..., addends=...)``)."""
    _require_cuda("bgmv_lora_delta_multi", slots, *xs, *a_pools, *b_pools, *deltas)
    torch.ops.persona.bgmv_lora_delta_multi(list(xs), list(a_pools), list(b_pools), slots, list(deltas))
    return deltas
