"""CPU oracle for the BGMV shrink/expand path -- TEST INFRASTRUCTURE ONLY.

This module restates, in numpy, the reference's fp32 torch implementation of
the multi-LoRA BGMV ops (SirBastion2/Multi-LoRA-LLM-Kernel, ``persona/ops.py``).
It is the checker the parity tests compare the CUDA kernels against, and the
CPU baseline that ``bench.py`` times.  The product package never imports it:
only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
leg do.

Parity pinning: the functions here are checked against golden vectors that
``tests/golden/make_golden.py`` produced by running the reference's own
``persona.ops.bgmv_*_ref`` functions on the same seeded inputs, and against the
reference's torch-free known-answer test (``standalone/test_bgmv.cu:36-86``).

Semantics restated (reference file:line):

* shrink  ``v[t, r] = sum_k A[slot[t], r, k] * x[t, k]`` in fp32; a row whose
  slot is -1 gets zeros (``persona/ops.py:12-34``).
* expand  ``y[t, n] = round(y[t, n] + sum_r B[slot[t], n, r] * v[t, r])``,
  accumulated in fp32 and rounded once to the storage type; a row whose slot
  is -1 is left bit-identical (``persona/ops.py:37-56``).
* forward ``expand(shrink(x))`` into a zero ``y`` (``persona/ops.py:59-68``).
* The LoRA scale ``alpha / r`` is not an argument: it is folded into B when
  the pool is built (``persona/adapter_pool.py:30-34, 98``).

Storage types: ``"f16"`` arrays are ``np.float16``; ``"bf16"`` arrays are
``np.uint16`` bit patterns (numpy has no bfloat16), converted here with
round-to-nearest-even exactly like torch's ``float -> bfloat16`` cast.
"""

from __future__ import annotations

import numpy as np

__all__ = [
    "to_f32",
    "from_f32",
    "bgmv_shrink_ref",
    "bgmv_expand_ref",
    "bgmv_forward_ref",
    "sgmv_slots",
    "sgmv_shrink_ref",
    "sgmv_expand_ref",
    "plan_ref",
    "kat_inputs",
    "algorithmic_bytes",
]


# ---------------------------------------------------------------- dtypes ---

def to_f32(a: np.ndarray, dtype: str) -> np.ndarray:
    """Exact widening of 16-bit storage to fp32 (``x.float()`` in the reference)."""
    if dtype == "f16":
        return np.asarray(a, dtype=np.float16).astype(np.float32)
    if dtype == "bf16":
        u = np.asarray(a, dtype=np.uint16).astype(np.uint32) << np.uint32(16)
        return u.view(np.float32)
    raise ValueError(f"unknown dtype {dtype!r}")


def from_f32(a32: np.ndarray, dtype: str) -> np.ndarray:
    """Round fp32 to 16-bit storage, nearest-even (``y32.to(y.dtype)``)."""
    a32 = np.ascontiguousarray(a32, dtype=np.float32)
    if dtype == "f16":
        return a32.astype(np.float16)
    if dtype == "bf16":
        u = a32.view(np.uint32).astype(np.uint64)
        nan = np.isnan(a32)
        rounded = (u + np.uint64(0x7FFF) + ((u >> np.uint64(16)) & np.uint64(1))) >> np.uint64(16)
        out = rounded.astype(np.uint16)
        # quiet NaN keeps its sign, like torch
        out[nan] = ((u[nan] >> np.uint64(16)).astype(np.uint16) | np.uint16(0x0040))
        return out
    raise ValueError(f"unknown dtype {dtype!r}")


# --------------------------------------------------------------- BGMV ops --

def bgmv_shrink_ref(x: np.ndarray, a_pool: np.ndarray, slots: np.ndarray,
                    dtype: str = "f16") -> np.ndarray:
    """``v[T,R] = A[slot] @ x`` in fp32 (reference ``persona/ops.py:12-34``).

    x: [T, K]; a_pool: [S, R, K]; slots: [T] int32 with -1 meaning "no
    adapter".  Like the reference, the whole pool is widened to fp32 once per
    call and each row is a separate fp32 matrix-vector product.
    """
    T, K = x.shape
    S, R, K2 = a_pool.shape
    if K != K2:
        raise ValueError("a_pool shape mismatch")
    x32 = to_f32(x, dtype)
    a32 = to_f32(a_pool, dtype)
    v = np.zeros((T, R), dtype=np.float32)
    for t in range(T):
        s = int(slots[t])
        if s < 0:
            continue
        if s >= S:
            raise IndexError("slot out of range")
        v[t] = a32[s] @ x32[t]
    return v


def bgmv_expand_ref(v: np.ndarray, b_pool: np.ndarray, slots: np.ndarray,
                    y: np.ndarray, dtype: str = "f16") -> np.ndarray:
    """``y[t] += B[slot] @ v[t]`` with one rounding (``persona/ops.py:37-56``).

    Updates ``y`` in place (the reference's in-place contract) and returns it.
    """
    T, R = v.shape
    S, N, R2 = b_pool.shape
    if R != R2:
        raise ValueError("b_pool rank dim mismatch")
    y32 = to_f32(y, dtype)
    b32 = to_f32(b_pool, dtype)
    v32 = np.asarray(v, dtype=np.float32)
    for t in range(T):
        s = int(slots[t])
        if s < 0:
            continue
        if s >= S:
            raise IndexError("slot out of range")
        y32[t] += b32[s] @ v32[t]
    y[...] = from_f32(y32, dtype)
    return y


def bgmv_forward_ref(x: np.ndarray, a_pool: np.ndarray, b_pool: np.ndarray,
                     slots: np.ndarray, dtype: str = "f16",
                     y: np.ndarray | None = None) -> np.ndarray:
    """``expand(shrink(x))`` (``persona/ops.py:59-68``); ``y`` defaults to zeros."""
    v = bgmv_shrink_ref(x, a_pool, slots, dtype)
    if y is None:
        y = from_f32(np.zeros((x.shape[0], b_pool.shape[1]), np.float32), dtype)
    return bgmv_expand_ref(v, b_pool, slots, y, dtype)


# ------------------------------------------------------------------- SGMV --

def sgmv_slots(indptr: np.ndarray, seg_slots: np.ndarray, T: int) -> np.ndarray:
    """Per-row slots of a segmented batch.

    The reference has no segmented op; its callers express a prefill of
    contiguous same-adapter rows as per-token slots
    (``LoRAContext.set_batch_slots``, ``persona/lora_layer.py:21-28``).  SGMV
    is therefore checked against BGMV on the expanded slots.  Rows outside
    every segment carry slot -1.  A segment is used only if
    ``0 <= lo <= hi <= T`` and no earlier ``indptr`` entry exceeds ``lo`` (so
    used segments never overlap); other segments, and slots outside
    ``[-1, S)``, leave their rows at -1 (the device reports them).
    """
    slots = np.full((T,), -1, dtype=np.int32)
    run_max = None
    for i in range(len(seg_slots)):
        lo, hi = int(indptr[i]), int(indptr[i + 1])
        run_max = lo if run_max is None else max(run_max, lo)
        if lo < 0 or hi < lo or hi > T or run_max > lo:
            continue
        slots[lo:hi] = int(seg_slots[i])
    return slots


def sgmv_shrink_ref(x, a_pool, indptr, seg_slots, dtype="f16"):
    return bgmv_shrink_ref(x, a_pool, sgmv_slots(indptr, seg_slots, x.shape[0]), dtype)


def sgmv_expand_ref(v, b_pool, indptr, seg_slots, y, dtype="f16"):
    return bgmv_expand_ref(v, b_pool, sgmv_slots(indptr, seg_slots, v.shape[0]), y, dtype)


# ------------------------------------------------------------ row grouping -

def plan_ref(slots: np.ndarray, S: int, rows_per_item: int):
    """Stable grouping of a batch's rows by adapter slot.

    Not a reference function: the reference visits rows one by one
    (``csrc/bgmv_shrink.cu:16-22``).  The B200 kernels instead stream each
    adapter's A/B once for all rows that use it, so they first group rows.
    This is the integer contract the device planner must meet bit-exactly:

    * ``perm``: rows with a valid slot, sorted by slot, ties in row order;
      then the rows with slot -1 in row order; then rows with an invalid
      slot (< -1 or >= S) in row order.
    * ``items``: ``(slot, begin, count)`` chunks of at most ``rows_per_item``
      consecutive entries of ``perm`` that share a slot; first every full
      chunk (``count == rows_per_item``) in ``perm`` order, then the partial
      chunks in ``perm`` order (heaviest work first).
    * counts ``n_valid, n_null, n_bad``.
    """
    slots = np.asarray(slots, dtype=np.int64)
    T = slots.shape[0]
    rows = np.arange(T)
    valid = (slots >= 0) & (slots < S)
    null = slots == -1
    bad = ~valid & ~null
    v_rows = rows[valid]
    order = np.argsort(slots[valid], kind="stable")
    v_sorted = v_rows[order]
    perm = np.concatenate([v_sorted, rows[null], rows[bad]]).astype(np.int32)
    items = []
    i = 0
    nv = v_sorted.shape[0]
    while i < nv:
        s = int(slots[v_sorted[i]])
        j = i
        while j < nv and int(slots[v_sorted[j]]) == s:
            j += 1
        b = i
        while b < j:
            c = min(rows_per_item, j - b)
            items.append((s, b, c))
            b += c
        i = j
    items = [it for it in items if it[2] == rows_per_item] + \
        [it for it in items if it[2] < rows_per_item]
    items = np.array(items, dtype=np.int32).reshape(-1, 3)
    return perm, items, int(nv), int(null.sum()), int(bad.sum())


# ------------------------------------------------------- known answers ----

def kat_inputs():
    """Deterministic inputs of the reference's torch-free shrink test
    (``standalone/test_bgmv.cu:41-55``): T=4, K=128, R=16, S=2,
    ``x[i] = 0.01*(i%17)``, ``a[i] = 0.001*(i%11)``, slots ``{0,1,-1,0}``.
    Pass criterion there: max abs error <= 1e-2 (``:85``)."""
    T, K, R, S = 4, 128, 16, 2
    x = (np.float32(0.01) * (np.arange(T * K) % 17).astype(np.float32)).astype(np.float16)
    a = (np.float32(0.001) * (np.arange(S * R * K) % 11).astype(np.float32)).astype(np.float16)
    slots = np.array([0, 1, -1, 0], dtype=np.int32)
    return x.reshape(T, K), a.reshape(S, R, K), slots


# ---------------------------------------------------------- byte counting -

def algorithmic_bytes(T: int, K: int, N: int, R: int, slots: np.ndarray,
                      elem: int = 2, fused: bool = True) -> int:
    """Bytes one shrink+expand call must move at minimum.

    ``u*(R*K + N*R)*e + Ta*K*e + 2*Ta*N*e + 4*T`` with ``u`` the number of
    distinct valid slots and ``Ta`` the rows that carry an adapter: each used
    adapter's A and B read once, an active row's x read once and its y read
    and written once, every slot read once.  Rows with slot -1 move no x/y
    bytes, so they earn no credit.  The separate (unfused) path also writes
    and re-reads v: ``+ 2*Ta*R*4`` (reported as overhead, not credit).
    """
    slots = np.asarray(slots)
    act = slots >= 0
    u = int(np.unique(slots[act]).shape[0])
    Ta = int(act.sum())
    b = u * (R * K + N * R) * elem + Ta * K * elem + 2 * Ta * N * elem + 4 * T
    if not fused:
        b += 2 * Ta * R * 4
    return int(b)
