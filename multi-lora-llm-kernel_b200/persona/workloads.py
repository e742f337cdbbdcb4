"""Seeded synthetic BGMV / SGMV workloads (numpy PCG64, host memory).

These are the five benchmark configurations of the multi-LoRA decode path,
generated deterministically so that the parity tests, the golden fixtures
and the benchmark all see bit-identical inputs on any machine:

* ``single_projection``: 8 rows, 4096->4096, rank 16, 4 adapters, fp16.
* ``decode_set``: the seven Mistral-7B projections at decode, 8 rows, rank 16,
  8 adapters (one per row, a permutation), fp16.
* ``mixed_batch``: 512 rows, the seven projection shapes, rank 64, a pool of
  256 adapters, slots drawn from a truncated Zipf(1.1) with 5 % of rows -1.
* ``segmented_prefill``: 32 requests x 512 rows, contiguous by adapter, rank
  16, bf16, gate/up (4096->14336) and down (14336->4096).

Value distributions: ``x ~ N(0, 1)``, ``A ~ U(-1/sqrt(h_in), 1/sqrt(h_in))``,
``B ~ N(0, 0.02)`` multiplied by the LoRA scale ``alpha/r = 2`` (the scale is
folded into B when a pool is built, as ``persona/adapter_pool.py:98`` of the
reference does).  bf16 tensors are returned as ``np.uint16`` bit patterns.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Dict, List, Optional

import numpy as np

# Mistral-7B projection geometry (h_in, h_out).
PROJECTIONS: Dict[str, tuple] = {
    "q_proj": (4096, 4096),
    "k_proj": (4096, 1024),
    "v_proj": (4096, 1024),
    "o_proj": (4096, 4096),
    "gate_proj": (4096, 14336),
    "up_proj": (4096, 14336),
    "down_proj": (14336, 4096),
}

LORA_SCALE = 2.0


def _f32_to_bf16_bits(a: np.ndarray) -> np.ndarray:
    u = np.ascontiguousarray(a, np.float32).view(np.uint32).astype(np.uint64)
    r = (u + np.uint64(0x7FFF) + ((u >> np.uint64(16)) & np.uint64(1))) >> np.uint64(16)
    return r.astype(np.uint16)


def _store(a32: np.ndarray, dtype: str) -> np.ndarray:
    if dtype == "f16":
        return a32.astype(np.float16)
    if dtype == "bf16":
        return _f32_to_bf16_bits(a32)
    raise ValueError(dtype)


@dataclass
class Projection:
    """One LoRA-wrapped linear: inputs for a shrink+expand call."""

    name: str
    K: int
    N: int
    R: int
    S: int
    dtype: str
    x: np.ndarray          # [T, K]
    a_pool: np.ndarray     # [S, R, K]
    b_pool: np.ndarray     # [S, N, R] (scale folded in)
    y: np.ndarray          # [T, N] initial base output


@dataclass
class Workload:
    name: str
    T: int
    slots: np.ndarray                  # [T] int32
    projections: List[Projection] = field(default_factory=list)
    indptr: Optional[np.ndarray] = None     # segmented only: [D+1]
    seg_slots: Optional[np.ndarray] = None  # segmented only: [D]


def make_projection(rng: np.random.Generator, name: str, T: int, K: int, N: int,
                    R: int, S: int, dtype: str, y_init: str = "zeros") -> Projection:
    lim = 1.0 / np.sqrt(K)
    x = _store(rng.standard_normal((T, K), dtype=np.float32), dtype)
    a = _store(rng.uniform(-lim, lim, size=(S, R, K)).astype(np.float32), dtype)
    b = _store((rng.standard_normal((S, N, R), dtype=np.float32) * np.float32(0.02)
                * np.float32(LORA_SCALE)), dtype)
    if y_init == "zeros":
        y = _store(np.zeros((T, N), np.float32), dtype)
    else:
        y = _store(rng.standard_normal((T, N), dtype=np.float32), dtype)
    return Projection(name, K, N, R, S, dtype, x, a, b, y)


def zipf_slots(rng: np.random.Generator, T: int, S: int, s: float = 1.1,
               null_frac: float = 0.05) -> np.ndarray:
    """Truncated Zipf ``P(k) ~ (k+1)^-s`` over ``[0, S)``, then an independent
    Bernoulli(null_frac) sets rows to -1 (no adapter)."""
    p = (np.arange(S, dtype=np.float64) + 1.0) ** (-s)
    p /= p.sum()
    slots = rng.choice(S, size=T, p=p).astype(np.int32)
    slots[rng.random(T) < null_frac] = -1
    return slots


def single_projection(seed: int = 0) -> Workload:
    rng = np.random.Generator(np.random.PCG64(seed))
    T, K, N, R, S = 8, 4096, 4096, 16, 4
    proj = make_projection(rng, "q_proj", T, K, N, R, S, "f16")
    slots = rng.integers(0, S, size=T).astype(np.int32)
    return Workload("single_projection", T, slots, [proj])


def decode_set(seed: int = 1, T: int = 8, R: int = 16, D: int = 8,
               names: Optional[List[str]] = None) -> Workload:
    rng = np.random.Generator(np.random.PCG64(seed))
    names = names or list(PROJECTIONS)
    slots = rng.permutation(D).astype(np.int32)[:T] if T <= D else \
        rng.integers(0, D, size=T).astype(np.int32)
    projs = [make_projection(rng, n, T, *PROJECTIONS[n], R, D, "f16") for n in names]
    return Workload("decode_set", T, slots, projs)


def mixed_batch(seed: int = 2, T: int = 512, R: int = 64, S: int = 256,
                names: Optional[List[str]] = None, dtype: str = "f16") -> Workload:
    rng = np.random.Generator(np.random.PCG64(seed))
    names = names or list(PROJECTIONS)
    slots = zipf_slots(rng, T, S)
    projs = [make_projection(rng, n, T, *PROJECTIONS[n], R, S, dtype) for n in names]
    return Workload("mixed_batch", T, slots, projs)


def segmented_prefill(seed: int = 3, requests: int = 32, rows_per_request: int = 512,
                      R: int = 16, names: Optional[List[str]] = None,
                      dtype: str = "bf16") -> Workload:
    rng = np.random.Generator(np.random.PCG64(seed))
    names = names or ["gate_proj", "down_proj"]
    T = requests * rows_per_request
    indptr = (np.arange(requests + 1) * rows_per_request).astype(np.int32)
    seg_slots = rng.permutation(requests).astype(np.int32)
    slots = np.repeat(seg_slots, rows_per_request).astype(np.int32)
    projs = [make_projection(rng, n, T, *PROJECTIONS[n], R, requests, dtype) for n in names]
    return Workload("segmented_prefill", T, slots, projs, indptr=indptr, seg_slots=seg_slots)


def checksum(*arrays: np.ndarray) -> str:
    """Stable digest of input arrays (guards fixtures against generator drift)."""
    import hashlib

    h = hashlib.sha256()
    for a in arrays:
        a = np.ascontiguousarray(a)
        h.update(str(a.dtype).encode())
        h.update(str(a.shape).encode())
        h.update(a.tobytes())
    return h.hexdigest()


def bgmv_bytes(K: int, N: int, R: int, slots: np.ndarray, elem: int = 2) -> int:
    """Algorithmic HBM bytes of one fused shrink+expand call.

    Each distinct adapter's A (R*K) and B (N*R) once, each active row's x
    (K) once and y (N) read and written once, every slot once; rows with
    slot -1 move no x/y bytes.
    """
    s = np.asarray(slots)
    act = s >= 0
    u = int(np.unique(s[act]).size)
    ta = int(act.sum())
    return int(u * (R * K + N * R) * elem + ta * K * elem + 2 * ta * N * elem + 4 * s.size)
