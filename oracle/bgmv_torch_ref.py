"""CPU torch restatement of the reference's fp32 BGMV -- TEST INFRASTRUCTURE.

The reference's CPU path is torch code (``persona/ops.py:12-68``): it widens
the whole adapter pool to fp32 on every call, then does one fp32
matrix-vector product per row and rounds y once.  ``bench.py``'s CPU legs
(the ``cpu_baseline`` leg and ``--impl reference``) time this restatement on
the host cores, because it runs the same torch operations on the same
threads as the reference's own code would; ``oracle/bgmv_oracle.py`` (numpy)
stays the checker.  Both are pinned by ``tests/test_oracle.py`` against the
golden vectors that the reference's own functions produced.

Nothing in the product imports this module.
"""

from __future__ import annotations

import torch


def bgmv_shrink_ref(x: torch.Tensor, a_pool: torch.Tensor, slots: torch.Tensor) -> torch.Tensor:
    """``v[t] = A[slots[t]] @ x[t]`` in fp32; slot -1 rows give zeros
    (reference ``persona/ops.py:12-34``)."""
    T = x.shape[0]
    R = a_pool.shape[1]
    x32 = x.float()
    a32 = a_pool.float()  # the whole pool, every call, as the reference does
    v = torch.zeros(T, R, dtype=torch.float32)
    sl = slots.tolist()
    for t in range(T):
        s = sl[t]
        if s < 0:
            continue
        v[t] = a32[s] @ x32[t]
    return v


def bgmv_expand_ref(v: torch.Tensor, b_pool: torch.Tensor, slots: torch.Tensor, y: torch.Tensor) -> torch.Tensor:
    """``y[t] = round(y[t] + B[slots[t]] @ v[t])`` in place, fp32 sum and one
    rounding; slot -1 rows untouched (reference ``persona/ops.py:37-56``)."""
    y32 = y.float()
    b32 = b_pool.float()
    sl = slots.tolist()
    for t in range(v.shape[0]):
        s = sl[t]
        if s < 0:
            continue
        y32[t] += b32[s] @ v[t]
    y.copy_(y32.to(y.dtype))
    return y


def bgmv_forward_ref(x: torch.Tensor, a_pool: torch.Tensor, b_pool: torch.Tensor, slots: torch.Tensor,
                     y: torch.Tensor) -> torch.Tensor:
    """``expand(shrink(x))`` into ``y`` (reference ``persona/ops.py:59-68``)."""
    return bgmv_expand_ref(bgmv_shrink_ref(x, a_pool, slots), b_pool, slots, y)
