"""LoRAContext and MultiLoRALinear: the callers of the BGMV ops inside a model
(drop-in for the reference's ``persona/lora_layer.py``).

Per projection the reference runs shrink, then expand, through two launches
and a fp32 ``v`` in HBM (``persona/lora_layer.py:48-58``).  Here the layer
runs ONE fused launch (``ops.bgmv_fused``; the rank-R intermediate stays on
chip) and every projection of a forward pass shares one row-grouping plan
that the context builds once per slot vector.  Results equal shrink followed
by expand up to fp32 summation order.
"""

from __future__ import annotations

from typing import Dict, Optional

import torch
from torch import nn

from persona import ops


class LoRAContext:
    """One per engine.  Holds the per-token adapter slots for the current
    forward pass (``-1`` = no adapter) and the plans built from them."""

    def __init__(self, max_tokens: int, device: torch.device):
        self.token_slots = torch.full((max_tokens,), -1, dtype=torch.int32, device=device)
        self.row_slots: Optional[torch.Tensor] = None
        self.enabled = True
        self._plans: Dict[tuple, torch.Tensor] = {}

    @property
    def max_tokens(self) -> int:
        return self.token_slots.shape[0]

    def set_batch_slots(self, row_slots: torch.Tensor, seq_len: int) -> None:
        """Per-request slots -> per-token slots (prefill: ``seq_len`` tokens per
        request; decode: 1), reference ``persona/lora_layer.py:21-28``."""
        if row_slots.dtype != torch.int32:
            row_slots = row_slots.to(dtype=torch.int32)
        self.row_slots = row_slots
        self._fill(row_slots, seq_len)

    def _fill(self, row_slots: torch.Tensor, seq_len: int) -> None:
        ntok = row_slots.shape[0] * seq_len
        if ntok > self.max_tokens:
            raise ValueError(f"LoRAContext: {ntok} tokens exceed max_tokens={self.max_tokens}")
        self.token_slots[:ntok] = row_slots.to(self.token_slots.device).repeat_interleave(seq_len)
        self._plans.clear()

    def slots(self, t: int) -> torch.Tensor:
        if t > self.max_tokens:
            raise ValueError(f"LoRAContext: {t} tokens exceed max_tokens={self.max_tokens}")
        return self.token_slots[:t]

    def plan(self, t: int, num_slots: int) -> torch.Tensor:
        """Row-grouping plan of the first ``t`` token slots for a pool of
        ``num_slots`` slots; built once and reused by every projection until
        the slots change (``set_batch_slots`` or the model's pre-hook)."""
        key = (t, num_slots)
        p = self._plans.get(key)
        if p is None:
            p = ops.bgmv_plan(self.slots(t), num_slots)
            self._plans[key] = p
        return p

    def invalidate(self) -> None:
        """Call after writing ``token_slots`` directly."""
        self._plans.clear()


class MultiLoRALinear(nn.Module):
    """Wraps a base linear (e.g. an NF4 ``Linear4bit``) and adds each token's
    own adapter: ``y = base(x) + B[slot] @ (A[slot] @ x)``."""

    def __init__(self, base: nn.Module, ctx: LoRAContext, a_pool: torch.Tensor, b_pool: torch.Tensor):
        super().__init__()
        self.base = base
        self.ctx = ctx
        self.a_pool = a_pool  # [S, r, K]; may be a rank block of a packed pool
        self.b_pool = b_pool  # [S, N, r]

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        y = self.base(x)
        if not self.ctx.enabled:
            return y
        x2d = x.reshape(-1, x.shape[-1])
        if x2d.stride(-1) != 1:
            x2d = x2d.contiguous()
        y2d = y.reshape(-1, y.shape[-1])
        if y2d.stride(-1) != 1:
            y2d = y2d.contiguous()
        t = x2d.shape[0]
        plan = self.ctx.plan(t, self.a_pool.shape[0])
        ops.bgmv_fused(x2d, self.a_pool, self.b_pool, self.ctx.slots(t), y2d, plan=plan)
        if y2d.data_ptr() != y.data_ptr():
            y.copy_(y2d.view(y.shape))  # reshape had to copy: write the result back
        return y


def make_slot_hook(ctx: LoRAContext):
    """Model forward pre-hook: expand ``ctx.row_slots`` to per-token slots
    from the batch's ``input_ids`` shape (reference
    ``persona/lora_layer.py:61-71``)."""

    def hook(module, args, kwargs):
        input_ids = kwargs.get("input_ids", args[0] if args else None)
        if input_ids is None or ctx.row_slots is None:
            return
        batch, seq = input_ids.shape
        ctx._fill(ctx.row_slots[:batch], seq)

    return hook
