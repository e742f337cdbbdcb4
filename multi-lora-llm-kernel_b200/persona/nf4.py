"""NF4 base linears: the 4-bit base weights under the LoRA layers.

The reference's base model is loaded through bitsandbytes with NF4, blocksize
64, double-quantised scales and fp16 compute (reference ``bench/e2e.py:70-90``)
and each patched projection calls ``self.base(x)`` before the LoRA ops
(``persona/lora_layer.py:30-45``).  Here the base weight is held in this
package's tiled NF4 format (``persona_nf4_*`` in ``include/persona_bgmv.h``)
and applied by ``torch.ops.persona.nf4_linear``: at decode sizes (up to 64
rows per launch) a kernel that streams the 4-bit codes once; for longer
inputs (prefill) the weight is expanded to fp16 by
``torch.ops.persona.nf4_dequantize`` and multiplied with cuBLAS.
"""

from __future__ import annotations

import os
from dataclasses import dataclass
from typing import List, Optional, Sequence

import torch
import torch.nn as nn

from persona import ops

# Rows of x up to which the streaming kernel is used; above it the weight is
# dequantised and multiplied densely.  PERSONA_NF4_DENSE_ABOVE overrides it.
DENSE_ABOVE_ROWS = int(os.environ.get("PERSONA_NF4_DENSE_ABOVE", "64"))


@dataclass
class NF4Weight:
    """One quantised matrix W[N, K] (fp16 semantics)."""

    packed: torch.Tensor  # uint8 [N / 128, K / 128, 8464]
    offset: torch.Tensor  # float32 [1]
    N: int
    K: int

    @property
    def nbytes(self) -> int:
        return self.packed.numel() + 4


def quantize(w: torch.Tensor) -> NF4Weight:
    """Quantise an fp16 CUDA matrix [N, K] (N, K multiples of 128)."""
    ops._load()
    if w.dtype != torch.float16:
        raise TypeError("nf4.quantize: w must be float16")
    packed, offset = torch.ops.persona.nf4_quantize(w.contiguous())
    return NF4Weight(packed, offset, int(w.shape[0]), int(w.shape[1]))


def dequantize(q: NF4Weight) -> torch.Tensor:
    """fp16 [N, K] copy of the weight."""
    ops._load()
    return torch.ops.persona.nf4_dequantize(q.packed, q.offset, q.N, q.K)


def linear(x: torch.Tensor, weights: Sequence[NF4Weight], outs: Optional[Sequence[torch.Tensor]] = None,
           dense_above: Optional[int] = None,
           addends: Optional[Sequence[torch.Tensor]] = None) -> List[torch.Tensor]:
    """``y_i = x @ W_i^T`` (``+ addends[i]``, fp32 [M, N_i], before the one
    rounding) for up to four weights that share x ([M, K] fp16, unit inner
    stride); one launch at decode sizes."""
    ops._load()
    if x.dim() != 2:
        raise ValueError("nf4.linear: x must be [M, K]")
    M = x.shape[0]
    if dense_above is None:
        dense_above = DENSE_ABOVE_ROWS
    if outs is None:
        outs = [torch.empty(M, w.N, dtype=torch.float16, device=x.device) for w in weights]
    if M > dense_above:
        for i, (w, y) in enumerate(zip(weights, outs)):
            if addends is None:
                torch.matmul(x, dequantize(w).t(), out=y)
            else:
                y.copy_(torch.matmul(x.float(), dequantize(w).float().t()) + addends[i])
        return list(outs)
    xc = x if x.stride(1) == 1 else x.contiguous()
    if addends is None:
        torch.ops.persona.nf4_linear(xc, [w.packed for w in weights], [w.offset for w in weights], list(outs))
    else:
        torch.ops.persona.nf4_linear_add(xc, [w.packed for w in weights], [w.offset for w in weights],
                                         list(addends), list(outs))
    return list(outs)


class NF4Linear(nn.Module):
    """Drop-in for a bias-free fp16 ``nn.Linear`` whose weight is NF4."""

    def __init__(self, weight: NF4Weight):
        super().__init__()
        self.weight_q = weight
        self.in_features = weight.K
        self.out_features = weight.N

    @classmethod
    def from_dense(cls, w: torch.Tensor) -> "NF4Linear":
        return cls(quantize(w))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        shp = x.shape
        x2 = x.reshape(-1, shp[-1])
        y = linear(x2, [self.weight_q])[0]
        return y.reshape(*shp[:-1], self.out_features)
