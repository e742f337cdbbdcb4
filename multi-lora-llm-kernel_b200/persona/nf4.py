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


# ---- bitsandbytes NF4 checkpoints -------------------------------------------
# The 16 NF4 values as the kernels hold them (fp16 bit patterns, increasing
# order; csrc/nf4_table.h).
NF4_F16_BITS = (0xBC00, 0xB992, 0xB833, 0xB652, 0xB48D, 0xB1EA, 0xADD4, 0x0000,
                0x2D18, 0x3126, 0x33E0, 0x3568, 0x370D, 0x3880, 0x39C9, 0x3C00)
_TILE, _BLOCK, _CODE_BYTES = 128, 64, 8192
_SCALE_OFF, _S127_OFF, _CHUNK_BYTES = 8192, 8448, 8464


def _fragment_order(device) -> tuple:
    """(row, col) inside a 128 x 128 tile of the first of the two weights of
    every code byte, in storage order (the A-fragment order of
    mma.m16n8k16: warp tile, K half, lane, k-step, register byte)."""
    i = torch.arange(_CODE_BYTES, device=device)
    j, ks, lane, kh, wt = i & 3, (i >> 2) & 3, (i >> 4) & 31, (i >> 9) & 1, i >> 10
    g, t = lane >> 2, lane & 3
    return 16 * wt + g + 8 * (j & 1), 64 * kh + 16 * ks + 2 * t + 8 * (j >> 1)


def from_bitsandbytes(packed: torch.Tensor, absmax: torch.Tensor, shape: Sequence[int], quant_map: torch.Tensor,
                      blocksize: int = 64, nested_absmax: Optional[torch.Tensor] = None,
                      nested_quant_map: Optional[torch.Tensor] = None, nested_offset: float = 0.0,
                      nested_blocksize: int = 256, device=None) -> NF4Weight:
    """Convert a bitsandbytes NF4 weight to this package's tiled format.

    The reference's base linears are bitsandbytes ``Linear4bit`` layers
    (reference ``bench/e2e.py:73-88``: nf4, blocksize 64, double quantisation,
    fp16 compute).  Their storage, as its quantisation state describes it:

    * ``packed``: uint8, two 4-bit codes per byte over the row-major weight
      ``[N, K]`` flattened (element ``2i`` in the high nibble, ``2i + 1`` in
      the low one); a code indexes ``quant_map`` (the 16 NF4 values, fp32).
    * one scale (absmax) per ``blocksize`` consecutive elements; with double
      quantisation ``absmax`` holds uint8 codes and the scale of block ``b``
      is ``nested_quant_map[absmax[b]] * nested_absmax[b // nested_blocksize]
      + nested_offset``, else ``absmax`` holds the fp32 scales.

    The 4-bit codes carry over unchanged (both formats take 64 consecutive
    weights of a row per scale and the same NF4 values).  The scales are
    stored again in this format's double quantisation (int8 codes per 128 x
    128 tile with an fp32 step, one fp32 offset per matrix), which moves a
    scale by at most half a step: ``(max - min) / 508`` of the tile's scales.
    N and K must be multiples of 128, ``blocksize`` 64.
    """
    N, K = int(shape[0]), int(shape[1])
    if N % _TILE or K % _TILE or N <= 0 or K <= 0:
        raise ValueError("from_bitsandbytes: N and K must be positive multiples of 128")
    if blocksize != _BLOCK:
        raise ValueError("from_bitsandbytes: only blocksize 64 maps onto this format")
    dev = torch.device(device) if device is not None else packed.device
    ours = torch.tensor(NF4_F16_BITS, dtype=torch.int32).to(torch.int16).view(torch.float16).float()
    qm = quant_map.detach().to("cpu", torch.float32).reshape(-1)
    if qm.numel() != 16 or not torch.allclose(qm, ours, rtol=0, atol=1e-3):
        raise ValueError("from_bitsandbytes: quant_map is not the NF4 table")
    nblocks = N * K // _BLOCK
    b = packed.detach().to(dev).reshape(-1)
    if b.dtype != torch.uint8 or b.numel() != N * K // 2:
        raise ValueError("from_bitsandbytes: packed must hold N * K / 2 uint8 bytes")
    codes = torch.stack([b >> 4, b & 15], dim=1).reshape(N, K)
    if nested_absmax is not None:
        q = absmax.detach().to(dev).reshape(-1).long()
        nm = nested_quant_map.detach().to(dev, torch.float32).reshape(-1)
        na = nested_absmax.detach().to(dev, torch.float32).reshape(-1)
        scale = nm[q] * na.repeat_interleave(nested_blocksize)[: q.numel()] + float(nested_offset)
    else:
        scale = absmax.detach().to(dev, torch.float32).reshape(-1)
    if scale.numel() != nblocks:
        raise ValueError("from_bitsandbytes: one scale per 64 weights expected")
    scale = scale.reshape(N, K // _BLOCK)
    # this format's double quantisation of the scales (as the quantiser kernel)
    offset = (scale.min() + scale.max()) * 0.5
    nt, kt = N // _TILE, K // _TILE
    d = (scale - offset).reshape(nt, _TILE, kt, 2).permute(0, 2, 1, 3)  # [nt, kt, 128, 2]
    s127 = d.abs().amax(dim=(2, 3)) / 127.0
    qs = torch.where(s127[..., None, None] > 0, d / torch.where(s127 > 0, s127, 1.0)[..., None, None],
                     torch.zeros_like(d))
    qs = torch.round(qs).clamp_(-127, 127).to(torch.int8)
    out = torch.zeros(nt, kt, _CHUNK_BYTES, dtype=torch.uint8, device=dev)
    out[:, :, _SCALE_OFF:_S127_OFF] = qs.reshape(nt, kt, 2 * _TILE).view(torch.uint8)
    out[:, :, _S127_OFF:_S127_OFF + 4] = s127.reshape(nt, kt, 1).contiguous().view(torch.uint8).reshape(nt, kt, 4)
    row, col = _fragment_order(dev)
    tiles = codes.reshape(nt, _TILE, kt, _TILE).permute(0, 2, 1, 3)  # [nt, kt, 128, 128]
    out[:, :, :_CODE_BYTES] = (tiles[:, :, row, col] << 4) | tiles[:, :, row, col + 1]
    return NF4Weight(out, offset.reshape(1).to(torch.float32), N, K)


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
