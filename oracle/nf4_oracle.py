"""CPU restatement of the NF4 base-weight format and of the base linear that
reads it.  Test infrastructure only: the product never imports this module.

The reference's base linears are bitsandbytes ``Linear4bit`` layers with
``bnb_4bit_quant_type="nf4"``, blocksize 64, ``bnb_4bit_use_double_quant``
and fp16 compute (reference ``bench/e2e.py:70-90``).  bitsandbytes is an
unpinned dev dependency of the reference (``pyproject.toml:18-24``), is not
installed here, and no reference test or fixture pins NF4 results, so
**parity is unpinned** for this format.  What is restated is the published
algorithm:

* NF4 (QLoRA, Dettmers et al. 2023): the 16 values are quantiles of
  N(0, 1), 8 from the positive half (9 quantiles between delta and 1/2,
  the last, 0, dropped), 7 from the negative half (8 quantiles, the last
  dropped), plus an exact 0, normalised so that the extremes are +-1;
  delta = 1 - (1/32 + 1/30) / 2.  ``nf4_values`` computes them here with
  scipy's normal quantile function.
* Blockwise absmax quantisation: every 64 consecutive weights of a row share
  one scale, absmax = max |w|; a weight's code is the NF4 value nearest to
  w / absmax (ties toward the lower code).
* Double quantisation of the scales: here each group of 256 block scales
  (one 128 x 128 tile: 128 rows x 2 blocks) is stored as int8 codes
  ``round((absmax - offset) / s127)`` with ``s127 = max |absmax - offset| /
  127`` per group, ``offset`` one fp32 per matrix = (min + max) / 2 of all
  block absmax values.  This grouping and the linear int8 code are this
  package's choice (bitsandbytes groups 256 consecutive blocks and uses its
  dynamic 8-bit map); they only change how the scales are stored.

Storage (``packed[N / 128, K / 128, CHUNK_BYTES]``), one chunk per 128 x 128
tile, chunks of a tile row adjacent:

* bytes [0, 8192): the codes in ``mma.sync.m16n8k16`` A-fragment order:
  ``((wt * 2 + kh) * 32 + lane) * 16 + ks * 4 + j`` for warp tile ``wt``
  (rows 16 wt .. 16 wt + 15), K half ``kh`` (one absmax block), lane
  (g = lane / 4, t = lane % 4), k-step ``ks`` (16 K) and byte ``j``;
  byte j holds rows (g, g + 8, g, g + 8)[j] and columns
  (2t, 2t, 2t + 8, 2t + 8)[j] and the column after, the first in the high
  nibble;
* bytes [8192, 8448): int8 scale codes, ``row * 2 + kh``;
* bytes [8448, 8452): fp32 ``s127``; then 12 zero bytes.

The linear: ``y[m, n] = sum_b absmax_q[n, b] * sum_{k in b} NF4[c[n, k]] *
x[m, k]`` with ``absmax_q = f32(code) * s127 + offset`` (two fp32
roundings), accumulated in fp32 and rounded once to fp16.
"""

from __future__ import annotations

import numpy as np

TILE = 128
BLOCK = 64
CODE_BYTES = TILE * TILE // 2
SCALE_OFF = CODE_BYTES
S127_OFF = SCALE_OFF + TILE * 2
CHUNK_BYTES = S127_OFF + 16
DELTA = 1.0 - (1.0 / 32.0 + 1.0 / 30.0) / 2.0


def nf4_values() -> np.ndarray:
    """The 16 NF4 values in increasing order (float64)."""
    from scipy.stats import norm

    pos = norm.ppf(np.linspace(DELTA, 0.5, 9)[:-1])
    neg = -norm.ppf(np.linspace(DELTA, 0.5, 8)[:-1])
    v = np.sort(np.concatenate([pos, [0.0], neg]))
    return v / v.max()


def nf4_f16() -> np.ndarray:
    """The values as the kernels hold them: fp16."""
    return nf4_values().astype(np.float16)


def nf4_midpoints() -> np.ndarray:
    """fp32 decision points between consecutive values (15)."""
    v = nf4_values()
    return ((v[:-1] + v[1:]) / 2.0).astype(np.float32)


def _codes(w: np.ndarray, absmax_rows: np.ndarray) -> np.ndarray:
    """NF4 index of every weight; w [N, K] fp32, absmax_rows [N, K/64]."""
    N, K = w.shape
    am = np.repeat(absmax_rows, BLOCK, axis=1)
    with np.errstate(divide="ignore", invalid="ignore"):
        r = np.where(am > 0, w / np.where(am > 0, am, np.float32(1)), np.float32(0)).astype(np.float32)
    mids = nf4_midpoints()
    return (r[..., None] > mids).sum(axis=-1).astype(np.uint8)


def quantize(w: np.ndarray) -> tuple[np.ndarray, np.float32]:
    """Quantise fp32 (or fp16) weights [N, K] (N, K multiples of 128) into
    the tiled format; returns (packed uint8 [N/128, K/128, CHUNK_BYTES],
    offset)."""
    w = np.asarray(w, dtype=np.float32)
    N, K = w.shape
    if N % TILE or K % TILE:
        raise ValueError("N and K must be multiples of 128")
    absmax = np.abs(w.reshape(N, K // BLOCK, BLOCK)).max(axis=2).astype(np.float32)
    offset = np.float32((np.float32(absmax.min()) + np.float32(absmax.max())) * np.float32(0.5))
    idx = _codes(w, absmax)
    nt, kt = N // TILE, K // TILE
    packed = np.zeros((nt, kt, CHUNK_BYTES), np.uint8)
    # scale codes per 128 x 128 tile
    d = (absmax - offset).astype(np.float32).reshape(nt, TILE, kt, 2).transpose(0, 2, 1, 3)  # [nt, kt, 128, 2]
    scale = np.abs(d).max(axis=(2, 3)).astype(np.float32)
    s127 = (scale / np.float32(127)).astype(np.float32)
    with np.errstate(divide="ignore", invalid="ignore"):
        q = np.where(s127[..., None, None] > 0, d / np.where(s127 > 0, s127, 1)[..., None, None], 0)
    q = np.clip(np.rint(q.astype(np.float32)), -127, 127).astype(np.int8)
    packed[:, :, SCALE_OFF:S127_OFF] = q.reshape(nt, kt, TILE * 2).view(np.uint8)
    packed[:, :, S127_OFF:S127_OFF + 4] = s127.reshape(nt, kt, 1).view(np.uint8).reshape(nt, kt, 4)
    # codes in fragment order
    packed[:, :, :CODE_BYTES] = _pack_codes(idx, nt, kt)
    return packed, offset


def _fragment_index():
    """(row, col) of the first element of every code byte of a chunk, in
    storage order: arrays of shape [8192]."""
    wt, kh, lane, ks, j = np.meshgrid(np.arange(8), np.arange(2), np.arange(32), np.arange(4), np.arange(4),
                                      indexing="ij")
    g, t = lane // 4, lane % 4
    row = 16 * wt + g + 8 * (j % 2)
    col = 64 * kh + 16 * ks + 2 * t + 8 * (j // 2)
    return row.reshape(-1), col.reshape(-1)


def _pack_codes(idx: np.ndarray, nt: int, kt: int) -> np.ndarray:
    row, col = _fragment_index()
    tiles = idx.reshape(nt, TILE, kt, TILE).transpose(0, 2, 1, 3)  # [nt, kt, 128, 128]
    hi = tiles[:, :, row, col]
    lo = tiles[:, :, row, col + 1]
    return ((hi << 4) | lo).astype(np.uint8)


def unpack(packed: np.ndarray, offset: np.float32, N: int, K: int):
    """(codes [N, K] uint8, absmax_q [N, K/64] fp32) from the tiled format."""
    nt, kt = N // TILE, K // TILE
    packed = packed.reshape(nt, kt, CHUNK_BYTES)
    row, col = _fragment_index()
    tiles = np.zeros((nt, kt, TILE, TILE), np.uint8)
    b = packed[:, :, :CODE_BYTES]
    tiles[:, :, row, col] = b >> 4
    tiles[:, :, row, col + 1] = b & 15
    codes = tiles.transpose(0, 2, 1, 3).reshape(N, K)
    q = packed[:, :, SCALE_OFF:S127_OFF].copy().view(np.int8).reshape(nt, kt, TILE, 2).astype(np.float32)
    s127 = packed[:, :, S127_OFF:S127_OFF + 4].copy().view(np.float32).reshape(nt, kt, 1, 1)
    am = (q * s127).astype(np.float32) + np.float32(offset)
    absmax_q = am.astype(np.float32).transpose(0, 2, 1, 3).reshape(N, K // BLOCK)
    return codes, absmax_q


def dequantize_f32(packed, offset, N, K) -> np.ndarray:
    """Weights as the linear uses them: NF4 (fp16 values) x absmax_q, fp32."""
    codes, am = unpack(packed, offset, N, K)
    vals = nf4_f16().astype(np.float32)[codes]
    return (vals * np.repeat(am, BLOCK, axis=1)).astype(np.float32)


def dequantize_f16(packed, offset, N, K) -> np.ndarray:
    """The dequantisation kernel's output: fp16(fp32(NF4) * absmax_q)."""
    return dequantize_f32(packed, offset, N, K).astype(np.float16)


def linear_ref(x: np.ndarray, packed, offset, N: int, K: int) -> np.ndarray:
    """y[M, N] = x[M, K] W^T in fp64 over the fp32 dequantised weights,
    rounded to fp16."""
    w = dequantize_f32(packed, offset, N, K).astype(np.float64)
    return (np.asarray(x, np.float64) @ w.T).astype(np.float16)
