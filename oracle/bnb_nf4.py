"""CPU restatement of bitsandbytes' NF4 weight storage -- TEST INFRASTRUCTURE.

The reference's base linears are bitsandbytes ``Linear4bit`` layers (nf4,
blocksize 64, double quantisation; reference ``bench/e2e.py:73-88``).
bitsandbytes is an unpinned development dependency of the reference
(``pyproject.toml:18-24``; 0.50.2 in the environment its profiles record,
``profiles/env_2026-10-05.txt:6``).  It is not installed here, so this module
restates its published storage format from the QLoRA paper (NF4, double
quantisation) and the 8-bit optimizers paper (blockwise quantisation with a
dynamic 8-bit map), and **parity with bitsandbytes itself is unpinned**.
``tests/test_nf4.py`` uses it to produce weights in that storage for the
product's converter, ``persona.nf4.from_bitsandbytes``.

Storage restated:
* the row-major weight [N, K] is flattened and cut into blocks of 64; each
  block's absmax scales it to [-1, 1]; a weight's code is the NF4 value
  nearest to w / absmax (decision points halfway between the values);
* codes are packed two per byte, element 2i in the high nibble;
* double quantisation: offset = mean of the absmax values; (absmax - offset)
  is cut into blocks of 256, each scaled by its own absmax (fp32) and coded
  as the index of the nearest entry of a signed 8-bit dynamic map.
"""

from __future__ import annotations

import numpy as np

from oracle import nf4_oracle


def dynamic_map_signed(max_exponent_bits: int = 7, total_bits: int = 8) -> np.ndarray:
    """The signed dynamic 8-bit map (sorted, 256 entries): for each decimal
    exponent e = 0 .. max_exponent_bits - 1, 2**e linearly spaced fractions
    (midpoints of linspace(0.1, 1, 2**e + 1)) times 10**(e - max_exponent_bits
    + 1), both signs; plus 0 and 1."""
    vals = []
    for e in range(max_exponent_bits):
        n = 2 ** (e + (total_bits - 1) - max_exponent_bits) + 1
        b = np.linspace(0.1, 1.0, n)
        mids = (b[:-1] + b[1:]) / 2.0
        scale = 10.0 ** (e - (max_exponent_bits - 1))
        vals += list(scale * mids) + list(-scale * mids)
    vals += [0.0, 1.0]
    vals += [0.0] * (2 ** total_bits - len(vals))
    return np.sort(np.asarray(vals, np.float32))


def quantize_blockwise(v: np.ndarray, code: np.ndarray, blocksize: int):
    """(codes uint8, absmax fp32 per block): nearest map entry of v / absmax."""
    v = np.asarray(v, np.float32).reshape(-1)
    nb = (v.size + blocksize - 1) // blocksize
    pad = np.zeros(nb * blocksize, np.float32)
    pad[: v.size] = v
    blocks = pad.reshape(nb, blocksize)
    absmax = np.abs(blocks).max(axis=1).astype(np.float32)
    with np.errstate(divide="ignore", invalid="ignore"):
        r = np.where(absmax[:, None] > 0, blocks / np.where(absmax > 0, absmax, 1)[:, None], 0).astype(np.float32)
    q = np.abs(r[..., None] - code[None, None, :]).argmin(axis=-1).astype(np.uint8)
    return q.reshape(-1)[: v.size], absmax


def quantize_nf4(w: np.ndarray, blocksize: int = 64, double_quant: bool = True) -> dict:
    """bitsandbytes-style NF4 storage of w [N, K] (fp32)."""
    w = np.asarray(w, np.float32)
    flat = w.reshape(-1, blocksize)
    absmax = np.abs(flat).max(axis=1).astype(np.float32)
    codes = nf4_oracle._codes(w.reshape(-1, blocksize), absmax[:, None])  # one block per row
    codes = codes.reshape(-1)
    packed = ((codes[0::2] << 4) | codes[1::2]).astype(np.uint8)
    st = {"packed": packed, "quant_map": nf4_oracle.nf4_values().astype(np.float32), "shape": w.shape,
          "blocksize": blocksize}
    if double_quant:
        offset = np.float32(absmax.mean())
        dmap = dynamic_map_signed()
        q, absmax2 = quantize_blockwise(absmax - offset, dmap, 256)
        st.update(absmax=q, nested_absmax=absmax2, nested_quant_map=dmap, nested_offset=float(offset),
                  nested_blocksize=256)
    else:
        st.update(absmax=absmax)
    return st


def scales(st: dict) -> np.ndarray:
    """The fp32 block scales the storage describes."""
    if "nested_absmax" in st:
        q = st["absmax"].astype(np.int64)
        return (st["nested_quant_map"][q] * np.repeat(st["nested_absmax"], st["nested_blocksize"])[: q.size]
                + np.float32(st["nested_offset"])).astype(np.float32)
    return st["absmax"].astype(np.float32)


def codes(st: dict) -> np.ndarray:
    b = st["packed"]
    return np.stack([b >> 4, b & 15], axis=1).reshape(st["shape"])


def dequantize(st: dict) -> np.ndarray:
    """fp32 weights: NF4[code] * scale of its block."""
    N, K = st["shape"]
    vals = st["quant_map"][codes(st).astype(np.int64)]
    return (vals * np.repeat(scales(st).reshape(N, K // st["blocksize"]), st["blocksize"], axis=1)).astype(np.float32)
