"""NF4 base-weight format on the CPU: the constants compiled into the kernels
against their construction, the tiled layout, and the oracle's quantiser
(parity with bitsandbytes is unpinned: it is not installed here)."""

import re
from pathlib import Path

import numpy as np
import pytest

from oracle import nf4_oracle as Q
from oracle import nf4_oracle as O

ROOT = Path(__file__).resolve().parents[1]
TABLE_H = ROOT / "multi-lora-llm-kernel_b200" / "csrc" / "nf4_table.h"


def _header_array(name):
    txt = TABLE_H.read_text()
    m = re.search(name + r"\[\d+\]\s*=\s*\{([^}]*)\}", txt)
    assert m, name
    return [int(v.strip(), 16) for v in m.group(1).split(",") if v.strip()]


def test_values_follow_the_published_construction():
    v = Q.nf4_values()
    assert v.shape == (16,) and v[0] == -1.0 and v[-1] == 1.0 and v[7] == 0.0
    assert np.all(np.diff(v) > 0)
    # the values printed in the QLoRA paper, to 4 decimals
    paper = [-1.0, -0.6962, -0.5251, -0.3949, -0.2844, -0.1848, -0.0911, 0.0, 0.0796, 0.1609, 0.2461,
             0.3379, 0.4407, 0.5626, 0.7230, 1.0]
    np.testing.assert_allclose(v, paper, atol=1.5e-4)


def test_kernel_constants_match_the_construction():
    assert _header_array("kNf4Half") == Q.nf4_f16().view(np.uint16).tolist()
    assert _header_array("kNf4Mid") == Q.nf4_midpoints().view(np.uint32).tolist()
    txt = TABLE_H.read_text()
    assert f"kNf4ChunkBytes = kNf4S127Off + 16" in txt and Q.CHUNK_BYTES == 8464


def test_fragment_order_covers_every_weight_once():
    row, col = Q._fragment_index()
    seen = np.zeros((128, 128), np.int32)
    np.add.at(seen, (row, col), 1)
    np.add.at(seen, (row, col + 1), 1)
    assert np.all(seen == 1)
    assert np.all(col % 2 == 0)


@pytest.mark.parametrize("N,K", [(128, 128), (256, 384), (384, 256)])
def test_quantise_round_trip_and_error_bound(N, K):
    rng = np.random.default_rng(N + K)
    w = (rng.standard_normal((N, K)) * 0.02).astype(np.float16).astype(np.float32)
    w[5, :64] = 0.0  # a block of zeros: absmax 0, every code is the value 0
    w[7, 100] = 0.5  # an outlier
    packed, offset = Q.quantize(w)
    assert packed.shape == (N // 128, K // 128, Q.CHUNK_BYTES)
    assert np.all(packed[:, :, Q.S127_OFF + 4:] == 0)
    codes, am = Q.unpack(packed, offset, N, K)
    absmax = np.abs(w.reshape(N, K // 64, 64)).max(axis=2)
    assert np.array_equal(codes, Q._codes(w, absmax))
    assert np.all(codes[5, :64] == 7)
    # scale codes: within half a step of the true absmax
    step = np.repeat(np.repeat(packed[:, :, Q.S127_OFF:Q.S127_OFF + 4].copy().view(np.float32)[..., 0], 128, 0), 2, 1)
    assert np.all(np.abs(am - absmax) <= 0.5 * step + 1e-6)
    # every weight is within half the largest NF4 gap of its block's scale
    deq = Q.dequantize_f32(packed, offset, N, K)
    gap = np.diff(Q.nf4_values()).max() / 2
    bound = np.repeat(np.maximum(absmax, am), 64, axis=1) * (gap + 1e-3) + np.repeat(np.abs(am - absmax), 64, 1) + 1e-6
    assert np.all(np.abs(deq - w) <= bound)


def test_linear_reference_is_the_dense_product():
    rng = np.random.default_rng(3)
    N, K, M = 256, 256, 5
    w = (rng.standard_normal((N, K)) * 0.02).astype(np.float16).astype(np.float32)
    packed, offset = Q.quantize(w)
    x = rng.standard_normal((M, K)).astype(np.float16)
    y = Q.linear_ref(x, packed, offset, N, K)
    want = (x.astype(np.float64) @ Q.dequantize_f32(packed, offset, N, K).astype(np.float64).T).astype(np.float16)
    assert np.array_equal(y, want)
    assert Q.dequantize_f16(packed, offset, N, K).dtype == np.float16


# ---- bitsandbytes storage -> this format (persona.nf4.from_bitsandbytes) ----

def _bnb_tensors(st):
    import torch

    kw = dict(packed=torch.from_numpy(st["packed"]), absmax=torch.from_numpy(st["absmax"]),
              shape=st["shape"], quant_map=torch.from_numpy(st["quant_map"]), blocksize=st["blocksize"])
    if "nested_absmax" in st:
        kw.update(nested_absmax=torch.from_numpy(st["nested_absmax"]),
                  nested_quant_map=torch.from_numpy(st["nested_quant_map"]),
                  nested_offset=st["nested_offset"], nested_blocksize=st["nested_blocksize"])
    return kw


@pytest.mark.parametrize("double_quant", [True, False])
def test_bitsandbytes_storage_converts(double_quant):
    """Codes carry over bit for bit; every scale moves by at most half a step
    of this format's per-tile int8 code (parity with bitsandbytes itself is
    unpinned: it is not installed, its storage is restated in oracle/)."""
    from oracle import bnb_nf4
    from persona import nf4

    rng = np.random.default_rng(7)
    N, K = 256, 384
    w = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    st = bnb_nf4.quantize_nf4(w, double_quant=double_quant)
    q = nf4.from_bitsandbytes(**_bnb_tensors(st), device="cpu")
    codes, am = O.unpack(q.packed.numpy(), np.float32(q.offset.item()), N, K)
    assert np.array_equal(codes, bnb_nf4.codes(st))
    want = bnb_nf4.scales(st).reshape(N, K // 64)
    s127 = q.packed.numpy()[:, :, O.S127_OFF:O.S127_OFF + 4].copy().view(np.float32).reshape(N // 128, K // 128)
    step = np.repeat(np.repeat(s127, 128, axis=0), 2, axis=1)
    assert np.all(np.abs(am - want) <= 0.5 * step * 1.001 + 1e-9)
    w_ours = O.dequantize_f32(q.packed.numpy(), np.float32(q.offset.item()), N, K)
    w_bnb = bnb_nf4.dequantize(st)
    assert np.abs(w_ours - w_bnb).max() <= 0.5 * step.max() * 1.001 + 1e-3 * np.abs(w_bnb).max()


def test_bitsandbytes_storage_rejects_other_layouts():
    import torch

    from oracle import bnb_nf4
    from persona import nf4

    st = bnb_nf4.quantize_nf4(np.zeros((128, 128), np.float32) + 0.01)
    kw = _bnb_tensors(st)
    with pytest.raises(ValueError, match="blocksize"):
        nf4.from_bitsandbytes(**{**kw, "blocksize": 128})
    with pytest.raises(ValueError, match="NF4 table"):
        nf4.from_bitsandbytes(**{**kw, "quant_map": torch.linspace(-1, 1, 16)})
    with pytest.raises(ValueError, match="multiples of 128"):
        nf4.from_bitsandbytes(**{**kw, "shape": (128, 64)})


def test_dynamic_map_shape():
    from oracle import bnb_nf4

    m = bnb_nf4.dynamic_map_signed()
    assert m.shape == (256,) and np.all(np.diff(m) >= 0) and m[0] >= -1 and m[-1] == 1.0
    assert np.sum(m == 0) >= 1 and np.abs(m).max() == 1.0
