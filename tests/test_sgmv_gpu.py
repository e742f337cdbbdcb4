"""SGMV on the tensor-core path (ranks 16 / 32 / 64, K % 64 == 0, N % 64 == 0)
against the oracle: ragged segments that straddle the 128-row items, holes,
slot -1 segments, both 16-bit types, strided y, and the C ABI."""

import ctypes

import numpy as np
import pytest
import torch

import capi_lib
from oracle import bgmv_oracle as O
from persona import ops

pytestmark = pytest.mark.gpu

TOL = dict(rtol=1e-2, atol=1e-2)


def dev():
    return torch.device("cuda", 0)


def t16(a, dtype):
    if dtype == "f16":
        return torch.from_numpy(np.ascontiguousarray(a)).to(dev())
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).to(dev()).view(torch.bfloat16)


def n16(t, dtype):
    t = t.detach().cpu()
    if dtype == "f16":
        return t.numpy()
    return t.view(torch.int16).numpy().view(np.uint16)


def f32(a, dtype):
    return O.to_f32(a, dtype)


def ti(a):
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.int32)).to(dev())


def no_device_error():
    ops.check_errors(dev())


def ragged_case(seed, lens, K, N, R, S, dtype, x_scale=1.0, null_segments=()):
    """Segments of the given lengths (0 = empty) packed back to back, random
    slots, pools scaled like trained LoRA weights."""
    rng = np.random.default_rng(seed)
    T = int(sum(lens))
    indptr = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    seg = rng.integers(0, S, size=len(lens)).astype(np.int32)
    for i in null_segments:
        seg[i] = -1
    x = (rng.standard_normal((T, K)) * x_scale).astype(np.float32)
    a = rng.uniform(-1, 1, (S, R, K)).astype(np.float32) / np.sqrt(K)
    b = (rng.standard_normal((S, N, R)) * 0.04).astype(np.float32)
    y = rng.standard_normal((T, N)).astype(np.float32)
    return (indptr, seg, O.from_f32(x, dtype), O.from_f32(a, dtype), O.from_f32(b, dtype),
            O.from_f32(y, dtype))


CASES = [
    # lens, K, N
    ([128, 300, 37, 0, 256, 1], 512, 256),
    ([5, 129, 127, 640], 1024, 384),
    ([128] * 3, 192, 128),
    ([200, 57], 128, 192),  # N a multiple of 64, not of 128
    ([64], 64, 64),
    ([130] * 160, 128, 128),  # 320 items: more than one per SM, the ring wraps across items
]


@pytest.mark.parametrize("dtype", ["bf16", "f16"])
@pytest.mark.parametrize("R", [16, 32, 64])
@pytest.mark.parametrize("ci", range(len(CASES)))
def test_sgmv_tensor_core_matches_oracle(dtype, R, ci):
    lens, K, N = CASES[ci]
    S = 7
    indptr, seg, x, a, b, y0 = ragged_case(10 + ci, lens, K, N, R, S, dtype, null_segments=(1,) if ci == 1 else ())
    T = x.shape[0]
    slots = O.sgmv_slots(indptr, seg, T)
    ip, ss = ti(indptr), ti(seg)
    v_ref = O.bgmv_shrink_ref(x, a, slots, dtype)
    v = ops.sgmv_shrink(t16(x, dtype), t16(a, dtype), ip, ss)
    np.testing.assert_allclose(v.cpu().numpy(), v_ref, **TOL)
    assert np.all(v.cpu().numpy()[slots < 0] == 0)

    y_ref = y0.copy()
    O.bgmv_expand_ref(v_ref, b, slots, y_ref, dtype)
    y = t16(y0, dtype)
    ops.sgmv_expand(v, t16(b, dtype), ip, ss, y)
    got = n16(y, dtype)
    np.testing.assert_allclose(f32(got, dtype), f32(y_ref, dtype), **TOL)
    assert np.array_equal(got[slots < 0], y0[slots < 0])

    y2 = t16(y0, dtype)
    ops.sgmv_fused(t16(x, dtype), t16(a, dtype), t16(b, dtype), ip, ss, y2)
    got2 = n16(y2, dtype)
    np.testing.assert_allclose(f32(got2, dtype), f32(y_ref, dtype), **TOL)
    assert np.array_equal(got2[slots < 0], y0[slots < 0])
    no_device_error()


@pytest.mark.parametrize("R", [16, 64])
def test_sgmv_tensor_core_f16_large_intermediate(R):
    """|v| far above the f16 range: the per-row power-of-two scale keeps the
    16-bit halves of v finite; y stays within f16."""
    dtype, K, N, S = "f16", 256, 256, 3
    indptr, seg, x, a, b, y0 = ragged_case(5, [200, 60], K, N, R, S, dtype, x_scale=4000.0)
    a = O.from_f32(f32(a, dtype) * 32.0, dtype)
    b = O.from_f32(f32(b, dtype) * 1e-3, dtype)
    T = x.shape[0]
    slots = O.sgmv_slots(indptr, seg, T)
    v_ref = O.bgmv_shrink_ref(x, a, slots, dtype)
    assert np.abs(v_ref).max() > 65504
    y_ref = y0.copy()
    O.bgmv_expand_ref(v_ref, b, slots, y_ref, dtype)
    y = t16(y0, dtype)
    ops.sgmv_fused(t16(x, dtype), t16(a, dtype), t16(b, dtype), ti(indptr), ti(seg), y)
    np.testing.assert_allclose(f32(n16(y, dtype), dtype), f32(y_ref, dtype), **TOL)
    no_device_error()


def test_sgmv_tensor_core_strided_y_and_c_abi():
    """y is a column window of a wider buffer (ldy > N); called through the
    C ABI with an explicit workspace; columns outside the window untouched."""
    lib = capi_lib.load()
    dtype, R, K, N, S = "bf16", 32, 320, 256, 4
    indptr, seg, x, a, b, y0 = ragged_case(6, [130, 0, 70, 256], K, N, R, S, dtype)
    T = x.shape[0]
    ld = N + 128
    rng = np.random.default_rng(1)
    wide = O.from_f32(rng.standard_normal((T, ld)).astype(np.float32), dtype)
    wide[:, 64:64 + N] = y0
    yw = t16(wide, dtype)
    xd, ad, bd = t16(x, dtype), t16(a, dtype), t16(b, dtype)
    ip, ss = ti(indptr), ti(seg)
    ws_bytes = lib.persona_sgmv_workspace_size(T)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev())
    err = torch.zeros(1, dtype=torch.int32, device=dev())
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    capi_lib.check(lib.persona_sgmv_fused(
        xd.data_ptr(), K, ad.data_ptr(), R * K, K, bd.data_ptr(), N * R, ip.data_ptr(), ss.data_ptr(),
        len(seg), yw.data_ptr() + 64 * 2, ld, T, K, N, R, S, capi_lib.BF16, ws.data_ptr(), ws_bytes,
        err.data_ptr(), stream))
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    slots = O.sgmv_slots(indptr, seg, T)
    y_ref = y0.copy()
    O.bgmv_forward_ref(x, a, b, slots, dtype, y=y_ref)
    got = n16(yw, dtype)
    np.testing.assert_allclose(f32(got[:, 64:64 + N], dtype), f32(y_ref, dtype), **TOL)
    assert np.array_equal(got[:, :64], wide[:, :64])
    assert np.array_equal(got[:, 64 + N:], wide[:, 64 + N:])


def test_sgmv_tensor_core_overlapping_segments_are_rejected():
    """An indptr that steps back makes the later segments overlap earlier
    rows; those segments are skipped and the segment error is raised."""
    dtype, R, K, N, S = "bf16", 16, 256, 128, 3
    indptr, seg, x, a, b, y0 = ragged_case(8, [150, 150, 150], K, N, R, S, dtype)
    bad = indptr.copy()
    bad[2] = 100  # segment 1 = [150, 100): decreasing; segment 2 = [100, 450) overlaps segment 0
    y = t16(y0, dtype)
    ops.sgmv_fused(t16(x, dtype), t16(a, dtype), t16(b, dtype), ti(bad), ti(seg), y)
    with pytest.raises(RuntimeError, match="invalid segment table"):
        ops.check_errors(dev())
    slots = O.sgmv_slots(bad, seg, x.shape[0])
    assert np.all(slots[150:] == -1)
    y_ref = y0.copy()
    O.bgmv_forward_ref(x, a, b, slots, dtype, y=y_ref)
    got = n16(y, dtype)
    np.testing.assert_allclose(f32(got, dtype), f32(y_ref, dtype), **TOL)
    assert np.array_equal(got[150:], y0[150:])
