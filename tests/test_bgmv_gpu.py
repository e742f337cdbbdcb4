"""GPU parity of the B200 BGMV kernels against the oracle and the reference's
golden vectors.  Tolerance for 16-bit outputs: atol = rtol = 1e-2 (the
reference's own CUDA-vs-fp32 tolerance, tests/test_bgmv_cuda.py:29,43);
adapter routing and rows without an adapter are checked bit for bit."""

import ctypes

import numpy as np
import pytest
import torch

import capi_lib
from oracle import bgmv_oracle as O
from persona import ops, workloads

pytestmark = pytest.mark.gpu
TOL = dict(rtol=1e-2, atol=1e-2)


def dev():
    return torch.device("cuda", 0)


def t16(a, dtype):
    a = np.ascontiguousarray(a)
    if dtype == "f16":
        return torch.from_numpy(a.astype(np.float16)).to(dev())
    return torch.from_numpy(a.astype(np.uint16).view(np.int16)).view(torch.bfloat16).to(dev())


def n16(t, dtype):
    t = t.detach().cpu().contiguous()
    if dtype == "f16":
        return t.numpy()
    return t.view(torch.int16).numpy().view(np.uint16)


def f32(a, dtype):
    return O.to_f32(a, dtype)


def ti(a):
    return torch.from_numpy(np.ascontiguousarray(a, np.int32)).to(dev())


def case(golden, name):
    pre = name + "/"
    return {k[len(pre):]: golden[k] for k in golden.files if k.startswith(pre)}


def no_device_error():
    ops.check_errors(dev())


# ------------------------------------------------------------ golden cases --

@pytest.mark.parametrize("dtype", ["f16", "bf16"])
@pytest.mark.parametrize("R", [8, 16, 32, 64])
def test_shrink_golden(golden, dtype, R):
    c = case(golden, f"shrink_{dtype}_r{R}")
    v = ops.bgmv_shrink(t16(c["x"], dtype), t16(c["a"], dtype), ti(c["slots"]))
    torch.cuda.synchronize()
    np.testing.assert_allclose(v.cpu().numpy(), c["v"], **TOL)
    assert not v[torch.from_numpy(c["slots"] < 0).to(dev())].any()
    no_device_error()


@pytest.mark.parametrize("dtype", ["f16", "bf16"])
@pytest.mark.parametrize("R", [8, 16, 32, 64])
def test_expand_golden(golden, dtype, R):
    c = case(golden, f"expand_{dtype}_r{R}")
    y = t16(c["y_in"], dtype)
    out = ops.bgmv_expand(torch.from_numpy(c["v"]).to(dev()), t16(c["b"], dtype), ti(c["slots"]), y)
    assert out is y
    got = n16(y, dtype)
    np.testing.assert_allclose(f32(got, dtype), f32(c["y_out"], dtype), **TOL)
    null = c["slots"] < 0
    assert np.array_equal(got[null].view(np.uint16), c["y_in"][null].view(np.uint16))
    no_device_error()


def test_forward_golden_fused_and_separate(golden):
    c = case(golden, "forward_f16")
    x, a, b, sl = t16(c["x"], "f16"), t16(c["a"], "f16"), t16(c["b"], "f16"), ti(c["slots"])
    y = torch.zeros(3, 64, dtype=torch.float16, device=dev())
    ops.bgmv_fused(x, a, b, sl, y)
    np.testing.assert_allclose(y.float().cpu().numpy(), c["y"].astype(np.float32), **TOL)
    y2 = torch.zeros_like(y)
    ops.bgmv_expand(ops.bgmv_shrink(x, a, sl), b, sl, y2)
    np.testing.assert_allclose(y2.float().cpu().numpy(), c["y"].astype(np.float32), **TOL)
    no_device_error()


def test_null_rows_golden(golden):
    c = case(golden, "null_bf16")
    x, a, b, sl = (t16(c["x"], "bf16"), t16(c["a"], "bf16"), t16(c["b"], "bf16"), ti(c["slots"]))
    v = ops.bgmv_shrink(x, a, sl)
    assert not v.any()
    y = torch.ones(8, 128, dtype=torch.bfloat16, device=dev())
    ops.bgmv_expand(v, b, sl, y)
    ops.bgmv_fused(x, a, b, sl, y)
    assert np.array_equal(n16(y, "bf16"), c["y"])
    no_device_error()


def test_single_projection_golden(golden):
    """8 rows, 4096 -> 4096, rank 16, 4 adapters (the CPU-runnable case)."""
    c = case(golden, "single_projection")
    wl = workloads.single_projection(0)
    p = wl.projections[0]
    x, a, b, sl = t16(p.x, "f16"), t16(p.a_pool, "f16"), t16(p.b_pool, "f16"), ti(wl.slots)
    v = ops.bgmv_shrink(x, a, sl)
    np.testing.assert_allclose(v.cpu().numpy(), c["v"], **TOL)
    y = t16(p.y, "f16")
    ops.bgmv_expand(v, b, sl, y)
    np.testing.assert_allclose(y.float().cpu().numpy(), c["y"].astype(np.float32), **TOL)
    yf = t16(p.y, "f16")
    ops.bgmv_fused(x, a, b, sl, yf)
    np.testing.assert_allclose(yf.float().cpu().numpy(), c["y"].astype(np.float32), **TOL)
    no_device_error()


def test_mixed_small_golden(golden):
    c = case(golden, "mixed_small")
    wl = workloads.mixed_batch(seed=5, T=64, R=64, S=16, names=["k_proj"])
    p = wl.projections[0]
    x, a, b, sl = t16(p.x, "f16"), t16(p.a_pool, "f16"), t16(p.b_pool, "f16"), ti(wl.slots)
    v = ops.bgmv_shrink(x, a, sl)
    np.testing.assert_allclose(v.cpu().numpy(), c["v"], **TOL)
    y = t16(p.y, "f16")
    ops.bgmv_fused(x, a, b, sl, y)
    np.testing.assert_allclose(y.float().cpu().numpy(), c["y"].astype(np.float32), **TOL)
    no_device_error()


# ----------------------------------------------------- benchmark workloads --

def _check_projection(p, slots, plan=None, fused=True, separate=True):
    x, a, b, sl = t16(p.x, p.dtype), t16(p.a_pool, p.dtype), t16(p.b_pool, p.dtype), ti(slots)
    v_ref = O.bgmv_shrink_ref(p.x, p.a_pool, slots, p.dtype)
    y_ref = p.y.copy()
    O.bgmv_expand_ref(v_ref, p.b_pool, slots, y_ref, p.dtype)
    y_ref32 = f32(y_ref, p.dtype)
    if separate:
        v = ops.bgmv_shrink(x, a, sl, plan=plan)
        np.testing.assert_allclose(v.cpu().numpy(), v_ref, **TOL)
        y = t16(p.y, p.dtype)
        ops.bgmv_expand(v, b, sl, y, plan=plan)
        np.testing.assert_allclose(f32(n16(y, p.dtype), p.dtype), y_ref32, **TOL)
    if fused:
        y = t16(p.y, p.dtype)
        ops.bgmv_fused(x, a, b, sl, y, plan=plan)
        got = n16(y, p.dtype)
        np.testing.assert_allclose(f32(got, p.dtype), y_ref32, **TOL)
        null = slots < 0
        assert np.array_equal(got[null].view(np.uint16), p.y[null].view(np.uint16))
    no_device_error()


def test_decode_set_all_projections():
    """Seven Mistral-7B projections at decode: 8 rows, rank 16, 8 adapters."""
    wl = workloads.decode_set()
    plan = ops.bgmv_plan(ti(wl.slots), 8)
    for p in wl.projections:
        _check_projection(p, wl.slots)
        _check_projection(p, wl.slots, plan=plan)


@pytest.mark.parametrize("name", ["q_proj", "k_proj", "gate_proj", "down_proj"])
def test_mixed_batch_full_size(name):
    """512 rows, Zipf(1.1) over 256 adapters + 5 % -1 rows, rank 64."""
    wl = workloads.mixed_batch(names=[name])
    _check_projection(wl.projections[0], wl.slots)


def test_segmented_prefill_rows_bf16_small():
    """Contiguous same-adapter rows (the prefill layout) through BGMV, bf16."""
    wl = workloads.segmented_prefill(requests=4, rows_per_request=40, names=["down_proj"])
    _check_projection(wl.projections[0], wl.slots)


# ------------------------------------------------------------- edge cases --

@pytest.mark.parametrize("dtype", ["f16", "bf16"])
@pytest.mark.parametrize("R", [8, 16, 32, 64])
@pytest.mark.parametrize("T,K,N,S", [(1, 64, 8, 1), (37, 136, 200, 5), (100, 512, 1032, 3)])
def test_odd_shapes(dtype, R, T, K, N, S):
    rng = np.random.default_rng(T * 1000 + K + R)
    p = workloads.make_projection(rng, "odd", T, K, N, R, S, dtype, y_init="randn")
    slots = rng.integers(-1, S, size=T).astype(np.int32)
    _check_projection(p, slots)


def test_many_rows_one_adapter_and_chunking():
    rng = np.random.default_rng(7)
    p = workloads.make_projection(rng, "hot", 300, 1024, 2048, 16, 3, "f16", y_init="randn")
    slots = np.full(300, 1, np.int32)
    slots[::7] = 2
    slots[::11] = -1
    _check_projection(p, slots)


def test_large_batch_over_one_plan_chunk():
    rng = np.random.default_rng(11)
    T = 2500  # more rows than one plan chunk (2048)
    p = workloads.make_projection(rng, "big", T, 128, 256, 8, 40, "bf16", y_init="randn")
    slots = rng.integers(-1, 40, size=T).astype(np.int32)
    _check_projection(p, slots)


def test_routing_is_bit_exact():
    """One-hot adapters: adapter s copies x[t, s] into y[t, s]; any wrong
    routing or a touched -1 row changes an exact integer result."""
    S, T, K, N, R = 6, 40, 64, 64, 16
    a = np.zeros((S, R, K), np.float16)
    b = np.zeros((S, N, R), np.float16)
    for s in range(S):
        a[s, 3, s] = 1.0
        b[s, s, 3] = 1.0
    rng = np.random.default_rng(3)
    x = rng.integers(-8, 9, size=(T, K)).astype(np.float16)
    y0 = rng.integers(-8, 9, size=(T, N)).astype(np.float16)
    slots = rng.integers(-1, S, size=T).astype(np.int32)
    want = y0.copy()
    for t in range(T):
        if slots[t] >= 0:
            want[t, slots[t]] += x[t, slots[t]]
    y = t16(y0, "f16")
    ops.bgmv_fused(t16(x, "f16"), t16(a, "f16"), t16(b, "f16"), ti(slots), y)
    assert np.array_equal(n16(y, "f16").view(np.uint16), want.view(np.uint16))
    y = t16(y0, "f16")
    ops.bgmv_expand(ops.bgmv_shrink(t16(x, "f16"), t16(a, "f16"), ti(slots)), t16(b, "f16"), ti(slots), y)
    assert np.array_equal(n16(y, "f16").view(np.uint16), want.view(np.uint16))
    no_device_error()


def test_packed_pool_slices_in_place():
    """q/k/v share a packed A_qkv [S, 3r, K]; slices are used without copies."""
    rng = np.random.default_rng(5)
    S, r, K, N, T = 4, 16, 512, 256, 24
    a_qkv = (rng.standard_normal((S, 3 * r, K)) * 0.02).astype(np.float16)
    b = (rng.standard_normal((S, N, r)) * 0.02).astype(np.float16)
    x = rng.standard_normal((T, K)).astype(np.float16)
    slots = rng.integers(-1, S, size=T).astype(np.int32)
    A = t16(a_qkv, "f16")
    for j in range(3):
        view = A[:, j * r:(j + 1) * r, :]
        assert not view.is_contiguous()
        v_ref = O.bgmv_shrink_ref(x, a_qkv[:, j * r:(j + 1) * r, :], slots)
        v = ops.bgmv_shrink(t16(x, "f16"), view, ti(slots))
        np.testing.assert_allclose(v.cpu().numpy(), v_ref, **TOL)
        y_ref = np.zeros((T, N), np.float16)
        O.bgmv_expand_ref(v_ref, b, slots, y_ref)
        y = torch.zeros(T, N, dtype=torch.float16, device=dev())
        ops.bgmv_fused(t16(x, "f16"), view, t16(b, "f16"), ti(slots), y)
        np.testing.assert_allclose(y.float().cpu().numpy(), y_ref.astype(np.float32), **TOL)
    no_device_error()


def test_y_is_a_view_of_a_wider_buffer():
    rng = np.random.default_rng(9)
    p = workloads.make_projection(rng, "v", 16, 256, 128, 16, 4, "f16", y_init="randn")
    slots = rng.integers(-1, 4, size=16).astype(np.int32)
    wide = torch.zeros(16, 384, dtype=torch.float16, device=dev())
    wide[:, 64:192] = t16(p.y, "f16")
    y = wide[:, 64:192]
    ops.bgmv_fused(t16(p.x, "f16"), t16(p.a_pool, "f16"), t16(p.b_pool, "f16"), ti(slots), y)
    y_ref = p.y.copy()
    O.bgmv_forward_ref(p.x, p.a_pool, p.b_pool, slots, y=y_ref)
    np.testing.assert_allclose(y.float().cpu().numpy(), y_ref.astype(np.float32), **TOL)
    assert not wide[:, :64].any() and not wide[:, 192:].any()
    no_device_error()


def test_out_of_range_slot_is_reported():
    rng = np.random.default_rng(1)
    p = workloads.make_projection(rng, "bad", 8, 128, 64, 16, 4, "f16", y_init="randn")
    slots = np.array([0, 1, 4, 2, -3, 3, -1, 0], np.int32)  # 4 and -3 are invalid
    y = t16(p.y, "f16")
    ops.bgmv_fused(t16(p.x, "f16"), t16(p.a_pool, "f16"), t16(p.b_pool, "f16"), ti(slots), y)
    with pytest.raises(RuntimeError, match="slot out of range"):
        ops.check_errors(dev())
    got = n16(y, "f16")
    bad = (slots >= 4) | (slots < -1) | (slots == -1)
    assert np.array_equal(got[bad].view(np.uint16), p.y[bad].view(np.uint16))
    ok = ~bad
    y_ref = p.y.copy()
    O.bgmv_forward_ref(p.x, p.a_pool, p.b_pool, np.where(ok, slots, -1).astype(np.int32), y=y_ref)
    np.testing.assert_allclose(got.astype(np.float32), y_ref.astype(np.float32), **TOL)
    # the error is sticky until read, and then cleared
    no_device_error()


def test_other_ranks_run_rowwise_shrink():
    rng = np.random.default_rng(2)
    for R in (4, 12, 80):
        p = workloads.make_projection(rng, "r", 10, 256, 64, R, 3, "bf16")
        slots = rng.integers(-1, 3, size=10).astype(np.int32)
        v = ops.bgmv_shrink(t16(p.x, "bf16"), t16(p.a_pool, "bf16"), ti(slots))
        np.testing.assert_allclose(v.cpu().numpy(), O.bgmv_shrink_ref(p.x, p.a_pool, slots, "bf16"), **TOL)
    with pytest.raises(RuntimeError, match="R must be 8, 16, 32, or 64"):
        y = torch.zeros(10, 64, dtype=torch.bfloat16, device=dev())
        ops.bgmv_expand(torch.zeros(10, 12, device=dev()), torch.zeros(3, 64, 12, dtype=torch.bfloat16,
                                                                        device=dev()), ti(slots), y)
    no_device_error()


def test_zero_rows_is_a_noop():
    x = torch.zeros(0, 64, dtype=torch.float16, device=dev())
    a = torch.zeros(2, 16, 64, dtype=torch.float16, device=dev())
    b = torch.zeros(2, 64, 16, dtype=torch.float16, device=dev())
    sl = torch.zeros(0, dtype=torch.int32, device=dev())
    y = torch.zeros(0, 64, dtype=torch.float16, device=dev())
    assert ops.bgmv_shrink(x, a, sl).shape == (0, 16)
    ops.bgmv_fused(x, a, b, sl, y)
    no_device_error()


def test_fused_is_deterministic():
    wl = workloads.mixed_batch(seed=4, T=256, names=["o_proj"])
    p = wl.projections[0]
    outs = []
    for _ in range(2):
        y = t16(p.y, "f16")
        ops.bgmv_fused(t16(p.x, "f16"), t16(p.a_pool, "f16"), t16(p.b_pool, "f16"), ti(wl.slots), y)
        outs.append(n16(y, "f16"))
    assert np.array_equal(outs[0].view(np.uint16), outs[1].view(np.uint16))


# ------------------------------------------------------------------- plan --

@pytest.mark.parametrize("T,S", [(1, 1), (8, 8), (255, 7), (256, 300), (257, 3), (512, 256), (600, 2), (300, 600), (1500, 2000),
                                 (2048, 256), (2049, 5), (5000, 3)])
def test_plan_matches_oracle(T, S):
    rng = np.random.default_rng(T + S)
    slots = rng.integers(-2, S + 1, size=T).astype(np.int32)
    plan = ops.bgmv_plan(ti(slots), S).cpu().numpy().view(np.int32)
    if ((slots < -1) | (slots >= S)).any():
        with pytest.raises(RuntimeError, match="slot out of range"):
            ops.check_errors(dev())
    else:
        ops.check_errors(dev())
    tp = (T + 3) // 4 * 4
    hdr, perm = plan[:8], plan[8:8 + T]
    items = plan[8 + tp:8 + tp + 4 * tp].reshape(-1, 4)
    # chunked like the device planner (2048 rows per chunk above 256 rows)
    ch = 256 if T <= 256 else 512 if T <= 512 else 1024 if T <= 1024 else 2048
    exp_items, nv_tot = [], 0
    for base in range(0, T, ch):
        sl = slots[base:base + ch]
        p_ref, it_ref, nv, nn, nb = O.plan_ref(sl, S, 16)
        assert np.array_equal(perm[base:base + len(sl)], p_ref + base)
        for s, b, c in it_ref:
            exp_items.append((s, b + base, c))
        nv_tot += nv
    n_items = hdr[0]
    assert n_items == len(exp_items)
    assert np.array_equal(items[:n_items, :3], np.array(exp_items, np.int32).reshape(-1, 3))
    assert hdr[1] == nv_tot and hdr[4] == T and hdr[5] == S and hdr[6] == 16


# ------------------------------------------------------------ the C ABI ----

def test_c_abi_fused_and_planned():
    lib = capi_lib.load()
    wl = workloads.mixed_batch(seed=6, T=128, names=["k_proj"])
    p = wl.projections[0]
    x, a, b, sl = t16(p.x, "f16"), t16(p.a_pool, "f16"), t16(p.b_pool, "f16"), ti(wl.slots)
    T, K, N, R, S = 128, p.K, p.N, p.R, p.S
    ws_bytes = lib.persona_bgmv_workspace_size(T)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev())
    err = torch.zeros(1, dtype=torch.int32, device=dev())
    stream = torch.cuda.current_stream().cuda_stream
    y_ref = p.y.copy()
    O.bgmv_forward_ref(p.x, p.a_pool, p.b_pool, wl.slots, y=y_ref)
    y = t16(p.y, "f16")
    capi_lib.check(lib.persona_bgmv_fused(x.data_ptr(), K, a.data_ptr(), R * K, K, b.data_ptr(), N * R,
                                          sl.data_ptr(), y.data_ptr(), N, T, K, N, R, S, capi_lib.F16,
                                          ws.data_ptr(), ws_bytes, 0, err.data_ptr(), stream))
    torch.cuda.synchronize()
    np.testing.assert_allclose(y.float().cpu().numpy(), y_ref.astype(np.float32), **TOL)
    # plan once, reuse for shrink + expand
    capi_lib.check(lib.persona_bgmv_plan(sl.data_ptr(), T, S, ws.data_ptr(), ws_bytes, err.data_ptr(), stream))
    v = torch.empty(T, R, dtype=torch.float32, device=dev())
    capi_lib.check(lib.persona_bgmv_shrink(x.data_ptr(), K, a.data_ptr(), R * K, K, sl.data_ptr(), v.data_ptr(),
                                           T, K, R, S, capi_lib.F16, ws.data_ptr(), ws_bytes,
                                           capi_lib.REUSE_PLAN, err.data_ptr(), stream))
    y2 = t16(p.y, "f16")
    capi_lib.check(lib.persona_bgmv_expand(v.data_ptr(), b.data_ptr(), N * R, sl.data_ptr(), y2.data_ptr(), N,
                                           T, N, R, S, capi_lib.F16, ws.data_ptr(), ws_bytes,
                                           capi_lib.REUSE_PLAN, err.data_ptr(), stream))
    torch.cuda.synchronize()
    np.testing.assert_allclose(y2.float().cpu().numpy(), y_ref.astype(np.float32), **TOL)
    assert int(err.item()) == 0


def test_c_abi_reused_plan_must_match_the_call():
    """PERSONA_REUSE_PLAN on a workspace whose plan belongs to another batch
    (a smaller T) or that was never planned: the split kernel checks the
    plan header, flags PERSONA_DEV_ERR_PLAN and leaves y alone; the same
    workspace then serves a normal call."""
    lib = capi_lib.load()
    T, T_other = 300, 100
    wl = workloads.mixed_batch(seed=8, T=T, S=32, names=["q_proj"])
    p = wl.projections[0]
    x, a, b, sl = t16(p.x, "f16"), t16(p.a_pool, "f16"), t16(p.b_pool, "f16"), ti(wl.slots)
    K, N, R, S = p.K, p.N, p.R, p.S
    ws_bytes = lib.persona_bgmv_workspace_size(T)
    stream = torch.cuda.current_stream().cuda_stream
    PLAN_BIT = 8  # PERSONA_DEV_ERR_PLAN
    for planned_rows in (T_other, None):
        ws = torch.zeros(ws_bytes, dtype=torch.uint8, device=dev())
        err = torch.zeros(1, dtype=torch.int32, device=dev())
        if planned_rows is not None:
            capi_lib.check(lib.persona_bgmv_plan(sl.data_ptr(), planned_rows, S, ws.data_ptr(), ws_bytes,
                                                 err.data_ptr(), stream))
        y = t16(p.y, "f16")
        capi_lib.check(lib.persona_bgmv_fused(x.data_ptr(), K, a.data_ptr(), R * K, K, b.data_ptr(), N * R,
                                              sl.data_ptr(), y.data_ptr(), N, T, K, N, R, S, capi_lib.F16,
                                              ws.data_ptr(), ws_bytes, capi_lib.REUSE_PLAN, err.data_ptr(), stream))
        torch.cuda.synchronize()
        assert int(err.item()) & PLAN_BIT
        assert np.array_equal(n16(y, "f16").view(np.uint16), p.y.view(np.uint16))
        # the same workspace, planned by the call itself
        err.zero_()
        capi_lib.check(lib.persona_bgmv_fused(x.data_ptr(), K, a.data_ptr(), R * K, K, b.data_ptr(), N * R,
                                              sl.data_ptr(), y.data_ptr(), N, T, K, N, R, S, capi_lib.F16,
                                              ws.data_ptr(), ws_bytes, 0, err.data_ptr(), stream))
        torch.cuda.synchronize()
        assert int(err.item()) == 0
        y_ref = p.y.copy()
        O.bgmv_forward_ref(p.x, p.a_pool, p.b_pool, wl.slots, y=y_ref)
        np.testing.assert_allclose(y.float().cpu().numpy(), y_ref.astype(np.float32), **TOL)


def test_gemv_fp16():
    rng = np.random.default_rng(0)
    W = rng.standard_normal((300, 520)).astype(np.float16)
    x = rng.standard_normal(520).astype(np.float16)
    y = torch.empty(300, dtype=torch.float16, device=dev())
    ops.gemv_fp16(t16(x, "f16"), t16(W, "f16"), y)
    want = W.astype(np.float32) @ x.astype(np.float32)
    np.testing.assert_allclose(y.float().cpu().numpy(), want, rtol=1e-2, atol=5e-2)


# ------------------------------------------------------------------- SGMV --

def _sgmv_case(requests, rows, names, dtype="bf16", seed=3, holes=False):
    wl = workloads.segmented_prefill(seed=seed, requests=requests, rows_per_request=rows, names=names, dtype=dtype)
    indptr, seg = wl.indptr.copy(), wl.seg_slots.copy()
    if holes:  # drop a segment (rows without adapter) and mark one as -1
        seg[1] = -1
    return wl, indptr, seg


@pytest.mark.parametrize("holes", [False, True])
def test_sgmv_matches_oracle_small(holes):
    wl, indptr, seg = _sgmv_case(6, 37, ["gate_proj"], holes=holes)
    p = wl.projections[0]
    x, a, b = t16(p.x, "bf16"), t16(p.a_pool, "bf16"), t16(p.b_pool, "bf16")
    ip, ss = ti(indptr), ti(seg)
    slots = O.sgmv_slots(indptr, seg, wl.T)
    v_ref = O.bgmv_shrink_ref(p.x, p.a_pool, slots, "bf16")
    v = ops.sgmv_shrink(x, a, ip, ss)
    np.testing.assert_allclose(v.cpu().numpy(), v_ref, **TOL)
    y_ref = p.y.copy()
    O.bgmv_expand_ref(v_ref, p.b_pool, slots, y_ref, "bf16")
    y = t16(p.y, "bf16")
    ops.sgmv_expand(v, b, ip, ss, y)
    np.testing.assert_allclose(f32(n16(y, "bf16"), "bf16"), f32(y_ref, "bf16"), **TOL)
    y2 = t16(p.y, "bf16")
    ops.sgmv_fused(x, a, b, ip, ss, y2)
    got = n16(y2, "bf16")
    np.testing.assert_allclose(f32(got, "bf16"), f32(y_ref, "bf16"), **TOL)
    assert np.array_equal(got[slots < 0], p.y[slots < 0])
    no_device_error()


def test_sgmv_bad_segment_table_is_reported():
    wl, indptr, seg = _sgmv_case(4, 16, ["down_proj"])
    p = wl.projections[0]
    bad = indptr.copy()
    bad[2] = bad[1] - 3  # decreasing
    y = t16(p.y, "bf16")
    ops.sgmv_fused(t16(p.x, "bf16"), t16(p.a_pool, "bf16"), t16(p.b_pool, "bf16"), ti(bad), ti(seg), y)
    with pytest.raises(RuntimeError, match="invalid segment table"):
        ops.check_errors(dev())


def test_sgmv_prefill_full_size_down_proj_sampled():
    """32 requests x 512 rows, rank 16, bf16, 14336 -> 4096: full-size run,
    oracle on a sample of rows (every 97th row) to bound CPU time."""
    wl = workloads.segmented_prefill(names=["down_proj"])
    p = wl.projections[0]
    x, a, b = t16(p.x, "bf16"), t16(p.a_pool, "bf16"), t16(p.b_pool, "bf16")
    ip, ss = ti(wl.indptr), ti(wl.seg_slots)
    y = t16(p.y, "bf16")
    ops.sgmv_fused(x, a, b, ip, ss, y)
    got = n16(y, "bf16")
    rows = np.arange(0, wl.T, 97)
    sl = wl.slots[rows]
    y_ref = p.y[rows].copy()
    O.bgmv_forward_ref(p.x[rows], p.a_pool, p.b_pool, sl, "bf16", y=y_ref)
    np.testing.assert_allclose(f32(got[rows], "bf16"), f32(y_ref, "bf16"), **TOL)
    no_device_error()
