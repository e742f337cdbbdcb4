"""bgmv_fused_multi: several projections that share the batch's slots in one
launch, each against the oracle and against bgmv_fused on that projection;
plan reuse, the C ABI, odd and strided shapes, and the full-size layer."""

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


def layer_case(seed, T, R, S, dtype, names=None, null_frac=0.1):
    rng = np.random.default_rng(seed)
    slots = rng.integers(0, S, size=T).astype(np.int32)
    slots[rng.random(T) < null_frac] = -1
    projs = []
    for name in names or list(workloads.PROJECTIONS):
        K, N = workloads.PROJECTIONS[name] if isinstance(name, str) else name
        x = O.from_f32(rng.standard_normal((T, K)).astype(np.float32), dtype)
        a = O.from_f32((rng.uniform(-1, 1, (S, R, K)) / np.sqrt(K)).astype(np.float32), dtype)
        b = O.from_f32((rng.standard_normal((S, N, R)) * 0.04).astype(np.float32), dtype)
        y = O.from_f32(rng.standard_normal((T, N)).astype(np.float32), dtype)
        projs.append(dict(K=K, N=N, x=x, a=a, b=b, y=y))
    return slots, projs


def check_against_oracle(slots, projs, ys, dtype, rows=None):
    for p, yd in zip(projs, ys):
        got = n16(yd, dtype)
        sel = np.arange(len(slots)) if rows is None else rows
        want = p["y"][sel].copy()
        O.bgmv_forward_ref(p["x"][sel], p["a"], p["b"], slots[sel], dtype, y=want)
        np.testing.assert_allclose(f32(got[sel], dtype), f32(want, dtype), **TOL)
        null = slots[sel] < 0
        assert np.array_equal(got[sel][null], p["y"][sel][null])


@pytest.mark.parametrize("dtype", ["f16", "bf16"])
@pytest.mark.parametrize("R", [8, 16, 64])
def test_multi_layer_matches_oracle_and_single(dtype, R):
    T, S = 48, 12
    slots, projs = layer_case(R + (dtype == "bf16"), T, R, S, dtype)
    sd = torch.from_numpy(slots).to(dev())
    xs = [t16(p["x"], dtype) for p in projs]
    a_s = [t16(p["a"], dtype) for p in projs]
    b_s = [t16(p["b"], dtype) for p in projs]
    ys = [t16(p["y"], dtype) for p in projs]
    ops.bgmv_fused_multi(xs, a_s, b_s, sd, ys)
    check_against_oracle(slots, projs, ys, dtype)
    for i, p in enumerate(projs):
        y1 = t16(p["y"], dtype)
        ops.bgmv_fused(xs[i], a_s[i], b_s[i], sd, y1)
        np.testing.assert_allclose(f32(n16(ys[i], dtype), dtype), f32(n16(y1, dtype), dtype), **TOL)
    ops.check_errors(dev())


def test_multi_reuses_a_plan_and_runs_twice():
    dtype, T, R, S = "f16", 40, 16, 6
    slots, projs = layer_case(3, T, R, S, dtype, names=["q_proj", "k_proj", "down_proj"])
    sd = torch.from_numpy(slots).to(dev())
    plan = ops.bgmv_plan(sd, S)
    xs = [t16(p["x"], dtype) for p in projs]
    a_s = [t16(p["a"], dtype) for p in projs]
    b_s = [t16(p["b"], dtype) for p in projs]
    for _ in range(2):  # the second launch runs on the state the first one left
        ys = [t16(p["y"], dtype) for p in projs]
        ops.bgmv_fused_multi(xs, a_s, b_s, sd, ys, plan=plan)
        check_against_oracle(slots, projs, ys, dtype)
    # single-projection calls on the same plan in between and after
    y1 = t16(projs[1]["y"], dtype)
    ops.bgmv_fused(xs[1], a_s[1], b_s[1], sd, y1, plan=plan)
    ys = [t16(p["y"], dtype) for p in projs]
    ops.bgmv_fused_multi(xs, a_s, b_s, sd, ys, plan=plan)
    check_against_oracle(slots, projs, ys, dtype)
    ops.check_errors(dev())


def test_multi_odd_shapes_and_strided_outputs_through_c_abi():
    """N below one 128-row tile, N not a multiple of 128, K not a multiple of
    the stage width; each y a column window of a wider buffer."""
    lib = capi_lib.load()
    dtype, T, R, S = "bf16", 37, 32, 5
    shapes = [(64, 64), (200, 136), (4096, 1024), (328, 520)]
    slots, projs = layer_case(9, T, R, S, dtype, names=shapes)
    sd = torch.from_numpy(slots).to(dev())
    keep, probs = [], []
    wides = []
    for p in projs:
        K, N = p["K"], p["N"]
        x, a, b = t16(p["x"], dtype), t16(p["a"], dtype), t16(p["b"], dtype)
        wide = torch.zeros(T, N + 64, dtype=torch.bfloat16, device=dev())
        wide[:, 32:32 + N] = t16(p["y"], dtype)
        before = wide.clone()
        keep += [x, a, b, wide]
        wides.append((wide, before))
        probs.append(capi_lib.Problem(x.data_ptr(), K, a.data_ptr(), R * K, K, b.data_ptr(), N * R,
                                      wide.data_ptr() + 32 * 2, N + 64, K, N))
    arr = (capi_lib.Problem * len(probs))(*probs)
    ws_bytes = lib.persona_bgmv_multi_workspace_size(T, len(probs))
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev())
    err = torch.zeros(1, dtype=torch.int32, device=dev())
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    capi_lib.check(lib.persona_bgmv_fused_multi(arr, len(probs), sd.data_ptr(), T, R, S, capi_lib.BF16,
                                                ws.data_ptr(), ws_bytes, 0, err.data_ptr(), stream))
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    for p, (wide, before) in zip(projs, wides):
        N = p["N"]
        check_against_oracle(slots, [p], [wide[:, 32:32 + N]], dtype)
        assert torch.equal(wide[:, :32], before[:, :32]) and torch.equal(wide[:, 32 + N:], before[:, 32 + N:])
    # too small a workspace, too many problems
    assert lib.persona_bgmv_fused_multi(arr, len(probs), sd.data_ptr(), T, R, S, capi_lib.BF16, ws.data_ptr(),
                                        lib.persona_bgmv_multi_workspace_size(T, 1), 0, err.data_ptr(),
                                        stream) == 6
    assert lib.persona_bgmv_fused_multi(arr, 9, sd.data_ptr(), T, R, S, capi_lib.BF16, ws.data_ptr(), ws_bytes,
                                        0, err.data_ptr(), stream) == 1


def _oracle_on_rows(rows, slots, x, a_pool, b_pool, y0, dtype="f16"):
    """The oracle on a subset of rows: only the adapters those rows use are
    copied from the device and widened (same math per row, far less CPU)."""
    sl = slots[rows]
    used = np.unique(sl[sl >= 0])
    remap = np.full(int(slots.max()) + 2, -1, np.int32)
    remap[used] = np.arange(len(used), dtype=np.int32)
    sl_c = np.where(sl >= 0, remap[np.maximum(sl, 0)], -1).astype(np.int32)
    idx = torch.from_numpy(used.astype(np.int64)).to(a_pool.device)
    a_np = a_pool.index_select(0, idx).cpu().numpy()
    b_np = b_pool.index_select(0, idx).cpu().numpy()
    ri = torch.from_numpy(np.asarray(rows, np.int64)).to(x.device)
    y_ref = y0.index_select(0, ri).cpu().numpy()
    O.bgmv_forward_ref(x.index_select(0, ri).cpu().numpy(), a_np, b_np, sl_c, dtype, y=y_ref)
    return y_ref


def test_multi_full_size_mixed_decode_layer():
    """The seven projections at 512 rows, rank 64, 256 adapters (Zipf slots +
    5% rows without adapter), fp16, generated on the device: every projection
    of the one launch against the oracle (all rows of q/k/v/o, every third
    row of gate/up/down), and rows without adapter untouched bit for bit."""
    rng = np.random.Generator(np.random.PCG64(4))
    T, R, S = 512, 64, 256
    slots = workloads.zipf_slots(rng, T, S)
    sd = torch.from_numpy(slots).to(dev())
    g = torch.Generator(device=dev()).manual_seed(4)
    names, xs, a_s, b_s, ys = [], [], [], [], []
    for name, (K, N) in workloads.PROJECTIONS.items():
        lim = 1.0 / np.sqrt(K)
        names.append(name)
        a_s.append(((torch.rand(S, R, K, generator=g, device=dev()) * 2 - 1) * lim).half())
        b_s.append((torch.randn(S, N, R, generator=g, device=dev()) * 0.04).half())
        xs.append(torch.randn(T, K, generator=g, device=dev()).half())
        ys.append(torch.randn(T, N, generator=g, device=dev()).half())
    y0 = [y.clone() for y in ys]
    ops.bgmv_fused_multi(xs, a_s, b_s, sd, ys)
    ops.check_errors(dev())
    null = torch.from_numpy(slots < 0).to(dev())
    for i, name in enumerate(names):
        rows = np.arange(T) if xs[i].shape[1] == 4096 and ys[i].shape[1] <= 4096 else np.arange(0, T, 3)
        y_ref = _oracle_on_rows(rows, slots, xs[i], a_s[i], b_s[i], y0[i])
        got = ys[i].index_select(0, torch.from_numpy(rows).to(dev())).float().cpu().numpy()
        np.testing.assert_allclose(got, y_ref.astype(np.float32), err_msg=name, **TOL)
        assert torch.equal(ys[i][null], y0[i][null]), name


@pytest.mark.parametrize("dtype", ["f16", "bf16"])
@pytest.mark.parametrize("R", [8, 16, 32, 64])
@pytest.mark.parametrize("T", [1, 5, 8, 64])
def test_decode_sized_fused_matches_split_kernels_and_oracle(dtype, R, T):
    """At most PERSONA_SMALL_MAX_ROWS rows run the kernel without cross-CTA
    steps; it matches the oracle and the split kernels (PERSONA_SPLIT_ONLY)
    on the same projections, rows without adapter stay untouched."""
    lib = capi_lib.load()
    S = 6
    shapes = [(4096, 4096), (4096, 1024), (14336, 4096), (256, 392)]
    slots, projs = layer_case(100 + T + R, T, R, S, dtype, names=shapes, null_frac=0.25)
    sd = torch.from_numpy(slots).to(dev())
    keep, probs = [], {}
    outs = {}
    for flag in (0, 2):  # 2 = PERSONA_SPLIT_ONLY
        ps, ys = [], []
        for p in projs:
            K, N = p["K"], p["N"]
            x, a, b, y = t16(p["x"], dtype), t16(p["a"], dtype), t16(p["b"], dtype), t16(p["y"], dtype)
            keep += [x, a, b, y]
            ys.append(y)
            ps.append(capi_lib.Problem(x.data_ptr(), K, a.data_ptr(), R * K, K, b.data_ptr(), N * R, y.data_ptr(),
                                       N, K, N))
        arr = (capi_lib.Problem * len(ps))(*ps)
        ws_bytes = lib.persona_bgmv_multi_workspace_size(T, len(ps))
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev())
        err = torch.zeros(1, dtype=torch.int32, device=dev())
        stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
        capi_lib.check(lib.persona_bgmv_fused_multi(arr, len(ps), sd.data_ptr(), T, R, S,
                                                    capi_lib.BF16 if dtype == "bf16" else capi_lib.F16,
                                                    ws.data_ptr(), ws_bytes, flag, err.data_ptr(), stream))
        torch.cuda.synchronize()
        assert int(err.item()) == 0
        outs[flag] = ys
        check_against_oracle(slots, projs, ys, dtype)
    for a_, b_ in zip(outs[0], outs[2]):
        np.testing.assert_allclose(f32(n16(a_, dtype), dtype), f32(n16(b_, dtype), dtype), **TOL)


def test_decode_sized_fused_flags_out_of_range_slots():
    dtype, T, R, S = "f16", 4, 16, 3
    slots, projs = layer_case(77, T, R, S, dtype, names=[(512, 256)], null_frac=0.0)
    slots[2] = 5  # out of range: the row is left alone and the slot error is raised
    p = projs[0]
    y = t16(p["y"], dtype)
    ops.bgmv_fused(t16(p["x"], dtype), t16(p["a"], dtype), t16(p["b"], dtype), torch.from_numpy(slots).to(dev()), y)
    with pytest.raises(RuntimeError, match="slot"):
        ops.check_errors(dev())
    got = n16(y, dtype)
    assert np.array_equal(got[2], p["y"][2])
    ok = np.array([0, 1, 3])
    want = p["y"][ok].copy()
    O.bgmv_forward_ref(p["x"][ok], p["a"], p["b"], slots[ok], dtype, y=want)
    np.testing.assert_allclose(f32(got[ok], dtype), f32(want, dtype), **TOL)


@pytest.mark.parametrize("dtype", ["f16", "bf16"])
@pytest.mark.parametrize("T", [1, 8, 64])
def test_lora_delta_matches_oracle(dtype, T):
    """The LoRA term alone, fp32, at decode sizes: B[s] (A[s] x) per row, exact
    zeros for rows without adapter."""
    R, S = 16, 5
    shapes = [(4096, 4096), (4096, 1024), (14336, 4096)]
    slots, projs = layer_case(300 + T, T, R, S, dtype, names=shapes, null_frac=0.3)
    sd = torch.from_numpy(slots).to(dev())
    xs = [t16(p["x"], dtype) for p in projs]
    a_s = [t16(p["a"], dtype) for p in projs]
    b_s = [t16(p["b"], dtype) for p in projs]
    ds = [torch.full((T, p["N"]), 7.0, dtype=torch.float32, device=dev()) for p in projs]
    ops.bgmv_lora_delta_multi(xs, a_s, b_s, sd, ds)
    ops.check_errors(dev())
    for p, d in zip(projs, ds):
        got = d.cpu().numpy()
        v = O.bgmv_shrink_ref(p["x"], p["a"], slots, dtype).astype(np.float64)
        b = f32(p["b"], dtype).astype(np.float64)
        for t in range(T):
            if slots[t] < 0:
                assert np.all(got[t] == 0)
            else:
                want = b[slots[t]] @ v[t]
                np.testing.assert_allclose(got[t], want, rtol=1e-3, atol=1e-3)
