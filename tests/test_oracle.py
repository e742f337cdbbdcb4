"""The oracle pinned against the reference's own outputs (golden vectors) and
its torch-free known-answer test.  CPU only."""

import numpy as np
import pytest

from oracle import bgmv_oracle as O
from persona import workloads


def _case(golden, name):
    pre = name + "/"
    return {k[len(pre):]: golden[k] for k in golden.files if k.startswith(pre)}


@pytest.mark.parametrize("dtype", ["f16", "bf16"])
@pytest.mark.parametrize("R", [8, 16, 32, 64])
def test_shrink_matches_reference(golden, dtype, R):
    c = _case(golden, f"shrink_{dtype}_r{R}")
    v = O.bgmv_shrink_ref(c["x"], c["a"], c["slots"], dtype)
    # same fp32 math as the reference; only the summation order differs
    np.testing.assert_allclose(v, c["v"], rtol=1e-5, atol=1e-5)
    assert np.all(v[c["slots"] < 0] == 0)


@pytest.mark.parametrize("dtype", ["f16", "bf16"])
@pytest.mark.parametrize("R", [8, 16, 32, 64])
def test_expand_matches_reference(golden, dtype, R):
    c = _case(golden, f"expand_{dtype}_r{R}")
    y = c["y_in"].copy()
    O.bgmv_expand_ref(c["v"], c["b"], c["slots"], y, dtype)
    got, want = O.to_f32(y, dtype), O.to_f32(c["y_out"], dtype)
    # one rounding of an fp32 sum: at most one storage ulp apart
    np.testing.assert_allclose(got, want, rtol=1e-2, atol=1e-2)
    ulp = 2.0 ** -10 if dtype == "f16" else 2.0 ** -7
    assert np.all(np.abs(got - want) <= ulp * np.maximum(np.abs(want), 2.0 ** -14) * 1.01)
    null = c["slots"] < 0
    assert np.array_equal(y[null].view(np.uint16), c["y_in"][null].view(np.uint16))


def test_forward_matches_reference(golden):
    c = _case(golden, "forward_f16")
    y = O.bgmv_forward_ref(c["x"], c["a"], c["b"], c["slots"], "f16")
    np.testing.assert_allclose(y.astype(np.float32), c["y"].astype(np.float32), rtol=1e-3, atol=1e-3)


def test_all_null_rows_bit_identical(golden):
    c = _case(golden, "null_bf16")
    v = O.bgmv_shrink_ref(c["x"], c["a"], c["slots"], "bf16")
    assert np.array_equal(v, c["v"]) and not v.any()
    y = O.from_f32(np.ones(c["y"].shape, np.float32), "bf16")
    y0 = y.copy()
    O.bgmv_expand_ref(v, c["b"], c["slots"], y, "bf16")
    assert np.array_equal(y, y0) and np.array_equal(y, c["y"])


@pytest.mark.parametrize("name,maker", [("single_projection", lambda: workloads.single_projection(0)),
                                        ("mixed_small", lambda: workloads.mixed_batch(
                                            seed=5, T=64, R=64, S=16, names=["k_proj"]))])
def test_workload_fixture(golden, name, maker):
    c = _case(golden, name)
    wl = maker()
    p = wl.projections[0]
    digest = workloads.checksum(p.x, p.a_pool, p.b_pool, wl.slots, p.y)
    assert digest == bytes(c["checksum"]).decode(), "workload generator drifted"
    v = O.bgmv_shrink_ref(p.x, p.a_pool, wl.slots)
    np.testing.assert_allclose(v, c["v"], rtol=1e-4, atol=1e-4)
    y = p.y.copy()
    O.bgmv_expand_ref(v, p.b_pool, wl.slots, y)
    np.testing.assert_allclose(y.astype(np.float32), c["y"].astype(np.float32), rtol=1e-2, atol=1e-2)


def test_bf16_rounding_matches_torch(golden):
    c = _case(golden, "bf16_round")
    got = O.from_f32(c["f32"], "bf16")
    want = c["bits"]
    nan = np.isnan(c["f32"])
    assert np.array_equal(got[~nan], want[~nan])
    assert np.all(np.isnan(O.to_f32(got[nan], "bf16")))


def test_standalone_known_answer():
    # standalone/test_bgmv.cu:36-86 -- CPU reference of the deterministic KAT
    x, a, slots = O.kat_inputs()
    v = O.bgmv_shrink_ref(x, a, slots)
    x32, a32 = x.astype(np.float32), a.astype(np.float32)
    for t in range(4):
        for r in range(16):
            want = 0.0 if slots[t] < 0 else float(np.dot(a32[slots[t], r].astype(np.float64),
                                                       x32[t].astype(np.float64)))
            assert abs(v[t, r] - want) <= 1e-2
    assert not v[2].any()


def test_plan_ref_contract():
    rng = np.random.default_rng(0)
    S = 7
    slots = rng.integers(-3, S + 2, size=300).astype(np.int32)
    perm, items, nv, nn, nb = O.plan_ref(slots, S, 5)
    assert sorted(perm.tolist()) == list(range(300))
    valid = (slots >= 0) & (slots < S)
    assert nv == valid.sum() and nn == (slots == -1).sum() and nb == 300 - nv - nn
    ps = slots[perm[:nv]]
    assert np.all(np.diff(ps) >= 0)
    for s in range(S):  # stable within a slot
        rows = perm[:nv][ps == s]
        assert np.all(np.diff(rows) > 0)
    covered = np.zeros(300, bool)
    seen_partial = False
    for s, b, c in items:
        assert 1 <= c <= 5 and np.all(slots[perm[b:b + c]] == s)
        assert not covered[b:b + c].any()
        covered[b:b + c] = True
        seen_partial |= c < 5
        assert c < 5 or not seen_partial, "full items come first"
    assert covered.sum() == nv and covered[:nv].all()


def test_sgmv_slots_expand_segments_and_skip_bad_ones():
    indptr = np.array([0, 3, 3, 7, 9], dtype=np.int32)
    seg = np.array([2, 5, -1, 1], dtype=np.int32)
    assert O.sgmv_slots(indptr, seg, 10).tolist() == [2, 2, 2, -1, -1, -1, -1, 1, 1, -1]
    # a step back: segment 1 is decreasing, segment 2 overlaps segment 0 -> both skipped
    bad = np.array([0, 5, 2, 8, 9], dtype=np.int32)
    assert O.sgmv_slots(bad, seg, 10).tolist() == [2] * 5 + [-1] * 3 + [1, -1]
    # past the end
    assert O.sgmv_slots(np.array([0, 4, 12], np.int32), np.array([0, 1], np.int32), 10).tolist() == \
        [0] * 4 + [-1] * 6


# ---- the torch restatement that bench.py's CPU legs time --------------------

def _torch16(a, dtype):
    import torch

    a = np.ascontiguousarray(a)
    if dtype == "f16":
        return torch.from_numpy(a)
    return torch.from_numpy(a.view(np.int16)).view(torch.bfloat16)


@pytest.mark.parametrize("dtype", ["f16", "bf16"])
@pytest.mark.parametrize("R", [8, 64])
def test_torch_restatement_matches_reference(golden, dtype, R):
    import torch

    from oracle import bgmv_torch_ref as TR

    c = _case(golden, f"shrink_{dtype}_r{R}")
    v = TR.bgmv_shrink_ref(_torch16(c["x"], dtype), _torch16(c["a"], dtype), torch.from_numpy(c["slots"]))
    np.testing.assert_allclose(v.numpy(), c["v"], rtol=1e-5, atol=1e-5)
    c = _case(golden, f"expand_{dtype}_r{R}")
    y = _torch16(c["y_in"].copy(), dtype)
    TR.bgmv_expand_ref(torch.from_numpy(c["v"]), _torch16(c["b"], dtype), torch.from_numpy(c["slots"]), y)
    got = y.numpy() if dtype == "f16" else y.view(torch.int16).numpy().view(np.uint16)
    np.testing.assert_allclose(O.to_f32(got, dtype), O.to_f32(c["y_out"], dtype), rtol=1e-2, atol=1e-2)
    null = c["slots"] < 0
    assert np.array_equal(got[null].view(np.uint16), c["y_in"][null].view(np.uint16))


def test_torch_restatement_forward_matches_reference(golden):
    import torch

    from oracle import bgmv_torch_ref as TR

    c = _case(golden, "forward_f16")
    y = torch.zeros(c["y"].shape, dtype=torch.float16)
    TR.bgmv_forward_ref(torch.from_numpy(c["x"]), torch.from_numpy(c["a"]), torch.from_numpy(c["b"]),
                        torch.from_numpy(c["slots"]), y)
    np.testing.assert_allclose(y.float().numpy(), c["y"].astype(np.float32), rtol=1e-3, atol=1e-3)
