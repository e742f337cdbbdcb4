"""The callers of the BGMV ops on the CPU: adapter pool (slot table, PEFT
parsing, scale folding, packing), LoRAContext / MultiLoRALinear plumbing and
model patching.  Mirrors the reference's tests/test_adapter_pool.py and
tests/test_lora_layer.py and adds the layout checks."""

import json
from pathlib import Path

import pytest
import torch

from persona.adapter_pool import (HIDDEN, KV_OUT, MLP_INTER, AdapterConfig, AdapterPool, LayerPools,
                                  load_peft_adapter_tensors, validate_uniform_adapters)
from persona.lora_layer import LoRAContext, MultiLoRALinear, make_slot_hook
from persona.model_patch import _resolve_a_pool, patch_model_with_pools, resolve_a_pool

from peft_fixture import tensor_digest, write_adapter

CPU = torch.device("cpu")


# ---------------------------------------------------------------- pool ----

def test_pool_random_slot():
    """Reference tests/test_adapter_pool.py:22-29, full 32-layer geometry."""
    pool = AdapterPool(max_slots=4, r=16, device=CPU, dtype=torch.float16)
    s0 = pool.load_random_adapter("a")
    s1 = pool.load_random_adapter("b")
    assert s0 != s1
    assert pool.name_to_slot["a"] == s0
    pool.release_slot("a")
    assert "a" not in pool.name_to_slot
    assert pool.acquire_slot("b") == s1  # idempotent for a held name
    assert pool.acquire_slot("c") == s0  # released slot is reused


def test_slot_table_exhaustion():
    pool = AdapterPool(max_slots=2, r=8, device=CPU, num_layers=1)
    assert [pool.acquire_slot(n) for n in "ab"] == [1, 0]
    with pytest.raises(RuntimeError, match="no free slots"):
        pool.acquire_slot("c")


def test_random_adapter_draw_order_is_fixed():
    """Same generator seed -> same weights; draws are per layer, per pool."""
    p1 = AdapterPool(3, 8, CPU, num_layers=2)
    p2 = AdapterPool(3, 8, CPU, num_layers=2)
    s1 = p1.load_random_adapter("x", generator=torch.Generator().manual_seed(7))
    s2 = p2.load_random_adapter("x", generator=torch.Generator().manual_seed(7))
    g = torch.Generator().manual_seed(7)
    first = torch.randn(p1.layers[0].A_qkv[s1].shape, dtype=torch.float16, generator=g) * 0.01
    assert torch.equal(p1.layers[0].A_qkv[s1], first)
    for f in LayerPools.__dataclass_fields__:
        assert torch.equal(getattr(p1.layers[1], f)[s1], getattr(p2.layers[1], f)[s2])


def test_layer_pools_share_one_aligned_slab():
    pool = AdapterPool(2, 16, CPU, num_layers=1)
    lp = pool.layers[0]
    base = lp.A_qkv.untyped_storage().data_ptr()
    for f in LayerPools.__dataclass_fields__:
        t = getattr(lp, f)
        assert t.untyped_storage().data_ptr() == base
        assert (t.data_ptr() - base) % 256 == 0  # the slab itself is allocator-aligned
        assert t.is_contiguous()
    assert lp.A_qkv.shape == (2, 48, HIDDEN) and lp.B_gate.shape == (2, MLP_INTER, 16)
    assert lp.A_down.shape == (2, 16, MLP_INTER) and lp.B_k.shape == (2, KV_OUT, 16)


# ------------------------------------------------------------ PEFT load ----

def test_validate_uniform(tmp_path):
    """Reference tests/test_adapter_pool.py:32-36, plus the mismatches."""
    a, _ = write_adapter(tmp_path / "a")
    b, _ = write_adapter(tmp_path / "b")
    assert validate_uniform_adapters([a, b]).r == 16
    c, _ = write_adapter(tmp_path / "c", alpha=16)
    with pytest.raises(ValueError, match="share r and lora_alpha"):
        validate_uniform_adapters([a, c])
    d, _ = write_adapter(tmp_path / "d", modules=("q_proj",))
    with pytest.raises(ValueError, match="target_modules"):
        validate_uniform_adapters([a, d])


def test_scale():
    assert AdapterConfig(16, 32.0, []).scale == 2.0
    assert AdapterConfig(16, 32.0, [], use_rslora=True).scale == 8.0


@pytest.mark.parametrize("rslora", [False, True])
def test_load_peft_folds_scale_after_the_cast(tmp_path, rslora):
    d, t = write_adapter(tmp_path / "a", rslora=rslora)
    cfg, per_layer = load_peft_adapter_tensors(d, dtype=torch.float16)
    assert sorted(per_layer) == [0, 1]
    assert sorted(per_layer[0]) == ["q_proj", "v_proj"]  # down_proj is not targeted
    a, b = per_layer[1]["v_proj"]
    src_b = t["base_model.model.model.layers.1.self_attn.v_proj.lora_B.weight"]
    want_b = (src_b.to(torch.float16).float() * cfg.scale).to(torch.float16)
    assert torch.equal(b, want_b)
    assert torch.equal(a, t["base_model.model.model.layers.1.self_attn.v_proj.lora_A.weight"].half())


def test_load_peft_missing_half_raises(tmp_path):
    d, _ = write_adapter(tmp_path / "a", drop_b=(1, "q_proj"))
    with pytest.raises(ValueError, match="Missing A or B for layer 1 q_proj"):
        load_peft_adapter_tensors(d)


def test_load_peft_requires_safetensors(tmp_path):
    d = tmp_path / "a"
    d.mkdir()
    (d / "adapter_config.json").write_text(json.dumps({"r": 8, "lora_alpha": 8, "target_modules": []}))
    with pytest.raises(FileNotFoundError):
        load_peft_adapter_tensors(d)


def test_load_adapter_packs_rank_blocks(tmp_path):
    d, _ = write_adapter(tmp_path / "a", modules=("q_proj", "v_proj", "up_proj", "down_proj"))
    pool = AdapterPool(3, 16, CPU, num_layers=2)
    slot = pool.load_adapter("a", d)
    cfg, per_layer = load_peft_adapter_tensors(d)
    for li in (0, 1):
        lp = pool.layers[li]
        aq, bq = per_layer[li]["q_proj"]
        av, bv = per_layer[li]["v_proj"]
        au, bu = per_layer[li]["up_proj"]
        ad, bd = per_layer[li]["down_proj"]
        assert torch.equal(lp.A_qkv[slot, 0:16], aq) and torch.equal(lp.B_q[slot], bq)
        assert torch.equal(lp.A_qkv[slot, 32:48], av) and torch.equal(lp.B_v[slot], bv)
        assert not lp.A_qkv[slot, 16:32].any() and not lp.B_k[slot].any()  # k not in the adapter
        assert torch.equal(lp.A_gu[slot, 16:32], au) and torch.equal(lp.B_up[slot], bu)
        assert not lp.A_gu[slot, 0:16].any()
        assert torch.equal(lp.A_down[slot], ad) and torch.equal(lp.B_down[slot], bd)
        assert torch.equal(pool.a_pool(li, "v_proj")[slot], av)
        assert pool.b_pool(li, "up_proj") is lp.B_up
    # other slots untouched
    others = [s for s in range(3) if s != slot]
    assert not pool.layers[0].A_qkv[others].any()


def test_load_adapter_rank_mismatch(tmp_path):
    d, _ = write_adapter(tmp_path / "a", r=8)
    with pytest.raises(ValueError, match="rank 8 != pool rank 16"):
        AdapterPool(2, 16, CPU, num_layers=1).load_adapter("a", d)


# ---------------------------------------------------- layer and context ----

class ZeroBase(torch.nn.Module):
    def forward(self, x):
        return torch.zeros_like(x)


def test_multi_lora_disabled():
    """Reference tests/test_lora_layer.py:11-19."""
    ctx = LoRAContext(max_tokens=4, device=CPU)
    ctx.enabled = False
    layer = MultiLoRALinear(ZeroBase(), ctx, torch.randn(2, 8, 16), torch.randn(2, 16, 8))
    x = torch.randn(2, 16)
    assert torch.allclose(layer(x), torch.zeros_like(x))


def test_enabled_layer_refuses_cpu_tensors():
    ctx = LoRAContext(max_tokens=4, device=CPU)
    ctx.set_batch_slots(torch.tensor([0, 1]), 1)
    layer = MultiLoRALinear(ZeroBase(), ctx, torch.randn(2, 8, 16).half(), torch.randn(2, 16, 8).half())
    with pytest.raises(RuntimeError):
        layer(torch.randn(2, 16).half())


def test_context_expands_slots_and_bounds_tokens():
    ctx = LoRAContext(max_tokens=8, device=CPU)
    ctx.set_batch_slots(torch.tensor([3, -1], dtype=torch.int64), 3)
    assert ctx.token_slots.dtype == torch.int32
    assert ctx.token_slots[:6].tolist() == [3, 3, 3, -1, -1, -1]
    assert ctx.token_slots[6:].tolist() == [-1, -1]
    with pytest.raises(ValueError, match="exceed max_tokens"):
        ctx.set_batch_slots(torch.tensor([0, 1, 2]), 3)
    with pytest.raises(ValueError, match="exceed max_tokens"):
        ctx.slots(9)


def test_slot_hook_uses_input_shape():
    ctx = LoRAContext(max_tokens=16, device=CPU)
    ctx.set_batch_slots(torch.tensor([1, 2]), 1)
    hook = make_slot_hook(ctx)
    hook(None, (), {"input_ids": torch.zeros(2, 4, dtype=torch.long)})
    assert ctx.token_slots[:8].tolist() == [1] * 4 + [2] * 4
    hook(None, (torch.zeros(2, 1, dtype=torch.long),), {})
    assert ctx.token_slots[:2].tolist() == [1, 2]


# ------------------------------------------------------------ patching ----

def _tiny_model(n_layers):
    class Attn(torch.nn.Module):
        def __init__(self):
            super().__init__()
            for m in ("q_proj", "k_proj", "v_proj", "o_proj"):
                setattr(self, m, torch.nn.Identity())

    class Mlp(torch.nn.Module):
        def __init__(self):
            super().__init__()
            for m in ("gate_proj", "up_proj", "down_proj"):
                setattr(self, m, torch.nn.Identity())

    class Block(torch.nn.Module):
        def __init__(self):
            super().__init__()
            self.self_attn, self.mlp = Attn(), Mlp()

    model = torch.nn.Module()
    model.model = torch.nn.Module()
    model.model.layers = torch.nn.ModuleList([Block() for _ in range(n_layers)])
    return model


def test_resolve_a_pool_is_a_view():
    pool = AdapterPool(2, 8, CPU, num_layers=1)
    lp = pool.layers[0]
    a_k = resolve_a_pool(lp, "A_qkv", "B_k", 8)
    assert a_k.shape == (2, 8, HIDDEN) and a_k.data_ptr() == lp.A_qkv[:, 8:16].data_ptr()
    assert a_k.stride() == lp.A_qkv.stride()
    assert resolve_a_pool(lp, "A_gu", "B_up", 8).data_ptr() == lp.A_gu[:, 8:].data_ptr()
    assert resolve_a_pool(lp, "A_down", "B_down", 8) is lp.A_down
    assert _resolve_a_pool is resolve_a_pool
    with pytest.raises(ValueError):
        resolve_a_pool(lp, "A_qkv", "B_gate", 8)
    pool.load_random_adapter("late")  # loaded after resolving: visible through the view
    assert a_k.abs().sum() > 0


def test_patch_model_with_pools():
    model = _tiny_model(2)
    pool = AdapterPool(2, 8, CPU, num_layers=2)
    ctx = LoRAContext(8, CPU)
    patch_model_with_pools(model, pool, ctx, target_modules=["q_proj", "down_proj", "up_proj"])
    blk = model.model.layers[1]
    assert isinstance(blk.self_attn.q_proj, MultiLoRALinear)
    assert isinstance(blk.self_attn.k_proj, torch.nn.Identity)
    assert blk.mlp.up_proj.b_pool is pool.layers[1].B_up
    assert blk.mlp.up_proj.a_pool.data_ptr() == pool.layers[1].A_gu[:, 8:].data_ptr()
    assert blk.mlp.down_proj.a_pool is pool.layers[1].A_down
    hooks = len(model._forward_pre_hooks)
    wrapped = blk.self_attn.q_proj
    patch_model_with_pools(model, pool, ctx)  # re-entry: no double wrap, one hook
    assert blk.self_attn.q_proj is wrapped
    assert isinstance(blk.self_attn.k_proj, MultiLoRALinear)
    assert len(model._forward_pre_hooks) == hooks == 1


# ------------------------------------------- pinned to the reference loader ----

def _golden_pool():
    return json.loads((Path(__file__).parent / "golden" / "golden_pool.json").read_text())


@pytest.mark.parametrize("name,dt", [("f16", torch.float16), ("bf16", torch.bfloat16)])
def test_peft_load_matches_reference_digests(tmp_path, name, dt):
    """Digests the reference's load_peft_adapter_tensors produced for the same
    seeded adapter (tests/golden/make_golden_pool.py): bit-identical A and
    scale-folded B, same layers and modules."""
    g = _golden_pool()
    spec = g["adapter"]
    d, _ = write_adapter(tmp_path / "a", r=spec["r"], alpha=spec["alpha"], modules=tuple(spec["modules"]),
                         layers=tuple(spec["layers"]), seed=spec["seed"])
    cfg, per_layer = load_peft_adapter_tensors(d, dtype=dt)
    assert cfg.scale == g[f"scale_{name}"]
    got = {f"{li}.{m}.{ab}": tensor_digest(t) for li, mods in per_layer.items() for m, pair in mods.items()
           for ab, t in zip("AB", pair)}
    assert got == g[f"load_{name}"]


def test_random_adapter_matches_reference_digests():
    g = _golden_pool()
    spec = g["random"]
    pool = AdapterPool(spec["slots"], spec["r"], CPU, torch.float16)
    slot = pool.load_random_adapter("x", generator=torch.Generator().manual_seed(spec["seed"]))
    assert slot == g["random_slot"]
    got = {f"{li}.{f}": tensor_digest(getattr(pool.layers[li], f)[slot])
           for li in spec["layers"] for f in LayerPools.__dataclass_fields__}
    assert got == spec["digests"]
