"""The callers on the GPU: MultiLoRALinear (fused op + shared plan) against the
oracle, and a patched model whose forward pre-hook routes per-request
adapters, including pools loaded after patching."""

import numpy as np
import pytest
import torch

from oracle import bgmv_oracle as O
from persona.adapter_pool import AdapterPool
from persona.lora_layer import LoRAContext, MultiLoRALinear
from persona.model_patch import patch_model_with_pools

pytestmark = pytest.mark.gpu

TOL = dict(rtol=1e-2, atol=1e-2)
DEV = torch.device("cuda", 0)


def _lora_ref(x2d, a, b, slots):
    """fp32 oracle of the LoRA term alone (y = 0 in, rounded to fp16)."""
    xs = x2d.detach().cpu().numpy().astype(np.float16)
    y = np.zeros((xs.shape[0], b.shape[1]), np.float16)
    O.bgmv_forward_ref(xs, a.detach().cpu().numpy().astype(np.float16),
                       b.detach().cpu().numpy().astype(np.float16), slots, "f16", y=y)
    return y.astype(np.float32)


def test_multi_lora_linear_matches_oracle_and_shares_the_plan():
    g = torch.Generator(device=DEV).manual_seed(0)
    K, N, R, S = 256, 384, 16, 5
    base = torch.nn.Linear(K, N, bias=False).to(DEV).half()
    with torch.no_grad():
        base.weight.zero_()  # isolate the LoRA term
    a = (torch.rand(S, R, K, generator=g, device=DEV) - 0.5).half() * 0.1
    b = (torch.randn(S, N, R, generator=g, device=DEV) * 0.05).half()
    ctx = LoRAContext(max_tokens=64, device=DEV)
    layer = MultiLoRALinear(base, ctx, a, b)
    layer2 = MultiLoRALinear(base, ctx, a, b)
    row_slots = torch.tensor([2, -1, 4, 0], dtype=torch.int32)
    ctx.set_batch_slots(row_slots, 5)  # prefill: 4 requests x 5 tokens
    x = torch.randn(4, 5, K, generator=g, device=DEV).half()
    with torch.no_grad():
        y = layer(x)
        plan = ctx._plans[(20, S)]
        y2 = layer2(x)
    assert ctx._plans[(20, S)] is plan  # one plan for both projections
    slots = np.repeat(row_slots.numpy(), 5)
    want = _lora_ref(x.reshape(-1, K), a, b, slots)
    np.testing.assert_allclose(y.reshape(-1, N).float().cpu().numpy(), want, **TOL)
    assert torch.equal(y, y2)
    assert not y.reshape(-1, N)[torch.from_numpy(slots < 0)].any()


def test_multi_lora_linear_non_contiguous_output_is_written_back():
    """A base whose output is a transposed view: reshape copies, and the layer
    writes the result back into the base output."""
    K, N, R, S = 128, 256, 8, 2

    class TBase(torch.nn.Module):
        def forward(self, x):
            return torch.zeros(N, x.shape[0], device=x.device, dtype=x.dtype).t()

    g = torch.Generator(device=DEV).manual_seed(1)
    a = (torch.randn(S, R, K, generator=g, device=DEV) * 0.05).half()
    b = (torch.randn(S, N, R, generator=g, device=DEV) * 0.05).half()
    ctx = LoRAContext(16, DEV)
    ctx.set_batch_slots(torch.tensor([1, 0, 1]), 1)
    x = torch.randn(3, K, generator=g, device=DEV).half()
    with torch.no_grad():
        y = MultiLoRALinear(TBase(), ctx, a, b)(x)
    assert not y.is_contiguous()
    np.testing.assert_allclose(y.float().cpu().numpy(), _lora_ref(x, a, b, np.array([1, 0, 1])), **TOL)


class _TinyMistral(torch.nn.Module):
    """One decoder layer's q_proj and down_proj on an embedding, enough to run
    the patched linears through the model's forward pre-hook."""

    def __init__(self):
        super().__init__()
        self.emb = torch.nn.Embedding(32, 4096)
        blk = torch.nn.Module()
        blk.self_attn = torch.nn.Module()
        blk.self_attn.q_proj = torch.nn.Linear(4096, 4096, bias=False)
        blk.mlp = torch.nn.Module()
        blk.mlp.down_proj = torch.nn.Linear(14336, 4096, bias=False)
        self.model = torch.nn.Module()
        self.model.layers = torch.nn.ModuleList([blk])

    def forward(self, input_ids):
        h = self.emb(input_ids)
        blk = self.model.layers[0]
        return blk.self_attn.q_proj(h), blk.mlp.down_proj(torch.cat([h] * 4, -1)[..., :14336])


def test_patched_model_routes_each_request():
    torch.manual_seed(0)
    model = _TinyMistral().to(DEV).half()
    pool = AdapterPool(max_slots=4, r=16, device=DEV, dtype=torch.float16, num_layers=1)
    ctx = LoRAContext(max_tokens=64, device=DEV)
    patch_model_with_pools(model, pool, ctx, target_modules=["q_proj", "down_proj"])
    # adapters loaded AFTER patching are visible (the A pools are views)
    s_a = pool.load_random_adapter("a", generator=torch.Generator(device=DEV).manual_seed(1))
    s_b = pool.load_random_adapter("b", generator=torch.Generator(device=DEV).manual_seed(2))
    ctx.row_slots = torch.tensor([s_b, -1, s_a], dtype=torch.int32, device=DEV)
    ids = torch.randint(0, 32, (3, 6), device=DEV)
    with torch.no_grad():
        q, d = model(input_ids=ids)
        ctx.enabled = False
        q0, d0 = model(input_ids=ids)
        ctx.enabled = True
    slots = np.repeat(np.array([s_b, -1, s_a]), 6)
    lp = pool.layers[0]
    with torch.no_grad():
        h = model.emb(ids).reshape(-1, 4096)
        hd = torch.cat([model.emb(ids)] * 4, -1)[..., :14336].reshape(-1, 14336)
    want_q = _lora_ref(h, lp.A_qkv[:, :16], lp.B_q, slots)
    np.testing.assert_allclose((q.float() - q0.float()).reshape(-1, 4096).cpu().numpy(), want_q,
                               rtol=2e-2, atol=2e-2)
    want_d = _lora_ref(hd, lp.A_down, lp.B_down, slots)
    np.testing.assert_allclose((d.float() - d0.float()).reshape(-1, 4096).cpu().numpy(), want_d,
                               rtol=2e-2, atol=2e-2)
    # the request without an adapter is exactly the base output
    assert torch.equal(q[1], q0[1]) and torch.equal(d[1], d0[1])
