"""The end-to-end decode on the GPU: the fused glue kernels against plain
torch fp32 references of the same steps, and a small Mistral-architecture
model (2 layers, hidden 512, 4 / 2 heads, NF4 base, rank-16 adapters)
through prefill and CUDA-graph decode steps against an fp32 reference of the
whole model on the same (dequantised) weights, teacher-forced with the
engine's own tokens; graph and eager decoding give the same tokens."""

import math

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from oracle import nf4_oracle as Q
from persona import ops
from persona.adapter_pool import AdapterPool
from persona.engine import Request, StaticBatchEngine
from persona.mistral import MistralConfig, MistralLoRAModel

pytestmark = pytest.mark.gpu


def _dev():
    return torch.device("cuda", 0)


def _rope_ref(x, pos, theta):
    """Rotate-half rotary embedding in fp32; x [rows, H, 128], pos [rows]."""
    j = torch.arange(64, device=x.device, dtype=torch.float32)
    inv = theta ** (-2 * j / 128)
    ang = pos.float()[:, None] * inv[None, :]
    c, s = torch.cos(ang)[:, None, :], torch.sin(ang)[:, None, :]
    x1, x2 = x[..., :64].float(), x[..., 64:].float()
    return torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], dim=-1)


def test_add_rmsnorm_matches_reference():
    g = torch.Generator(device=_dev()).manual_seed(1)
    h = torch.randn(5, 4096, generator=g, device=_dev()).half()
    d = torch.randn(5, 4096, generator=g, device=_dev()).half()
    w = (1 + 0.1 * torch.randn(4096, generator=g, device=_dev())).half()
    want_h = (h.float() + d.float()).half()
    hf = want_h.float()
    want = w.float() * (hf * torch.rsqrt(hf.pow(2).mean(-1, keepdim=True) + 1e-5)).half().float()
    out = torch.empty_like(h)
    ops.add_rmsnorm(h, d, w, out, 1e-5)
    assert torch.equal(h, want_h)
    torch.testing.assert_close(out.float(), want, rtol=2e-3, atol=2e-3)
    out2 = torch.empty_like(h)
    ops.add_rmsnorm(h, None, w, out2, 1e-5)  # no delta: h unchanged
    assert torch.equal(h, want_h) and torch.equal(out2, out)


def test_rope_cache_matches_reference_and_fills_the_cache():
    g = torch.Generator(device=_dev()).manual_seed(2)
    B, T, Hq, Hkv, L = 3, 5, 8, 2, 16
    q = torch.randn(B * T, Hq, 128, generator=g, device=_dev()).half()
    k = torch.randn(B * T, Hkv, 128, generator=g, device=_dev()).half()
    v = torch.randn(B * T, Hkv, 128, generator=g, device=_dev()).half()
    kc = torch.zeros(B, Hkv, L, 128, dtype=torch.float16, device=_dev())
    vc = torch.zeros_like(kc)
    start = torch.tensor([4], dtype=torch.int32, device=_dev())
    pos = (4 + torch.arange(B * T, device=_dev()) % T)
    q_want, k_want = _rope_ref(q, pos, 1e6), _rope_ref(k, pos, 1e6)
    q2, k2 = q.clone(), k.clone()
    ops.rope_cache(q2, k2, v, kc, vc, start, T, 1e6)
    torch.testing.assert_close(q2.float(), q_want, rtol=2e-3, atol=4e-3)
    torch.testing.assert_close(k2.float(), k_want, rtol=2e-3, atol=4e-3)
    for b in range(B):
        assert torch.equal(kc[b, :, 4:4 + T].transpose(0, 1), k2[b * T:(b + 1) * T])
        assert torch.equal(vc[b, :, 4:4 + T].transpose(0, 1), v[b * T:(b + 1) * T])
    assert torch.all(kc[:, :, :4] == 0) and torch.all(kc[:, :, 4 + T:] == 0)


def test_silu_mul_matches_reference():
    g = torch.Generator(device=_dev()).manual_seed(3)
    a = (3 * torch.randn(7, 1024, generator=g, device=_dev())).half()
    b = torch.randn(7, 1024, generator=g, device=_dev()).half()
    out = torch.empty_like(a)
    ops.silu_mul(a, b, out)
    torch.testing.assert_close(out.float(), (F.silu(a.float()).half().float() * b.float()), rtol=2e-3, atol=2e-3)


@pytest.mark.parametrize("length", [1, 31, 32, 33, 200])
def test_decode_attention_matches_reference(length):
    g = torch.Generator(device=_dev()).manual_seed(length)
    B, Hq, Hkv, L = 3, 32, 8, 256
    q = torch.randn(B, Hq, 128, generator=g, device=_dev()).half()
    kc = torch.randn(B, Hkv, L, 128, generator=g, device=_dev()).half()
    vc = torch.randn(B, Hkv, L, 128, generator=g, device=_dev()).half()
    out = torch.empty_like(q)
    ln = torch.tensor([length], dtype=torch.int32, device=_dev())
    ops.decode_attention(q, kc, vc, ln, out, 1 / math.sqrt(128))
    kk = kc[:, :, :length].float().repeat_interleave(Hq // Hkv, dim=1)
    vv = vc[:, :, :length].float().repeat_interleave(Hq // Hkv, dim=1)
    p = torch.softmax(torch.einsum("bhd,bhld->bhl", q.float(), kk) / math.sqrt(128), dim=-1)
    want = torch.einsum("bhl,bhld->bhd", p, vv)
    torch.testing.assert_close(out.float(), want, rtol=2e-3, atol=2e-3)



@pytest.mark.parametrize("pos,G", [(0, 4), (37, 4), (255, 8), (256, 4)])
def test_rope_decode_attention_equals_rope_cache_then_attention(pos, G):
    """The one-launch rotary + attention gives the bits of rope_cache (one
    token per sequence at pos) followed by decode_attention: the attention
    output, q and k rotated in place, and both caches.  pos = L writes
    nothing and rotates nothing, as rope_cache does."""
    g = torch.Generator(device=_dev()).manual_seed(40 + pos)
    B, Hkv, L = 3, 8, 256
    Hq = Hkv * G
    q = torch.randn(B, Hq, 128, generator=g, device=_dev()).half()
    k = torch.randn(B, Hkv, 128, generator=g, device=_dev()).half()
    v = torch.randn(B, Hkv, 128, generator=g, device=_dev()).half()
    kc = torch.randn(B, Hkv, L, 128, generator=g, device=_dev()).half()
    vc = torch.randn(B, Hkv, L, 128, generator=g, device=_dev()).half()
    p_t = torch.tensor([pos], dtype=torch.int32, device=_dev())
    ln = torch.tensor([min(pos + 1, L)], dtype=torch.int32, device=_dev())
    scale = 1 / math.sqrt(128)
    q1, k1, kc1, vc1 = q.clone(), k.clone(), kc.clone(), vc.clone()
    out1 = torch.empty_like(q)
    ops.rope_cache(q1, k1, v, kc1, vc1, p_t, 1, 1e6)
    ops.decode_attention(q1, kc1, vc1, ln, out1, scale)
    q2, k2, kc2, vc2 = q.clone(), k.clone(), kc.clone(), vc.clone()
    out2 = torch.empty_like(q)
    ops.rope_decode_attention(q2, k2, v, kc2, vc2, p_t, ln, out2, 1e6, scale)
    torch.cuda.synchronize()
    for a, b in ((out1, out2), (q1, q2), (k1, k2), (kc1, kc2), (vc1, vc2)):
        assert torch.equal(a, b)
    if pos >= L:
        assert torch.equal(q2, q) and torch.equal(kc2, kc)

# ------------------------------------------------------------ small model --
CFG = MistralConfig(num_layers=2, hidden=512, n_heads=4, n_kv_heads=2, head_dim=128, intermediate=1024, vocab=1024)


def _small_model():
    pool = AdapterPool(max_slots=4, r=16, device=_dev(), num_layers=CFG.num_layers,
                       geometry=(CFG.hidden, CFG.kv_dim, CFG.intermediate))
    g = torch.Generator(device=_dev()).manual_seed(11)
    for i in range(3):
        pool.load_random_adapter(f"a{i}", generator=g)
    return pool, MistralLoRAModel(CFG, pool, _dev(), seed=5)


def _dense(w):
    return torch.from_numpy(Q.dequantize_f32(w.packed.cpu().numpy(), np.float32(w.offset.item()), w.N, w.K)).to(_dev())


def _reference_logits(model, pool, tokens, slots):
    """fp32 forward of the whole sequence [B, L]; logits [B, L, V]."""
    cfg = model.cfg
    B, L = tokens.shape
    h = model.embed[tokens].float()
    pos = torch.arange(L, device=_dev())

    def rms(x, w):
        return w.float() * (x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + cfg.rms_eps))

    def lora(x, li, mod):
        a = pool.a_pool(li, mod).float()
        b = pool.b_pool(li, mod).float()
        out = torch.zeros(B, L, b.shape[1], device=_dev())
        for i in range(B):
            if slots[i] >= 0:
                out[i] = (x[i] @ a[slots[i]].t()) @ b[slots[i]].t()
        return out

    for li, lw in enumerate(model.layers):
        xn = rms(h, lw.in_norm)
        q = xn @ _dense(lw.q).t() + lora(xn, li, "q_proj")
        k = xn @ _dense(lw.k).t() + lora(xn, li, "k_proj")
        v = xn @ _dense(lw.v).t() + lora(xn, li, "v_proj")
        q = _rope_ref(q.view(B * L, cfg.n_heads, 128), pos.repeat(B), cfg.rope_theta).view(B, L, cfg.n_heads, 128)
        k = _rope_ref(k.view(B * L, cfg.n_kv_heads, 128), pos.repeat(B), cfg.rope_theta).view(B, L, cfg.n_kv_heads, 128)
        v = v.view(B, L, cfg.n_kv_heads, 128)
        rep = cfg.n_heads // cfg.n_kv_heads
        kk, vv = k.repeat_interleave(rep, dim=2), v.repeat_interleave(rep, dim=2)
        att = F.scaled_dot_product_attention(q.transpose(1, 2), kk.transpose(1, 2), vv.transpose(1, 2), is_causal=True)
        att = att.transpose(1, 2).reshape(B, L, cfg.q_dim)
        h = h + att @ _dense(lw.o).t() + lora(att, li, "o_proj")
        xn = rms(h, lw.post_norm)
        g_ = xn @ _dense(lw.gate).t() + lora(xn, li, "gate_proj")
        u_ = xn @ _dense(lw.up).t() + lora(xn, li, "up_proj")
        act = F.silu(g_) * u_
        h = h + act @ _dense(lw.down).t() + lora(act, li, "down_proj")
    return rms(h, model.final_norm) @ model.lm_head.float().t()


def test_small_model_prefill_and_graph_decode_match_fp32_reference():
    """Prefill (LoRA per request segment through the segmented kernel) and
    graph-replayed decode against an fp32 reference of the whole network."""
    pool, model = _small_model()
    B, T, steps = 3, 20, 4
    g = torch.Generator(device=_dev()).manual_seed(7)
    prompts = torch.randint(0, CFG.vocab, (B, T), generator=g, device=_dev())
    slots = [pool.name_to_slot["a0"], -1, pool.name_to_slot["a2"]]
    st = model.new_state(torch.tensor(slots, dtype=torch.int32), T + steps)
    seq = prompts.clone()
    got = [model.prefill(st, prompts).float()]
    st.tok.copy_(got[0].argmax(-1))
    for _ in range(steps):
        seq = torch.cat([seq, st.tok[:, None]], dim=1)
        model.decode_step(st, use_graph=True)
        got.append(st.bufs["logits"].float().clone())
    ops.check_errors(_dev())
    ref = _reference_logits(model, pool, seq, slots)
    for i, lg in enumerate(got):
        want = ref[:, T - 1 + i]
        scale = want.abs().max().item()
        torch.testing.assert_close(lg, want, rtol=0, atol=0.03 * scale)


def test_engine_graph_and_eager_generate_the_same_tokens():
    pool, model = _small_model()
    g = torch.Generator().manual_seed(9)
    reqs = [Request(f"r{i}", f"a{i}", torch.randint(0, CFG.vocab, (12,), generator=g).tolist(),
                    slot=pool.name_to_slot[f"a{i}"]) for i in range(3)]
    eng = StaticBatchEngine(model, pool, max_batch=4, max_seq_len=64)
    a = eng.run_static_generate(reqs, max_new_tokens=8, use_cuda_graph=True)
    b = eng.run_static_generate(reqs, max_new_tokens=8, use_cuda_graph=False)
    assert a["tokens"].shape == (3, 8) and a["new_tokens"] == 24
    assert torch.equal(a["tokens"], b["tokens"])
    assert a["tok_per_s"] > 0
    with pytest.raises(ValueError):
        eng.run_static_generate(reqs + reqs[:2], max_new_tokens=4)


def test_engine_pages_adapters_through_the_cache():
    """Three adapters, two slots: the second batch evicts one adapter; each
    row's tokens equal those of the same adapter in a fresh pool (rows are
    computed independently)."""
    from persona.adapter_pool import AdapterCache

    geom = (CFG.hidden, CFG.kv_dim, CFG.intermediate)
    dims = {"q_proj": (CFG.hidden, CFG.q_dim), "k_proj": (CFG.hidden, CFG.kv_dim), "v_proj": (CFG.hidden, CFG.kv_dim),
            "o_proj": (CFG.q_dim, CFG.hidden), "gate_proj": (CFG.hidden, CFG.intermediate),
            "up_proj": (CFG.hidden, CFG.intermediate), "down_proj": (CFG.intermediate, CFG.hidden)}
    g = torch.Generator().manual_seed(4)
    ads = {f"c{i}": {li: {m: ((torch.randn(16, k, generator=g) * 0.02).half(), (torch.randn(n, 16, generator=g) * 0.02)
                              .half()) for m, (k, n) in dims.items()} for li in range(CFG.num_layers)} for i in range(3)}
    prompt = torch.randint(0, CFG.vocab, (10,), generator=g).tolist()

    def engine(names):
        pool = AdapterPool(max_slots=2, r=16, device=_dev(), num_layers=CFG.num_layers, geometry=geom)
        cache = AdapterCache(pool)
        for n in names:
            cache.register(n, layers=ads[n])
        model = MistralLoRAModel(CFG, pool, _dev(), seed=5)
        return cache, StaticBatchEngine(model, pool, max_batch=2, max_seq_len=64, cache=cache)

    cache, eng = engine(["c0", "c1", "c2"])
    out1 = eng.run_static_generate([Request("r0", "c0", prompt), Request("r1", "c1", prompt)], max_new_tokens=6)
    out2 = eng.run_static_generate([Request("r2", "c2", prompt), Request("r0", "c0", prompt)], max_new_tokens=6)
    assert cache.evictions == 1 and "c1" not in cache.resident
    assert torch.equal(out1["tokens"][0], out2["tokens"][1])
    _, fresh = engine(["c2"])
    out3 = fresh.run_static_generate([Request("r2", "c2", prompt), Request("x", "c2", prompt)], max_new_tokens=6)
    assert torch.equal(out3["tokens"][0], out2["tokens"][0])
