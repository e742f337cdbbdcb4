"""A Mistral-7B-architecture decoder whose base linears are NF4 and whose
seven projections carry per-row LoRA adapters from an ``AdapterPool``: the
model the end-to-end mixed-adapter decode runs.

The reference loads the real Mistral-7B through Hugging Face with
bitsandbytes NF4 (reference ``bench/e2e.py:70-90``), patches the projections
with ``MultiLoRALinear`` (``persona/model_patch.py``) and decodes with
``model.generate`` (``persona/engine.py:101-107``).  Here the weights are
random (N(0, 0.02), as for a freshly initialised model; norms are ones), the
architecture is the same (RMSNorm, rotary embedding with base 1e6, grouped
query attention, SwiGLU MLP, untied fp16 LM head) and every step runs this
package's kernels:

* base projections: ``nf4.linear`` (one launch for q / k / v, one for gate /
  up, one each for o and down);
* LoRA: ``ops.bgmv_fused_multi`` on a plan computed once per batch at decode;
  ``ops.sgmv_fused`` over the request segments at prefill;
* the rest: ``ops.add_rmsnorm`` (residual add fused into the
  next norm), ``rope_cache`` (rotary embedding + KV-cache write) at prefill,
  ``rope_decode_attention`` (the same and the attention, one launch) at
  decode, ``silu_mul``; the LM head and the prefill attention are library
  calls (cuBLAS, scaled_dot_product_attention).

A decode step has fixed shapes and reads the position from device memory,
so it is captured once as a CUDA graph and replayed for every token.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import List, Optional

import torch
import torch.nn.functional as F

from persona import nf4, ops
from persona.adapter_pool import AdapterPool

@dataclass
class MistralConfig:
    num_layers: int = 32
    hidden: int = 4096
    n_heads: int = 32
    n_kv_heads: int = 8
    head_dim: int = 128
    intermediate: int = 14336
    vocab: int = 32000
    rope_theta: float = 1e6
    rms_eps: float = 1e-5

    @property
    def q_dim(self) -> int:
        return self.n_heads * self.head_dim

    @property
    def kv_dim(self) -> int:
        return self.n_kv_heads * self.head_dim


@dataclass
class LayerWeights:
    in_norm: torch.Tensor
    post_norm: torch.Tensor
    q: nf4.NF4Weight
    k: nf4.NF4Weight
    v: nf4.NF4Weight
    o: nf4.NF4Weight
    gate: nf4.NF4Weight
    up: nf4.NF4Weight
    down: nf4.NF4Weight


@dataclass
class DecodeState:
    """Static buffers of one batch (CUDA-graph friendly)."""

    B: int
    max_seq: int
    tok: torch.Tensor             # [B] int64: the token each row feeds next
    pos: torch.Tensor             # [1] int32: its position
    length: torch.Tensor          # [1] int32: pos + 1
    slots: torch.Tensor           # [B] int32 adapter slot per row
    plan: torch.Tensor            # BGMV plan of ``slots``
    k_cache: List[torch.Tensor]   # per layer [B, Hkv, max_seq, 128]
    v_cache: List[torch.Tensor]
    bufs: dict = field(default_factory=dict)
    graph: Optional[torch.cuda.CUDAGraph] = None


class MistralLoRAModel:
    """Random-init Mistral-architecture decoder with NF4 base weights."""

    def __init__(self, cfg: MistralConfig, pool: AdapterPool, device, seed: int = 0):
        if pool.num_layers != cfg.num_layers:
            raise ValueError("adapter pool and model disagree on the layer count")
        if cfg.head_dim != 128:
            raise ValueError("the decode kernels take head_dim 128")
        self.cfg = cfg
        self.pool = pool
        self.device = torch.device(device)
        g = torch.Generator(device=self.device)
        g.manual_seed(seed)
        h, d = cfg.hidden, self.device
        self.embed = (torch.randn(cfg.vocab, h, generator=g, device=d) * 0.02).half()
        self.layers: List[LayerWeights] = []
        for _ in range(cfg.num_layers):
            def q(n_out, n_in):
                w = (torch.randn(n_out, n_in, generator=g, device=d) * 0.02).half()
                return nf4.quantize(w)

            self.layers.append(LayerWeights(
                in_norm=torch.ones(h, dtype=torch.float16, device=d),
                post_norm=torch.ones(h, dtype=torch.float16, device=d),
                q=q(cfg.q_dim, h), k=q(cfg.kv_dim, h), v=q(cfg.kv_dim, h), o=q(h, cfg.q_dim),
                gate=q(cfg.intermediate, h), up=q(cfg.intermediate, h), down=q(h, cfg.intermediate)))
        self.final_norm = torch.ones(h, dtype=torch.float16, device=d)
        self.lm_head = (torch.randn(cfg.vocab, h, generator=g, device=d) * 0.02).half()
        self._lora = [self._lora_pools(i) for i in range(cfg.num_layers)]

    # ---- weights ---------------------------------------------------------
    def _lora_pools(self, layer: int):
        p = self.pool
        mods = ("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj")
        return {m: (p.a_pool(layer, m), p.b_pool(layer, m)) for m in mods}

    def base_bytes(self) -> int:
        """HBM bytes of the weights one decode step streams (NF4 + head)."""
        n = sum(w.nbytes for lw in self.layers for w in (lw.q, lw.k, lw.v, lw.o, lw.gate, lw.up, lw.down))
        return n + self.lm_head.numel() * 2

    # ---- batch state -------------------------------------------------------
    def new_state(self, slots: torch.Tensor, max_seq: int) -> DecodeState:
        cfg, d = self.cfg, self.device
        B = int(slots.numel())
        slots = slots.to(d, torch.int32).contiguous()
        plan = ops.bgmv_plan(slots, self.pool.max_slots)
        kc = [torch.zeros(B, cfg.n_kv_heads, max_seq, 128, dtype=torch.float16, device=d)
              for _ in range(cfg.num_layers)]
        vc = [torch.zeros_like(t) for t in kc]
        st = DecodeState(B=B, max_seq=max_seq, tok=torch.zeros(B, dtype=torch.int64, device=d),
                         pos=torch.zeros(1, dtype=torch.int32, device=d),
                         length=torch.ones(1, dtype=torch.int32, device=d), slots=slots, plan=plan,
                         k_cache=kc, v_cache=vc)
        f16 = dict(dtype=torch.float16, device=d)
        st.bufs = dict(
            h=torch.empty(B, cfg.hidden, **f16), xn=torch.empty(B, cfg.hidden, **f16),
            q=torch.empty(B, cfg.q_dim, **f16), k=torch.empty(B, cfg.kv_dim, **f16),
            v=torch.empty(B, cfg.kv_dim, **f16), attn=torch.empty(B, cfg.q_dim, **f16),
            o=torch.empty(B, cfg.hidden, **f16), g=torch.empty(B, cfg.intermediate, **f16),
            u=torch.empty(B, cfg.intermediate, **f16), act=torch.empty(B, cfg.intermediate, **f16),
            d=torch.empty(B, cfg.hidden, **f16), logits=torch.empty(B, cfg.vocab, **f16))
        return st

    # ---- prefill -------------------------------------------------------------
    @torch.inference_mode()
    def prefill(self, st: DecodeState, tokens: torch.Tensor) -> torch.Tensor:
        """Run the prompts ([B, T] token ids, all of length T) through the
        model, fill the caches, and return the last position's logits [B, V]."""
        cfg = self.cfg
        B, T = tokens.shape
        if B != st.B or T > st.max_seq:
            raise ValueError("prompt batch does not fit the decode state")
        R = B * T
        rows = tokens.reshape(-1).to(self.device)
        h = self.embed.index_select(0, rows)
        xn = torch.empty_like(h)
        indptr = torch.arange(0, R + 1, T, dtype=torch.int32, device=self.device)
        start = torch.zeros(1, dtype=torch.int32, device=self.device)
        # LoRA over the request segments (one adapter per prompt): the
        # segmented kernel splits its work evenly over the SMs whatever the
        # number of prompts (the reference's caller expands the same segments
        # into per-token slots, persona/lora_layer.py:21-28).
        def lora_apply(x, lora, names, ys):
            for name, y in zip(names, ys):
                ops.sgmv_fused(x, *lora[name], indptr, st.slots, y)

        delta = None
        for li, lw in enumerate(self.layers):
            lora = self._lora[li]
            ops.add_rmsnorm(h, delta, lw.in_norm, xn, cfg.rms_eps)
            q, k, v = nf4.linear(xn, [lw.q, lw.k, lw.v])
            lora_apply(xn, lora, ("q_proj", "k_proj", "v_proj"), (q, k, v))
            q3, k3, v3 = (t.view(R, -1, 128) for t in (q, k, v))
            ops.rope_cache(q3, k3, v3, st.k_cache[li], st.v_cache[li], start, T, cfg.rope_theta)
            qa = q3.view(B, T, cfg.n_heads, 128).transpose(1, 2)
            ka = k3.view(B, T, cfg.n_kv_heads, 128).transpose(1, 2)
            va = v3.view(B, T, cfg.n_kv_heads, 128).transpose(1, 2)
            attn = F.scaled_dot_product_attention(qa, ka, va, is_causal=True, enable_gqa=True)
            attn = attn.transpose(1, 2).reshape(R, cfg.q_dim).contiguous()
            o = nf4.linear(attn, [lw.o])[0]
            lora_apply(attn, lora, ("o_proj",), (o,))
            ops.add_rmsnorm(h, o, lw.post_norm, xn, cfg.rms_eps)
            g_, u_ = nf4.linear(xn, [lw.gate, lw.up])
            lora_apply(xn, lora, ("gate_proj", "up_proj"), (g_, u_))
            act = torch.empty_like(g_)
            ops.silu_mul(g_, u_, act)
            dn = nf4.linear(act, [lw.down])[0]
            lora_apply(act, lora, ("down_proj",), (dn,))
            delta = dn
        ops.add_rmsnorm(h, delta, self.final_norm, xn, cfg.rms_eps)
        last = xn.view(B, T, cfg.hidden)[:, -1, :]
        logits = torch.matmul(last, self.lm_head.t())
        st.pos.fill_(T)
        st.length.fill_(T + 1)
        return logits

    # ---- decode --------------------------------------------------------------
    def _decode_body(self, st: DecodeState) -> None:
        cfg, b = self.cfg, st.bufs
        B = st.B
        torch.index_select(self.embed, 0, st.tok, out=b["h"])
        scale = 1.0 / math.sqrt(128)
        delta = None
        for li, lw in enumerate(self.layers):
            lora = self._lora[li]
            ops.add_rmsnorm(b["h"], delta, lw.in_norm, b["xn"], cfg.rms_eps)
            nf4.linear(b["xn"], [lw.q, lw.k, lw.v], outs=[b["q"], b["k"], b["v"]])
            ops.bgmv_fused_multi([b["xn"]] * 3, [lora[m][0] for m in ("q_proj", "k_proj", "v_proj")],
                                 [lora[m][1] for m in ("q_proj", "k_proj", "v_proj")], st.slots,
                                 [b["q"], b["k"], b["v"]], plan=st.plan)
            # rotary embedding, cache write and attention in one launch
            ops.rope_decode_attention(b["q"].view(B, cfg.n_heads, 128), b["k"].view(B, cfg.n_kv_heads, 128),
                                      b["v"].view(B, cfg.n_kv_heads, 128), st.k_cache[li], st.v_cache[li], st.pos,
                                      st.length, b["attn"].view(B, cfg.n_heads, 128), cfg.rope_theta, scale)
            nf4.linear(b["attn"], [lw.o], outs=[b["o"]])
            ops.bgmv_fused(b["attn"], *lora["o_proj"], st.slots, b["o"], plan=st.plan)
            ops.add_rmsnorm(b["h"], b["o"], lw.post_norm, b["xn"], cfg.rms_eps)
            nf4.linear(b["xn"], [lw.gate, lw.up], outs=[b["g"], b["u"]])
            ops.bgmv_fused_multi([b["xn"]] * 2, [lora[m][0] for m in ("gate_proj", "up_proj")],
                                 [lora[m][1] for m in ("gate_proj", "up_proj")], st.slots, [b["g"], b["u"]],
                                 plan=st.plan)
            ops.silu_mul(b["g"], b["u"], b["act"])
            nf4.linear(b["act"], [lw.down], outs=[b["d"]])
            ops.bgmv_fused(b["act"], *lora["down_proj"], st.slots, b["d"], plan=st.plan)
            delta = b["d"]
        ops.add_rmsnorm(b["h"], delta, self.final_norm, b["xn"], cfg.rms_eps)
        torch.matmul(b["xn"], self.lm_head.t(), out=b["logits"])
        st.tok.copy_(torch.argmax(b["logits"], dim=-1))
        st.pos.add_(1)
        st.length.add_(1)

    @torch.inference_mode()
    def decode_step(self, st: DecodeState, use_graph: bool = True) -> torch.Tensor:
        """Feed ``st.tok`` at ``st.pos``; greedy next tokens land in
        ``st.tok`` (returned) and the position advances."""
        if not use_graph:
            self._decode_body(st)
            return st.tok
        if st.graph is None:
            # warm up on a side stream (the first calls make the workspaces),
            # then capture; the warm-up step is undone by rewinding pos.
            pos0, tok0 = st.pos.clone(), st.tok.clone()
            s = torch.cuda.Stream(self.device)
            s.wait_stream(torch.cuda.current_stream(self.device))
            with torch.cuda.stream(s):
                self._decode_body(st)
            torch.cuda.current_stream(self.device).wait_stream(s)
            st.pos.copy_(pos0)
            st.length.copy_(pos0 + 1)
            st.tok.copy_(tok0)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                self._decode_body(st)
            st.graph = g
            # capture does not run the body: run it now
        st.graph.replay()
        return st.tok
