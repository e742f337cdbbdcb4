"""Static-batch mixed-adapter generation (reference ``persona/engine.py``):
every request starts together, each row keeps one adapter slot for the
whole generation.

Where the reference hands a patched Hugging Face model to ``model.generate``
(``persona/engine.py:101-107``), this engine runs its own loop over
``MistralLoRAModel``: one prefill over all prompts, then one CUDA-graph
replay per new token, greedy inside the graph (the reference's
``decode_step_greedy`` / ``sample_next_token`` semantics; rows that sample
at a temperature overwrite the greedy token from the step's logits).
Prompts are token ids: this build ships no tokenizer.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import List, Optional, Sequence

import torch

from persona.adapter_pool import AdapterCache, AdapterPool
from persona.mistral import MistralLoRAModel
from persona.sampling import SamplingParams, sample_next_token


@dataclass
class Request:
    request_id: str
    persona_name: str
    prompt: Sequence[int]
    slot: int = -1
    sampling: SamplingParams = field(default_factory=SamplingParams)


class StaticBatchEngine:
    """All requests of a batch share the prompt length and start together."""

    def __init__(self, model: MistralLoRAModel, pool: AdapterPool, max_batch: int = 8, max_seq_len: int = 2048,
                 cache: Optional[AdapterCache] = None):
        """With ``cache``, a request whose ``persona_name`` is registered there
        gets its slot from ``cache.acquire`` (its adapter paged in if needed);
        other requests keep the slot they carry."""
        if cache is not None and cache.pool is not pool:
            raise ValueError("the adapter cache must page this engine's pool")
        self.model = model
        self.pool = pool
        self.cache = cache
        self.max_batch = max_batch
        self.max_seq_len = max_seq_len
        self.device = model.device
        # decode states (caches, plan, captured graph) by (slots, cache length):
        # a batch with the same adapters reuses its graph
        self._states = {}

    def plan_batch(self, requests: Sequence[Request]) -> torch.Tensor:
        if len(requests) > self.max_batch:
            raise ValueError("Static batch exceeds max_batch")
        if self.cache is not None:
            names = [r.persona_name for r in requests if r.persona_name in self.cache.registered]
            slots = iter(self.cache.acquire(names))
            for r in requests:
                if r.persona_name in self.cache.registered:
                    r.slot = next(slots)
        return torch.tensor([r.slot for r in requests], dtype=torch.int32, device=self.device)

    @torch.inference_mode()
    def run_static_generate(self, requests: Sequence[Request], max_new_tokens: int = 128,
                            use_cuda_graph: bool = True) -> dict:
        """Generate ``max_new_tokens`` per request; returns the new token ids
        [batch, max_new_tokens] (CPU) and the device time of the prefill and of
        the decode loop (CUDA events)."""
        slots = self.plan_batch(requests)  # fills r.slot from the cache first
        lens = {len(r.prompt) for r in requests}
        if len(lens) != 1:
            raise ValueError("static batching needs prompts of one length")
        T = lens.pop()
        if T + max_new_tokens > self.max_seq_len:
            raise ValueError("prompt + new tokens exceed max_seq_len")
        prompts = torch.tensor([list(r.prompt) for r in requests], dtype=torch.int64, device=self.device)
        key = (tuple(r.slot for r in requests), T + max_new_tokens)
        st = self._states.get(key)
        if st is None:
            st = self._states[key] = self.model.new_state(slots, T + max_new_tokens)
        sampled = [i for i, r in enumerate(requests) if r.sampling.temperature > 0]
        out = torch.empty(len(requests), max_new_tokens, dtype=torch.int64, device=self.device)
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
        ev[0].record()
        logits = self.model.prefill(st, prompts)
        st.tok.copy_(self._next(logits, requests, sampled))
        out[:, 0] = st.tok
        ev[1].record()
        for i in range(1, max_new_tokens):
            self.model.decode_step(st, use_graph=use_cuda_graph)
            if sampled:
                st.tok.copy_(self._next(st.bufs["logits"], requests, sampled))
            out[:, i] = st.tok
        ev[2].record()
        torch.cuda.synchronize(self.device)
        prefill_ms = ev[0].elapsed_time(ev[1])
        decode_ms = ev[1].elapsed_time(ev[2])
        new = len(requests) * max_new_tokens
        return {"tokens": out.cpu(), "prefill_ms": prefill_ms, "decode_ms": decode_ms, "new_tokens": new,
                "tok_per_s": new / ((prefill_ms + decode_ms) * 1e-3)}

    @staticmethod
    def _next(logits: torch.Tensor, requests: Sequence[Request], sampled: List[int]) -> torch.Tensor:
        nxt = logits.argmax(dim=-1)
        for i in sampled:
            nxt[i] = sample_next_token(logits[i:i + 1], requests[i].sampling)[0]
        return nxt

    def decode_step_greedy(self, logits: torch.Tensor) -> torch.Tensor:
        """Single-step greedy decode helper (reference ``engine.py:109-111``)."""
        return sample_next_token(logits, SamplingParams(temperature=0.0))
