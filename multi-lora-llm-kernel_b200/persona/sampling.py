"""Per-request sampling (reference ``persona/sampling.py:8-33``): greedy at
temperature 0, else softmax sampling with an optional top-p cut."""

from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass
class SamplingParams:
    temperature: float = 0.0
    top_p: float = 1.0
    max_tokens: int = 128


def sample_next_token(logits: torch.Tensor, params: SamplingParams) -> torch.Tensor:
    """logits [batch, vocab] -> next token ids [batch] (int64)."""
    if params.temperature <= 0:
        return logits.argmax(dim=-1)
    probs = torch.softmax(logits.float() / params.temperature, dim=-1)
    if params.top_p < 1.0:
        p_sorted, idx = torch.sort(probs, descending=True, dim=-1)
        # keep the smallest prefix whose mass reaches top_p (the first token always)
        drop = torch.cumsum(p_sorted, dim=-1) - p_sorted > params.top_p
        p_sorted = p_sorted.masked_fill(drop, 0.0)
        p_sorted = p_sorted / p_sorted.sum(dim=-1, keepdim=True)
        pick = torch.multinomial(p_sorted, num_samples=1)
        return idx.gather(-1, pick).squeeze(-1)
    return torch.multinomial(probs, num_samples=1).squeeze(-1)
