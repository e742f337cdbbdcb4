"""Per-request sampling parameters and next-token choice.

The parameter set is the reference's (``persona/sampling.py:8-13``:
temperature, top-p, a token budget).  The choice itself is written around
the Gumbel-max identity instead of an explicit draw from a renormalised
distribution: ``argmax(z + G)`` with ``G`` i.i.d. standard Gumbel noise picks
index ``i`` with probability ``softmax(z)_i``.  That needs no renormalisation,
no ``multinomial`` and no host round trip, and a top-p cut becomes a mask on
``z`` (a per-row log-probability threshold), so every row of a batch is
handled in one set of tensor ops on the device.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import torch


@dataclass
class SamplingParams:
    temperature: float = 0.0
    top_p: float = 1.0
    max_tokens: int = 128


def _nucleus_mask(z: torch.Tensor, top_p: float) -> torch.Tensor:
    """``z`` with every token outside the top-p nucleus set to -inf.

    The nucleus of a row is the most probable tokens, taken in order of
    probability while the mass of the tokens before them is at most
    ``top_p`` (so the most probable token always stays).  It is applied as a
    threshold on the log-probability of the last token kept; tokens tied
    with that one stay as well.
    """
    lp = torch.log_softmax(z, dim=-1)
    lp_sorted = torch.sort(lp, dim=-1, descending=True).values
    p_sorted = lp_sorted.exp()
    mass_before = torch.cumsum(p_sorted, dim=-1) - p_sorted
    keep = (mass_before <= top_p).sum(dim=-1, keepdim=True).clamp_(min=1)
    threshold = lp_sorted.gather(-1, keep - 1)
    return z.masked_fill(lp < threshold, float("-inf"))


def sample_next_token(logits: torch.Tensor, params: SamplingParams,
                      generator: Optional[torch.Generator] = None) -> torch.Tensor:
    """logits [batch, vocab] -> next token ids [batch] (int64).

    Temperature 0 (or below) is greedy.  Otherwise the logits are divided by
    the temperature, cut to the top-p nucleus when ``top_p < 1``, and one
    token per row is drawn by Gumbel-max.
    """
    if params.temperature <= 0:
        return logits.argmax(dim=-1)
    z = logits.float() / params.temperature
    if params.top_p < 1.0:
        z = _nucleus_mask(z, params.top_p)
    u = torch.rand(z.shape, device=z.device, generator=generator)
    gumbel = -torch.log(-torch.log(u.clamp_(min=torch.finfo(torch.float32).tiny)))
    return (z + gumbel).argmax(dim=-1)
