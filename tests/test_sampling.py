"""Next-token choice (persona/sampling.py): greedy at temperature 0, the
top-p nucleus, and Gumbel-max draws that follow softmax(logits / T).  CPU."""

import numpy as np
import torch

from persona.sampling import SamplingParams, _nucleus_mask, sample_next_token


def test_greedy_is_argmax():
    g = torch.Generator().manual_seed(0)
    logits = torch.randn(5, 100, generator=g)
    assert torch.equal(sample_next_token(logits, SamplingParams(temperature=0.0)), logits.argmax(-1))


def test_nucleus_keeps_the_reference_prefix():
    # probabilities 0.5, 0.25, 0.15, 0.1 (already sorted, token order shuffled)
    p = torch.tensor([[0.15, 0.5, 0.1, 0.25]])
    z = p.log()
    # the reference's rule: drop a token when the mass before it exceeds top_p
    for top_p, kept in ((0.4, {1}), (0.45, {1}), (0.6, {1, 3}), (0.8, {1, 3, 0}), (0.95, {1, 3, 0, 2})):
        m = _nucleus_mask(z, top_p)
        assert set(torch.nonzero(torch.isfinite(m[0])).flatten().tolist()) == kept, top_p


def test_draws_follow_the_tempered_softmax():
    g = torch.Generator().manual_seed(1)
    logits = torch.tensor([[2.0, 1.0, 0.0, -1.0]]).repeat(20000, 1)
    params = SamplingParams(temperature=0.7)
    tok = sample_next_token(logits, params, generator=g)
    freq = np.bincount(tok.numpy(), minlength=4) / tok.numel()
    want = torch.softmax(logits[0] / 0.7, -1).numpy()
    assert np.all(np.abs(freq - want) < 0.015), (freq, want)


def test_top_p_draws_stay_in_the_nucleus():
    g = torch.Generator().manual_seed(2)
    logits = torch.tensor([[3.0, 2.0, 0.0, -2.0, -3.0]]).repeat(5000, 1)
    params = SamplingParams(temperature=1.0, top_p=0.8)
    tok = sample_next_token(logits, params, generator=g)
    p = torch.softmax(logits[0], -1)
    assert p[0] < 0.8 <= p[0] + p[1]
    assert set(tok.unique().tolist()) == {0, 1}
    freq = (tok == 0).float().mean().item()
    assert abs(freq - (p[0] / (p[0] + p[1])).item()) < 0.02
