"""Prefix-overlap objective (CPU): unbiasedness by enumeration, EOS handling, gradients, and the
online learner training the draft with it during generation."""

import itertools

import pytest
import torch

from online_speculation_b200.blockspec.generation import MaskedAttentionBranch, generate
from online_speculation_b200.blockspec.model import DualViewConfig, DualViewDecoder
from online_speculation_b200.blockspec.online import SuffixConfig
from online_speculation_b200.blockspec.prefix_objective import PrefixLearner, PrefixOnlineFeedback, prefix_overlap
from online_speculation_b200.blockspec.sampling import SamplingConfig


def test_expectation_is_the_expected_accepted_prefix():
    g = torch.Generator().manual_seed(0)
    n, V = 3, 4
    q = torch.softmax(torch.randn(n, V, generator=g, dtype=torch.float64), -1)
    p = torch.softmax(torch.randn(n, V, generator=g, dtype=torch.float64), -1)
    expected = 0.0
    for combo in itertools.product(range(V), repeat=n):
        c = torch.tensor(combo)
        weight = float(q[torch.arange(n), c].prod())
        expected += weight * float(prefix_overlap(q, p, c, q[torch.arange(n), c]))
    a = torch.minimum(q, p).sum(-1)
    exact = float(a[0] + a[0] * a[1] + a[0] * a[1] * a[2])
    assert expected == pytest.approx(exact, rel=1e-10)


def test_eos_ends_the_reachable_output_and_gradients_flow():
    q = torch.softmax(torch.randn(3, 5, dtype=torch.float64), -1).requires_grad_(True)
    p = torch.softmax(torch.randn(3, 5, dtype=torch.float64), -1)
    c = torch.tensor([2, 1, 0])
    taken = q.detach()[torch.arange(3), c]
    v = prefix_overlap(q, p, c, taken, eos_id=2)
    live0 = float((torch.minimum(q, p)[0].detach() * (torch.arange(5) != 2)).sum())
    assert float(v.detach()) == pytest.approx(live0)   # the first candidate is EOS: nothing beyond it
    v2 = prefix_overlap(q, p, c, taken)
    v2.backward()
    assert q.grad is not None and float(q.grad.abs().sum()) > 0
    with pytest.raises(ValueError):
        prefix_overlap(q, p, c, torch.zeros(3, dtype=torch.float64))


def test_prefix_learner_trains_during_generation():
    torch.manual_seed(2)
    cfg = DualViewConfig(vocab_size=17, hidden_size=16, intermediate_size=32, num_hidden_layers=2,
                         num_attention_heads=4, num_key_value_heads=2, head_dim=4, block_size=4, mask_token_id=1)
    m = DualViewDecoder(cfg).eval().requires_grad_(False)
    learner = PrefixLearner(m, SuffixConfig(stride=2, replay_blocks=1, learning_rate=1e-2))
    before = {n: p.clone() for n, p in m.named_parameters()}
    res = generate(MaskedAttentionBranch(m), torch.tensor([[2, 4, 6]]), 24, sampling=SamplingConfig(1.0),
                   generator=torch.Generator().manual_seed(0),
                   feedback=PrefixOnlineFeedback(learner=learner, output_budget=24))
    assert len(res.tokens) == 24 and res.updates >= 1 and learner.version == res.updates
    changed = {n for n, p in m.named_parameters() if not torch.equal(before[n], p)}
    assert changed and all(".attention.draft." in n for n in changed)
