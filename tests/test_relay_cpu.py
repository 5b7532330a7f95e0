"""PrefixRelay heads (CPU): a zero head is the parallel proposal, greedy relay decoding equals
AR decoding, sampled relay outputs follow the target law, and the online learner lowers TV."""

import pytest
import torch

from online_speculation_b200.blockspec.generation import generate, generate_ar
from online_speculation_b200.blockspec.model import DualViewConfig, DualViewDecoder
from online_speculation_b200.blockspec.relay import (RelayBranch, RelayConfig, RelayFeedback, RelayHead,
                                                     RelayLearner, relay_candidates, relay_loss)
from online_speculation_b200.blockspec.sampling import SamplingConfig


def _model(seed=0, vocab=48):
    torch.manual_seed(seed)
    m = DualViewDecoder(DualViewConfig(vocab_size=vocab, block_size=4, mask_token_id=1)).eval()
    with torch.no_grad():
        for layer in m.layers:
            for p in layer.attention.draft.parameters():
                p.add_(torch.randn_like(p) * 0.05)
    return m


def test_zero_head_is_the_parallel_proposal():
    head = RelayHead(RelayConfig(40, 16, rank=8))
    logits = torch.randn(3, 40)
    d = relay_candidates(head, logits, torch.randn(3, 16), 5, sampling=SamplingConfig(0.0))
    assert torch.equal(d.tokens, logits.argmax(-1)) and d.q is None
    d1 = relay_candidates(head, logits, torch.randn(3, 16), 5, sampling=SamplingConfig(1.0),
                          generator=torch.Generator().manual_seed(0))
    assert torch.allclose(d1.q, logits.softmax(-1), atol=1e-6)
    with pytest.raises(ValueError):
        relay_candidates(head, logits, torch.randn(2, 16), 5)
    m = _model()
    head2 = RelayHead(RelayConfig(48, m.config.hidden_size, rank=8))
    head2.initialize_from_embedding(m.embedding.weight)
    assert torch.allclose(head2.embedding.weight.norm(dim=-1), torch.ones(48), atol=1e-5)


@pytest.mark.parametrize("threshold", [0.0, 0.6])
def test_greedy_relay_decoding_equals_ar(threshold):
    m = _model(1)
    head = RelayHead(RelayConfig(48, m.config.hidden_size, rank=8))
    with torch.no_grad():
        head.projection.weight.normal_(0, 0.5)
        head.confidence.bias.fill_(0.5)
    br = RelayBranch(m, head, threshold=threshold)
    prompt = torch.tensor([[5, 9, 13, 2, 7]])
    g = SamplingConfig(0.0)
    assert generate(br, prompt, 20, sampling=g).tokens == generate_ar(br, prompt, 20, sampling=g).tokens


def test_sampled_relay_outputs_follow_the_target_law():
    m = _model(2, vocab=8)
    head = RelayHead(RelayConfig(8, m.config.hidden_size, rank=4))
    with torch.no_grad():
        head.projection.weight.normal_(0, 1.0)         # a relay law far from the parallel one
    br = RelayBranch(m, head)
    prompt = torch.tensor([[3, 5]])
    with torch.no_grad():
        p1 = m(prompt).logits[0, -1].float().softmax(-1)
        exact = torch.zeros(8, 8)
        for a in range(8):
            p2 = m(torch.tensor([[3, 5, a]])).logits[0, -1].float().softmax(-1)
            for b in range(8):
                p3 = m(torch.tensor([[3, 5, a, b]])).logits[0, -1].float().softmax(-1)
                exact[b] += p1[a] * p2[b] * p3
    g = torch.Generator().manual_seed(5)
    counts = torch.zeros(8, 8)
    n = 2000
    for _ in range(n):
        out = generate(br, prompt, 3, sampling=SamplingConfig(1.0), generator=g)
        counts[out.tokens[1], out.tokens[2]] += 1
    assert 0.5 * float((counts / n - exact).abs().sum()) < 0.08


def test_relay_learner_lowers_tv():
    torch.manual_seed(3)
    V, H = 30, 16
    head = RelayHead(RelayConfig(V, H, rank=8))
    prev = torch.randint(0, V, (64,))
    logits = torch.randn(64, V)
    shift = torch.randn(V, V) * 2
    teacher = logits + shift[prev]                     # the target depends on the previous token
    fb = RelayFeedback(logits, torch.randn(64, H), prev, teacher)
    learner = RelayLearner(head, lr=3e-2, interval=1)
    before = float(relay_loss(head, fb)[1])
    for _ in range(60):
        learner.observe(fb)
    after = float(relay_loss(head, fb)[1])
    assert learner.updates == 60 and after < 0.7 * before


def test_relay_trains_online_while_decoding():
    m = _model(4)
    head = RelayHead(RelayConfig(48, m.config.hidden_size, rank=8))
    br = RelayBranch(m, head)
    learner = RelayLearner(head, lr=1e-2, interval=2)
    out = generate(br, torch.tensor([[5, 9, 13]]), 24, sampling=SamplingConfig(1.0),
                   generator=torch.Generator().manual_seed(1), feedback=br.feedback(learner))
    assert len(out.tokens) == 24 and learner.feedback_blocks >= 2 and learner.updates >= 1
