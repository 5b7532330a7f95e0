"""Full-answer work audit and screening gate (CPU): the visit recurrence against exact
enumeration of accept / reject outcomes, trace scoring against per-round draft forwards,
the timing estimate, and the screening state machine."""

import itertools
import math

import pytest
import torch

from online_speculation_b200.blockspec.generation import MaskedAttentionBranch, ProposalSampler, generate
from online_speculation_b200.blockspec.model import DualViewConfig, DualViewDecoder, draft_block_mask, trim_cache
from online_speculation_b200.blockspec.sampling import SamplingConfig
from online_speculation_b200.blockspec.virtual_work import (FullAnswerGate, TraceSupportError, calibration_starts,
                                                            estimate_trace, expected_work, inverse_acceptance,
                                                            score_trace)


def _enumerate(acc, n, budget, block):
    """Expected draft / tail visits by walking every accept / reject outcome."""
    draft, tail = [0.0] * (n - 1), [0.0] * (n - 1)

    def go(j, w):
        if j >= n or w == 0:
            return
        if budget - j == 1:
            tail[j - 1] += w
            return
        draft[j - 1] += w
        m = min(block, budget - j + 1) - 1
        alive = w
        for o in range(1, m + 1):
            if j + o >= n:          # the delivered answer ends within this round
                return
            a = float(acc[j - 1, o - 1])
            go(j + o, alive * (1 - a))
            alive *= a
        go(j + m + 1, alive)

    go(1, 1.0)
    return draft, tail


@pytest.mark.parametrize("n,budget,block", [(7, 7, 4), (9, 12, 3), (6, 6, 2), (10, 10, 5), (2, 5, 4)])
def test_expected_work_matches_enumeration(n, budget, block):
    g = torch.Generator().manual_seed(n * 100 + block)
    acc = torch.rand(n - 1, block - 1, generator=g, dtype=torch.float64)
    w = expected_work(acc, output_tokens=n, output_budget=budget, block_size=block)
    d, t = _enumerate(acc, n, budget, block)
    assert torch.allclose(w.draft_visits, torch.tensor(d, dtype=torch.float64), atol=1e-12)
    assert torch.allclose(w.tail_visits, torch.tensor(t, dtype=torch.float64), atol=1e-12)
    assert float(w.decode_forwards) == pytest.approx(2 * sum(d) + sum(t))


def test_expected_work_limits_and_gradient():
    n, block = 9, 4
    ones = torch.ones(n - 1, block - 1, dtype=torch.float64)
    w = expected_work(ones, output_tokens=n, output_budget=n, block_size=block)
    # always accepted: rounds after 1 and 5 deliver 4 tokens each (3 drafts + the bonus token)
    assert w.draft_visits.tolist() == [1, 0, 0, 0, 1, 0, 0, 0] and w.tail_visits.tolist() == [0] * 8
    zeros = torch.zeros(n - 1, block - 1, dtype=torch.float64)
    w0 = expected_work(zeros, output_tokens=n, output_budget=n, block_size=block)
    assert float(w0.draft_forwards) == 7 and float(w0.tail_ar_forwards) == 1   # one token per round
    a = torch.full((n - 1, block - 1), 0.5, dtype=torch.float64, requires_grad=True)
    cost = expected_work(a, output_tokens=n, output_budget=n, block_size=block).cost(2.0, 1.0)
    cost.backward()
    assert bool(torch.isfinite(a.grad).all()) and float(a.grad.sum()) < 0   # more acceptance, less work
    with pytest.raises(ValueError):
        expected_work(torch.ones(3, 2), output_tokens=5, output_budget=5, block_size=3)


def test_inverse_acceptance_and_calibration_starts():
    q = torch.tensor([-1.0, -3.0])
    p = torch.tensor([-2.0, -1.0])
    assert torch.allclose(inverse_acceptance(q, p), torch.tensor([1.0, math.exp(-2.0)]))
    with pytest.raises(TraceSupportError):
        inverse_acceptance(q, torch.tensor([-1.0, float("-inf")]))
    assert calibration_starts(torch.tensor([1.0, 1.0, 1.0, 1.0]), 2) == [1, 3]
    assert calibration_starts(torch.zeros(3), 2) == []


def _model(seed=0):
    torch.manual_seed(seed)
    cfg = DualViewConfig(vocab_size=48, block_size=4, mask_token_id=1)
    m = DualViewDecoder(cfg).eval()
    with torch.no_grad():                       # make the draft view differ from the AR view
        for layer in m.layers:
            for p in layer.attention.draft.parameters():
                p.add_(torch.randn_like(p) * 0.05)
    return m


def test_score_trace_matches_per_round_draft_forwards():
    m = _model()
    prompt = torch.tensor([[5, 9, 13, 2]])
    outputs = torch.tensor([7, 11, 3, 20, 8, 30, 4, 17, 22])
    n, budget, P = outputs.numel(), outputs.numel(), prompt.shape[1]
    sampling = SamplingConfig(1.0)
    s = score_trace(m, prompt, outputs, output_budget=budget, sampling=sampling, anchors_per_pass=3, chunk_rows=5)
    clean = torch.cat((prompt, outputs[None]), 1)
    with torch.no_grad():
        full = m(clean)
        ar_logp = full.logits[0].float().log_softmax(-1)
        for j in range(1, n - 1):
            L = min(4, budget - j + 1)
            a = P + j - 1
            cache = trim_cache(full.cache, a)
            inp = torch.full((1, L), 1, dtype=torch.long)
            inp[0, 0] = clean[0, a]
            out = m(inp, view="draft", cache=cache, allowed=draft_block_mask(a, L, inp.device))
            q = out.logits[0].float().log_softmax(-1)
            for o in range(1, L):
                if j + o > n - 1:
                    assert not s.valid[j - 1, o - 1]
                    continue
                tok = int(outputs[j + o - 1])
                assert bool(s.valid[j - 1, o - 1])
                assert float(s.proposal_logp[j - 1, o - 1]) == pytest.approx(float(q[o - 1, tok]), abs=1e-4)
                assert float(s.target_logp[j - 1, o - 1]) == pytest.approx(float(ar_logp[a + o - 1, tok]),
                                                                           abs=1e-4)
    w = s.work()
    assert float(w.draft_forwards) > 0 and w.draft_visits.shape == (n - 1,)


def test_estimate_trace_predicts_a_time():
    m = _model(1)
    branch = MaskedAttentionBranch(m)
    sampling = SamplingConfig(1.0)
    sampler = ProposalSampler(sampling)
    prompt = torch.tensor([[5, 9, 13, 2]])
    g = torch.Generator().manual_seed(3)
    res = generate(branch, prompt, 12, sampling=sampling, generator=g)
    outputs = torch.tensor(res.tokens)
    t = estimate_trace(branch, prompt, outputs, output_budget=12, prefill_seconds=0.001, sampler=sampler,
                       generator=torch.Generator().manual_seed(4), sampling=sampling, calibration_points=2)
    assert t.predicted_seconds > 0.001 and len(t.round_seconds) == 2 and t.measured_seconds >= t.score_seconds
    assert float(t.work.draft_forwards) >= 1


def _row(step=3, ref=2.0, pred=1.0, tokens=100):
    return {"step": step, "reference_tokens": tokens, "reference_seconds": ref, "predicted_seconds": pred}


def test_full_answer_gate_screening():
    g = FullAnswerGate(count=2, margin=1.1)
    r = g.observe(_row(), 0.5)
    assert not r["screen_passed"] and not r["complete"] and g.estimate == pytest.approx(0.6)
    r = g.observe(dict(_row(), evaluation_seconds=0.2), 0.5)
    assert r["screen_passed"] and r["awaiting_confirmation"] and r["candidate_over_ar"] == pytest.approx(2.0)
    assert g.ready and g.estimate == pytest.approx(1.2 * (1.0 + 0.0 + 0.3))
    with pytest.raises(ValueError):
        g.observe(_row(), 0.5)                      # no new evidence while awaiting confirmation
    st = g.state_dict()
    h = FullAnswerGate(count=2, margin=1.1)
    h.load_state_dict(st, step=3, next_probe=3, speculating=False, requests=5)
    assert h.ready and h.pending == g.pending
    g.confirmed()
    assert not g.ready and g.pending == []
    # a failing screen is discarded once complete
    g2 = FullAnswerGate(count=2, margin=1.5)
    g2.observe(_row(ref=1.0), 0.4)
    r = g2.observe(_row(ref=1.0), 0.4)
    assert r["complete"] and not r["screen_passed"] and g2.pending == []
    with pytest.raises(ValueError):
        FullAnswerGate(margin=0.9)
    with pytest.raises(ValueError):
        g2.observe(_row(step=0), 0.4)
    g3 = FullAnswerGate(count=3)
    g3.observe(_row(step=4), 0.4)
    with pytest.raises(ValueError):
        g3.observe(_row(step=5), 0.4)               # evidence must come from one version
    with pytest.raises(ValueError):                 # restored evidence must match the service position
        FullAnswerGate(count=3).load_state_dict(g3.state_dict(), step=5, next_probe=5, speculating=False,
                                                requests=5)


def test_full_answer_gate_against_the_serving_speculative_version():
    g = FullAnswerGate(count=1, margin=1.0, reuse_speculative=True)
    with pytest.raises(ValueError):
        g.observe(dict(_row(step=6), reference_step=2), 0.5)   # needs a measured AR rate first
    g.confirmed(ar_tps=200.0)
    r = g.observe(dict(_row(step=6), reference_step=2), 0.5)
    assert r["candidate_over_serving"] == pytest.approx(2.0) and g.ready
    assert g.estimate == pytest.approx(1.2 * (1.0 + 100 / 200.0 + 0.5))
    st = g.state_dict()
    h = FullAnswerGate(count=1, margin=1.0, reuse_speculative=True)
    h.load_state_dict(st, step=6, next_probe=6, speculating=True, requests=3, serving_step=2)
    assert h.ready and h.ar_tps == 200.0
    for bad in (dict(step=6, next_probe=6, speculating=True, requests=3, serving_step=6),
                dict(step=7, next_probe=6, speculating=True, requests=3, serving_step=2)):
        with pytest.raises(ValueError):
            FullAnswerGate(count=1, margin=1.0, reuse_speculative=True).load_state_dict(st, **bad)
    assert list(itertools.islice(iter(st["pending"]), 1))[0]["reference_step"] == 2
