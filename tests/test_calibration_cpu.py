"""Online temperature calibration (CPU): simplex projection, tempered-expert mixtures,
convergence towards the temperature that matches the target, and state round trips."""

import pytest
import torch

from online_speculation_b200.blockspec.calibration import OverlapMix, mix_rows, project_simplex


def _bisection_projection(v):
    lo, hi = float(v.min()) - 1.0, float(v.max())
    for _ in range(200):
        mid = 0.5 * (lo + hi)
        if float((v - mid).clamp_min(0).sum()) > 1:
            lo = mid
        else:
            hi = mid
    return (v - 0.5 * (lo + hi)).clamp_min(0)


def test_project_simplex():
    g = torch.Generator().manual_seed(0)
    v = torch.randn(20, 7, generator=g, dtype=torch.float64) * 2
    x = project_simplex(v)
    assert bool((x >= 0).all()) and torch.allclose(x.sum(-1), torch.ones(20, dtype=torch.float64))
    for i in range(20):
        assert torch.allclose(x[i], _bisection_projection(v[i]), atol=1e-9)
    on = torch.tensor([[0.2, 0.3, 0.5], [1.0, 0.0, 0.0]], dtype=torch.float64)
    assert torch.allclose(project_simplex(on), on)


def test_mix_rows_experts_and_protected_row():
    g = torch.Generator().manual_seed(1)
    base = torch.softmax(torch.randn(4, 30, generator=g), -1)
    temps = (0.5, 1.0, 2.0)
    powers = torch.tensor(temps).reciprocal()[None, :, None]
    k = 6
    w = torch.zeros(3, 3)
    w[:, 1] = 1                                        # identity expert only
    q, fb = mix_rows(base, w, powers, 1, k, protected_rows=1)
    assert torch.equal(q[0], base[0])                  # the anchor row passes through
    vals, idx = base[1:].topk(k, -1)
    assert torch.allclose(q[1:].gather(-1, idx), vals) and torch.allclose(q[1:].sum(-1), vals.sum(-1))
    w2 = torch.zeros(3, 3)
    w2[:, 0] = 1                                       # T = 0.5: squared and renormalised on the top-k
    q2, _ = mix_rows(base, w2, powers, 1, k)
    want = vals.pow(2) / vals.pow(2).sum(-1, keepdim=True)
    assert torch.allclose(q2[1:].gather(-1, idx), want, atol=1e-6)
    assert torch.allclose(q2[1:].sum(-1), torch.ones(3), atol=1e-6)
    assert fb.experts.shape == (3, 3, k)


def test_overlap_mix_learns_the_matching_temperature():
    torch.manual_seed(2)
    block, V, k = 4, 40, 8
    cal = OverlapMix(block, k, temperatures=(0.5, 1.0, 2.0), learning_rate=0.5, interval=2, diagnostics=True)
    first_tv = last_tv = None
    for it in range(400):
        base = torch.softmax(torch.randn(block, V) * 1.5, -1)
        q, fb = cal.propose(base)
        vals, idx = base[1:].topk(k, -1)
        target = torch.zeros(block - 1, V).scatter_(-1, idx, vals.pow(2) / vals.pow(2).sum(-1, keepdim=True))
        tv = float((1 - torch.minimum(target, q[1:]).sum(-1)).mean())
        if it == 0:
            first_tv = tv
        last_tv = tv
        cal.observe(fb, target[:2])                     # the block reached two drafted depths
    w = cal.weights
    assert float(w[0, 0]) > 0.8 and float(w[1, 0]) > 0.8  # T = 0.5 wins on the observed depths
    assert torch.equal(w[2], torch.tensor([0.0, 1.0, 0.0]))   # an unobserved depth keeps its start
    assert last_tv < 0.5 * first_tv and cal.updates == 200
    m = cal.metrics()
    assert m["depth_observations"][:2] == [400.0, 400.0] and m["depth_observations"][2] == 0.0


def test_overlap_mix_state_round_trip_and_validation():
    a = OverlapMix(4, 8, interval=1)
    base = torch.softmax(torch.randn(4, 20), -1)
    _, fb = a.propose(base)
    a.observe(fb, torch.softmax(torch.randn(3, 20), -1))
    st = a.state_dict()
    b = OverlapMix(4, 8, interval=1)
    b.load_state_dict(st)
    assert torch.equal(a.weights, b.weights) and b.updates == a.updates == 1
    with pytest.raises(ValueError):
        OverlapMix(4, 8, interval=2).load_state_dict(st)
    bad = {**st, "tensors": {**st["tensors"], "weights": st["tensors"]["weights"] * 2}}
    with pytest.raises(ValueError):
        b.load_state_dict(bad)
    with pytest.raises(ValueError):
        OverlapMix(4, 8, temperatures=(0.5, 2.0))      # the identity temperature is required
    with pytest.raises(ValueError):
        a.propose(torch.softmax(torch.randn(6, 20), -1))   # more rows than the block has
