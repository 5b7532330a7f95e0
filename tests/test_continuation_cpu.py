"""Request-local continuation mixtures (CPU): suffix index, the parallel copy walk against the
sequential walk, the TV gradient against finite differences, and online learning."""

import pytest
import torch

from online_speculation_b200.blockspec.continuation import (ContinuationMix, SuffixLookup, copy_mixture,
                                                            copy_tv_gradient)


def test_suffix_lookup_finds_the_longest_repeated_suffix():
    s = SuffixLookup([7, 1, 2, 3, 9, 8, 5, 1, 2, 3], lookahead=2)
    cont, n = s.find(4)
    assert n == 3 and cont == [9, 8, 5, 1]
    assert SuffixLookup([1, 2, 3, 4]).find(3) == ([], 0)
    s.extend([4])                                  # the suffix "2 3 4" has not occurred before
    assert s.find(2)[1] == 0
    with pytest.raises(ValueError):
        s.find(1)


def _sequential(baseline, weights, copied, e):
    tokens, rows, on_copy = [], [], True
    for i in range(baseline.shape[0]):
        row = baseline[i].clone()
        if i > 0 and on_copy and copied[i] >= 0:
            row = row * (1 - weights[i - 1])
            row[copied[i]] += weights[i - 1]
        tok = int((row / e[i]).argmax())
        tokens.append(tok)
        rows.append(row)
        on_copy = on_copy and tok == int(copied[i])
    return torch.tensor(tokens), torch.stack(rows)


@pytest.mark.parametrize("seed", range(6))
def test_parallel_copy_walk_equals_the_sequential_walk(seed):
    g = torch.Generator().manual_seed(seed)
    L, V = 5, 7
    base = torch.softmax(torch.randn(L, V, generator=g, dtype=torch.float64) * 2, -1)
    w = torch.rand(L - 1, generator=g, dtype=torch.float64)
    copied = torch.randint(0, V, (L,), generator=g)
    copied[-1] = -1 if seed % 2 else copied[-1]
    e = torch.empty(L, V, dtype=torch.float64).exponential_(generator=g)
    tok, q, fb = copy_mixture(base, w, copied, e)
    tok2, q2 = _sequential(base, w, copied, e)
    assert torch.equal(tok, tok2) and torch.allclose(q, q2)
    assert torch.equal(q[0], base[0])              # the root row is exact


def test_copy_tv_gradient_matches_finite_differences():
    g = torch.Generator().manual_seed(3)
    n, V = 4, 9
    q0 = torch.softmax(torch.randn(n, V, generator=g, dtype=torch.float64), -1)
    p = torch.softmax(torch.randn(n, V, generator=g, dtype=torch.float64), -1)
    c = torch.randint(0, V, (n,), generator=g)
    lam = torch.full((n,), 0.3, dtype=torch.float64)

    class FB:
        baseline, copied, weights, active = q0, c, lam, torch.ones(n, dtype=torch.bool)

    grad, _ = copy_tv_gradient(FB, p)

    def tv(l):
        q = q0 * (1 - l[:, None])
        q[torch.arange(n), c] += l
        return 1 - torch.minimum(q, p).sum(-1)

    h = 1e-6
    fd = (tv(lam + h) - tv(lam - h)) / (2 * h)
    assert torch.allclose(grad, fd, atol=1e-5)


def test_continuation_mix_learns_to_trust_repeated_text():
    mix = ContinuationMix(4, learning_rate=0.5, interval=1, diagnostics=True)
    text = [5, 6, 7, 8, 9, 10, 5, 6, 7]
    V = 16
    for _ in range(30):
        mix.begin_request(text)
        base = torch.full((4, V), 1.0 / V)
        base[0] = 0.0
        base[0, 8] = 1.0                               # the root (exact) continues the repetition
        tokens, q, fb = mix.draft(base, generator=torch.Generator().manual_seed(0))
        assert fb is not None and mix.copied[:3] == [8, 9, 10] and int(tokens[0]) == 8
        teacher = torch.zeros(3, V)
        teacher[torch.arange(3), torch.tensor(mix.copied[1:4])] = 1.0   # the text really repeats
        mix.observe(fb, teacher)
    group = min(3 - 2, 2)
    assert float(mix.weights[group, 0]) > 0.9
    st = mix.state_dict()
    other = ContinuationMix(4, learning_rate=0.5, interval=1)
    other.load_state_dict(st)
    assert torch.equal(other.weights, mix.weights)
    with pytest.raises(ValueError):
        ContinuationMix(4, interval=2).load_state_dict(st)
