"""Prefix-budget trees (CPU): best-first prefixes against brute force, ancestor masks,
greedy equality with AR decoding, and the target law of sampled outputs."""

import itertools
import math

import pytest
import torch

from online_speculation_b200.blockspec.generation import MaskedAttentionBranch, generate_ar
from online_speculation_b200.blockspec.model import DualViewConfig, DualViewDecoder
from online_speculation_b200.blockspec.sampling import SamplingConfig
from online_speculation_b200.blockspec.tree import build_tree, generate_tree, traverse_greedy


def test_build_tree_keeps_the_best_prefixes():
    g = torch.Generator().manual_seed(0)
    q = torch.softmax(torch.randn(3, 6, generator=g) * 2, -1)
    k, budget = 3, 9
    tree = build_tree(2, q, top_k=k, prefix_budget=budget)
    assert len(tree.tokens) == budget and tree.tokens[0] == 2
    top = [q[d].topk(k).indices.tolist() for d in range(3)]
    prefixes = []
    for depth in range(1, 4):
        for combo in itertools.product(*top[:depth]):
            prefixes.append((sum(math.log(float(q[d, t])) for d, t in enumerate(combo)), combo))
    best = sorted(prefixes, reverse=True)[: budget - 1]
    got = {tuple(tree.tokens[n] for n in tree.path(node)[1:]) for node in range(1, budget)}
    assert got == {p for _, p in best}
    for node in range(1, budget):                      # prefix-closed, scores = log products
        assert tree.parents[node] < node
        assert tree.scores[node] == pytest.approx(sum(math.log(float(q[d, tree.tokens[n]]))
                                                      for d, n in enumerate(tree.path(node)[1:])))


def test_layout_sees_only_ancestors():
    q = torch.softmax(torch.randn(2, 5), -1)
    tree = build_tree(1, q, top_k=2, prefix_budget=5)
    ids, pos, allowed = tree.layout(3, device="cpu")
    assert ids.shape == (1, 5) and pos[0, 0] == 3
    for node in range(5):
        seen = set((allowed[0, 0, node, 3:].nonzero().flatten()).tolist())
        assert seen == set(tree.path(node)) and bool(allowed[0, 0, node, :3].all())
        assert int(pos[0, node]) == 3 + tree.depths[node]
    walk = traverse_greedy(tree, torch.tensor([tree.tokens[1]] + [0] * 4), budget=10)
    assert walk.matched >= 1 and walk.path[:2] == [0, 1]


def _model(seed=0, vocab=48):
    torch.manual_seed(seed)
    m = DualViewDecoder(DualViewConfig(vocab_size=vocab, block_size=4, mask_token_id=1)).eval()
    with torch.no_grad():
        for layer in m.layers:
            for p in layer.attention.draft.parameters():
                p.add_(torch.randn_like(p) * 0.05)
    return m


@pytest.mark.parametrize("top_k,budget,block", [(2, 6, 4), (4, 16, 5), (1, 3, 3)])
def test_greedy_tree_decoding_equals_ar(top_k, budget, block):
    m = _model(1)
    br = MaskedAttentionBranch(m)
    prompt = torch.tensor([[5, 9, 13, 2, 7]])
    greedy = SamplingConfig(0.0)
    ar = generate_ar(br, prompt, 20, sampling=greedy)
    tr = generate_tree(br, prompt, 20, block_size=block, top_k=top_k, prefix_budget=budget, sampling=greedy)
    assert tr.tokens == ar.tokens
    assert tr.rounds >= 1 and sum(tr.proposed_per_round) >= tr.rounds


def test_sampled_tree_outputs_follow_the_target_law():
    """Tokens 2 and 3 come from the tree traversal (token 1 from the prefill); their joint law
    must be the AR model's, summed over token 1."""
    m = _model(2, vocab=8)
    br = MaskedAttentionBranch(m)
    prompt = torch.tensor([[3, 5]])
    s = SamplingConfig(1.0)
    with torch.no_grad():
        p1 = m(prompt).logits[0, -1].float().softmax(-1)
        exact = torch.zeros(8, 8)
        for a in range(8):
            p2 = m(torch.tensor([[3, 5, a]])).logits[0, -1].float().softmax(-1)
            for b in range(8):
                p3 = m(torch.tensor([[3, 5, a, b]])).logits[0, -1].float().softmax(-1)
                exact[b] += p1[a] * p2[b] * p3
    g = torch.Generator().manual_seed(4)
    counts = torch.zeros(8, 8)
    n = 2000
    for _ in range(n):
        out = generate_tree(br, prompt, 3, block_size=4, top_k=3, prefix_budget=6, sampling=s, generator=g)
        counts[out.tokens[1], out.tokens[2]] += 1
    assert torch.allclose(exact.sum(), torch.tensor(1.0), atol=1e-5)
    tv = 0.5 * float((counts / n - exact.view(8, 8)).abs().sum())
    assert tv < 0.08
