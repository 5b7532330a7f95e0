"""Prefix-budget candidate trees with exact target-path traversal.

Each round drafts one block from the committed anchor (the draft view, as in
:func:`online_speculation_b200.blockspec.generation.generate`), then spends a
budget of tree nodes on the most probable draft *prefixes*: a best-first search
over products of the per-depth top-k draft probabilities (a product never grows
when a prefix is extended, so the heap yields the globally best prefixes without
enumerating K**depth leaves).  One AR forward scores every node with an
ancestor-only attention mask.  Decoding then walks the tree: at the current node
it samples the TARGET distribution p(. | path), and moves to the child holding
that token if the tree has one; the first sampled token without a child ends the
round and becomes the next anchor.

The tree is a computation schedule, not a proposal law: tokens are always drawn
from the target, so the output law is exactly the target's (no p / q ratio is
involved), and under greedy decoding the output equals plain AR decoding.  Only
the KV rows of the committed ancestral path are kept for the next round.

Reference behaviour: online-speculation/ablation/src/blockspec_ablation/tree.py
(``build_tree``, ``CandidateTree.layout``, ``traverse_target`` / ``traverse_greedy``,
``compact_tree_cache``, ``generate_tree``).
"""

from __future__ import annotations

import heapq
import math
import time
from dataclasses import dataclass, field

import torch
from torch import Tensor

from .generation import Generation, MaskedAttentionBranch, ProposalSampler, _sync
from .model import cache_length
from .sampling import SamplingConfig, draw, greedy_tokens, probabilities, validate_distribution


def tree_scores(logits: Tensor, sampling: SamplingConfig = SamplingConfig()) -> Tensor:
    """Ranking scores of the draft rows: softmax at the sampling temperature (1 when greedy).

    They only order candidate prefixes; they never enter an acceptance ratio."""
    return probabilities(logits, SamplingConfig(temperature=sampling.temperature or 1.0))


@dataclass
class CandidateTree:
    tokens: list[int]
    parents: list[int]
    depths: list[int]
    scores: list[float]                     # log of the prefix product
    children: list[dict[int, int]] = field(default_factory=list)

    def path(self, node: int) -> list[int]:
        out = []
        while node >= 0:
            out.append(node)
            node = self.parents[node]
        return out[::-1]

    def layout(self, prefix_length: int, *, device):
        """(ids [1, n], positions [1, n], allowed [1, 1, n, prefix + n]): every node sees the
        prefix and its own ancestors (itself included), at position prefix + depth."""
        n = len(self.tokens)
        allowed = torch.zeros(n, prefix_length + n, dtype=torch.bool)
        allowed[:, :prefix_length] = True
        for node in range(n):
            allowed[node, [prefix_length + a for a in self.path(node)]] = True
        ids = torch.tensor([self.tokens], device=device)
        positions = torch.tensor([self.depths], device=device) + prefix_length
        return ids, positions, allowed[None, None].to(device)


def build_tree(root: int, q: Tensor, *, top_k: int = 4, prefix_budget: int = 16) -> CandidateTree:
    """Best-first tree of the highest-product draft prefixes; ``prefix_budget`` counts the root.

    ``q`` [depths, V]: draft probabilities of the tokens after the root, per depth.
    Ties are broken by the token path (deterministic)."""
    validate_distribution(q)
    if q.ndim != 2 or top_k < 1 or prefix_budget < 1 or not 0 <= root < q.shape[-1]:
        raise ValueError("a [depths, V] distribution, top_k >= 1, a positive budget and a valid root are required")
    vals, ids = q.detach().topk(min(top_k, q.shape[-1]), dim=-1, sorted=True)
    vals, ids = vals.cpu().tolist(), ids.cpu().tolist()
    tree = CandidateTree([root], [-1], [0], [0.0], [{}])
    heap: list = []

    def push_children(parent: int, path: tuple):
        d = tree.depths[parent]
        if d >= q.shape[0]:
            return
        for pr, tok in zip(vals[d], ids[d]):
            if pr > 0:
                heapq.heappush(heap, (-(tree.scores[parent] + math.log(pr)), path + (tok,), parent, tok))

    push_children(0, ())
    while heap and len(tree.tokens) < prefix_budget:
        neg, path, parent, tok = heapq.heappop(heap)
        node = len(tree.tokens)
        tree.tokens.append(tok)
        tree.parents.append(parent)
        tree.depths.append(tree.depths[parent] + 1)
        tree.scores.append(-neg)
        tree.children.append({})
        tree.children[parent][tok] = node
        push_children(node, path)
    return tree


@dataclass
class TreeTraversal:
    tokens: list[int]        # sampled tokens, in order (the root is not included)
    path: list[int]          # visited nodes: the root, then every matched child
    teachers: list[int]      # node whose target row produced each sampled token
    matched: int


def _walk(tree: CandidateTree, next_token, budget: int, eos_id) -> TreeTraversal:
    out, path, teachers = [], [0], []
    node = matched = 0
    while len(out) < budget and (not out or out[-1] != eos_id):
        tok = next_token(node)
        teachers.append(node)
        out.append(tok)
        child = tree.children[node].get(tok)
        if child is None:
            break
        matched += 1
        node = child
        path.append(node)
    return TreeTraversal(out, path, teachers, matched)


def traverse_target(tree: CandidateTree, target: Tensor, *, budget: int, eos_id=None, generator=None) -> TreeTraversal:
    """Sample the target distribution at each reached node (``target`` [nodes, V] probabilities)."""
    validate_distribution(target)
    if target.ndim != 2 or target.shape[0] != len(tree.tokens) or budget < 1:
        raise ValueError("one target row per tree node and a positive token budget are required")
    return _walk(tree, lambda node: int(draw(target[node], generator)), budget, eos_id)


def traverse_greedy(tree: CandidateTree, target_ids: Tensor, *, budget: int, eos_id=None) -> TreeTraversal:
    if (tuple(target_ids.shape) != (len(tree.tokens),) or budget < 1
            or target_ids.dtype not in (torch.int32, torch.int64)):
        raise ValueError("one integer greedy target per tree node is required")
    t = target_ids.tolist()
    if any(v < 0 for v in t):
        raise ValueError("negative target id")
    return _walk(tree, lambda node: t[node], budget, eos_id)


def compact_tree_cache(cache, prefix_length: int, path: list[int]):
    """Keep the prefix and exactly the committed ancestral path's KV rows (no siblings)."""
    total = cache_length(cache)
    if cache is None or not 0 <= prefix_length <= total:
        raise ValueError("invalid tree cache prefix")
    if len(set(path)) != len(path) or any(n < 0 or prefix_length + n >= total for n in path):
        raise ValueError("invalid tree path indices")
    dev = cache[0][0].device
    idx = torch.cat((torch.arange(prefix_length, device=dev),
                     prefix_length + torch.tensor(path, dtype=torch.long, device=dev)))
    if not idx.numel():
        return None
    return tuple((k.index_select(2, idx).detach(), v.index_select(2, idx).detach()) for k, v in cache)


@torch.no_grad()
def generate_tree(branch: MaskedAttentionBranch, prompt: Tensor, max_new_tokens: int, *, block_size=None,
                  top_k: int = 4, prefix_budget: int = 16, sampling: SamplingConfig = SamplingConfig(),
                  eos_id=None, generator=None, sampler: ProposalSampler | None = None) -> Generation:
    """Tree speculation with the dual-view model; same ``Generation`` record as ``generate``
    (``accepted_per_round`` counts matched tree nodes, ``proposed_per_round`` tree nodes)."""
    if prompt.ndim != 2 or prompt.shape[0] != 1 or prompt.shape[1] < 1:
        raise ValueError("nonempty batch-one prompt required")
    block = branch.default_block_size if block_size is None else block_size
    if block < 2 or top_k < 1 or prefix_budget < 1:
        raise ValueError("block >= 2, top_k >= 1 and a positive node budget are required")
    model = branch.model
    sampler = sampler or ProposalSampler(sampling)
    result = Generation()
    if max_new_tokens == 0:
        return result
    _sync(prompt.device)
    t0 = time.perf_counter()
    logits, cache = branch.ar(prompt, logits_to_keep=1)
    tok = sampler.sample_ar(logits[0, -1], generator)
    result.tokens.append(tok)
    result.prefill_forwards = result.prefill_output_tokens = 1
    while len(result.tokens) < max_new_tokens and tok != eos_id:
        result.rounds += 1
        remaining = max_new_tokens - len(result.tokens)
        prefix = prompt.shape[1] + len(result.tokens) - 1          # history before the anchor
        anchor = prompt.new_tensor([[tok]])
        if remaining == 1:
            logits, cache = branch.ar(anchor, cache=cache, logits_to_keep=1)
            tok = sampler.sample_ar(logits[0, -1], generator)
            result.tokens.append(tok)
            result.tail_ar_forwards += 1
            break
        length = min(block, remaining + 1)
        inp = anchor.new_full((1, length), model.config.mask_token_id)
        inp[:, 0] = anchor[0, 0]
        draft = model(inp, view="draft", cache=cache).logits[0, :-1]     # depths 1 .. length-1
        result.draft_forwards += 1
        tree = build_tree(tok, tree_scores(draft, sampling), top_k=top_k, prefix_budget=prefix_budget)
        ids, pos, allowed = tree.layout(prefix, device=prompt.device)
        out = model(ids, cache=cache, positions=pos, allowed=allowed)
        result.verifier_forwards += 1
        if sampling.temperature == 0:
            walk = traverse_greedy(tree, greedy_tokens(out.logits[0]), budget=remaining, eos_id=eos_id)
        else:
            walk = traverse_target(tree, probabilities(out.logits[0], sampling), budget=remaining, eos_id=eos_id,
                                   generator=generator)
        result.tokens.extend(walk.tokens)
        # the anchor and every committed token but the last (the next anchor) keep their KV rows
        cache = compact_tree_cache(out.cache, prefix, walk.path[:len(walk.tokens)])
        tok = result.tokens[-1]
        result.accepted_per_round.append(walk.matched)
        result.proposed_per_round.append(len(tree.tokens) - 1)
        result.fully_covered_rounds += walk.matched == length - 1
    del result.tokens[max_new_tokens:]
    _sync(prompt.device)
    result.seconds = time.perf_counter() - t0
    return result


__all__ = ["CandidateTree", "TreeTraversal", "build_tree", "compact_tree_cache", "generate_tree",
           "traverse_greedy", "traverse_target", "tree_scores"]
