"""Rao-Blackwellised prefix-overlap objective for a factorised parallel draft.

A drafted block's value is how far the exact p / q correction gets into it.  Given
the candidates c_1..c_n that the serving proposal q_taken actually drew, the number
of positions a round advances is estimated by

    sum_k reach_k * sum_v min(q_k, p_k)(v),   reach_k = prod_{j<k} min(q_j, p_j)(c_j) / q_taken_j(c_j),

where row k integrates its own categorical draw analytically and the earlier rows
use importance weights against the proposal that generated the candidates.  With
q = q_taken its expectation over the candidates is the expected accepted prefix
length, sum_k prod_{j<k} a_j * a_k with a_j = sum min(q_j, p_j).  Maximising it
trains the draft towards what speculation rewards -- long accepted prefixes --
rather than a per-row divergence.  EOS (when given) ends the reachable output.

:class:`PrefixLearner` is the online suffix learner with this objective (the
gradient reaches the draft attention through q); the estimator needs candidates
drawn by the current draft version, so only on-version replay enters an update.
:class:`PrefixOnlineFeedback` collects the candidates and their proposal
probabilities from :func:`online_speculation_b200.blockspec.generation.generate`.

Reference behaviour: online-speculation/ablation/src/blockspec_ablation/prefix_objective.py
(``prefix_overlap``, ``PrefixLearner``, ``PrefixOnlineFeedback``).
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch

from .online import Feedback, OnlineFeedback, SuffixConfig, SuffixLearner


def prefix_overlap(q: torch.Tensor, p: torch.Tensor, candidates: torch.Tensor, proposal_taken: torch.Tensor, *,
                   eos_id: int | None = None) -> torch.Tensor:
    """Estimated additional output positions of one round (differentiable in ``q``).

    ``q`` [n, V] current draft rows, ``p`` [n, V] target rows, ``candidates`` [n] the drawn
    tokens, ``proposal_taken`` [n] their probabilities under the proposal that drew them."""
    if (q.ndim != 2 or q.shape != p.shape or len(q) < 1 or tuple(candidates.shape) != (len(q),)
            or proposal_taken.shape != candidates.shape):
        raise ValueError("aligned [n, V] rows, n candidates and n proposal probabilities are required")
    if candidates.dtype != torch.long or bool(((candidates < 0) | (candidates >= q.shape[1])).any()):
        raise ValueError("integer candidates inside the vocabulary are required")
    if (not bool(torch.isfinite(proposal_taken).all()) or bool((proposal_taken <= 0).any())
            or bool((proposal_taken > 1).any())):
        raise ValueError("proposal probabilities in (0, 1] are required")
    if eos_id is not None and not 0 <= eos_id < q.shape[1]:
        raise ValueError("EOS must lie inside the vocabulary")
    overlap = torch.minimum(q, p.detach())
    live = overlap if eos_id is None else overlap * (torch.arange(q.shape[1], device=q.device) != eos_id)[None]
    ratio = overlap.gather(1, candidates[:, None]).squeeze(1) / proposal_taken.detach()
    if eos_id is not None:
        ratio = ratio * (candidates != eos_id)
    reach = torch.cat((ratio.new_ones(1), ratio[:-1].cumprod(0)))
    return (reach * live.sum(-1)).sum()


@dataclass
class PrefixFeedback(Feedback):
    candidates: torch.Tensor | None = None
    proposal_taken: torch.Tensor | None = None
    version: int = 0

    def detached(self, cache_start: int = 0) -> "PrefixFeedback":
        base = super().detached(cache_start=cache_start)
        return PrefixFeedback(base.inputs, base.cache, base.teacher_logits, base.valid, base.boundary,
                              base.fully_covered, self.candidates.detach().clone(),
                              self.proposal_taken.detach().clone(), self.version)


class PrefixLearner(SuffixLearner):
    """Online suffix learner maximising the prefix-overlap estimate (temperature ``temperature``)."""

    def __init__(self, model, config: SuffixConfig = SuffixConfig(), *, temperature: float = 1.0):
        if not math.isfinite(temperature) or temperature <= 0:
            raise ValueError("a positive finite temperature is required")
        super().__init__(model, config)
        self.temperature = temperature

    def observe(self, fb, *, may_update: bool = True):
        if not isinstance(fb, PrefixFeedback) or fb.version != self.version:
            raise ValueError("feedback must carry candidates drawn by the current draft version")
        return super().observe(fb, may_update=may_update)

    def _replay_items(self) -> list:
        return [fb for fb in self.replay if getattr(fb, "version", -1) == self.version]

    def _replay_loss(self, fb, logits, rows, blocks):
        q = (logits.float() / self.temperature).softmax(-1)
        p = (fb.teacher_logits.float() / self.temperature).softmax(-1)
        return -prefix_overlap(q, p, fb.candidates, fb.proposal_taken,
                               eos_id=self.model.config.eos_token_id) / blocks


class PrefixOnlineFeedback(OnlineFeedback):
    """Generation hooks collecting every drafted candidate (not only accepted ones) with the
    probability its proposal gave it; ``output_budget`` is the request's max_new_tokens."""

    def __init__(self, *, learner: PrefixLearner, output_budget: int):
        super().__init__(learner=learner)
        self.output_budget = output_budget

    def begin(self, prompt):
        super().begin(prompt)
        self.emitted = self.last_commit = 0

    def commit(self, tokens):
        self.last_commit = len(tokens)
        self.emitted += self.last_commit

    def observe(self, proposal, teacher_logits, target, *, used, fully_covered, done):
        if not proposal.collect_feedback or proposal.boundary is None:
            self.learner.skip()
            return
        remaining = self.output_budget - (self.emitted - self.last_commit)
        rows = min(proposal.candidates.numel(), remaining - 1)
        if rows < 1 or proposal.proposal is None:
            self.learner.skip()
            return
        cand = proposal.candidates[:rows].long()
        taken = proposal.proposal[:rows].gather(1, cand[:, None]).squeeze(1)
        fb = PrefixFeedback(proposal.draft_inputs, proposal.cache, teacher_logits[:rows], rows, proposal.boundary,
                            fully_covered, cand, taken, self.learner.version)
        self.learner.observe(fb, may_update=not done)


__all__ = ["PrefixFeedback", "PrefixLearner", "PrefixOnlineFeedback", "prefix_overlap"]
