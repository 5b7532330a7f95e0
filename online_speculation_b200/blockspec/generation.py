"""Batch-one block-speculative decoding with a pending committed anchor.

A :class:`_Decoder` holds the state of one request (branch, sampler, KV history,
anchor, result) and moves through three kinds of step:

1. prefill: the prompt goes through the AR view and the first token is sampled
   exactly from it;
2. a speculative round: the branch drafts ``[anchor, MASK x (K - 1)]`` through the
   draft view (read-only AR history, bidirectional block), the sampler proposes
   K - 1 candidates, the AR view verifies ``[anchor, candidates]`` causally, the
   exact correction commits the accepted prefix plus one corrected token, the KV
   history is cut back to the committed prefix, and feedback hooks (the online
   learner) may observe the round;
3. a tail step: with one token of budget left the AR view samples it directly.

Branches: :class:`MaskedAttentionBranch` (the PyTorch dual-view module) and
``KernelBranch`` (the same weights on the sm_100a engine, ``kernel_branch.py``).
The counters of :class:`Generation` are the reference's report fields
(online-speculation/src/blockspec/parallel/generation.py).
"""

from __future__ import annotations

import time
from dataclasses import asdict, dataclass, field

import torch
from torch import Tensor

from .model import DualViewDecoder, cache_length, trim_cache
from .sampling import (SamplingConfig, draw, greedy_tokens, probabilities, sample_logits, verify_greedy,
                       verify_linear)


@dataclass
class Generation:
    tokens: list[int] = field(default_factory=list)
    seconds: float = 0.0
    prefill_forwards: int = 0
    prefill_output_tokens: int = 0
    draft_forwards: int = 0
    verifier_forwards: int = 0
    tail_ar_forwards: int = 0
    accepted_per_round: list[int] = field(default_factory=list)
    proposed_per_round: list[int] = field(default_factory=list)
    rounds: int = 0
    fully_covered_rounds: int = 0
    updates: int = 0
    update_seconds: float = 0.0
    feedback_blocks: int = 0
    # generate_ar(prefix_tokens=k): time at which the first min(k, delivered) tokens were
    # out, and the synchronisation time spent taking that measurement
    prefix_tokens: int = 0
    prefix_seconds: float = 0.0
    prefix_capture_seconds: float = 0.0

    @property
    def tps(self) -> float:
        return len(self.tokens) / self.seconds if self.seconds else 0.0

    @property
    def decode_forwards(self) -> int:
        return self.draft_forwards + self.verifier_forwards + self.tail_ar_forwards

    def summary(self) -> dict:
        v = asdict(self)
        v["tokens"] = len(self.tokens)
        v["tps"] = self.tps
        v["decode_forwards"] = self.decode_forwards
        v["decode_tpf"] = ((len(self.tokens) - self.prefill_output_tokens) / self.decode_forwards
                           if self.decode_forwards else None)
        return v


@dataclass
class DraftBatch:
    verifier_inputs: Tensor
    candidates: Tensor
    proposal: Tensor | None
    cache: object
    guaranteed: list
    draft_inputs: Tensor | None = None
    boundary: object = None
    collect_feedback: bool = False


class ProposalSampler:
    """Draft proposals and the exact correction under one probability policy."""

    def __init__(self, config: SamplingConfig = SamplingConfig()):
        self.config = config

    def sample_ar(self, logits: Tensor, generator) -> int:
        return int(sample_logits(logits, self.config, generator))

    def propose(self, logits: Tensor, generator):
        if self.config.temperature == 0:
            return greedy_tokens(logits), None
        q = probabilities(logits, self.config)
        return draw(q, generator), q

    def verify(self, proposal: DraftBatch, target_logits: Tensor, generator):
        if self.config.temperature == 0:
            return verify_greedy(proposal.candidates, greedy_tokens(target_logits)), None
        p = probabilities(target_logits, self.config)
        return verify_linear(proposal.candidates, proposal.proposal, p, generator=generator), p


class MaskedAttentionBranch:
    """Draft with the PyTorch dual-view module (anchor reprocessed with a masked block)."""

    initial_ar_token = True
    input_budget_extra = 1

    def __init__(self, model: DualViewDecoder):
        self.model = model
        self.default_block_size = model.config.block_size

    def ar(self, tokens: Tensor, cache=None, logits_to_keep: int = 0):
        out = self.model(tokens, cache=cache, logits_to_keep=logits_to_keep)
        return out.logits, out.cache

    def draft(self, anchor: Tensor, cache, block_size: int, sampler: ProposalSampler, generator=None, feedback=None):
        inputs = anchor.new_full((1, block_size), self.model.config.mask_token_id)
        inputs[:, :1] = anchor
        capture = None if feedback is None else feedback.capture_layer
        out = self.model(inputs, view="draft", cache=cache, capture_layer=capture)
        cand, q = sampler.propose(out.logits[0, :-1], generator)
        return DraftBatch(torch.cat((anchor, cand[None]), 1), cand, q, cache, [], inputs, out.boundary,
                          feedback is not None and capture is not None)


def _sync(device) -> None:
    if device.type == "cuda":
        torch.cuda.synchronize(device)


def _check_prompt(prompt: Tensor) -> None:
    if prompt.ndim != 2 or prompt.shape[0] != 1 or prompt.shape[1] == 0:
        raise ValueError("decoding takes one non-empty prompt of shape [1, T]")


class _Decoder:
    """State of one batch-one decode."""

    def __init__(self, branch, prompt: Tensor, budget: int, sampler: ProposalSampler, eos_id, generator, feedback):
        self.branch = branch
        self.prompt = prompt
        self.budget = budget
        self.sampler = sampler
        self.eos = eos_id
        self.generator = generator
        self.feedback = feedback
        self.result = Generation()
        self.cache = None
        self.stopped = False

    # ---- cache helpers (branches may bring their own cache type)
    def _cache_length(self, cache) -> int:
        measure = getattr(self.branch, "cache_length", None)
        return measure(cache) if measure is not None else cache_length(cache)

    def _trim(self, cache, n: int):
        cut = getattr(self.branch, "trim", None)
        return cut(cache, n) if cut is not None else trim_cache(cache, n)

    def emit(self, tokens) -> list[int]:
        """Append tokens until the budget or EOS; returns the tokens actually kept."""
        kept = []
        for t in tokens:
            if len(self.result.tokens) >= self.budget:
                break
            self.result.tokens.append(int(t))
            kept.append(int(t))
            if int(t) == self.eos:
                self.stopped = True
                break
        if len(self.result.tokens) >= self.budget:
            self.stopped = True
        if self.feedback is not None and kept:
            self.feedback.commit(kept)
        return kept

    @property
    def anchor(self) -> Tensor:
        return self.prompt.new_tensor([[self.result.tokens[-1]]])

    def prefill(self) -> None:
        logits, self.cache = self.branch.ar(self.prompt, logits_to_keep=1)
        self.result.prefill_forwards = self.result.prefill_output_tokens = 1
        self.emit([self.sampler.sample_ar(logits[0, -1], self.generator)])

    def tail_step(self) -> None:
        logits, self.cache = self.branch.ar(self.anchor, cache=self.cache, logits_to_keep=1)
        self.result.tail_ar_forwards += 1
        self.emit([self.sampler.sample_ar(logits[0, -1], self.generator)])

    def speculative_round(self, block: int) -> None:
        r = self.result
        r.rounds += 1
        expected = self.prompt.shape[1] + len(r.tokens) - 1
        if self._cache_length(self.cache) != expected:
            raise RuntimeError("the KV history must end right before the committed anchor")
        remaining = self.budget - len(r.tokens)
        if remaining == 1:
            self.tail_step()
            return
        length = min(block, remaining + self.branch.input_budget_extra)
        proposal = self.branch.draft(self.anchor, self.cache, length, self.sampler, self.generator, self.feedback)
        r.draft_forwards += 1
        logits, verified_cache = self.branch.ar(proposal.verifier_inputs, cache=proposal.cache)
        r.verifier_forwards += 1
        verdict, target = self.sampler.verify(proposal, logits[0], self.generator)
        feedback, self.feedback = self.feedback, None          # commit the round's tokens only once, below
        submitted = self.emit(list(proposal.guaranteed) + list(verdict.tokens))
        self.feedback = feedback
        n = proposal.candidates.numel()
        kept = min(verdict.accepted, len(submitted))
        r.accepted_per_round.append(kept)
        r.proposed_per_round.append(n)
        r.fully_covered_rounds += kept == n
        self.cache = self._trim(verified_cache, self.prompt.shape[1] + len(r.tokens) - 1)
        if feedback is not None:
            feedback.commit(submitted)
            feedback.observe(proposal, logits[0], target, used=min(verdict.supervised, len(submitted)),
                             fully_covered=kept == n, done=self.stopped)


@torch.no_grad()
def generate_ar(branch, prompt: Tensor, max_new_tokens: int, *, sampling=SamplingConfig(), eos_id=None,
                generator=None, sampler=None, prefix_tokens: int | None = None) -> Generation:
    """Plain autoregressive decoding with the AR view (the speed-up denominator).

    ``prefix_tokens``: also record when the first ``prefix_tokens`` outputs were out
    (``prefix_seconds``; the end of the answer when it is shorter), the reference time
    of a live AR-prefix trial; the device synchronisation that measurement needs is
    reported as ``prefix_capture_seconds``.
    """
    if prefix_tokens is not None and (type(prefix_tokens) is not int or prefix_tokens < 1):
        raise ValueError("prefix_tokens has to be a positive integer")
    _check_prompt(prompt)
    if max_new_tokens == 0:
        return Generation()
    d = _Decoder(branch, prompt, max_new_tokens, sampler or ProposalSampler(sampling), eos_id, generator, None)
    _sync(prompt.device)
    started = time.perf_counter()

    def note_prefix() -> None:
        r = d.result
        if prefix_tokens is None or r.prefix_tokens or not (len(r.tokens) >= prefix_tokens or d.stopped):
            return
        before = time.perf_counter()
        _sync(prompt.device)
        after = time.perf_counter()
        r.prefix_tokens = len(r.tokens)
        r.prefix_seconds = after - started
        r.prefix_capture_seconds = after - before

    d.prefill()
    note_prefix()
    while not d.stopped:
        d.tail_step()
        note_prefix()
    _sync(prompt.device)
    d.result.seconds = time.perf_counter() - started
    d.result.rounds = len(d.result.tokens)
    return d.result


@torch.no_grad()
def generate(branch, prompt: Tensor, max_new_tokens: int, *, block_size=None, sampling=SamplingConfig(),
             eos_id=None, generator=None, sampler=None, feedback=None) -> Generation:
    _check_prompt(prompt)
    block = branch.default_block_size if block_size is None else block_size
    if block < 2:
        raise ValueError("block drafting needs block_size >= 2")
    if feedback is not None:
        feedback.begin(prompt)
    if max_new_tokens == 0:
        empty = Generation()
        if feedback is not None:
            feedback.finish(empty)
        return empty
    d = _Decoder(branch, prompt, max_new_tokens, sampler or ProposalSampler(sampling), eos_id, generator, feedback)
    _sync(prompt.device)
    started = time.perf_counter()
    d.prefill()
    while not d.stopped:
        d.speculative_round(block)
    if feedback is not None:
        feedback.finish(d.result)
    _sync(prompt.device)
    d.result.seconds = time.perf_counter() - started
    return d.result
