"""Batch-one block-speculative decoding with a pending committed anchor.

Loop (online-speculation/src/blockspec/parallel/generation.py:74-212):

1. prefill the prompt and sample the first token exactly from the AR view;
2. each round: the branch drafts ``[anchor, MASK x (K-1)]`` through the draft
   view (read-only AR history, bidirectional block), the sampler proposes K-1
   candidates, the AR view verifies ``[anchor, candidates]`` causally, the
   exact correction commits the accepted prefix plus one corrected token, the
   KV history is trimmed to the committed prefix, and feedback hooks may
   observe the round (online learner);
3. with one token left the AR view samples it directly.

Branches: :class:`MaskedAttentionBranch` (the PyTorch dual-view module) and
``KernelBranch`` (the same weights on the sm_100a engine, in
``kernel_branch.py``).  Samplers: :class:`ProposalSampler` (tensor maths of
``sampling.py``).
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


def _length(branch, cache) -> int:
    return branch.cache_length(cache) if hasattr(branch, "cache_length") else cache_length(cache)


def _trim(branch, cache, n: int):
    return branch.trim(cache, n) if hasattr(branch, "trim") else trim_cache(cache, n)


def _append(result: Generation, tokens, budget: int, eos) -> bool:
    for t in tokens:
        if len(result.tokens) == budget:
            return True
        result.tokens.append(int(t))
        if t == eos:
            return True
    return len(result.tokens) == budget


def _sync(device):
    if device.type == "cuda":
        torch.cuda.synchronize(device)


@torch.no_grad()
def generate_ar(branch, prompt: Tensor, max_new_tokens: int, *, sampling=SamplingConfig(), eos_id=None,
                generator=None, sampler=None, prefix_tokens: int | None = None) -> Generation:
    """Plain autoregressive decoding with the AR view (the speed-up denominator).

    ``prefix_tokens``: also record when the first ``prefix_tokens`` outputs were
    delivered (``prefix_seconds``; the answer's end when it is shorter) -- the
    reference time of a live AR-prefix trial.  The device synchronisation that
    measurement needs is reported as ``prefix_capture_seconds``.
    """
    if prefix_tokens is not None and (type(prefix_tokens) is not int or prefix_tokens < 1):
        raise ValueError("a positive prefix length is required")
    if prompt.ndim != 2 or prompt.shape[0] != 1 or prompt.shape[1] < 1:
        raise ValueError("nonempty batch-one prompt required")
    result = Generation()
    if max_new_tokens == 0:
        return result
    sampler = sampler or ProposalSampler(sampling)
    _sync(prompt.device)
    start = time.perf_counter()
    logits, cache = branch.ar(prompt, logits_to_keep=1)
    token = sampler.sample_ar(logits[0, -1], generator)
    result.prefill_forwards = result.prefill_output_tokens = 1
    stopped = _append(result, [token], max_new_tokens, eos_id)

    def capture():
        if prefix_tokens is not None and not result.prefix_tokens and (
                len(result.tokens) >= prefix_tokens or stopped):
            c0 = time.perf_counter()
            _sync(prompt.device)
            c1 = time.perf_counter()
            result.prefix_tokens = len(result.tokens)
            result.prefix_seconds = c1 - start
            result.prefix_capture_seconds = c1 - c0

    capture()
    while not stopped:
        logits, cache = branch.ar(prompt.new_tensor([[token]]), cache=cache, logits_to_keep=1)
        token = sampler.sample_ar(logits[0, -1], generator)
        result.tail_ar_forwards += 1
        stopped = _append(result, [token], max_new_tokens, eos_id)
        capture()
    _sync(prompt.device)
    result.seconds = time.perf_counter() - start
    result.rounds = len(result.tokens)
    return result


@torch.no_grad()
def generate(branch, prompt: Tensor, max_new_tokens: int, *, block_size=None, sampling=SamplingConfig(),
             eos_id=None, generator=None, sampler=None, feedback=None) -> Generation:
    if prompt.ndim != 2 or prompt.shape[0] != 1 or prompt.shape[1] < 1:
        raise ValueError("nonempty batch-one prompt required")
    block = branch.default_block_size if block_size is None else block_size
    if block < 2:
        raise ValueError("parallel drafting requires block_size >= 2")
    result = Generation()
    if feedback is not None:
        feedback.begin(prompt)
    if max_new_tokens == 0:
        if feedback is not None:
            feedback.finish(result)
        return result
    sampler = sampler or ProposalSampler(sampling)
    _sync(prompt.device)
    start = time.perf_counter()
    logits, cache = branch.ar(prompt, logits_to_keep=1)
    token = sampler.sample_ar(logits[0, -1], generator)
    result.prefill_forwards = result.prefill_output_tokens = 1
    stopped = _append(result, [token], max_new_tokens, eos_id)
    if feedback is not None:
        feedback.commit([token])
    anchor = prompt.new_tensor([[token]])
    while not stopped:
        result.rounds += 1
        if _length(branch, cache) != prompt.shape[1] + len(result.tokens) - 1:
            raise RuntimeError("history must end right before the committed anchor")
        remaining = max_new_tokens - len(result.tokens)
        if remaining == 1:
            logits, cache = branch.ar(anchor, cache=cache, logits_to_keep=1)
            token = sampler.sample_ar(logits[0, -1], generator)
            result.tail_ar_forwards += 1
            stopped = _append(result, [token], max_new_tokens, eos_id)
            if feedback is not None:
                feedback.commit([token])
            continue
        length = min(block, remaining + branch.input_budget_extra)
        proposal = branch.draft(anchor, cache, length, sampler, generator, feedback)
        result.draft_forwards += 1
        logits, verified_cache = branch.ar(proposal.verifier_inputs, cache=proposal.cache)
        result.verifier_forwards += 1
        verified, target = sampler.verify(proposal, logits[0], generator)
        begin = len(result.tokens)
        stopped = _append(result, proposal.guaranteed + verified.tokens, max_new_tokens, eos_id)
        submitted = result.tokens[begin:]
        kept = min(verified.accepted, len(submitted))
        used = min(verified.supervised, len(submitted))
        n = proposal.candidates.numel()
        result.accepted_per_round.append(kept)
        result.proposed_per_round.append(n)
        full = kept == n
        result.fully_covered_rounds += full
        cache = _trim(branch, verified_cache, prompt.shape[1] + len(result.tokens) - 1)
        anchor = prompt.new_tensor([[result.tokens[-1]]])
        if feedback is not None:
            feedback.commit(submitted)
            feedback.observe(proposal, logits[0], target, used=used, fully_covered=full, done=stopped)
    if feedback is not None:
        feedback.finish(result)
    _sync(prompt.device)
    result.seconds = time.perf_counter() - start
    return result
