"""Base-candidate conditional IS whose rollout weights reuse stored completions.

Per step: draw base candidates; for each candidate that still needs rollouts,
freeze a claim on up to ``max_history_per_candidate`` stored evaluation records
(before anything but their behaviour ids is revealed) and draw ``fresh_rollouts``
fresh base rollouts.  The candidate's weight combines truncated-IS history terms
min(c, p / b) exp(r / tau), with b the mixture of the behaviour policies that
produced the claimed records (re-scored exactly), and the fresh tail
(1 - c b / p)+ exp(r / tau) that keeps the estimate unbiased.  Revealed history and
fresh draws join the design pool; optional reserve rollouts write evaluation records
for later steps.  The work of one run lives in a :class:`_ReplayRun`; random-stream
names and record / request ids follow
src/inference_scaling/arllm/algorithms/base_replay.py so frozen designs replay.
"""

from __future__ import annotations

from collections.abc import Sequence
from dataclasses import dataclass

import numpy as np

from ...shared.importance import (ProbabilityObservation, ReplayWeightEstimate as _SharedEstimate,
                                  TruncatedReplayRolloutWeightProvider, logmeanexp)
from ...shared.rng import SeedStream
from ...shared.stepwise import normalize_log_weights
from ...shared.types import TokenSequence
from ..config import BaseReplayConfig, SamplingConfig
from ..replay import (BehaviorPolicy, BehaviorRegistry, FrozenReplayClaim, InMemoryReplayStore, ReplayKey,
                      ReplayRecord, ReplaySampleRequest, mixture_logprobabilities, sample_replay_records,
                      validate_record_probabilities)
from ..types import AutoregressiveBackend, ScoreRequest, SequenceSample
from .conditional_is import _full_support, sample_candidates


@dataclass(frozen=True, slots=True)
class ReplayWeightEstimate(_SharedEstimate):
    history_record_ids: tuple[str, ...] = ()
    behavior_counts: tuple[tuple[str, int], ...] = ()


@dataclass(frozen=True, slots=True)
class BaseReplayCandidate:
    token_ids: TokenSequence
    base_token_logprobs: tuple[float, ...]
    estimate: ReplayWeightEstimate


@dataclass(frozen=True, slots=True)
class BaseReplayStep:
    generated_length_before: int
    candidates: tuple[BaseReplayCandidate, ...]
    selected_index: int

    @property
    def selected(self) -> BaseReplayCandidate:
        return self.candidates[self.selected_index]


@dataclass(frozen=True, slots=True)
class BaseReplayResult:
    prompt: TokenSequence
    token_ids: TokenSequence
    steps: tuple[BaseReplayStep, ...]
    reserve_records_written: int


def _score_base(backend, key: ReplayKey, completions, sampling) -> tuple[float, ...]:
    """Base-policy log-probabilities of completions; they must lie in the base support."""
    if not completions:
        return ()
    scores = backend.score_batch([ScoreRequest(key.rollout_prefix, tuple(completions), sampling)])
    if len(scores) != len(completions) or any(len(s) != len(c) for s, c in zip(scores, completions)):
        raise RuntimeError("the base backend's scores do not match the completions")
    totals = np.asarray([float(np.sum(s)) for s in scores])
    if not np.isfinite(totals).all():
        raise ValueError("a replayed completion has zero probability under the base policy")
    return tuple(totals.tolist())


def build_fresh_replay_requests(*, key: ReplayKey, count: int, rollout_length: int, seeds: SeedStream,
                                step_index: int, candidate_index: int) -> tuple[ReplaySampleRequest, ...]:
    def one(f: int) -> ReplaySampleRequest:
        seed = seeds.derive("base_replay", step_index, "candidate", candidate_index, "fresh", f)
        tag = seeds.derive("fresh-id", step_index, candidate_index, f)
        return ReplaySampleRequest(key, rollout_length, seed, f"fresh:{step_index}:{candidate_index}:{f}:{tag}")

    return tuple(one(f) for f in range(count))


def _checked_fresh(claim: FrozenReplayClaim, base_policy: BehaviorPolicy, fresh: Sequence[ReplayRecord],
                   count: int) -> tuple[ReplayRecord, ...]:
    fresh = tuple(fresh)
    if len(fresh) != count:
        raise ValueError(f"{len(fresh)} fresh records were given for a design of {count}")
    if any(r.key != claim.key or r.behavior_id != base_policy.behavior_id for r in fresh):
        raise ValueError("the given fresh records belong to another candidate or behaviour policy")
    return fresh


def estimate_replay_weight(*, base_backend, base_policy: BehaviorPolicy, registry: BehaviorRegistry,
                           store: InMemoryReplayStore, claim: FrozenReplayClaim, fresh_count: int,
                           rollout_length: int, reward, reward_temperature: float, truncation: float,
                           seeds: SeedStream, step_index: int, candidate_index: int,
                           precomputed_fresh_records: Sequence[ReplayRecord] | None = None) -> ReplayWeightEstimate:
    if precomputed_fresh_records is None:
        requests = build_fresh_replay_requests(key=claim.key, count=fresh_count, rollout_length=rollout_length,
                                               seeds=seeds, step_index=step_index, candidate_index=candidate_index)
        fresh = sample_replay_records(base_policy, requests, reward)
    else:
        fresh = _checked_fresh(claim, base_policy, precomputed_fresh_records, fresh_count)
    history = store.reveal_and_consume(claim)
    if claim.count == 0:
        if history:
            raise RuntimeError("an empty claim revealed records")
        for r in fresh:
            store.add_design(r)
        terms = tuple(r.reward / reward_temperature for r in fresh)
        return ReplayWeightEstimate(logmeanexp(terms), (), terms, (), ())
    observe = getattr(base_backend, "observe_draft_sequences", None)
    if callable(observe):
        observe(claim.key.rollout_prefix + tuple(r.completion) for r in history)
    validate_record_probabilities(history, registry)
    counts = dict(claim.behavior_counts)
    h_completions = [r.completion for r in history]
    f_completions = [r.completion for r in fresh]
    base_h = _score_base(base_backend, claim.key, h_completions, base_policy.sampling)
    mix_h = mixture_logprobabilities(registry, claim.key, counts, h_completions)
    mix_f = mixture_logprobabilities(registry, claim.key, counts, f_completions)
    observed_history = [ProbabilityObservation(p, b, r.reward) for r, p, b in zip(history, base_h, mix_h)]
    observed_fresh = [ProbabilityObservation(r.behavior_logprob, b, r.reward) for r, b in zip(fresh, mix_f)]
    provider = TruncatedReplayRolloutWeightProvider(truncation=truncation, reward_temperature=reward_temperature)
    estimate = provider.estimate(observed_history, observed_fresh)
    for r in fresh:
        store.add_design(r)
    return ReplayWeightEstimate(estimate.log_weight, estimate.history_log_terms, estimate.fresh_log_terms,
                                tuple(r.record_id for r in history), claim.behavior_counts)


def _frozen_candidates_ok(cands, prefix, backend, sampling, step_index, count, block) -> None:
    if len(cands) != count:
        raise ValueError(f"{len(cands)} frozen candidates for a design of {count}")
    for i, c in enumerate(cands):
        if (c.prefix != prefix or c.model_id != backend.model_id or c.policy_id != sampling.policy_id
                or c.request_id != f"conditional-is:step:{step_index}:candidate:{i}" or not c.token_ids
                or len(c.token_ids) > block):
            raise ValueError(f"frozen candidate {i} does not answer its base-model generation request")


class _ReplayRun:
    """The fixed parts of one base-replay run (backend, stores, design, reward)."""

    def __init__(self, base_backend, registry, store, prompt, config: BaseReplayConfig, base_sampling, reward,
                 reward_version, seeds):
        self.backend = base_backend
        self.registry = registry
        self.store = store
        self.prompt = tuple(prompt)
        self.config = config
        self.sampling = base_sampling
        self.reward = reward
        self.reward_version = reward_version
        self.seeds = seeds
        self.eos = base_sampling.eos_token_id

    def _ends(self, tokens) -> bool:
        return self.eos is not None and bool(tokens) and tokens[-1] == self.eos

    def step(self, generated, step_index, candidate_samples=None) -> BaseReplayStep:
        cfg = self.config
        remaining = cfg.total_length - len(generated)
        if remaining <= 0:
            raise ValueError("the generated prefix already has total_length tokens")
        block = min(cfg.block_size, remaining)
        prefix = self.prompt + tuple(generated)
        if candidate_samples is None:
            cands = sample_candidates(self.backend, prefix, cfg.candidate_count, block, self.sampling, self.seeds,
                                      step_index)
        else:
            cands = list(candidate_samples)
            _frozen_candidates_ok(cands, prefix, self.backend, self.sampling, step_index, cfg.candidate_count, block)
        base = BehaviorPolicy.for_backend(self.backend, self.sampling, label="base")
        self.registry.register(base)
        rollout = max(0, remaining - block)
        keys = [ReplayKey(self.prompt, tuple(generated), c.token_ids, self.reward_version) for c in cands]
        needs = [rollout > 0 and not self._ends(c.token_ids) for c in cands]
        claims = [self.store.freeze_claims([k], cfg.max_history_per_candidate)[0] if need else None
                  for k, need in zip(keys, needs)]
        requests: list[ReplaySampleRequest] = []
        slices: list[slice | None] = []
        for i, (key, claim) in enumerate(zip(keys, claims)):
            if claim is None:
                slices.append(None)
                continue
            start = len(requests)
            requests.extend(build_fresh_replay_requests(key=key, count=cfg.fresh_rollouts, rollout_length=rollout,
                                                        seeds=self.seeds, step_index=step_index, candidate_index=i))
            slices.append(slice(start, len(requests)))
        fresh = sample_replay_records(base, requests, self.reward)
        scored = []
        for i, (cand, claim, part) in enumerate(zip(cands, claims, slices)):
            if claim is None:
                direct = float(self.reward(self.prompt, tuple(generated) + tuple(cand.token_ids))) / \
                    cfg.reward_temperature
                estimate = ReplayWeightEstimate(direct, (), (direct,), (), ())
            else:
                estimate = estimate_replay_weight(
                    base_backend=self.backend, base_policy=base, registry=self.registry, store=self.store,
                    claim=claim, fresh_count=cfg.fresh_rollouts, rollout_length=rollout, reward=self.reward,
                    reward_temperature=cfg.reward_temperature, truncation=cfg.truncation, seeds=self.seeds,
                    step_index=step_index, candidate_index=i, precomputed_fresh_records=fresh[part])
            scored.append(BaseReplayCandidate(cand.token_ids, cand.token_logprobs, estimate))
        probabilities = normalize_log_weights([c.estimate.log_weight for c in scored])
        chosen = int(self.seeds.generator("base_replay", step_index, "select").choice(len(scored), p=probabilities))
        return BaseReplayStep(len(generated), tuple(scored), chosen)

    def reserve(self, reserve_policy: BehaviorPolicy, generated, step_index) -> int:
        cfg = self.config
        remaining = cfg.total_length - len(generated)
        if remaining <= 0 or cfg.reserve_rollouts == 0:
            return 0
        block = min(cfg.block_size, remaining)
        cands = sample_candidates(self.backend, self.prompt + tuple(generated), cfg.reserve_rollouts, block,
                                  self.sampling, self.seeds, step_index + 1_000_000)
        requests = []
        for i, c in enumerate(cands):
            length = remaining - len(c.token_ids)
            if length <= 0 or self._ends(c.token_ids):
                continue
            key = ReplayKey(self.prompt, tuple(generated), c.token_ids, self.reward_version)
            requests.append(ReplaySampleRequest(key, length, self.seeds.derive("base_replay", step_index, "reserve", i),
                                                f"reserve:{step_index}:{i}:"
                                                f"{self.seeds.derive('reserve-id', step_index, i)}"))
        records = sample_replay_records(reserve_policy, requests, self.reward)
        for r in records:
            self.store.add_evaluation(r)
        return len(records)


def base_replay_step(*, base_backend: AutoregressiveBackend, registry: BehaviorRegistry, store: InMemoryReplayStore,
                     prompt: TokenSequence, generated_prefix: TokenSequence, config: BaseReplayConfig,
                     base_sampling: SamplingConfig, reward, reward_version: str, seeds: SeedStream, step_index: int,
                     candidate_samples: Sequence[SequenceSample] | None = None) -> BaseReplayStep:
    """One guidance step with a frozen replay design (``candidate_samples`` may reuse frozen candidate draws)."""
    _full_support(base_sampling, "base replay sampling")
    run = _ReplayRun(base_backend, registry, store, prompt, config, base_sampling, reward, reward_version, seeds)
    return run.step(generated_prefix, step_index, candidate_samples)


def write_reserve_records(*, base_backend, base_sampling: SamplingConfig, reserve_policy: BehaviorPolicy,
                          store: InMemoryReplayStore, prompt: TokenSequence, generated_prefix: TokenSequence,
                          config: BaseReplayConfig, reward, reward_version: str, seeds: SeedStream,
                          step_index: int) -> int:
    """Evaluation records for future steps, drawn by ``reserve_policy`` (independent of this step's draws)."""
    run = _ReplayRun(base_backend, None, store, prompt, config, base_sampling, reward, reward_version, seeds)
    return run.reserve(reserve_policy, generated_prefix, step_index)


def run_base_replay(base_backend: AutoregressiveBackend, registry: BehaviorRegistry, store: InMemoryReplayStore,
                    prompt: TokenSequence, config: BaseReplayConfig, base_sampling: SamplingConfig, reward,
                    seeds: SeedStream, *, reward_version: str = "reward",
                    reserve_policy: BehaviorPolicy | None = None) -> BaseReplayResult:
    _full_support(base_sampling, "base replay sampling")
    run = _ReplayRun(base_backend, registry, store, prompt, config, base_sampling, reward, reward_version, seeds)
    if reserve_policy is not None:
        registry.register(reserve_policy)
    generated: tuple = ()
    steps: list[BaseReplayStep] = []
    written = 0
    while len(generated) < config.total_length and not (steps and run._ends(generated)):
        if reserve_policy is not None:
            written += run.reserve(reserve_policy, generated, len(steps))
        step = run.step(generated, len(steps))
        steps.append(step)
        generated += tuple(step.selected.token_ids)
    return BaseReplayResult(tuple(prompt), generated, tuple(steps), written)


__all__ = ["BaseReplayCandidate", "BaseReplayResult", "BaseReplayStep", "ReplayWeightEstimate", "base_replay_step",
           "build_fresh_replay_requests", "estimate_replay_weight", "run_base_replay", "write_reserve_records"]
