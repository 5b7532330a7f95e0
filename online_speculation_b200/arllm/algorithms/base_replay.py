"""Base-candidate conditional IS whose rollout weights reuse stored completions.

Per step: draw base candidates; for each non-terminal candidate freeze a claim
on up to ``max_history_per_candidate`` stored evaluation records (before
revealing them), draw ``fresh_rollouts`` fresh base rollouts, then estimate the
candidate's weight from truncated-IS history terms min(c, p / b) exp(r / tau)
(b = the mixture of the behaviour policies that produced the claimed records,
re-scored exactly) plus the fresh tail (1 - c b / p)+ exp(r / tau)
(shared.importance).  Consumed history and the fresh draws join the design
pool; optional reserve rollouts write new evaluation records for later steps.

Reference behaviour: src/inference_scaling/arllm/algorithms/base_replay.py:157-532.
"""

from __future__ import annotations

from collections.abc import Sequence
from dataclasses import dataclass
from math import isfinite

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
    if not completions:
        return ()
    got = backend.score_batch([ScoreRequest(key.rollout_prefix, tuple(completions), sampling)])
    if len(got) != len(completions):
        raise RuntimeError("base backend returned an invalid number of scores")
    out = []
    for c, s in zip(completions, got):
        if len(c) != len(s):
            raise RuntimeError("base backend returned an invalid token score shape")
        t = float(sum(s))
        if not isfinite(t):
            raise ValueError("replay behavior generated a completion outside base support")
        out.append(t)
    return tuple(out)


def build_fresh_replay_requests(*, key: ReplayKey, count: int, rollout_length: int, seeds: SeedStream,
                                step_index: int, candidate_index: int) -> tuple[ReplaySampleRequest, ...]:
    return tuple(ReplaySampleRequest(
        key, rollout_length, seeds.derive("base_replay", step_index, "candidate", candidate_index, "fresh", f),
        f"fresh:{step_index}:{candidate_index}:{f}:{seeds.derive('fresh-id', step_index, candidate_index, f)}")
        for f in range(count))


def estimate_replay_weight(*, base_backend, base_policy: BehaviorPolicy, registry: BehaviorRegistry,
                           store: InMemoryReplayStore, claim: FrozenReplayClaim, fresh_count: int,
                           rollout_length: int, reward, reward_temperature: float, truncation: float,
                           seeds: SeedStream, step_index: int, candidate_index: int,
                           precomputed_fresh_records: Sequence[ReplayRecord] | None = None) -> ReplayWeightEstimate:
    if precomputed_fresh_records is None:
        fresh = sample_replay_records(base_policy, build_fresh_replay_requests(
            key=claim.key, count=fresh_count, rollout_length=rollout_length, seeds=seeds, step_index=step_index,
            candidate_index=candidate_index), reward)
    else:
        fresh = tuple(precomputed_fresh_records)
        if len(fresh) != fresh_count:
            raise ValueError("precomputed fresh record count does not match the frozen design")
        if any(r.key != claim.key or r.behavior_id != base_policy.behavior_id for r in fresh):
            raise ValueError("precomputed fresh records do not match the candidate and base policy")
    if claim.count == 0:
        if store.reveal_and_consume(claim):
            raise RuntimeError("an empty replay claim unexpectedly contained records")
        for r in fresh:
            store.add_design(r)
        terms = tuple(r.reward / reward_temperature for r in fresh)
        return ReplayWeightEstimate(logmeanexp(terms), (), terms, (), ())
    hist = store.reveal_and_consume(claim)
    observe = getattr(base_backend, "observe_draft_sequences", None)
    if callable(observe):
        observe(claim.key.rollout_prefix + r.completion for r in hist)
    validate_record_probabilities(hist, registry)
    counts = dict(claim.behavior_counts)
    hc, fc = [r.completion for r in hist], [r.completion for r in fresh]
    h_obs = tuple(ProbabilityObservation(p, b, r.reward) for r, p, b in zip(
        hist, _score_base(base_backend, claim.key, hc, base_policy.sampling),
        mixture_logprobabilities(registry, claim.key, counts, hc)))
    f_obs = tuple(ProbabilityObservation(r.behavior_logprob, b, r.reward) for r, b in zip(
        fresh, mixture_logprobabilities(registry, claim.key, counts, fc)))
    est = TruncatedReplayRolloutWeightProvider(truncation=truncation, reward_temperature=reward_temperature
                                               ).estimate(h_obs, f_obs)
    for r in fresh:
        store.add_design(r)
    return ReplayWeightEstimate(est.log_weight, est.history_log_terms, est.fresh_log_terms,
                                tuple(r.record_id for r in hist), claim.behavior_counts)


def base_replay_step(*, base_backend: AutoregressiveBackend, registry: BehaviorRegistry, store: InMemoryReplayStore,
                     prompt: TokenSequence, generated_prefix: TokenSequence, config: BaseReplayConfig,
                     base_sampling: SamplingConfig, reward, reward_version: str, seeds: SeedStream, step_index: int,
                     candidate_samples: Sequence[SequenceSample] | None = None) -> BaseReplayStep:
    """One guidance step with a frozen replay design (``candidate_samples`` may reuse frozen candidate draws)."""
    _full_support(base_sampling, "base replay sampling")
    remaining = config.total_length - len(generated_prefix)
    if remaining <= 0:
        raise ValueError("generated prefix has already reached total_length")
    block = min(config.block_size, remaining)
    cpre = prompt + generated_prefix
    if candidate_samples is None:
        cands = sample_candidates(base_backend, cpre, config.candidate_count, block, base_sampling, seeds, step_index)
    else:
        cands = list(candidate_samples)
        if len(cands) != config.candidate_count:
            raise ValueError("frozen candidate count does not match the replay design")
        for i, c in enumerate(cands):
            if (c.prefix != cpre or c.model_id != base_backend.model_id or c.policy_id != base_sampling.policy_id
                    or c.request_id != f"conditional-is:step:{step_index}:candidate:{i}" or not c.token_ids
                    or len(c.token_ids) > block):
                raise ValueError("a frozen candidate does not match its base-model generation request")
    base = BehaviorPolicy.for_backend(base_backend, base_sampling, label="base")
    registry.register(base)
    rollout_len = max(0, remaining - block)
    eos = base_sampling.eos_token_id
    keys = [ReplayKey(prompt, generated_prefix, c.token_ids, reward_version) for c in cands]
    claims = [None if rollout_len == 0 or (eos is not None and c.token_ids[-1] == eos)
              else store.freeze_claims([k], config.max_history_per_candidate)[0] for k, c in zip(keys, cands)]
    reqs, spans = [], []
    for i, (k, cl) in enumerate(zip(keys, claims)):
        if cl is None:
            spans.append(None)
            continue
        s = len(reqs)
        reqs += build_fresh_replay_requests(key=k, count=config.fresh_rollouts, rollout_length=rollout_len,
                                            seeds=seeds, step_index=step_index, candidate_index=i)
        spans.append((s, len(reqs)))
    fresh = sample_replay_records(base, reqs, reward)
    out = []
    for i, (c, cl, sp) in enumerate(zip(cands, claims, spans)):
        if cl is None:
            t = float(reward(prompt, generated_prefix + c.token_ids)) / config.reward_temperature
            est = ReplayWeightEstimate(t, (), (t,), (), ())
        else:
            est = estimate_replay_weight(base_backend=base_backend, base_policy=base, registry=registry, store=store,
                                         claim=cl, fresh_count=config.fresh_rollouts, rollout_length=rollout_len,
                                         reward=reward, reward_temperature=config.reward_temperature,
                                         truncation=config.truncation, seeds=seeds, step_index=step_index,
                                         candidate_index=i, precomputed_fresh_records=fresh[sp[0]:sp[1]])
        out.append(BaseReplayCandidate(c.token_ids, c.token_logprobs, est))
    probs = normalize_log_weights([c.estimate.log_weight for c in out])
    sel = int(seeds.generator("base_replay", step_index, "select").choice(len(out), p=probs))
    return BaseReplayStep(len(generated_prefix), tuple(out), sel)


def write_reserve_records(*, base_backend, base_sampling: SamplingConfig, reserve_policy: BehaviorPolicy,
                          store: InMemoryReplayStore, prompt: TokenSequence, generated_prefix: TokenSequence,
                          config: BaseReplayConfig, reward, reward_version: str, seeds: SeedStream,
                          step_index: int) -> int:
    """Generate evaluation records for future steps from ``reserve_policy`` (independent of this step's draws)."""
    remaining = config.total_length - len(generated_prefix)
    if remaining <= 0 or config.reserve_rollouts == 0:
        return 0
    block = min(config.block_size, remaining)
    cands = sample_candidates(base_backend, prompt + generated_prefix, config.reserve_rollouts, block, base_sampling,
                              seeds, step_index + 1_000_000)
    eos = base_sampling.eos_token_id
    reqs = []
    for i, c in enumerate(cands):
        rl = remaining - len(c.token_ids)
        if rl <= 0 or (eos is not None and c.token_ids[-1] == eos):
            continue
        reqs.append(ReplaySampleRequest(ReplayKey(prompt, generated_prefix, c.token_ids, reward_version), rl,
                                        seeds.derive("base_replay", step_index, "reserve", i),
                                        f"reserve:{step_index}:{i}:{seeds.derive('reserve-id', step_index, i)}"))
    recs = sample_replay_records(reserve_policy, reqs, reward)
    for r in recs:
        store.add_evaluation(r)
    return len(recs)


def run_base_replay(base_backend: AutoregressiveBackend, registry: BehaviorRegistry, store: InMemoryReplayStore,
                    prompt: TokenSequence, config: BaseReplayConfig, base_sampling: SamplingConfig, reward,
                    seeds: SeedStream, *, reward_version: str = "reward",
                    reserve_policy: BehaviorPolicy | None = None) -> BaseReplayResult:
    generated: TokenSequence = ()
    steps, written, i = [], 0, 0
    if reserve_policy is not None:
        registry.register(reserve_policy)
    eos = base_sampling.eos_token_id
    while len(generated) < config.total_length:
        if reserve_policy is not None:
            written += write_reserve_records(base_backend=base_backend, base_sampling=base_sampling,
                                             reserve_policy=reserve_policy, store=store, prompt=prompt,
                                             generated_prefix=generated, config=config, reward=reward,
                                             reward_version=reward_version, seeds=seeds, step_index=i)
        st = base_replay_step(base_backend=base_backend, registry=registry, store=store, prompt=prompt,
                              generated_prefix=generated, config=config, base_sampling=base_sampling, reward=reward,
                              reward_version=reward_version, seeds=seeds, step_index=i)
        steps.append(st)
        generated += st.selected.token_ids
        i += 1
        if eos is not None and generated and generated[-1] == eos:
            break
    return BaseReplayResult(prompt, generated, tuple(steps), written)


__all__ = ["BaseReplayCandidate", "BaseReplayResult", "BaseReplayStep", "ReplayWeightEstimate", "base_replay_step",
           "build_fresh_replay_requests", "estimate_replay_weight", "run_base_replay", "write_reserve_records"]
