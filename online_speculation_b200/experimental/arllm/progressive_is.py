"""Progressive conditional IS: a pilot phase sizes an independent evaluation phase.

Per block: K base candidates; pilot rollouts estimate, per candidate, the spread
of the normalised rollout weight and the relative cost of one rollout (tokens
times model parameters, plus base re-scoring when off-policy).  From those the
variance-cost allocator freezes how many evaluation rollouts each candidate
gets under ``evaluation_cost_budget``; only the freshly drawn evaluation
rollouts enter the candidate weight, so the pilot never counts as a second
observation of the same quantity (its trajectories remain usable as draft-cache
material by the backend).  Rewards stream from a worker pool as completions
finish, and a backend with ``submit_run_ahead`` may start low-priority
run-ahead rollouts once a phase's generation is done.

Reference behaviour: src/inference_scaling/experimental/arllm/progressive_is.py:42-538.
"""

from __future__ import annotations

from collections.abc import Sequence
from dataclasses import dataclass
from math import exp, isfinite

import numpy as np

from ...arllm.acceleration import StreamingRewardEvaluator, StreamingRewardSnapshot
from ...arllm.algorithms.conditional_is import (RolloutEvaluation, TokenBatchReward, TokenReward, _check_policies,
                                                 sample_candidates)
from ...arllm.config import ProgressiveISConfig, SamplingConfig
from ...arllm.types import AutoregressiveBackend, GenerationRequest, ScoreRequest, SequenceSample
from ...shared.budget import allocate_fresh_rollout_budget
from ...shared.importance import logmeanexp
from ...shared.rng import SeedStream
from ...shared.types import TokenSequence


@dataclass(frozen=True, slots=True)
class PilotSummary:
    rollout_count: int
    normalized_weight_std: float
    normalized_cost: float
    streaming: StreamingRewardSnapshot | None


@dataclass(frozen=True, slots=True)
class ProgressiveCandidate:
    token_ids: TokenSequence
    base_token_logprobs: tuple[float, ...]
    pilot: PilotSummary
    evaluation_rollouts: tuple[RolloutEvaluation, ...]
    evaluation_count: int
    log_weight: float


@dataclass(frozen=True, slots=True)
class ProgressiveISStep:
    generated_length_before: int
    candidates: tuple[ProgressiveCandidate, ...]
    selected_index: int
    frozen_evaluation_cost: float

    @property
    def selected(self) -> ProgressiveCandidate:
        return self.candidates[self.selected_index]


@dataclass(frozen=True, slots=True)
class ProgressiveISResult:
    prompt: TokenSequence
    token_ids: TokenSequence
    steps: tuple[ProgressiveISStep, ...]


def _parameter_count(backend) -> float:
    try:
        v = float(getattr(backend, "parameter_count", 1))
    except (TypeError, ValueError):
        return 1.0
    return v if isfinite(v) and v > 0 else 1.0


def _scalar_rewards(prompt, seqs, reward, reward_batch) -> list[float]:
    if reward_batch is not None:
        vals = [float(v) for v in reward_batch(prompt, list(seqs))]
        if len(vals) != len(seqs):
            raise ValueError("reward_batch returned an invalid number of rewards")
    else:
        if reward is None:
            raise ValueError("a reward callback is required")
        vals = [float(reward(prompt, s)) for s in seqs]
    if any(not isfinite(v) for v in vals):
        raise ValueError("reward must be finite")
    return vals


def _draw(*, base_backend, rollout_backend, prompt, generated_prefix, candidates: Sequence[SequenceSample],
          counts: Sequence[int], rollout_length, base_sampling, rollout_sampling, tau, clip, reward, reward_batch,
          seeds, step, phase, evaluator, run_ahead):
    """One phase of rollouts for every candidate; returns (per-candidate evaluations, stream snapshot)."""
    if len(counts) != len(candidates):
        raise ValueError("rollout counts must match candidates")
    eos = rollout_sampling.eos_token_id
    reqs, owner, prefixes, inputs, terminal = [], [], [], [], []
    for k, (c, n) in enumerate(zip(candidates, counts)):
        if n < 0:
            raise ValueError("rollout counts must be non-negative")
        gen = generated_prefix + c.token_ids
        if rollout_length == 0 or (eos is not None and c.token_ids[-1] == eos):
            terminal.append(k)
            continue
        for r in range(n):
            reqs.append(GenerationRequest(prompt + gen, rollout_length, rollout_sampling,
                                          seeds.derive("progressive_is", step, phase, k, r),
                                          f"progressive-is:{phase}:step:{step}:candidate:{k}:rollout:{r}"))
            owner.append(k)
            prefixes.append(prompt + gen)
            inputs.append((prompt, gen))
    snap = None
    if reqs and evaluator is not None:
        if reward is None or reward_batch is not None:
            raise ValueError("streaming rewards require the scalar reward callback")
        ahead = []
        submit = getattr(base_backend, "submit_run_ahead", None)
        if callable(submit) and run_ahead:
            for k, c in enumerate(candidates):
                if k in terminal:
                    continue
                gen = generated_prefix + c.token_ids
                ahead += [GenerationRequest(prompt + gen, rollout_length, base_sampling,
                                            seeds.derive("progressive_is", step, phase, "run_ahead", k, r),
                                            f"progressive-is:{phase}:run-ahead:step:{step}:candidate:{k}:rollout:{r}")
                          for r in range(run_ahead)]
        samples, rewards, snap = evaluator.sample_and_score(
            rollout_backend, reqs, inputs, reward,
            on_generation_complete=(lambda _s: submit(ahead)) if ahead else None)
        rewards = [float(v) for v in rewards]
        if any(not isfinite(v) for v in rewards):
            raise ValueError("reward must be finite")
    else:
        samples = rollout_backend.sample_batch(reqs) if reqs else []
        rewards = _scalar_rewards(prompt, [g + s.token_ids for (_, g), s in zip(inputs, samples)], reward,
                                  reward_batch) if reqs else []
    if len(samples) != len(reqs) or len(rewards) != len(reqs):
        raise RuntimeError("rollout backend or reward callback returned an invalid count")
    if rollout_backend is not base_backend:
        observe = getattr(base_backend, "observe_draft_samples", None)
        if callable(observe):
            observe(samples)
    on_policy = rollout_backend.model_id == base_backend.model_id and rollout_sampling == base_sampling
    if on_policy or not samples:
        base = [s.logprob for s in samples]
    else:
        base = [float(sum(v)) for v in base_backend.score_batch(
            [ScoreRequest(p, (s.token_ids,), base_sampling) for p, s in zip(prefixes, samples)])]
        if any(not isfinite(v) for v in base):
            raise ValueError("rollout proposal generated a completion outside base-model support")
    groups: list[list[RolloutEvaluation]] = [[] for _ in candidates]
    for k in terminal:
        v = _scalar_rewards(prompt, [generated_prefix + candidates[k].token_ids], reward, reward_batch)[0]
        groups[k].append(RolloutEvaluation((), v, 0.0, 0.0, 0.0, 0.0, v / tau, rollout_backend.model_id,
                                           rollout_sampling.policy_id))
    for k, s, b, v in zip(owner, samples, base, rewards):
        raw = float(b - s.logprob)
        app = raw if clip is None else max(-clip, min(clip, raw))
        groups[k].append(RolloutEvaluation(tuple(s.token_ids), v, float(b), s.logprob, raw, app, v / tau + app,
                                           s.model_id, s.policy_id))
    return tuple(tuple(g) for g in groups), snap


def _pilot_statistics(pilot, *, rollout_backend, base_backend, on_policy) -> tuple[list[float], list[float]]:
    logs = [e.log_weight for g in pilot for e in g]
    top = max(logs) if logs else 0.0
    per_param = _parameter_count(rollout_backend) + (0.0 if on_policy else _parameter_count(base_backend))
    stds, raw = [], []
    for g in pilot:
        w = np.asarray([exp(e.log_weight - top) for e in g], dtype=np.float64)
        stds.append(float(np.std(w, ddof=1)) if len(w) >= 2 else max(float(w[0]) if len(w) else 0.0, 1e-12))
        toks = max(1.0, float(np.mean([max(1, len(e.token_ids)) for e in g]))) if g else 1.0
        raw.append(toks * per_param)
    lo = min(raw) if raw else 1.0
    return stds, [max(1.0, c / lo) for c in raw]


def progressive_is_step(*, base_backend: AutoregressiveBackend, rollout_backend: AutoregressiveBackend,
                        prompt: TokenSequence, generated_prefix: TokenSequence, config: ProgressiveISConfig,
                        base_sampling: SamplingConfig, rollout_sampling: SamplingConfig,
                        reward: TokenReward | None, seeds: SeedStream, step_index: int,
                        reward_batch: TokenBatchReward | None = None,
                        streaming_evaluator: StreamingRewardEvaluator | None = None) -> ProgressiveISStep:
    _check_policies(base_sampling, rollout_sampling)
    if (reward is None) == (reward_batch is None):
        raise ValueError("provide exactly one of reward or reward_batch")
    prompt, generated_prefix = tuple(prompt), tuple(generated_prefix)
    left = config.total_length - len(generated_prefix)
    if left <= 0:
        raise ValueError("generated prefix has already reached total_length")
    block = min(config.block_size, left)
    cands = sample_candidates(base_backend, prompt + generated_prefix, config.candidate_count, block, base_sampling,
                              seeds, step_index)
    roll = max(0, left - block)
    eos = rollout_sampling.eos_token_id
    terminal = [roll == 0 or (eos is not None and c.token_ids[-1] == eos) for c in cands]
    common = dict(base_backend=base_backend, rollout_backend=rollout_backend, prompt=prompt,
                  generated_prefix=generated_prefix, candidates=cands, rollout_length=roll,
                  base_sampling=base_sampling, rollout_sampling=rollout_sampling, tau=config.reward_temperature,
                  clip=config.importance_log_ratio_clip, reward=reward, reward_batch=reward_batch, seeds=seeds,
                  step=step_index, evaluator=streaming_evaluator,
                  run_ahead=config.run_ahead_rollouts_per_candidate)
    pilot_counts = [0 if t else config.pilot_rollouts_per_candidate for t in terminal]
    pilot, snap = _draw(counts=pilot_counts, phase="pilot", **common)
    on_policy = rollout_backend.model_id == base_backend.model_id and rollout_sampling == base_sampling
    stds, costs = _pilot_statistics(pilot, rollout_backend=rollout_backend, base_backend=base_backend,
                                    on_policy=on_policy)
    active = [k for k, t in enumerate(terminal) if not t]
    counts = [0] * len(cands)
    frozen = 0.0
    if active:
        floor = sum(config.minimum_evaluation_per_candidate * costs[k] for k in active)
        budget = config.evaluation_cost_budget
        if config.evaluation_reference_rollouts_per_candidate is not None:
            # a fixed per-candidate count expressed as a cost budget from the frozen pilot costs
            mean_cost = sum(costs[k] for k in active) / len(active)
            budget = max(floor, len(active) * config.evaluation_reference_rollouts_per_candidate * mean_cost)
        if budget + 1e-12 < floor:
            raise ValueError("evaluation_cost_budget cannot cover the minimum independent evaluation rollouts")
        alloc = allocate_fresh_rollout_budget(outer_ratios=[1.0] * len(active),
                                              standard_deviations=[max(stds[k], 1e-12) for k in active],
                                              costs=[costs[k] for k in active], rollout_budget=budget,
                                              minimum_fresh=config.minimum_evaluation_per_candidate)
        for k, a in zip(active, alloc):
            counts[k] = a.fresh_count
            frozen += a.estimated_cost
    evaluation, _ = _draw(counts=counts, phase="evaluation", **common)
    out = []
    for k, c in enumerate(cands):
        # a terminal candidate's weight is deterministic: its single pilot evaluation is the weight
        evs = pilot[k] if terminal[k] else evaluation[k]
        if not evs:
            raise RuntimeError("each candidate needs an independent weight estimate")
        out.append(ProgressiveCandidate(c.token_ids, tuple(c.token_logprobs),
                                        PilotSummary(pilot_counts[k], stds[k], costs[k], snap), tuple(evs),
                                        1 if terminal[k] else counts[k], logmeanexp([e.log_weight for e in evs])))
    lw = np.asarray([c.log_weight for c in out], dtype=np.float64)
    p = np.exp(lw - lw.max())
    sel = int(seeds.generator("progressive_is", step_index, "select").choice(len(out), p=p / p.sum()))
    return ProgressiveISStep(len(generated_prefix), tuple(out), sel, frozen)


def run_progressive_conditional_is(base_backend: AutoregressiveBackend, prompt: TokenSequence,
                                   config: ProgressiveISConfig, reward: TokenReward | None, seeds: SeedStream, *,
                                   base_sampling: SamplingConfig | None = None,
                                   rollout_backend: AutoregressiveBackend | None = None,
                                   rollout_sampling: SamplingConfig | None = None,
                                   reward_batch: TokenBatchReward | None = None,
                                   streaming_rewards: bool = True) -> ProgressiveISResult:
    base_sampling = base_sampling or SamplingConfig()
    rollout_backend = rollout_backend or base_backend
    rollout_sampling = rollout_sampling or base_sampling
    _check_policies(base_sampling, rollout_sampling)
    prompt = tuple(prompt)
    evaluator = (StreamingRewardEvaluator(workers=config.reward_workers)
                 if streaming_rewards and reward is not None and reward_batch is None else None)
    gen: list[int] = []
    steps = []
    eos = base_sampling.eos_token_id
    try:
        while len(gen) < config.total_length:
            st = progressive_is_step(base_backend=base_backend, rollout_backend=rollout_backend, prompt=prompt,
                                     generated_prefix=tuple(gen), config=config, base_sampling=base_sampling,
                                     rollout_sampling=rollout_sampling, reward=reward, reward_batch=reward_batch,
                                     seeds=seeds, step_index=len(steps), streaming_evaluator=evaluator)
            gen.extend(st.selected.token_ids)
            steps.append(st)
            if eos is not None and eos in st.selected.token_ids:
                gen = gen[:gen.index(eos) + 1]
                break
    finally:
        if evaluator is not None:
            evaluator.close()
    return ProgressiveISResult(prompt, tuple(gen), tuple(steps))


__all__ = ["PilotSummary", "ProgressiveCandidate", "ProgressiveISResult", "ProgressiveISStep",
           "progressive_is_step", "run_progressive_conditional_is"]
