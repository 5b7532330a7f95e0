"""Conditional importance sampling over blocks (finite-candidate SIR).

At each step K candidate blocks are sampled from the base policy.  Each
candidate is weighted by R rollouts to the end of the budget: on-policy
rollouts weight exp(r / tau); off-policy rollouts from a full-support proposal
q add the base/proposal log-ratio log p - log q of the rollout (optionally
clipped).  The rollout weights combine by log-mean-exp and one candidate is
selected with an explicit uniform.

Stream names follow src/inference_scaling/arllm/algorithms/conditional_is.py:
("conditional_is", step, "candidate", k) and (..., "rollout", r), with selection
from ("conditional_is", step, "select").
"""

from __future__ import annotations

from collections.abc import Callable, Sequence
from dataclasses import dataclass
from math import isfinite

from ...shared.importance import MonteCarloRolloutWeightProvider, RolloutObservation, logmeanexp
from ...shared.rng import SeedStream
from ...shared.stepwise import StepwiseCandidate, run_stepwise_generation
from ...shared.types import TokenSequence
from ..config import ConditionalISConfig, SamplingConfig
from ..types import AutoregressiveBackend, GenerationRequest, ScoreRequest, SequenceSample

TokenReward = Callable[[TokenSequence, TokenSequence], float]
TokenBatchReward = Callable[[TokenSequence, Sequence[TokenSequence]], Sequence[float]]


@dataclass(frozen=True, slots=True)
class RolloutEvaluation:
    token_ids: TokenSequence
    reward: float
    base_logprob: float | None
    proposal_logprob: float
    raw_log_importance_ratio: float | None
    applied_log_importance_ratio: float | None
    log_weight: float
    proposal_model_id: str
    proposal_policy_id: str


@dataclass(frozen=True, slots=True)
class ConditionalCandidate:
    token_ids: TokenSequence
    base_token_logprobs: tuple[float, ...]
    rollouts: tuple[RolloutEvaluation, ...]
    log_weight: float
    planned_rollout_count: int = 0


@dataclass(frozen=True, slots=True)
class ConditionalISStep:
    generated_length_before: int
    candidates: tuple[ConditionalCandidate, ...]
    selected_index: int
    probabilities: tuple[float, ...] = ()

    @property
    def selected(self) -> ConditionalCandidate:
        return self.candidates[self.selected_index]


@dataclass(frozen=True, slots=True)
class ConditionalISResult:
    prompt: TokenSequence
    token_ids: TokenSequence
    steps: tuple[ConditionalISStep, ...]


def _full_support(sampling: SamplingConfig, what: str) -> None:
    if not sampling.full_support:
        raise ValueError(f"{what} must use a full-support policy: top_p=1 and top_k=None")


def sample_candidates(backend: AutoregressiveBackend, prefix: TokenSequence, count: int, block: int,
                      sampling: SamplingConfig, seeds: SeedStream, step: int) -> list[SequenceSample]:
    reqs = [GenerationRequest(prefix, block, sampling, seeds.derive("conditional_is", step, "candidate", k),
                              f"conditional-is:step:{step}:candidate:{k}") for k in range(count)]
    out = backend.sample_batch(reqs)
    if len(out) != count:
        raise RuntimeError("backend returned an invalid number of candidates")
    for c in out:
        if not c.token_ids:
            raise RuntimeError("a candidate block must contain at least one token")
        if c.policy_id != sampling.policy_id:
            raise RuntimeError("candidate was not sampled by the requested base policy")
    return out


def estimate_conditional_weights(*, base_backend: AutoregressiveBackend, rollout_backend: AutoregressiveBackend,
                                 prompt: TokenSequence, generated_prefix: TokenSequence,
                                 candidates: Sequence[SequenceSample], rollout_length: int, rollout_count: int,
                                 base_sampling: SamplingConfig, rollout_sampling: SamplingConfig,
                                 reward_temperature: float, importance_log_ratio_clip: float | None,
                                 apply_importance_correction: bool, reward: TokenReward | None, seeds: SeedStream,
                                 step_index: int, reward_batch: TokenBatchReward | None = None
                                 ) -> tuple[ConditionalCandidate, ...]:
    """Weight every candidate with its rollouts (one batched sample call for all K * R)."""
    _full_support(rollout_sampling, "off-policy rollouts")
    if rollout_count <= 0 or reward_temperature <= 0:
        raise ValueError("rollout_count and reward_temperature must be positive")
    if (reward is None) == (reward_batch is None):
        raise ValueError("provide exactly one of reward or reward_batch")
    eos = rollout_sampling.eos_token_id
    requests, owner, prefixes, terminal = [], [], [], set()
    for k, cand in enumerate(candidates):
        if rollout_length == 0 or (eos is not None and cand.token_ids[-1] == eos):
            terminal.add(k)
            continue
        prefix = prompt + generated_prefix + cand.token_ids
        for r in range(rollout_count):
            requests.append(GenerationRequest(
                prefix, rollout_length, rollout_sampling,
                seeds.derive("conditional_is", step_index, "candidate", k, "rollout", r),
                f"conditional-is:step:{step_index}:candidate:{k}:rollout:{r}"))
            owner.append(k)
            prefixes.append(prefix)
    samples = rollout_backend.sample_batch(requests) if requests else []
    if len(samples) != len(requests):
        raise RuntimeError("backend returned an invalid number of rollouts")
    on_policy = rollout_backend.model_id == base_backend.model_id and rollout_sampling == base_sampling
    if on_policy:
        base_totals = [s.logprob for s in samples]
    elif apply_importance_correction:
        base_id = base_sampling.policy_id
        base_totals, need = [], []
        for i, s in enumerate(samples):
            if s.reference_policy_id == base_id and s.reference_token_logprobs is not None:
                base_totals.append(float(sum(s.reference_token_logprobs)))
            else:
                base_totals.append(None)
                need.append(i)
        if need:
            scored = base_backend.score_batch([ScoreRequest(prefixes[i], (samples[i].token_ids,), base_sampling)
                                               for i in need])
            for i, vals in zip(need, scored):
                base_totals[i] = float(sum(vals))
        if any(v is None or not isfinite(v) for v in base_totals):
            raise ValueError("rollout proposal generated a completion outside base-model support")
    else:
        base_totals = [None] * len(samples)
    groups: list[list[tuple]] = [[] for _ in candidates]
    for k in terminal:
        groups[k].append(((), 0.0, 0.0, rollout_backend.model_id, rollout_sampling.policy_id,
                          generated_prefix + candidates[k].token_ids))
    for k, s, b in zip(owner, samples, base_totals):
        groups[k].append((s.token_ids, b, s.logprob, s.model_id, s.policy_id,
                          generated_prefix + candidates[k].token_ids + s.token_ids))
    flat = [g for grp in groups for g in grp]
    if reward_batch is not None:
        rewards = [float(v) for v in reward_batch(prompt, [g[-1] for g in flat])]
        if len(rewards) != len(flat):
            raise ValueError("reward_batch returned an invalid number of rewards")
    else:
        rewards = [float(reward(prompt, g[-1])) for g in flat]
    if any(not isfinite(v) for v in rewards):
        raise ValueError("reward must be finite")
    iw = MonteCarloRolloutWeightProvider(reward_temperature=reward_temperature, correction="importance",
                                         log_ratio_clip=importance_log_ratio_clip)
    plain = MonteCarloRolloutWeightProvider(reward_temperature=reward_temperature, correction="none")
    out, idx = [], 0
    for k, grp in enumerate(groups):
        evals = []
        for toks, b, q, mid, pid, _ in grp:
            obs = RolloutObservation(rewards[idx], b, q, toks)
            idx += 1
            w = iw.weight(obs) if b is not None else plain.weight(obs)
            evals.append(RolloutEvaluation(toks, obs.reward, b, q, w.raw_log_importance_ratio,
                                           w.applied_log_importance_ratio, w.log_weight, mid, pid))
        base_logs = tuple(candidates[k].reference_token_logprobs or candidates[k].token_logprobs)
        out.append(ConditionalCandidate(candidates[k].token_ids, base_logs, tuple(evals),
                                        logmeanexp([e.log_weight for e in evals]), len(evals)))
    return tuple(out)


class AutoregressiveStepwiseAdapter:
    """Stepwise-generation adapter: state = generated tokens so far."""

    def __init__(self, *, base_backend, rollout_backend, prompt, config: ConditionalISConfig,
                 base_sampling: SamplingConfig, rollout_sampling: SamplingConfig, reward=None, reward_batch=None):
        _full_support(base_sampling, "base candidates")
        self.base_backend, self.rollout_backend = base_backend, rollout_backend
        self.prompt, self.config = tuple(prompt), config
        self.base_sampling, self.rollout_sampling = base_sampling, rollout_sampling
        self.reward, self.reward_batch = reward, reward_batch

    @property
    def initial_state(self) -> TokenSequence:
        return ()

    def is_terminal(self, state: TokenSequence) -> bool:
        eos = self.base_sampling.eos_token_id
        return len(state) >= self.config.total_length or (eos is not None and bool(state) and state[-1] == eos)

    def propose(self, state, step_index, seeds):
        block = min(self.config.block_size, self.config.total_length - len(state))
        return sample_candidates(self.base_backend, self.prompt + state, self.config.candidate_count, block,
                                 self.base_sampling, seeds, step_index)

    def evaluate(self, state, proposals, step_index, seeds):
        rollout_len = self.config.total_length - len(state) - len(proposals[0].token_ids)
        cands = estimate_conditional_weights(
            base_backend=self.base_backend, rollout_backend=self.rollout_backend, prompt=self.prompt,
            generated_prefix=state, candidates=proposals, rollout_length=max(rollout_len, 0),
            rollout_count=self.config.rollout_count, base_sampling=self.base_sampling,
            rollout_sampling=self.rollout_sampling, reward_temperature=self.config.reward_temperature,
            importance_log_ratio_clip=self.config.importance_log_ratio_clip,
            apply_importance_correction=self.config.apply_importance_correction, reward=self.reward, seeds=seeds,
            step_index=step_index, reward_batch=self.reward_batch)
        return [StepwiseCandidate(c, c.log_weight) for c in cands]

    def advance(self, state, selected: ConditionalCandidate, step_index):
        return state + selected.token_ids


def run_conditional_is(*, base_backend: AutoregressiveBackend, prompt: TokenSequence, config: ConditionalISConfig,
                       seeds: SeedStream, reward: TokenReward | None = None,
                       reward_batch: TokenBatchReward | None = None,
                       rollout_backend: AutoregressiveBackend | None = None,
                       base_sampling: SamplingConfig = SamplingConfig(),
                       rollout_sampling: SamplingConfig | None = None) -> ConditionalISResult:
    adapter = AutoregressiveStepwiseAdapter(
        base_backend=base_backend, rollout_backend=rollout_backend or base_backend, prompt=prompt, config=config,
        base_sampling=base_sampling, rollout_sampling=rollout_sampling or base_sampling, reward=reward,
        reward_batch=reward_batch)
    result = run_stepwise_generation(adapter, seeds, selection_namespace=("conditional_is",))
    steps = tuple(ConditionalISStep(len(s.state_before), tuple(c.value for c in s.candidates), s.selected_index,
                                    s.probabilities) for s in result.steps)
    return ConditionalISResult(tuple(prompt), result.final_state, steps)
