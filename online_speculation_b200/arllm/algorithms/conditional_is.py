"""Conditional importance sampling over blocks (finite-candidate SIR).

At each step K candidate blocks are sampled from the base policy.  Each
candidate is weighted by R rollouts to the end of the budget: on-policy
rollouts weight exp(r / tau); off-policy rollouts from a full-support proposal
q add the base/proposal log-ratio log p - log q of the rollout (optionally
clipped).  The rollout weights combine by log-mean-exp and one candidate is
selected with an explicit uniform.

Rollout designs: ``iid`` (independent seeds), ``scrambled_sobol`` (one
scrambled Sobol net per candidate, one coordinate per rollout token, inverse
CDF) and ``arithmetic_lattice`` (a randomly shifted lattice of arithmetic-coding
uniforms per candidate).  Every rollout stays marginally exact, so the
candidate weight stays unbiased; only the dependence between rollouts changes.

Exact early stopping: with declared bounds [a, b] on every rollout log-weight,
rollouts are evaluated in batches and the unseen ones bound each candidate
weight in [(S + m e^a) / R, (S + m e^b) / R].  As soon as the categorical
selection with the step's fixed uniform is the same for every weight vector in
that box, the remaining rollouts are skipped; the selected index is then the
one a full evaluation would have produced.

Stream names follow src/inference_scaling/arllm/algorithms/conditional_is.py:
("conditional_is", step, "candidate", k) and (..., "rollout", r), with selection
from ("conditional_is", step, "select").  Reference behaviour: same file,
:174-872.
"""

from __future__ import annotations

from collections.abc import Callable, Sequence
from dataclasses import dataclass
from math import exp, isfinite, log

from ...shared.importance import MonteCarloRolloutWeightProvider, RolloutObservation, logmeanexp
from ...shared.rng import SeedStream
from ...experimental.shared.bounded_selection import invariant_categorical_index
from ...experimental.shared.rqmc import randomized_lattice_uniforms, scrambled_sobol_uniforms
from ...shared.stepwise import (StepwiseCandidate, categorical_index_from_uniform, normalize_log_weights,
                                run_stepwise_generation, stepwise_generation_step)
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
    log_weight_lower_bound: float | None = None
    log_weight_upper_bound: float | None = None


@dataclass(frozen=True, slots=True)
class ConditionalISStep:
    generated_length_before: int
    candidates: tuple[ConditionalCandidate, ...]
    selected_index: int
    probabilities: tuple[float, ...] = ()
    rollout_evaluations_planned: int = 0
    rollout_evaluations_performed: int = 0
    rollout_evaluations_skipped: int = 0
    rollout_evaluation_batches: int = 0
    exact_early_stop: bool = False
    selection_invariant_verified: bool = False

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
                                 step_index: int, reward_batch: TokenBatchReward | None = None,
                                 rollout_design: str = "iid", rollout_index_offset: int = 0
                                 ) -> tuple[ConditionalCandidate, ...]:
    """Weight every candidate with its rollouts (one batched sample call for all K * R)."""
    _full_support(rollout_sampling, "off-policy rollouts")
    if rollout_count <= 0 or reward_temperature <= 0:
        raise ValueError("rollout_count and reward_temperature must be positive")
    if (reward is None) == (reward_batch is None):
        raise ValueError("provide exactly one of reward or reward_batch")
    if rollout_design not in ROLLOUT_DESIGNS:
        raise ValueError("unknown rollout_design")
    if rollout_index_offset < 0:
        raise ValueError("rollout_index_offset must be non-negative")
    if rollout_index_offset and rollout_design != "iid":
        raise ValueError("staged rollout offsets require iid rollouts")
    if rollout_design != "iid" and reward_batch is not None:
        raise ValueError("randomized QMC rollouts need a pointwise reward: a batch-coupled reward changes with "
                         "the dependence between rollouts")
    eos = rollout_sampling.eos_token_id
    requests, owner, prefixes, terminal = [], [], [], set()
    for k, cand in enumerate(candidates):
        if rollout_length == 0 or (eos is not None and cand.token_ids[-1] == eos):
            terminal.add(k)
            continue
        prefix = prompt + generated_prefix + cand.token_ids
        tok_u = arith_u = (None,) * rollout_count
        if rollout_design == "scrambled_sobol":
            tok_u = scrambled_sobol_uniforms(rollout_count, rollout_length, seed=seeds.derive(
                "conditional_is", step_index, "candidate", k, "scrambled_sobol"))
        elif rollout_design == "arithmetic_lattice":
            arith_u = randomized_lattice_uniforms(rollout_count, seed=seeds.derive(
                "conditional_is", step_index, "candidate", k, "arithmetic_lattice"))
        for j in range(rollout_count):
            r = rollout_index_offset + j
            requests.append(GenerationRequest(
                prefix, rollout_length, rollout_sampling,
                seeds.derive("conditional_is", step_index, "candidate", k, "rollout", r),
                f"conditional-is:step:{step_index}:candidate:{k}:rollout:{r}", tok_u[j], arith_u[j]))
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
            step_index=step_index, reward_batch=self.reward_batch, rollout_design=self.config.rollout_design)
        return [StepwiseCandidate(c, c.log_weight) for c in cands]

    def advance(self, state, selected: ConditionalCandidate, step_index):
        return state + selected.token_ids


def _bounded_conditional_is_step(*, base_backend, rollout_backend, prompt, generated_prefix, config, base_sampling,
                                 rollout_sampling, reward, seeds, step_index, reward_batch) -> ConditionalISStep:
    if reward is None or reward_batch is not None:
        raise ValueError("exact rollout early stopping requires a fixed pointwise reward")
    if config.rollout_log_weight_bounds is None:
        raise ValueError("exact rollout early stopping requires log-weight bounds")
    if config.rollout_design != "iid":
        raise ValueError("exact rollout early stopping requires iid rollouts")
    _full_support(base_sampling, "base candidates")
    left = config.total_length - len(generated_prefix)
    if left <= 0:
        raise ValueError("generated prefix has already reached total_length")
    props = sample_candidates(base_backend, prompt + generated_prefix, config.candidate_count,
                              min(config.block_size, left), base_sampling, seeds, step_index)
    roll_len = max(0, left - len(props[0].token_ids))
    eos = rollout_sampling.eos_token_id
    terminal = [roll_len == 0 or (eos is not None and p.token_ids[-1] == eos) for p in props]
    planned = [1 if t else config.rollout_count for t in terminal]
    u = float(seeds.generator("conditional_is", step_index, "select").random())
    a, b = config.rollout_log_weight_bounds
    try:
        w_min, w_max = exp(a), exp(b)
    except OverflowError as e:
        raise ValueError("rollout log-weight bounds cannot be exponentiated") from e
    if not (isfinite(w_min) and isfinite(w_max) and w_min > 0):
        raise ValueError("rollout log-weight bounds must map to finite positive weights")
    R = config.rollout_count
    seen: list[list[RolloutEvaluation]] = [[] for _ in props]
    lo_w, hi_w, fixed, done, batches = [], [], None, 0, 0
    while done < R:
        n = min(config.rollout_evaluation_batch_size, R - done)
        got = estimate_conditional_weights(
            base_backend=base_backend, rollout_backend=rollout_backend, prompt=prompt,
            generated_prefix=generated_prefix, candidates=props, rollout_length=roll_len, rollout_count=n,
            base_sampling=base_sampling, rollout_sampling=rollout_sampling,
            reward_temperature=config.reward_temperature,
            importance_log_ratio_clip=config.importance_log_ratio_clip,
            apply_importance_correction=config.apply_importance_correction, reward=reward, seeds=seeds,
            step_index=step_index, rollout_index_offset=done)
        batches += 1
        for k, c in enumerate(got):
            if terminal[k]:
                if not seen[k]:
                    seen[k].append(c.rollouts[0])
                continue
            for ev in c.rollouts:
                if not a <= ev.log_weight <= b:
                    raise ValueError("observed rollout log-weight lies outside the declared bounds")
            seen[k].extend(c.rollouts)
        done += n
        lo_w, hi_w = [], []
        for k, evs in enumerate(seen):
            tot = sum(exp(e.log_weight) for e in evs)
            if terminal[k]:
                lo_w.append(tot)
                hi_w.append(tot)
            else:
                m = R - len(evs)
                lo_w.append((tot + m * w_min) / R)
                hi_w.append((tot + m * w_max) / R)
        fixed = invariant_categorical_index(lo_w, hi_w, uniform=u)
        if fixed is not None:
            break
    cands = tuple(ConditionalCandidate(p.token_ids, tuple(p.reference_token_logprobs or p.token_logprobs),
                                       tuple(seen[k]), log(0.5 * (lo_w[k] + hi_w[k])), planned[k],
                                       log(lo_w[k]), log(hi_w[k])) for k, p in enumerate(props))
    probs = normalize_log_weights([c.log_weight for c in cands])
    sel = categorical_index_from_uniform(probs, u)
    if fixed is not None and sel != fixed:
        raise RuntimeError("bounded categorical decision disagrees with the representative weights")
    performed = sum(len(c.rollouts) for c in cands)
    skipped = sum(planned) - performed
    return ConditionalISStep(len(generated_prefix), cands, sel, probs, sum(planned), performed, skipped, batches,
                             skipped > 0, skipped > 0 and fixed is not None)


def _check_policies(base_sampling: SamplingConfig, rollout_sampling: SamplingConfig) -> None:
    _full_support(base_sampling, "base candidates")
    _full_support(rollout_sampling, "off-policy rollouts")
    if base_sampling.eos_token_id != rollout_sampling.eos_token_id:
        raise ValueError("candidate and rollout policies must agree on eos_token_id")


def conditional_is_step(*, base_backend: AutoregressiveBackend, rollout_backend: AutoregressiveBackend,
                        prompt: TokenSequence, generated_prefix: TokenSequence, config: ConditionalISConfig,
                        base_sampling: SamplingConfig, rollout_sampling: SamplingConfig,
                        reward: TokenReward | None, seeds: SeedStream, step_index: int,
                        reward_batch: TokenBatchReward | None = None) -> ConditionalISStep:
    """One conditional-IS block choice from an explicit generated prefix."""
    kw = dict(base_backend=base_backend, rollout_backend=rollout_backend, prompt=tuple(prompt), config=config,
              base_sampling=base_sampling, rollout_sampling=rollout_sampling, reward=reward,
              reward_batch=reward_batch)
    if config.exact_rollout_early_stop:
        return _bounded_conditional_is_step(generated_prefix=tuple(generated_prefix), seeds=seeds,
                                            step_index=step_index, **kw)
    sel = stepwise_generation_step(AutoregressiveStepwiseAdapter(**kw), tuple(generated_prefix), step_index, seeds,
                                   selection_namespace=("conditional_is",))
    cands = tuple(c.value for c in sel.candidates)
    n = sum(len(c.rollouts) for c in cands)
    return ConditionalISStep(len(generated_prefix), cands, sel.selected_index, sel.probabilities, n, n, 0, 1)


def run_conditional_is(base_backend: AutoregressiveBackend, prompt: TokenSequence, config: ConditionalISConfig,
                       reward: TokenReward | None = None, seeds: SeedStream | None = None, *,
                       base_sampling: SamplingConfig | None = None,
                       rollout_backend: AutoregressiveBackend | None = None,
                       rollout_sampling: SamplingConfig | None = None,
                       reward_batch: TokenBatchReward | None = None) -> ConditionalISResult:
    """Generate a sequence by repeated conditional-IS block choices."""
    if seeds is None:
        raise ValueError("run_conditional_is needs a SeedStream")
    base_sampling = base_sampling or SamplingConfig()
    rollout_sampling = rollout_sampling or base_sampling
    rollout_backend = rollout_backend or base_backend
    _check_policies(base_sampling, rollout_sampling)
    prompt = tuple(prompt)
    if config.exact_rollout_early_stop:
        gen: TokenSequence = ()
        steps = []
        eos = base_sampling.eos_token_id
        while len(gen) < config.total_length and (eos is None or eos not in gen):
            st = conditional_is_step(base_backend=base_backend, rollout_backend=rollout_backend, prompt=prompt,
                                     generated_prefix=gen, config=config, base_sampling=base_sampling,
                                     rollout_sampling=rollout_sampling, reward=reward, seeds=seeds,
                                     step_index=len(steps), reward_batch=reward_batch)
            gen += st.selected.token_ids
            if eos is not None and eos in gen:
                gen = gen[:gen.index(eos) + 1]
            steps.append(st)
        return ConditionalISResult(prompt, gen, tuple(steps))
    adapter = AutoregressiveStepwiseAdapter(
        base_backend=base_backend, rollout_backend=rollout_backend, prompt=prompt, config=config,
        base_sampling=base_sampling, rollout_sampling=rollout_sampling, reward=reward, reward_batch=reward_batch)
    result = run_stepwise_generation(adapter, seeds, selection_namespace=("conditional_is",))
    steps = []
    for s in result.steps:
        cands = tuple(c.value for c in s.candidates)
        n = sum(len(c.rollouts) for c in cands)
        steps.append(ConditionalISStep(len(s.state_before), cands, s.selected_index, s.probabilities, n, n, 0, 1))
    return ConditionalISResult(prompt, result.final_state, tuple(steps))


ROLLOUT_DESIGNS = ("iid", "scrambled_sobol", "arithmetic_lattice")
