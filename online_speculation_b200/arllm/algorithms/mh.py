"""Suffix-resampling Metropolis--Hastings for sequence power and reward targets.

For a fixed generated length L the power target is p(y | x)^alpha.  An update
draws a suffix length from a full-support schedule, keeps the prefix, regenerates
the suffix from the proposal policy (temperature 1 / alpha by default), and
accepts with the full forward/reverse Hastings ratio using cached per-token
proposal (q) and base (p) log-probabilities of the current state.

Random streams use the same path names as the reference implementation
(src/inference_scaling/arllm/algorithms/mh.py:154-747) -- ("mh", chain, stage,
step, "cut" | "proposal" | "accept") and ("mh", chain, stage, "extend") -- so
batching chains changes scheduling, never random numbers.
"""

from __future__ import annotations

from collections.abc import Callable, Sequence
from dataclasses import dataclass
from math import isfinite

import numpy as np

from ...shared.mh import decide_metropolis_hastings
from ...shared.rng import SeedStream
from ...shared.types import TokenSequence
from ..config import MHConfig, RewardMHConfig, SamplingConfig
from ..types import AutoregressiveBackend, GenerationRequest, ScoreRequest


@dataclass(frozen=True, slots=True)
class MHStep:
    stage_length: int
    step: int
    cut: int
    proposed_suffix_length: int
    log_acceptance: float
    accepted: bool
    suffix_schedule: str
    suffix_probability: float
    proposed_token_changes: int
    accepted_token_changes: int


class _TraceStats:
    trace: tuple

    @property
    def attempts(self) -> int:
        return len(self.trace)

    @property
    def accepted(self) -> int:
        return sum(s.accepted for s in self.trace)

    @property
    def acceptance_rate(self) -> float:
        return self.accepted / self.attempts if self.attempts else 0.0

    def _mean(self, field: str) -> float:
        return sum(getattr(s, field) for s in self.trace) / self.attempts if self.attempts else 0.0

    @property
    def mean_proposed_suffix_length(self) -> float:
        return self._mean("proposed_suffix_length")

    @property
    def mean_proposed_token_changes(self) -> float:
        return self._mean("proposed_token_changes")

    @property
    def mean_accepted_token_changes(self) -> float:
        return self._mean("accepted_token_changes")


@dataclass(frozen=True, slots=True)
class MHChainResult(_TraceStats):
    prompt: TokenSequence
    token_ids: TokenSequence
    base_token_logprobs: tuple[float, ...]
    proposal_token_logprobs: tuple[float, ...]
    trace: tuple[MHStep, ...]
    chain_id: int


@dataclass(frozen=True, slots=True)
class RewardMHStep:
    step: int
    cut: int
    proposed_suffix_length: int
    current_reward: float
    proposed_reward: float
    log_acceptance: float
    accepted: bool
    suffix_schedule: str
    suffix_probability: float
    proposed_token_changes: int
    accepted_token_changes: int


@dataclass(frozen=True, slots=True)
class RewardMHChainResult(_TraceStats):
    prompt: TokenSequence
    token_ids: TokenSequence
    reward: float
    base_token_logprobs: tuple[float, ...]
    proposal_token_logprobs: tuple[float, ...]
    trace: tuple[RewardMHStep, ...]
    chain_id: int


def suffix_length_probabilities(stage_length: int, schedule: str) -> tuple[float, ...]:
    """Full-support probabilities of suffix lengths 1..L.

    ``multiscale`` puts 10% uniform mass everywhere and splits 90% evenly over
    the powers of two below L and L itself.
    """
    if stage_length <= 0:
        raise ValueError("stage_length must be positive")
    L = stage_length
    if schedule == "uniform":
        w = np.ones(L)
    elif schedule == "inverse_length":
        w = 1.0 / np.arange(1, L + 1, dtype=np.float64)
    elif schedule == "multiscale":
        w = np.full(L, 0.1 / L)
        favored = {1, L}
        k = 1
        while k < L:
            favored.add(k)
            k *= 2
        for s in favored:
            w[s - 1] += 0.9 / len(favored)
    else:
        raise ValueError(f"unknown suffix schedule {schedule!r}")
    w = w / w.sum()
    return tuple(float(x) for x in w)


def draw_suffix(stage_length: int, schedule: str, rng: np.random.Generator) -> tuple[int, int, float]:
    """Return (cut, suffix length, probability of that length)."""
    probs = suffix_length_probabilities(stage_length, schedule)
    if schedule == "uniform":
        cut = int(rng.integers(0, stage_length))
        length = stage_length - cut
    else:
        length = int(rng.choice(np.arange(1, stage_length + 1), p=probs))
        cut = stage_length - length
    return cut, length, probs[length - 1]


def validate_proposal(sampling: SamplingConfig) -> None:
    if sampling.eos_token_id is not None:
        raise ValueError("fixed-length MH treats every position as a token; eos_token_id must be None")
    if not sampling.full_support:
        raise ValueError("hard top-k/top-p truncation violates MH's equal-support condition; "
                         "use a full-support proposal")


def _is_base(sampling: SamplingConfig) -> bool:
    return sampling.temperature == 1 and sampling.full_support


def sample_fixed_lengths(backend: AutoregressiveBackend, prefixes: Sequence[TokenSequence], lengths: Sequence[int],
                         sampling: SamplingConfig, seeds: Sequence[int], request_ids: Sequence[str]):
    """Sample independent fixed-length suffixes in one backend call.

    Returns (tokens, proposal log-probs, base log-probs) per request; base
    log-probs come from the sample when the backend reports the reference
    policy, else one batched score call.
    """
    n = len(prefixes)
    if not n or not (len(lengths) == len(seeds) == len(request_ids) == n):
        raise ValueError("batched proposal inputs must have one entry per chain")
    samples = backend.sample_batch([GenerationRequest(tuple(p), int(l), sampling, int(s), r)
                                    for p, l, s, r in zip(prefixes, lengths, seeds, request_ids)])
    if len(samples) != n:
        raise RuntimeError("backend returned an invalid sample count")
    base_id = SamplingConfig().policy_id
    tokens, qs, ps, missing = [], [], [], []
    for i, (smp, length) in enumerate(zip(samples, lengths)):
        if len(smp.token_ids) != length:
            raise RuntimeError(f"MH requires a fixed-length suffix of {length} tokens, got {len(smp.token_ids)}")
        if smp.policy_id != sampling.policy_id:
            raise RuntimeError("backend did not score tokens under the requested proposal policy")
        tokens.append(tuple(smp.token_ids))
        qs.append(tuple(smp.token_logprobs))
        if smp.reference_policy_id == base_id:
            ps.append(tuple(smp.reference_token_logprobs))
        else:
            ps.append(None)
            missing.append(i)
    if missing:
        scored = backend.score_batch([ScoreRequest(tuple(prefixes[i]), (tokens[i],), None) for i in missing])
        for i, vals in zip(missing, scored):
            if len(vals) != lengths[i]:
                raise RuntimeError("backend returned an invalid score shape")
            ps[i] = tuple(vals)
    if any(not isfinite(v) for row in ps for v in row):
        raise ValueError("proposal generated a sequence outside the base model support")
    return tokens, qs, ps


def run_mh_chains_batched(backend: AutoregressiveBackend, prompt: TokenSequence, config: MHConfig,
                          proposal: SamplingConfig, seed_streams: Sequence[SeedStream], *,
                          chain_ids: Sequence[int] | None = None,
                          on_update: Callable[[int, int], None] | None = None) -> tuple[MHChainResult, ...]:
    """Independent power-target chains advanced in lock-step (one backend call per update)."""
    validate_proposal(proposal)
    if not seed_streams:
        raise ValueError("batched MH requires at least one seed stream")
    ids = tuple(chain_ids) if chain_ids is not None else (0,) * len(seed_streams)
    if len(ids) != len(seed_streams):
        raise ValueError("batched MH requires one chain id per seed stream")
    n = len(ids)
    prompt = tuple(prompt)
    tokens = [[] for _ in range(n)]
    base = [[] for _ in range(n)]
    prop = [[] for _ in range(n)]
    traces = [[] for _ in range(n)]
    for stage_index, L in enumerate(config.stages):
        ext = L - len(tokens[0])
        if ext > 0:
            t, q, p = sample_fixed_lengths(
                backend, [prompt + tuple(x) for x in tokens], [ext] * n, proposal,
                [s.derive("mh", c, stage_index, "extend") for s, c in zip(seed_streams, ids)],
                [f"mh:{c}:stage:{stage_index}:extend" for c in ids])
            for i in range(n):
                tokens[i].extend(t[i])
                prop[i].extend(q[i])
                base[i].extend(p[i])
        for step in range(config.stage_updates):
            draws = [draw_suffix(L, config.suffix_schedule, s.generator("mh", c, stage_index, step, "cut"))
                     for s, c in zip(seed_streams, ids)]
            cuts = [d[0] for d in draws]
            t, q, p = sample_fixed_lengths(
                backend, [prompt + tuple(tokens[i][:cuts[i]]) for i in range(n)], [L - c for c in cuts], proposal,
                [s.derive("mh", c, stage_index, step, "proposal") for s, c in zip(seed_streams, ids)],
                [f"mh:{c}:stage:{stage_index}:step:{step}" for c in ids])
            for i, (s, c) in enumerate(zip(seed_streams, ids)):
                cut = cuts[i]
                old_p, old_q = float(sum(base[i][cut:L])), float(sum(prop[i][cut:L]))
                new_p, new_q = float(sum(p[i])), float(sum(q[i]))
                decision = decide_metropolis_hastings(
                    current_target_log_density=config.alpha * old_p,
                    proposed_target_log_density=config.alpha * new_p,
                    forward_proposal_log_probability=new_q,
                    reverse_proposal_log_probability=old_q,
                    uniform=float(s.generator("mh", c, stage_index, step, "accept").random()),
                )
                changes = sum(a != b for a, b in zip(tokens[i][cut:L], t[i]))
                if decision.accepted:
                    tokens[i][cut:L] = t[i]
                    base[i][cut:L] = p[i]
                    prop[i][cut:L] = q[i]
                traces[i].append(MHStep(L, step, cut, L - cut, decision.log_acceptance, decision.accepted,
                                        config.suffix_schedule, draws[i][2], changes,
                                        changes if decision.accepted else 0))
            if on_update is not None:
                on_update(stage_index, step)
    return tuple(MHChainResult(prompt, tuple(tokens[i]), tuple(base[i]), tuple(prop[i]), tuple(traces[i]), ids[i])
                 for i in range(n))


def run_mh_chain(backend: AutoregressiveBackend, prompt: TokenSequence, config: MHConfig, proposal: SamplingConfig,
                 seeds: SeedStream, *, chain_id: int = 0) -> MHChainResult:
    """One staged power-target chain."""
    return run_mh_chains_batched(backend, prompt, config, proposal, (seeds,), chain_ids=(chain_id,))[0]


def run_mh_chains(backend: AutoregressiveBackend, prompt: TokenSequence, config: MHConfig, proposal: SamplingConfig,
                  seeds: SeedStream) -> tuple[MHChainResult, ...]:
    return run_mh_chains_batched(backend, prompt, config, proposal, (seeds,) * config.chains,
                                 chain_ids=tuple(range(config.chains)))


TokenReward = Callable[[TokenSequence, TokenSequence], float]


def run_reward_mh_chain(backend: AutoregressiveBackend, prompt: TokenSequence, config: RewardMHConfig,
                        proposal: SamplingConfig, reward: TokenReward, seeds: SeedStream, *, chain_id: int = 0,
                        on_state: Callable[[RewardMHChainResult], None] | None = None) -> RewardMHChainResult:
    """Sample p(y) exp(r(y) / tau) with full-length initialisation and suffix updates.

    With the base model as proposal the likelihood terms cancel and only the
    reward difference remains; the expanded ratio is exact for any
    full-support proposal.
    """
    validate_proposal(proposal)
    prompt = tuple(prompt)
    L = config.total_length
    t, q, p = sample_fixed_lengths(backend, [prompt], [L], proposal,
                                   [seeds.derive("reward_mh", chain_id, "initialize")],
                                   [f"reward-mh:{chain_id}:initialize"])
    toks, prop = list(t[0]), list(q[0])
    base = list(q[0]) if _is_base(proposal) else list(p[0])
    current = float(reward(prompt, tuple(toks)))
    if not isfinite(current):
        raise ValueError("reward must be finite")
    trace: list[RewardMHStep] = []

    def state() -> RewardMHChainResult:
        return RewardMHChainResult(prompt, tuple(toks), current, tuple(base), tuple(prop), tuple(trace), chain_id)

    if on_state is not None:
        on_state(state())
    for step in range(config.updates):
        cut, length, sprob = draw_suffix(L, config.suffix_schedule,
                                         seeds.generator("reward_mh", chain_id, step, "cut"))
        t, q, p = sample_fixed_lengths(backend, [prompt + tuple(toks[:cut])], [length], proposal,
                                       [seeds.derive("reward_mh", chain_id, step, "proposal")],
                                       [f"reward-mh:{chain_id}:step:{step}"])
        new_tokens, new_q = t[0], q[0]
        new_p = new_q if _is_base(proposal) else p[0]
        proposed_reward = float(reward(prompt, tuple(toks[:cut]) + new_tokens))
        if not isfinite(proposed_reward):
            raise ValueError("reward must be finite")
        decision = decide_metropolis_hastings(
            current_target_log_density=float(sum(base[cut:])) + current / config.reward_temperature,
            proposed_target_log_density=float(sum(new_p)) + proposed_reward / config.reward_temperature,
            forward_proposal_log_probability=float(sum(new_q)),
            reverse_proposal_log_probability=float(sum(prop[cut:])),
            uniform=float(seeds.generator("reward_mh", chain_id, step, "accept").random()),
        )
        changes = sum(a != b for a, b in zip(toks[cut:], new_tokens))
        previous = current
        if decision.accepted:
            toks[cut:] = new_tokens
            base[cut:] = new_p
            prop[cut:] = new_q
            current = proposed_reward
        trace.append(RewardMHStep(step, cut, length, previous, proposed_reward, decision.log_acceptance,
                                  decision.accepted, config.suffix_schedule, sprob, changes,
                                  changes if decision.accepted else 0))
        if on_state is not None:
            on_state(state())
    return state()


def run_reward_mh_chains(backend, prompt, config: RewardMHConfig, proposal: SamplingConfig, reward: TokenReward,
                         seeds: SeedStream, *, chains: int) -> tuple[RewardMHChainResult, ...]:
    if chains <= 0:
        raise ValueError("chains must be positive")
    return tuple(run_reward_mh_chain(backend, prompt, config, proposal, reward, seeds, chain_id=c)
                 for c in range(chains))
