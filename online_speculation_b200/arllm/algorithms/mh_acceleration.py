"""Exact accelerations of reward-tilted suffix MH (target p(y) exp(r(y) / tau)).

* Delayed acceptance: stage one uses a cheap surrogate reward in the full
  Hastings ratio; only proposals that pass pay for the exact reward, and stage
  two accepts with exp(((r' - s') - (r - s)) / tau), so the target is unchanged.
* Prefetched branches: while the exact reward of the current proposal is
  evaluated on a worker thread, the next step's proposals for both possible
  outcomes (reject: from the current state; accept: from the proposed state)
  are sampled in one backend call; the Hastings decision then picks the branch.
  The next step's cut and seed do not depend on the state, so this is the same
  chain; the unused branch is overhead only.
* Frozen replay proposal: the suffix proposal is the defensive mixture
  (1 - h) p_base + h * empirical(suffixes observed after the same prefix and of
  the same length), frozen before sampling, with exact forward and reverse
  mixture probabilities.

Reference behaviour: src/inference_scaling/arllm/algorithms/mh_acceleration.py:312-856.
"""

from __future__ import annotations

import threading
from collections import Counter, defaultdict
from collections.abc import Callable, Iterable
from concurrent.futures import ThreadPoolExecutor
from dataclasses import dataclass
from math import isfinite, log

import numpy as np

from ...shared.mh import decide_metropolis_hastings
from ...shared.rng import SeedStream
from ...shared.types import TokenSequence
from ..config import RewardMHConfig, SamplingConfig
from ..types import AutoregressiveBackend, ScoreRequest
from .mh import RewardMHChainResult, RewardMHStep, _is_base, draw_suffix, sample_fixed_lengths, validate_proposal

RewardFunction = Callable[[TokenSequence, TokenSequence], float]


def _reward(fn: RewardFunction, prompt, seq) -> float:
    v = float(fn(prompt, seq))
    if not isfinite(v):
        raise ValueError("reward must be finite")
    return v


@dataclass(frozen=True, slots=True)
class _State:
    tokens: TokenSequence
    base: tuple[float, ...]
    prop: tuple[float, ...]
    reward: float | None


@dataclass(frozen=True, slots=True)
class _Proposal:
    source: _State
    cut: int
    tokens: TokenSequence
    base: tuple[float, ...]
    prop: tuple[float, ...]
    schedule: str
    probability: float

    @property
    def sequence(self) -> TokenSequence:
        return self.source.tokens[:self.cut] + self.tokens


def _initial_state(backend, prompt, config, proposal, reward, seeds, chain_id) -> _State:
    t, q, p = sample_fixed_lengths(backend, [prompt], [config.total_length], proposal,
                                   [seeds.derive("reward_mh", chain_id, "initialize")],
                                   [f"reward-mh:{chain_id}:initialize"])
    base = q[0] if _is_base(proposal) else p[0]
    return _State(t[0], tuple(base), tuple(q[0]), _reward(reward, prompt, t[0]))


def _proposals(backend, states, *, prompt, config, proposal, seeds, chain_id, step) -> tuple[_Proposal, ...]:
    cut, n, prob = draw_suffix(config.total_length, config.suffix_schedule,
                               seeds.generator("reward_mh", chain_id, step, "cut"))
    t, q, p = sample_fixed_lengths(backend, [prompt + s.tokens[:cut] for s in states], [n] * len(states), proposal,
                                   [seeds.derive("reward_mh", chain_id, step, "proposal")] * len(states),
                                   [f"reward-mh:{chain_id}:step:{step}"] * len(states))
    return tuple(_Proposal(s, cut, tt, tuple(qq if _is_base(proposal) else pp), tuple(qq), config.suffix_schedule,
                           prob) for s, tt, qq, pp in zip(states, t, q, p))


def _hastings(state: _State, pr: _Proposal, cur_val: float, new_val: float, tau: float, u: float):
    c = pr.cut
    return decide_metropolis_hastings(
        current_target_log_density=sum(state.base[c:]) + cur_val / tau,
        proposed_target_log_density=sum(pr.base) + new_val / tau,
        forward_proposal_log_probability=sum(pr.prop), reverse_proposal_log_probability=sum(state.prop[c:]),
        uniform=u)


def _accepted_state(state: _State, pr: _Proposal, reward: float | None) -> _State:
    return _State(pr.sequence, state.base[:pr.cut] + pr.base, state.prop[:pr.cut] + pr.prop, reward)


def _changes(state: _State, pr: _Proposal) -> int:
    return sum(a != b for a, b in zip(state.tokens[pr.cut:], pr.tokens))


# -------------------------------------------------------- delayed acceptance --
@dataclass(frozen=True, slots=True)
class DelayedRewardMHStep:
    step: int
    cut: int
    proposed_suffix_length: int
    current_reward: float
    proposed_reward: float | None
    current_surrogate_reward: float
    proposed_surrogate_reward: float
    stage_one_log_acceptance: float
    stage_one_accepted: bool
    stage_two_log_acceptance: float | None
    exact_reward_evaluated: bool
    accepted: bool
    suffix_schedule: str
    suffix_probability: float
    proposed_token_changes: int
    accepted_token_changes: int


@dataclass(frozen=True, slots=True)
class DelayedRewardMHResult:
    prompt: TokenSequence
    token_ids: TokenSequence
    reward: float
    surrogate_reward: float
    base_token_logprobs: tuple[float, ...]
    proposal_token_logprobs: tuple[float, ...]
    trace: tuple[DelayedRewardMHStep, ...]
    chain_id: int
    exact_reward_evaluations: int
    surrogate_reward_evaluations: int

    @property
    def attempts(self) -> int:
        return len(self.trace)

    @property
    def accepted(self) -> int:
        return sum(s.accepted for s in self.trace)

    @property
    def acceptance_rate(self) -> float:
        return self.accepted / self.attempts if self.attempts else 0.0

    @property
    def exact_reward_fraction(self) -> float:
        return self.exact_reward_evaluations / self.surrogate_reward_evaluations


def run_reward_mh_chain_delayed(backend: AutoregressiveBackend, prompt: TokenSequence, config: RewardMHConfig,
                                proposal: SamplingConfig, reward: RewardFunction, surrogate_reward: RewardFunction,
                                seeds: SeedStream, *, chain_id: int = 0) -> DelayedRewardMHResult:
    validate_proposal(proposal)
    prompt = tuple(prompt)
    tau = config.reward_temperature
    st = _initial_state(backend, prompt, config, proposal, reward, seeds, chain_id)
    sur = _reward(surrogate_reward, prompt, st.tokens)
    exact, surs = 1, 1
    trace = []
    for step in range(config.updates):
        pr = _proposals(backend, (st,), prompt=prompt, config=config, proposal=proposal, seeds=seeds,
                        chain_id=chain_id, step=step)[0]
        ps = _reward(surrogate_reward, prompt, pr.sequence)
        surs += 1
        one = _hastings(st, pr, sur, ps, tau,
                        float(seeds.generator("reward_mh", chain_id, step, "delayed-stage-one").random()))
        pr_r, two_log, acc = None, None, False
        if one.accepted:
            pr_r = _reward(reward, prompt, pr.sequence)
            exact += 1
            two = decide_metropolis_hastings(
                current_target_log_density=(st.reward - sur) / tau, proposed_target_log_density=(pr_r - ps) / tau,
                uniform=float(seeds.generator("reward_mh", chain_id, step, "delayed-stage-two").random()))
            two_log, acc = two.log_acceptance, two.accepted
        prev_r, prev_s = st.reward, sur
        ch = _changes(st, pr)
        if acc:
            st = _accepted_state(st, pr, pr_r)
            sur = ps
        trace.append(DelayedRewardMHStep(step, pr.cut, config.total_length - pr.cut, prev_r, pr_r, prev_s, ps,
                                         one.log_acceptance, one.accepted, two_log, one.accepted, acc, pr.schedule,
                                         pr.probability, ch, ch if acc else 0))
    return DelayedRewardMHResult(prompt, st.tokens, st.reward, sur, st.base, st.prop, tuple(trace), chain_id, exact,
                                 surs)


# ---------------------------------------------------------------- prefetch --
@dataclass(frozen=True, slots=True)
class PrefetchSnapshot:
    used_proposals: int
    prefetched_proposals: int
    unused_prefetched_proposals: int
    reward_evaluations: int


@dataclass(frozen=True, slots=True)
class PrefetchedRewardMHResult:
    chain: RewardMHChainResult
    prefetch: PrefetchSnapshot


def run_reward_mh_chain_prefetched(backend: AutoregressiveBackend, prompt: TokenSequence, config: RewardMHConfig,
                                   proposal: SamplingConfig, reward: RewardFunction, seeds: SeedStream, *,
                                   chain_id: int = 0) -> PrefetchedRewardMHResult:
    validate_proposal(proposal)
    prompt = tuple(prompt)
    tau = config.reward_temperature
    st = _initial_state(backend, prompt, config, proposal, reward, seeds, chain_id)
    cur = _proposals(backend, (st,), prompt=prompt, config=config, proposal=proposal, seeds=seeds, chain_id=chain_id,
                     step=0)[0]
    trace, prefetched, used, evals = [], 1, 0, 1
    with ThreadPoolExecutor(max_workers=1, thread_name_prefix="mh-reward") as pool:
        for step in range(config.updates):
            if cur.source.tokens != st.tokens:
                raise RuntimeError("prefetched MH proposal does not match the selected branch")
            fut = pool.submit(_reward, reward, prompt, cur.sequence)
            nxt: tuple[_Proposal, ...] = ()
            if step + 1 < config.updates:
                nxt = _proposals(backend, (st, _accepted_state(st, cur, None)), prompt=prompt, config=config,
                                 proposal=proposal, seeds=seeds, chain_id=chain_id, step=step + 1)
                prefetched += len(nxt)
            pr_r = float(fut.result())
            evals += 1
            prev = st.reward
            ch = _changes(st, cur)
            d = _hastings(st, cur, st.reward, pr_r, tau,
                          float(seeds.generator("reward_mh", chain_id, step, "accept").random()))
            if d.accepted:
                st = _accepted_state(st, cur, pr_r)
            used += 1
            trace.append(RewardMHStep(step, cur.cut, config.total_length - cur.cut, prev, pr_r, d.log_acceptance,
                                      d.accepted, cur.schedule, cur.probability, ch, ch if d.accepted else 0))
            if nxt:
                cur = nxt[1 if d.accepted else 0]
    chain = RewardMHChainResult(prompt, st.tokens, st.reward, st.base, st.prop, tuple(trace), chain_id)
    return PrefetchedRewardMHResult(chain, PrefetchSnapshot(used, prefetched, prefetched - used, evals))


# ---------------------------------------------------------- replay proposal --
@dataclass(frozen=True, slots=True)
class ReplayProposalDraw:
    token_ids: TokenSequence
    base_token_logprobs: tuple[float, ...]
    proposal_logprob: float
    source: str


@dataclass(frozen=True, slots=True)
class ReplayProposalSnapshot:
    stored_suffixes: int
    stored_prefix_lengths: int
    base_draws: int
    history_draws: int
    logprob_queries: int


def _score(backend, prefix, suffix) -> tuple[float, ...]:
    got = backend.score_batch([ScoreRequest(tuple(prefix), (tuple(suffix),), None)])
    if len(got) != 1 or len(got[0]) != len(suffix):
        raise RuntimeError("backend returned an invalid score shape")
    return tuple(got[0])


class FrozenReplaySuffixProposal:
    """Defensive mixture of base suffixes and empirical replay suffixes (frozen before use)."""

    def __init__(self, backend: AutoregressiveBackend, *, history_mixture: float = 0.25,
                 sampling: SamplingConfig | None = None):
        if not 0 <= history_mixture < 1:
            raise ValueError("history_mixture must lie in [0, 1)")
        self.backend = backend
        self.sampling = sampling or SamplingConfig()
        validate_proposal(self.sampling)
        if not _is_base(self.sampling):
            raise ValueError("defensive replay proposal currently requires base sampling")
        self.history_mixture = float(history_mixture)
        self._suffixes: dict[tuple[TokenSequence, int], Counter] = defaultdict(Counter)
        self._frozen = False
        self._n = Counter()
        self._lock = threading.RLock()

    def observe_suffix(self, prefix: TokenSequence, suffix: TokenSequence) -> None:
        if self._frozen:
            raise RuntimeError("replay proposal is frozen")
        if not suffix:
            raise ValueError("replay proposal suffix cannot be empty")
        self._suffixes[(tuple(prefix), len(suffix))][tuple(suffix)] += 1

    def observe_sequence(self, prompt: TokenSequence, sequence: TokenSequence) -> None:
        seq = tuple(sequence)
        for cut in range(len(seq)):
            self.observe_suffix(tuple(prompt) + seq[:cut], seq[cut:])

    def observe_sequences(self, prompt: TokenSequence, sequences: Iterable[TokenSequence]) -> None:
        for s in sequences:
            self.observe_sequence(prompt, s)

    def freeze(self) -> None:
        self._frozen = True

    def _mix(self, base_lp: float, counts, suffix) -> float:
        if not counts or self.history_mixture == 0:
            return float(base_lp)
        hp = counts.get(tuple(suffix), 0) / sum(counts.values())
        terms = [log(1.0 - self.history_mixture) + float(base_lp)]
        if hp > 0:
            terms.append(log(self.history_mixture) + log(hp))
        return float(np.logaddexp.reduce(np.asarray(terms)))

    def draw(self, prefix: TokenSequence, length: int, *, seed: int, request_id: str) -> ReplayProposalDraw:
        if not self._frozen:
            raise RuntimeError("replay proposal must be frozen before sampling")
        if length <= 0:
            raise ValueError("replay proposal length must be positive")
        counts = self._suffixes.get((tuple(prefix), int(length)))
        use_hist = bool(counts) and float(SeedStream(seed).generator("replay-proposal-component").random()) < \
            self.history_mixture
        if use_hist:
            support = tuple(sorted(counts))
            m = np.asarray([counts[s] for s in support], dtype=np.float64)
            suffix = support[int(SeedStream(seed).generator("replay-proposal-history").choice(len(support),
                                                                                              p=m / m.sum()))]
            base = _score(self.backend, prefix, suffix)
            src = "history"
        else:
            t, q, p = sample_fixed_lengths(self.backend, [tuple(prefix)], [length], self.sampling,
                                           [SeedStream(seed).derive("replay-proposal-base")], [request_id])
            suffix, base, src = t[0], tuple(q[0]), "base"
        with self._lock:
            self._n[src] += 1
        return ReplayProposalDraw(tuple(suffix), tuple(base), self._mix(sum(base), counts, suffix), src)

    def logprob(self, prefix: TokenSequence, suffix: TokenSequence, *, base_logprob: float | None = None) -> float:
        if not self._frozen:
            raise RuntimeError("replay proposal must be frozen before scoring")
        if not suffix:
            raise ValueError("replay proposal suffix cannot be empty")
        if base_logprob is None:
            base_logprob = float(sum(_score(self.backend, prefix, suffix)))
        with self._lock:
            self._n["queries"] += 1
        return self._mix(base_logprob, self._suffixes.get((tuple(prefix), len(suffix))), suffix)

    def snapshot(self) -> ReplayProposalSnapshot:
        with self._lock:
            return ReplayProposalSnapshot(sum(sum(c.values()) for c in self._suffixes.values()), len(self._suffixes),
                                          self._n["base"], self._n["history"], self._n["queries"])


@dataclass(frozen=True, slots=True)
class ReplayProposalMHStep:
    step: int
    cut: int
    proposed_suffix_length: int
    current_reward: float
    proposed_reward: float
    old_proposal_logprob: float
    new_proposal_logprob: float
    log_acceptance: float
    accepted: bool
    proposal_source: str
    suffix_schedule: str
    suffix_probability: float
    proposed_token_changes: int
    accepted_token_changes: int


@dataclass(frozen=True, slots=True)
class ReplayProposalMHResult:
    prompt: TokenSequence
    token_ids: TokenSequence
    reward: float
    base_token_logprobs: tuple[float, ...]
    trace: tuple[ReplayProposalMHStep, ...]
    chain_id: int
    initial_source: str

    @property
    def attempts(self) -> int:
        return len(self.trace)

    @property
    def accepted(self) -> int:
        return sum(s.accepted for s in self.trace)

    @property
    def acceptance_rate(self) -> float:
        return self.accepted / self.attempts if self.attempts else 0.0


def run_reward_mh_chain_replay_proposal(proposal: FrozenReplaySuffixProposal, prompt: TokenSequence,
                                        config: RewardMHConfig, reward: RewardFunction, seeds: SeedStream, *,
                                        chain_id: int = 0) -> ReplayProposalMHResult:
    proposal.freeze()
    prompt = tuple(prompt)
    tau = config.reward_temperature
    init = proposal.draw(prompt, config.total_length, seed=seeds.derive("reward_mh", chain_id, "initialize"),
                         request_id=f"reward-mh-replay:{chain_id}:initialize")
    toks, base = init.token_ids, init.base_token_logprobs
    cur = _reward(reward, prompt, toks)
    trace = []
    for step in range(config.updates):
        cut, n, prob = draw_suffix(config.total_length, config.suffix_schedule,
                                   seeds.generator("reward_mh", chain_id, step, "cut"))
        kept, old = toks[:cut], toks[cut:]
        old_p = float(sum(base[cut:]))
        old_q = proposal.logprob(prompt + kept, old, base_logprob=old_p)
        d = proposal.draw(prompt + kept, config.total_length - cut,
                          seed=seeds.derive("reward_mh", chain_id, step, "proposal"),
                          request_id=f"reward-mh-replay:{chain_id}:step:{step}")
        new_r = _reward(reward, prompt, kept + d.token_ids)
        new_p = float(sum(d.base_token_logprobs))
        dec = decide_metropolis_hastings(current_target_log_density=old_p + cur / tau,
                                         proposed_target_log_density=new_p + new_r / tau,
                                         forward_proposal_log_probability=d.proposal_logprob,
                                         reverse_proposal_log_probability=old_q,
                                         uniform=float(seeds.generator("reward_mh", chain_id, step, "accept").random()))
        ch = sum(a != b for a, b in zip(old, d.token_ids))
        prev = cur
        if dec.accepted:
            toks, base, cur = kept + d.token_ids, base[:cut] + d.base_token_logprobs, new_r
        trace.append(ReplayProposalMHStep(step, cut, n, prev, new_r, old_q, d.proposal_logprob, dec.log_acceptance,
                                          dec.accepted, d.source, config.suffix_schedule, prob, ch,
                                          ch if dec.accepted else 0))
    return ReplayProposalMHResult(prompt, toks, cur, base, tuple(trace), chain_id, init.source)


def run_reward_mh_chains_replay_proposal(proposal: FrozenReplaySuffixProposal, prompt: TokenSequence,
                                         config: RewardMHConfig, reward: RewardFunction, seeds: SeedStream, *,
                                         chains: int) -> tuple[ReplayProposalMHResult, ...]:
    if chains <= 0:
        raise ValueError("chains must be positive")
    return tuple(run_reward_mh_chain_replay_proposal(proposal, prompt, config, reward, seeds, chain_id=c)
                 for c in range(chains))


__all__ = ["DelayedRewardMHResult", "DelayedRewardMHStep", "FrozenReplaySuffixProposal", "PrefetchSnapshot",
           "PrefetchedRewardMHResult", "ReplayProposalDraw", "ReplayProposalMHResult", "ReplayProposalMHStep",
           "ReplayProposalSnapshot", "run_reward_mh_chain_delayed", "run_reward_mh_chain_prefetched",
           "run_reward_mh_chain_replay_proposal", "run_reward_mh_chains_replay_proposal"]
