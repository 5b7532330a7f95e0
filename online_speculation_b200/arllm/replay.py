"""Replay records, behaviour policies and a single-use data-pool lifecycle.

A record stores a completion generated from ``key.rollout_prefix`` by a named
behaviour policy, its reward and its behaviour log-probability.  Evaluation
records are used at most once: ``freeze_claims`` reserves them before any
completion or reward is revealed (only behaviour-id counts are visible), and
``reveal_and_consume`` moves them to the design pool.  Mixture behaviour
log-probabilities (several behaviour policies) and re-validation of stored
probabilities are computed by re-scoring with the registered backends.

Reference behaviour: src/inference_scaling/arllm/replay.py:28-478.
"""

from __future__ import annotations

from collections import Counter, defaultdict
from collections.abc import Callable, Iterable, Mapping, Sequence
from dataclasses import dataclass
from math import isclose, isfinite, log

import numpy as np

from ..shared.types import TokenSequence
from .config import SamplingConfig
from .rollout_broker import AsyncRolloutBroker, PartialRollout, RolloutBrokerSnapshot
from .types import AutoregressiveBackend, GenerationRequest, ScoreRequest

TokenReward = Callable[[TokenSequence, TokenSequence], float]


@dataclass(frozen=True, slots=True)
class ReplayKey:
    prompt: TokenSequence
    generated_prefix: TokenSequence
    candidate: TokenSequence
    reward_version: str

    @property
    def rollout_prefix(self) -> TokenSequence:
        return self.prompt + self.generated_prefix + self.candidate


@dataclass(frozen=True, slots=True)
class ReplayRecord:
    record_id: str
    key: ReplayKey
    completion: TokenSequence
    reward: float
    behavior_id: str
    behavior_logprob: float

    def __post_init__(self) -> None:
        if not self.record_id or not self.behavior_id:
            raise ValueError("record_id and behavior_id cannot be empty")
        if not isfinite(self.reward):
            raise ValueError("stored reward must be finite")
        if not isfinite(self.behavior_logprob):
            raise ValueError("a generated completion must have finite behavior log-probability")


@dataclass(frozen=True, slots=True)
class ReplaySampleRequest:
    key: ReplayKey
    max_new_tokens: int
    seed: int
    record_id: str

    def __post_init__(self) -> None:
        if self.max_new_tokens < 0 or self.seed < 0:
            raise ValueError("max_new_tokens and seed must be non-negative")
        if not self.record_id:
            raise ValueError("record_id cannot be empty")


@dataclass(frozen=True, slots=True)
class BehaviorPolicy:
    behavior_id: str
    backend: AutoregressiveBackend
    sampling: SamplingConfig

    @classmethod
    def for_backend(cls, backend: AutoregressiveBackend, sampling: SamplingConfig, *, label: str | None = None):
        return cls(label or f"{backend.model_id}|{sampling.policy_id}", backend, sampling)


@dataclass(frozen=True, slots=True)
class BrokeredReplayState:
    """Replay metadata paired with a resumable, unfinished rollout."""

    request: ReplaySampleRequest
    rollout: PartialRollout

    def __post_init__(self) -> None:
        g = self.rollout.request
        if self.request.max_new_tokens <= 0:
            raise ValueError("brokered replay requires a positive rollout length")
        if g.request_id != f"replay:{self.request.record_id}":
            raise ValueError("brokered replay request id does not match its record")
        if (g.prefix, g.max_new_tokens, g.seed) != (self.request.key.rollout_prefix, self.request.max_new_tokens,
                                                    self.request.seed):
            raise ValueError("brokered replay rollout does not match its request")

    @classmethod
    def start(cls, policy: BehaviorPolicy, request: ReplaySampleRequest, *, priority: float = 0.0):
        if request.max_new_tokens <= 0:
            raise ValueError("brokered replay requires a positive rollout length")
        g = GenerationRequest(request.key.rollout_prefix, request.max_new_tokens, policy.sampling, request.seed,
                              f"replay:{request.record_id}")
        return cls(request, PartialRollout.from_request(g, priority=float(priority)))


@dataclass(frozen=True, slots=True)
class BrokeredReplayResult:
    records: tuple[ReplayRecord, ...]
    partial: tuple[BrokeredReplayState, ...]
    snapshot: RolloutBrokerSnapshot


class BehaviorRegistry:
    def __init__(self, policies: Iterable[BehaviorPolicy] = ()):
        self._p: dict[str, BehaviorPolicy] = {}
        for p in policies:
            self.register(p)

    def register(self, policy: BehaviorPolicy) -> None:
        old = self._p.get(policy.behavior_id)
        if old is not None:
            if old.backend.model_id != policy.backend.model_id or old.sampling != policy.sampling:
                raise ValueError(f"behavior id {policy.behavior_id!r} has conflicting definitions")
            return
        self._p[policy.behavior_id] = policy

    def get(self, behavior_id: str) -> BehaviorPolicy:
        try:
            return self._p[behavior_id]
        except KeyError as e:
            raise KeyError(f"unknown behavior policy {behavior_id!r}") from e

    def __contains__(self, behavior_id: str) -> bool:
        return behavior_id in self._p


@dataclass(frozen=True, slots=True)
class FrozenReplayClaim:
    """Metadata-only claim (behaviour counts) made before any completion is revealed."""

    claim_id: str
    key: ReplayKey
    behavior_counts: tuple[tuple[str, int], ...]

    @property
    def count(self) -> int:
        return sum(c for _, c in self.behavior_counts)


class InMemoryReplayStore:
    """Evaluation records are single use by construction; consumed records join the design pool."""

    def __init__(self):
        self._eval: dict[ReplayKey, list[ReplayRecord]] = defaultdict(list)
        self._design: list[ReplayRecord] = []
        self._reserved: dict[str, tuple[ReplayRecord, ...]] = {}
        self._ids: set[str] = set()
        self._claims = 0

    def _new(self, r: ReplayRecord) -> None:
        if r.record_id in self._ids:
            raise ValueError(f"duplicate replay record id {r.record_id!r}")
        self._ids.add(r.record_id)

    def add_evaluation(self, record: ReplayRecord) -> None:
        self._new(record)
        self._eval[record.key].append(record)

    def add_design(self, record: ReplayRecord) -> None:
        self._new(record)
        self._design.append(record)

    def inventory(self, key: ReplayKey) -> dict[str, int]:
        return dict(Counter(r.behavior_id for r in self._eval.get(key, ())))

    def freeze_claims(self, keys: Sequence[ReplayKey], max_records_per_candidate: int
                      ) -> tuple[FrozenReplayClaim, ...]:
        if max_records_per_candidate < 0:
            raise ValueError("max_records_per_candidate must be non-negative")
        out = []
        for k in keys:
            avail = self._eval.get(k, [])
            take = tuple(avail[:max_records_per_candidate])
            del avail[:len(take)]
            self._claims += 1
            cid = f"claim-{self._claims}"
            self._reserved[cid] = take
            out.append(FrozenReplayClaim(cid, k, tuple(sorted(Counter(r.behavior_id for r in take).items()))))
        return tuple(out)

    def reveal_and_consume(self, claim: FrozenReplayClaim) -> tuple[ReplayRecord, ...]:
        try:
            recs = self._reserved.pop(claim.claim_id)
        except KeyError as e:
            raise ValueError(f"claim {claim.claim_id!r} is unknown or already consumed") from e
        if any(r.key != claim.key for r in recs):
            raise RuntimeError("replay claim key mismatch")
        if tuple(sorted(Counter(r.behavior_id for r in recs).items())) != claim.behavior_counts:
            raise RuntimeError("replay claim metadata changed after freezing")
        self._design.extend(recs)
        return recs

    def design_records(self, key: ReplayKey | None = None) -> tuple[ReplayRecord, ...]:
        return tuple(self._design) if key is None else tuple(r for r in self._design if r.key == key)

    @property
    def evaluation_count(self) -> int:
        return sum(len(v) for v in self._eval.values())

    @property
    def design_count(self) -> int:
        return len(self._design)

    @property
    def reserved_count(self) -> int:
        return sum(len(v) for v in self._reserved.values())


def score_continuations(policy: BehaviorPolicy, key: ReplayKey, completions: Sequence[TokenSequence]
                        ) -> tuple[float, ...]:
    if not completions:
        return ()
    got = policy.backend.score_batch([ScoreRequest(key.rollout_prefix, tuple(completions), policy.sampling)])
    if len(got) != len(completions):
        raise RuntimeError("behavior backend returned an invalid number of scores")
    out = []
    for c, s in zip(completions, got):
        if len(s) != len(c):
            raise RuntimeError("behavior backend returned an invalid token score shape")
        out.append(float(sum(s)))
    return tuple(out)


def mixture_logprobabilities(registry: BehaviorRegistry, key: ReplayKey, behavior_counts: Mapping[str, int],
                             completions: Sequence[TokenSequence]) -> tuple[float, ...]:
    """log sum_b (n_b / n) q_b(completion) over the behaviour policies that produced the records."""
    total = sum(behavior_counts.values())
    if total <= 0:
        raise ValueError("a behavior mixture requires at least one selected record")
    comps = []
    for bid, n in sorted(behavior_counts.items()):
        if n <= 0:
            raise ValueError("behavior mixture counts must be positive")
        comps.append(np.asarray(score_continuations(registry.get(bid), key, completions)) + log(n / total))
    return tuple(float(v) for v in np.logaddexp.reduce(np.stack(comps), axis=0))


def validate_record_probabilities(records: Sequence[ReplayRecord], registry: BehaviorRegistry, *,
                                  absolute_tolerance: float = 1e-5, per_token_tolerance: float = 2e-4) -> None:
    """Re-score stored completions; reject a record whose stored behaviour probability is not reproduced."""
    if absolute_tolerance < 0 or per_token_tolerance < 0:
        raise ValueError("probability validation tolerances must be non-negative")
    groups: dict[tuple, list[ReplayRecord]] = defaultdict(list)
    for r in records:
        groups[(r.key, r.behavior_id)].append(r)
    for (k, bid), g in groups.items():
        for r, s in zip(g, score_continuations(registry.get(bid), k, [x.completion for x in g])):
            tol = absolute_tolerance + per_token_tolerance * len(r.completion)
            if not isclose(r.behavior_logprob, s, rel_tol=0.0, abs_tol=tol):
                raise ValueError(f"stored behavior probability for {r.record_id!r} cannot be reproduced within "
                                 f"tolerance {tol:g}")


def sample_replay_records(policy: BehaviorPolicy, requests: Sequence[ReplaySampleRequest], reward: TokenReward
                          ) -> tuple[ReplayRecord, ...]:
    """Generate replay completions for heterogeneous keys in one backend batch."""
    gen, where = [], []
    for i, r in enumerate(requests):
        if r.max_new_tokens:
            gen.append(GenerationRequest(r.key.rollout_prefix, r.max_new_tokens, policy.sampling, r.seed,
                                         f"replay:{r.record_id}"))
            where.append(i)
    got = policy.backend.sample_batch(gen) if gen else []
    if len(got) != len(gen):
        raise RuntimeError("replay backend returned an invalid number of samples")
    by = dict(zip(where, got))
    out = []
    for i, r in enumerate(requests):
        s = by.get(i)
        if s is None:
            comp, lp = (), 0.0
        else:
            if s.model_id != policy.backend.model_id or s.policy_id != policy.sampling.policy_id:
                raise RuntimeError("replay sample does not match its declared behavior policy")
            comp, lp = s.token_ids, s.logprob
        out.append(ReplayRecord(r.record_id, r.key, comp,
                                float(reward(r.key.prompt, r.key.generated_prefix + r.key.candidate + comp)),
                                policy.behavior_id, lp))
    return tuple(out)


def sample_replay_record(policy: BehaviorPolicy, key: ReplayKey, max_new_tokens: int, reward: TokenReward, *,
                         seed: int, record_id: str) -> ReplayRecord:
    return sample_replay_records(policy, [ReplaySampleRequest(key, max_new_tokens, seed, record_id)], reward)[0]


def sample_replay_records_brokered(policy: BehaviorPolicy, work: Sequence[ReplaySampleRequest | BrokeredReplayState],
                                   reward: TokenReward, broker: AsyncRolloutBroker, *,
                                   completion_target: int | None = None,
                                   on_record: Callable[[ReplayRecord], None] | None = None) -> BrokeredReplayResult:
    """Replay generation through the rollout broker; only finished trajectories become records."""
    if broker.backend is not policy.backend:
        raise ValueError("rollout broker must use the behavior policy backend")
    states = tuple(w if isinstance(w, BrokeredReplayState) else BrokeredReplayState.start(policy, w) for w in work)
    if not states:
        raise ValueError("brokered replay requires at least one rollout")
    by_id: dict[str, BrokeredReplayState] = {}
    for st in states:
        g = st.rollout.request
        if g.sampling != policy.sampling:
            raise ValueError("brokered replay state uses the wrong behavior policy")
        if st.rollout.complete:
            raise ValueError("completed replay state must not be resubmitted")
        if g.request_id in by_id:
            raise ValueError("brokered replay record ids must be unique")
        by_id[g.request_id] = st
    res = broker.run_until(tuple(s.rollout for s in states), completion_target=completion_target)
    recs = []
    for smp in res.completed:
        st = by_id.get(smp.request_id)
        if st is None:
            raise RuntimeError("broker completed an unknown replay request")
        if smp.model_id != policy.backend.model_id or smp.policy_id != policy.sampling.policy_id:
            raise RuntimeError("brokered replay sample used the wrong behavior policy")
        k = st.request.key
        rec = ReplayRecord(st.request.record_id, k, smp.token_ids,
                           float(reward(k.prompt, k.generated_prefix + k.candidate + smp.token_ids)),
                           policy.behavior_id, smp.logprob)
        recs.append(rec)
        if on_record is not None:
            on_record(rec)
    partial = tuple(BrokeredReplayState(by_id[p.request.request_id].request, p) for p in res.partial)
    return BrokeredReplayResult(tuple(recs), partial, res.snapshot)


__all__ = ["BehaviorPolicy", "BehaviorRegistry", "BrokeredReplayResult", "BrokeredReplayState", "FrozenReplayClaim",
           "InMemoryReplayStore", "ReplayKey", "ReplayRecord", "ReplaySampleRequest", "mixture_logprobabilities",
           "sample_replay_record", "sample_replay_records", "sample_replay_records_brokered", "score_continuations",
           "validate_record_probabilities"]
