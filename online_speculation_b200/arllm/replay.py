"""Replay records, behaviour policies, and a store whose evaluation records are used once.

A record is a completion generated from ``key.rollout_prefix`` by a named behaviour
policy, with its reward and behaviour log-probability.  The store tracks every record
in one table with a lifecycle state:

    evaluation  ->  reserved (by a frozen claim)  ->  design

``freeze_claims`` reserves up to n evaluation records per key before anything about
them except their behaviour ids is revealed; ``reveal_and_consume`` hands a claim's
records over and moves them to the design pool, so an evaluation record can inform
at most one estimate.  Mixture behaviour log-probabilities (records drawn by several
policies) and checks of stored probabilities re-score completions with the registered
backends.  Request ids ``replay:<record_id>`` and claim ids ``claim-<n>`` follow
src/inference_scaling/arllm/replay.py (they key caches and saved runs).
"""

from __future__ import annotations

from collections import Counter
from collections.abc import Callable, Iterable, Mapping, Sequence
from dataclasses import dataclass
from math import isfinite

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
        return tuple(self.prompt) + tuple(self.generated_prefix) + tuple(self.candidate)


@dataclass(frozen=True, slots=True)
class ReplayRecord:
    record_id: str
    key: ReplayKey
    completion: TokenSequence
    reward: float
    behavior_id: str
    behavior_logprob: float

    def __post_init__(self) -> None:
        if not (self.record_id and self.behavior_id):
            raise ValueError("a replay record needs a record id and a behaviour id")
        if not (isfinite(self.reward) and isfinite(self.behavior_logprob)):
            raise ValueError("a replay record's reward and behaviour log-probability have to be finite")


@dataclass(frozen=True, slots=True)
class ReplaySampleRequest:
    key: ReplayKey
    max_new_tokens: int
    seed: int
    record_id: str

    def __post_init__(self) -> None:
        if min(self.max_new_tokens, self.seed) < 0:
            raise ValueError("max_new_tokens and seed cannot be negative")
        if not self.record_id:
            raise ValueError("a replay request needs a record id")


def _request_id(record_id: str) -> str:
    return f"replay:{record_id}"


@dataclass(frozen=True, slots=True)
class BehaviorPolicy:
    behavior_id: str
    backend: AutoregressiveBackend
    sampling: SamplingConfig

    @classmethod
    def for_backend(cls, backend: AutoregressiveBackend, sampling: SamplingConfig, *, label: str | None = None):
        return cls(label if label else f"{backend.model_id}|{sampling.policy_id}", backend, sampling)


@dataclass(frozen=True, slots=True)
class BrokeredReplayState:
    """Replay metadata paired with its resumable, unfinished rollout."""

    request: ReplaySampleRequest
    rollout: PartialRollout

    def __post_init__(self) -> None:
        g = self.rollout.request
        expected = (_request_id(self.request.record_id), self.request.key.rollout_prefix,
                    self.request.max_new_tokens, self.request.seed)
        if self.request.max_new_tokens < 1:
            raise ValueError("a brokered replay rollout generates at least one token")
        if (g.request_id, g.prefix, g.max_new_tokens, g.seed) != expected:
            raise ValueError("the rollout does not belong to this replay request")

    @classmethod
    def start(cls, policy: BehaviorPolicy, request: ReplaySampleRequest, *, priority: float = 0.0):
        if request.max_new_tokens < 1:
            raise ValueError("a brokered replay rollout generates at least one token")
        generation = GenerationRequest(request.key.rollout_prefix, request.max_new_tokens, policy.sampling,
                                       request.seed, _request_id(request.record_id))
        return cls(request, PartialRollout.from_request(generation, priority=float(priority)))


@dataclass(frozen=True, slots=True)
class BrokeredReplayResult:
    records: tuple[ReplayRecord, ...]
    partial: tuple[BrokeredReplayState, ...]
    snapshot: RolloutBrokerSnapshot


class BehaviorRegistry:
    """Behaviour policies by id; registering the same id twice must describe the same policy."""

    def __init__(self, policies: Iterable[BehaviorPolicy] = ()):
        self._policies: dict[str, BehaviorPolicy] = {}
        for policy in policies:
            self.register(policy)

    def register(self, policy: BehaviorPolicy) -> None:
        known = self._policies.setdefault(policy.behavior_id, policy)
        if known is not policy and (known.backend.model_id, known.sampling) != (policy.backend.model_id,
                                                                                 policy.sampling):
            raise ValueError(f"behaviour id {policy.behavior_id!r} is already registered with another policy")

    def get(self, behavior_id: str) -> BehaviorPolicy:
        if behavior_id not in self._policies:
            raise KeyError(f"no behaviour policy is registered as {behavior_id!r}")
        return self._policies[behavior_id]

    def __contains__(self, behavior_id: str) -> bool:
        return behavior_id in self._policies


@dataclass(frozen=True, slots=True)
class FrozenReplayClaim:
    """Claim made before any completion is revealed: only behaviour counts are visible."""

    claim_id: str
    key: ReplayKey
    behavior_counts: tuple[tuple[str, int], ...]

    @property
    def count(self) -> int:
        return sum(n for _, n in self.behavior_counts)


def _behaviour_counts(records: Iterable[ReplayRecord]) -> tuple[tuple[str, int], ...]:
    return tuple(sorted(Counter(r.behavior_id for r in records).items()))


class InMemoryReplayStore:
    """One table of records, each in state "evaluation", "design" or a claim id (reserved)."""

    _EVAL, _DESIGN = "evaluation", "design"

    def __init__(self):
        self._records: list[ReplayRecord] = []
        self._state: list[str] = []
        self._ids: set[str] = set()
        self._claims = 0
        self._open_claims: set[str] = set()

    def _add(self, record: ReplayRecord, state: str) -> None:
        if record.record_id in self._ids:
            raise ValueError(f"replay record id {record.record_id!r} is already stored")
        self._ids.add(record.record_id)
        self._records.append(record)
        self._state.append(state)

    def add_evaluation(self, record: ReplayRecord) -> None:
        self._add(record, self._EVAL)

    def add_design(self, record: ReplayRecord) -> None:
        self._add(record, self._DESIGN)

    def _rows(self, state: str, key: ReplayKey | None = None) -> list[int]:
        return [i for i, (r, s) in enumerate(zip(self._records, self._state))
                if s == state and (key is None or r.key == key)]

    def inventory(self, key: ReplayKey) -> dict[str, int]:
        return dict(Counter(self._records[i].behavior_id for i in self._rows(self._EVAL, key)))

    def freeze_claims(self, keys: Sequence[ReplayKey], max_records_per_candidate: int
                      ) -> tuple[FrozenReplayClaim, ...]:
        if max_records_per_candidate < 0:
            raise ValueError("max_records_per_candidate cannot be negative")
        claims = []
        for key in keys:
            self._claims += 1
            claim_id = f"claim-{self._claims}"
            taken = self._rows(self._EVAL, key)[:max_records_per_candidate]
            for i in taken:
                self._state[i] = claim_id
            self._open_claims.add(claim_id)
            claims.append(FrozenReplayClaim(claim_id, key, _behaviour_counts(self._records[i] for i in taken)))
        return tuple(claims)

    def reveal_and_consume(self, claim: FrozenReplayClaim) -> tuple[ReplayRecord, ...]:
        if claim.claim_id not in self._open_claims:
            raise ValueError(f"claim {claim.claim_id!r} is unknown or was already consumed")
        rows = self._rows(claim.claim_id)
        records = tuple(self._records[i] for i in rows)
        if any(r.key != claim.key for r in records) or _behaviour_counts(records) != claim.behavior_counts:
            raise RuntimeError(f"the records reserved by {claim.claim_id!r} no longer match the claim")
        self._open_claims.discard(claim.claim_id)
        for i in rows:
            self._state[i] = self._DESIGN
        return records

    def design_records(self, key: ReplayKey | None = None) -> tuple[ReplayRecord, ...]:
        return tuple(self._records[i] for i in self._rows(self._DESIGN, key))

    @property
    def evaluation_count(self) -> int:
        return self._state.count(self._EVAL)

    @property
    def design_count(self) -> int:
        return self._state.count(self._DESIGN)

    @property
    def reserved_count(self) -> int:
        return sum(s not in (self._EVAL, self._DESIGN) for s in self._state)


def score_continuations(policy: BehaviorPolicy, key: ReplayKey, completions: Sequence[TokenSequence]
                        ) -> tuple[float, ...]:
    """Sequence log-probabilities of ``completions`` after the key's rollout prefix."""
    if not len(completions):
        return ()
    scores = policy.backend.score_batch([ScoreRequest(key.rollout_prefix, tuple(completions), policy.sampling)])
    if len(scores) != len(completions) or any(len(s) != len(c) for s, c in zip(scores, completions)):
        raise RuntimeError("the behaviour backend's scores do not match the completions")
    return tuple(float(np.sum(s)) for s in scores)


def mixture_logprobabilities(registry: BehaviorRegistry, key: ReplayKey, behavior_counts: Mapping[str, int],
                             completions: Sequence[TokenSequence]) -> tuple[float, ...]:
    """log sum_b (n_b / n) q_b(completion): the behaviour law of records pooled from several policies."""
    ids = sorted(behavior_counts)
    counts = np.asarray([behavior_counts[b] for b in ids], dtype=np.float64)
    if counts.size == 0 or counts.sum() <= 0:
        raise ValueError("a behaviour mixture needs at least one record")
    if (counts <= 0).any():
        raise ValueError("every behaviour in a mixture needs a positive count")
    table = np.asarray([score_continuations(registry.get(b), key, completions) for b in ids], dtype=np.float64)
    weights = np.log(counts / counts.sum())[:, None]
    return tuple(np.logaddexp.reduce(table + weights, axis=0).tolist())


def declared_logprob_tolerance(backend) -> tuple[float, float] | None:
    """(absolute, per-token) difference a backend declares between the log-probabilities it
    returns when sampling and when re-scoring the same tokens (its ``logprob_tolerance``),
    looked up through wrapper backends; None when no backend in the chain declares one."""
    for _ in range(8):
        if backend is None:
            return None
        tol = getattr(backend, "logprob_tolerance", None)
        if tol is not None:
            return float(tol[0]), float(tol[1])
        backend = getattr(backend, "_backend", None) or getattr(backend, "backend", None)
    return None


def validate_record_probabilities(records: Sequence[ReplayRecord], registry: BehaviorRegistry, *,
                                  absolute_tolerance: float = 1e-5, per_token_tolerance: float = 2e-4) -> None:
    """Re-score stored completions; a stored behaviour probability that is not reproduced is an error.

    A backend whose sampling and scoring passes differ numerically (bf16 activations through
    kernels of different shapes) declares that difference; the larger tolerance applies.
    """
    if min(absolute_tolerance, per_token_tolerance) < 0:
        raise ValueError("tolerances cannot be negative")
    groups: dict[tuple, list[ReplayRecord]] = {}
    for record in records:
        groups.setdefault((record.key, record.behavior_id), []).append(record)
    for (key, behavior), group in groups.items():
        policy = registry.get(behavior)
        fresh = np.asarray(score_continuations(policy, key, [r.completion for r in group]))
        stored = np.asarray([r.behavior_logprob for r in group])
        a_tol, t_tol = absolute_tolerance, per_token_tolerance
        declared = declared_logprob_tolerance(policy.backend)
        if declared is not None:
            a_tol, t_tol = max(a_tol, declared[0]), max(t_tol, declared[1])
        allowed = a_tol + t_tol * np.asarray([len(r.completion) for r in group])
        bad = np.flatnonzero(np.abs(stored - fresh) > allowed)
        if bad.size:
            r = group[int(bad[0])]
            raise ValueError(f"record {r.record_id!r}: stored behaviour log-probability {r.behavior_logprob:.6g} "
                             f"is not reproduced (re-scored {fresh[bad[0]]:.6g}, tolerance {allowed[bad[0]]:g})")


def _record(policy: BehaviorPolicy, request: ReplaySampleRequest, completion, logprob, reward: TokenReward):
    k = request.key
    value = float(reward(k.prompt, tuple(k.generated_prefix) + tuple(k.candidate) + tuple(completion)))
    return ReplayRecord(request.record_id, k, tuple(completion), value, policy.behavior_id, logprob)


def _check_policy(policy: BehaviorPolicy, sample) -> None:
    if sample.model_id != policy.backend.model_id or sample.policy_id != policy.sampling.policy_id:
        raise RuntimeError("a replay sample was not drawn by its declared behaviour policy")


def sample_replay_records(policy: BehaviorPolicy, requests: Sequence[ReplaySampleRequest], reward: TokenReward
                          ) -> tuple[ReplayRecord, ...]:
    """Generate completions for requests of different keys in one backend batch
    (zero-length requests record an empty completion of log-probability 0)."""
    active = [r for r in requests if r.max_new_tokens]
    batch = [GenerationRequest(r.key.rollout_prefix, r.max_new_tokens, policy.sampling, r.seed,
                               _request_id(r.record_id)) for r in active]
    samples = policy.backend.sample_batch(batch) if batch else []
    if len(samples) != len(batch):
        raise RuntimeError(f"{len(samples)} replay samples came back for {len(batch)} requests")
    drawn = {}
    for request, sample in zip(active, samples):
        _check_policy(policy, sample)
        drawn[request.record_id] = (sample.token_ids, sample.logprob)
    return tuple(_record(policy, r, *drawn.get(r.record_id, ((), 0.0)), reward) for r in requests)


def sample_replay_record(policy: BehaviorPolicy, key: ReplayKey, max_new_tokens: int, reward: TokenReward, *,
                         seed: int, record_id: str) -> ReplayRecord:
    return sample_replay_records(policy, [ReplaySampleRequest(key, max_new_tokens, seed, record_id)], reward)[0]


def sample_replay_records_brokered(policy: BehaviorPolicy, work: Sequence[ReplaySampleRequest | BrokeredReplayState],
                                   reward: TokenReward, broker: AsyncRolloutBroker, *,
                                   completion_target: int | None = None,
                                   on_record: Callable[[ReplayRecord], None] | None = None) -> BrokeredReplayResult:
    """Replay generation through a rollout broker; only finished trajectories become records."""
    if broker.backend is not policy.backend:
        raise ValueError("the broker has to sample from the behaviour policy's backend")
    states = [w if isinstance(w, BrokeredReplayState) else BrokeredReplayState.start(policy, w) for w in work]
    if not states:
        raise ValueError("brokered replay needs at least one rollout")
    by_request: dict[str, BrokeredReplayState] = {}
    for state in states:
        g = state.rollout.request
        if g.sampling != policy.sampling:
            raise ValueError(f"{g.request_id} samples from another behaviour policy")
        if state.rollout.complete:
            raise ValueError(f"{g.request_id} is already finished")
        if g.request_id in by_request:
            raise ValueError(f"{g.request_id} was submitted twice")
        by_request[g.request_id] = state
    result = broker.run_until([s.rollout for s in states], completion_target=completion_target)
    records = []
    for sample in result.completed:
        state = by_request.get(sample.request_id)
        if state is None:
            raise RuntimeError(f"the broker finished {sample.request_id!r}, which was not submitted")
        _check_policy(policy, sample)
        record = _record(policy, state.request, sample.token_ids, sample.logprob, reward)
        records.append(record)
        if on_record is not None:
            on_record(record)
    partial = tuple(BrokeredReplayState(by_request[p.request.request_id].request, p) for p in result.partial)
    return BrokeredReplayResult(tuple(records), partial, result.snapshot)


__all__ = ["BehaviorPolicy", "BehaviorRegistry", "BrokeredReplayResult", "BrokeredReplayState", "FrozenReplayClaim",
           "InMemoryReplayStore", "ReplayKey", "ReplayRecord", "ReplaySampleRequest", "mixture_logprobabilities",
           "sample_replay_record", "sample_replay_records", "sample_replay_records_brokered", "score_continuations",
           "declared_logprob_tolerance", "validate_record_probabilities"]
