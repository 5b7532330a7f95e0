"""Cold start: serve autoregressively, learn the draft view within a time budget, publish when faster.

The service starts from a dual-view model whose draft attention has never been
trained.  Its parts:

* :class:`TimeBudget` -- maintenance work (training, trials, publication,
  collection) may spend ``fraction`` of the delivered generation time.  An
  operation runs only when its estimate fits the credit; an operation that
  overruns leaves a debt that later deliveries repay.
* :class:`CleanReplay` -- a bounded store of completed responses.  A training
  micro-batch is a set of contiguous crops with random anchors (the offline
  distillation layout), so the draft only reads clean positions before its anchor.
* :class:`FullBlockLearner` -- fp32 masters of every draft-attention projection,
  started from the AR attention and trained with the offline distillation update;
  the serving copy changes only at :meth:`FullBlockLearner.publish`, and
  :meth:`FullBlockLearner.candidate` installs the masters for one trial.
* :class:`ColdStartService` -- answers every request in the current mode (AR until
  a version is published, speculative after), keeps the response, trains when the
  budget admits it, and asks its validation policy whether the learning version
  should be published (or, once speculative, whether to fall back to AR).

Validation policies (one per service, see :class:`ServiceConfig`):

* gate prompts (default): paired trials on held-out prompts every ``probe_every``
  learning steps; same prompt, output cap and seed per pair, alternating order;
  publish when every paired ratio clears ``publish_margin``;
* ``reuse_ar_prefix``: the first ``probe_tokens`` outputs of a delivered AR answer
  are the reference, the candidate answers the same prompt and seed for as many
  tokens; ``live_probe_requests`` such trials of one version are pooled;
* ``full_answer_screen``: the candidate is screened on delivered answers with the
  exact conditional work law (``virtual_work.estimate_trace``) against the
  measured answer time (``FullAnswerGate``); a passing screen earns one fresh
  paired confirmation, which decides.  With ``reuse_speculative_answers`` the
  screening continues after publication against the serving version.

``state_dict`` / ``load_state_dict`` (format ``cold-start-research-v1``) carry the
request-boundary state.  Behaviour follows
online-speculation/ablation/src/blockspec_ablation/cold_start.py.
"""

from __future__ import annotations

import math
import time
from collections import deque
from contextlib import contextmanager
from dataclasses import asdict, dataclass, fields

import torch
from torch import Tensor

from .fitting import FitConfig, frozen_fingerprint
from .generation import MaskedAttentionBranch, ProposalSampler, generate, generate_ar
from .sampling import SamplingConfig
from .training import distillation_update, sample_anchors
from .virtual_work import FullAnswerGate, TraceSupportError, estimate_trace

STATE_FORMAT = "cold-start-research-v1"


def _finite_at_least(value, low: float, *, strict: bool = False) -> bool:
    if not isinstance(value, (int, float)) or not math.isfinite(value):
        return False
    return value > low if strict else value >= low


def _device_of(model) -> torch.device:
    return next(model.parameters()).device


def _settle(model) -> None:
    device = _device_of(model)
    if device.type == "cuda":
        torch.cuda.synchronize(device)


class TimeBudget:
    """Maintenance credit earned at ``fraction`` of the delivered generation time."""

    def __init__(self, fraction: float = 0.01, service_seconds: float = 0.0, costs: dict | None = None):
        if not _finite_at_least(fraction, 0.0, strict=True) or fraction > 0.1:
            raise ValueError(f"the maintenance fraction {fraction} is outside (0, 0.1]")
        self.fraction = float(fraction)
        self.service_seconds = float(service_seconds)
        self.costs: dict[str, float] = dict(costs or {})

    @property
    def spent(self) -> float:
        return float(sum(self.costs.values()))

    @property
    def credit(self) -> float:
        return self.fraction * self.service_seconds - self.spent

    def delivered(self, seconds: float) -> None:
        if not _finite_at_least(seconds, 0.0):
            raise ValueError(f"a delivery lasts a finite, non-negative time, not {seconds}")
        self.service_seconds += seconds

    def charge(self, kind: str, seconds: float) -> None:
        if not _finite_at_least(seconds, 0.0):
            raise ValueError(f"maintenance '{kind}' lasted a finite, non-negative time, not {seconds}")
        self.costs[kind] = self.costs.get(kind, 0.0) + float(seconds)

    def admits(self, estimate: float) -> bool:
        if not _finite_at_least(estimate, 0.0, strict=True):
            raise ValueError(f"an operation estimate is finite and positive, not {estimate}")
        return self.credit >= estimate

    def summary(self) -> dict:
        spent, served = self.spent, self.service_seconds
        return {"fraction": self.fraction, "service_seconds": served, "costs": dict(self.costs),
                "extra_seconds": spent, "extra_over_service": spent / served if served else None,
                "remaining_credit_seconds": self.credit, "debt_seconds": max(0.0, -self.credit)}


class CleanReplay:
    """The last ``capacity`` completed responses and a seeded crop/anchor sampler over them."""

    def __init__(self, capacity: int, sequence_length: int, block_size: int, seed: int):
        if capacity < 1 or block_size < 2 or sequence_length < block_size:
            raise ValueError("the replay needs a positive capacity and windows that hold a draft block")
        self.records: deque = deque(maxlen=capacity)
        self.sequence_length = sequence_length
        self.block_size = block_size
        self.rng = torch.Generator().manual_seed(seed)
        self.anchors_rng = torch.Generator().manual_seed(seed + 1)

    def append(self, tokens: Tensor) -> None:
        """Keep one [1, T] integer record (records shorter than a block cannot train and are dropped)."""
        if tokens.ndim != 2 or tokens.shape[0] != 1 or tokens.dtype != torch.long:
            raise ValueError("a replay record is one [1, T] sequence of int64 token ids")
        if tokens.shape[1] >= self.block_size:
            self.records.append(tokens.detach().to("cpu", copy=True))

    def _crop(self) -> Tensor:
        record = self.records[int(torch.randint(len(self.records), (), generator=self.rng))][0]
        width = min(self.sequence_length, record.numel())
        offset = int(torch.randint(record.numel() - width + 1, (), generator=self.rng))
        return record[offset:offset + width]

    def batch(self, count: int, anchors_per_sequence: int, *, batch_size: int = 1) -> list[tuple[Tensor, Tensor]]:
        """``count`` micro-batches of ``batch_size`` crops each: (tokens [B, <= window], anchors [B, A])."""
        if not self.records:
            raise ValueError("the replay is empty")
        if count < 1 or batch_size < 1:
            raise ValueError("micro-batch and crop counts must be positive")
        micro = []
        for _ in range(count):
            crops = [self._crop() for _ in range(batch_size)]
            anchors = torch.cat([sample_anchors(c.unsqueeze(0), self.block_size, anchors_per_sequence,
                                                generator=self.anchors_rng) for c in crops])
            micro.append((torch.nn.utils.rnn.pad_sequence(crops, batch_first=True, padding_value=0), anchors))
        return micro


class FullBlockLearner:
    """fp32 master copies of the draft attention, trained beside a frozen serving model."""

    def __init__(self, model, config: FitConfig):
        if not isinstance(config, FitConfig):
            raise ValueError("the learner takes a FitConfig")
        if config.sequence_length < model.config.block_size:
            raise ValueError("training windows must hold a whole draft block")
        if any(p.requires_grad for p in model.parameters()):
            raise ValueError("the served model must be frozen (requires_grad_(False))")
        self.model, self.config = model, config
        model.initialize_draft_from_ar()
        model.eval()
        self.execution = {n: p for n, p in model.named_parameters() if ".attention.draft." in n}
        self.master = {n: torch.nn.Parameter(p.detach().float().clone()) for n, p in self.execution.items()}
        self.optimizer = config.make_optimizer(list(self.master.values()))
        # every non-draft parameter and its version counter: in-place writes to them are refused
        self._frozen = [(p, p._version) for n, p in model.named_parameters() if n not in self.execution]
        self.steps = 0
        self.serving_step = 0

    def check(self) -> None:
        grads = any(p.requires_grad for p in self.model.parameters())
        touched = any(p._version != version for p, version in self._frozen)
        if grads or touched:
            raise RuntimeError("the shared AR weights changed or started requiring gradients")

    def step(self, batches) -> dict:
        self.check()
        if self.steps >= self.config.steps:
            raise ValueError(f"all {self.config.steps} learning steps are done")
        device = _device_of(self.model)
        moved = [(tokens.to(device), anchors.to(device)) for tokens, anchors in batches]
        metrics = distillation_update(self.model, moved, self.optimizer, learning_rate=self.config.rate(self.steps),
                                      clip_grad=self.config.clip_grad, chunk_rows=self.config.chunk_rows,
                                      master=self.master)
        self.steps += 1
        self.check()
        return {"step": self.steps, **metrics}

    @torch.no_grad()
    def _install(self, source: dict) -> None:
        for name, param in self.execution.items():
            param.copy_(source[name])

    def publish(self) -> None:
        self.check()
        self._install(self.master)
        self.serving_step = self.steps

    @contextmanager
    def candidate(self):
        """Serve the latest masters inside the block; the serving weights come back even on error."""
        self.check()
        serving = {n: p.detach().clone() for n, p in self.execution.items()}
        serving_step = self.serving_step
        try:
            self.publish()
            yield
        finally:
            self._install(serving)
            self.serving_step = serving_step


@dataclass(frozen=True)
class ServiceConfig:
    fraction: float = 0.01
    replay_records: int = 128
    probe_every: int = 16
    probe_tokens: int = 64
    publish_margin: float = 1.10
    initial_step_estimate: float = 0.5
    seed: int = 731
    initial_probe_factor: float = 2.0
    reuse_ar_prefix: bool = False
    live_probe_requests: int = 1
    full_answer_screen: bool = False
    reuse_speculative_answers: bool = False
    screen_requests: int = 2
    screen_margin: float = 1.02
    initial_screen_estimate: float = 0.4

    def __post_init__(self):
        TimeBudget(self.fraction)
        FullAnswerGate(self.screen_requests, self.screen_margin, self.initial_screen_estimate)
        switches = (self.reuse_ar_prefix, self.full_answer_screen, self.reuse_speculative_answers)
        problems = []
        if not all(type(s) is bool for s in switches):
            problems.append("the policy switches are booleans")
        if self.reuse_ar_prefix and self.full_answer_screen:
            problems.append("choose one live validation policy, not both")
        if self.reuse_speculative_answers and not self.full_answer_screen:
            problems.append("reuse_speculative_answers extends full_answer_screen")
        if type(self.live_probe_requests) is not int or self.live_probe_requests < 1:
            problems.append("live_probe_requests is a positive integer")
        elif self.live_probe_requests > 1 and not self.reuse_ar_prefix:
            problems.append("pooling several live trials is part of reuse_ar_prefix")
        if min(self.replay_records, self.probe_every, self.probe_tokens) < 1:
            problems.append("replay size, probe interval and probe length are positive")
        if not _finite_at_least(self.publish_margin, 1.0, strict=True):
            problems.append("publish_margin is above 1")
        if not _finite_at_least(self.initial_step_estimate, 0.0, strict=True):
            problems.append("initial_step_estimate is positive")
        if not _finite_at_least(self.initial_probe_factor, 1.0):
            problems.append("initial_probe_factor is at least 1")
        if problems:
            raise ValueError("invalid service config: " + "; ".join(problems))

    @property
    def live(self) -> bool:
        return self.reuse_ar_prefix or self.full_answer_screen


def _to_cpu(value):
    """A detached CPU copy of a (nested) state value."""
    if isinstance(value, Tensor):
        return value.detach().to("cpu", copy=True)
    if isinstance(value, dict):
        return {k: _to_cpu(v) for k, v in value.items()}
    if isinstance(value, (list, tuple)):
        return type(value)(_to_cpu(v) for v in value)
    return value


def _rate(tokens: float, seconds: float) -> float:
    return tokens / seconds


class ColdStartService:
    """Budgeted learning and publication around a one-request-at-a-time service."""

    def __init__(self, model, fit: FitConfig, config: ServiceConfig = ServiceConfig(), *, gate_prompts=(),
                 sampling: SamplingConfig = SamplingConfig(1.0)):
        if config.live and not gate_prompts:
            raise ValueError("live validation still needs gate prompts for the trials after publication")
        _settle(model)
        opened = time.perf_counter()
        self.learner = FullBlockLearner(model, fit)
        self.model, self.fit, self.config = model, fit, config
        self.branch = MaskedAttentionBranch(model)
        self.sampling = sampling
        self.sampler = ProposalSampler(sampling)
        self.budget = TimeBudget(config.fraction)
        self.replay = CleanReplay(config.replay_records, fit.sequence_length, model.config.block_size, fit.seed)
        self.gate_prompts = tuple(p.detach().clone() for p in gate_prompts)
        self.speculating = False
        self.tokens = 0
        self.requests = 0
        self.next_probe = config.probe_every
        self.step_estimate = config.initial_step_estimate
        self.probe_estimate = 0.0
        self.last_probe = None
        self.pending_live: list[dict] = []
        self.full_gate = None
        if config.full_answer_screen:
            self.full_gate = FullAnswerGate(config.screen_requests, config.screen_margin,
                                            config.initial_screen_estimate,
                                            reuse_speculative=config.reuse_speculative_answers)
        _settle(model)
        self.budget.charge("setup", time.perf_counter() - opened)

    # ---- generation and accounting ----------------------------------------------------------------------------
    def _charged(self, kind: str, work):
        """Run ``work`` as maintenance of ``kind``; returns (its result, the seconds charged)."""
        _settle(self.model)
        started = time.perf_counter()
        try:
            result = work()
        finally:
            _settle(self.model)
            elapsed = time.perf_counter() - started
            self.budget.charge(kind, elapsed)
        return result, elapsed

    def _answer(self, prompt: Tensor, budget: int, *, speculative: bool, seed: int, prefix_tokens=None):
        generator = torch.Generator(device=prompt.device).manual_seed(seed)
        common = dict(sampling=self.sampling, eos_id=self.model.config.eos_token_id, generator=generator,
                      sampler=self.sampler)
        if speculative:
            return generate(self.branch, prompt, budget, **common)
        if prefix_tokens is not None:
            common["prefix_tokens"] = prefix_tokens
        return generate_ar(self.branch, prompt, budget, **common)

    def _run_pair(self, prompt: Tensor, budget: int, seed: int, legs: list[str]) -> dict:
        """Answer ``prompt`` once per leg ('candidate', 'ar' or 'serving'), in the given order."""
        out = {}
        for leg in legs:
            if leg == "candidate":
                with self.learner.candidate():
                    out[leg] = self._answer(prompt, budget, speculative=True, seed=seed)
            else:
                out[leg] = self._answer(prompt, budget, speculative=leg == "serving" and self.speculating,
                                        seed=seed)
        return out

    def _reference_kind(self) -> str:
        return "delivered_speculative_full" if self.speculating else "delivered_ar_full"

    # ---- decisions ---------------------------------------------------------------------------------------------
    def _settle_trial(self, record: dict) -> None:
        self.last_probe = record
        if not record.get("complete", True):
            return
        if record["passed"]:
            self._charged("publication", self.learner.publish)
            self.speculating = True
        elif record.get("fallback", False):
            self.speculating = False
        self.next_probe = self.learner.steps + self.config.probe_every

    # ---- gate-prompt trials ------------------------------------------------------------------------------------
    def _gate_trial(self) -> dict:
        legs = ["baseline", "candidate"] + (["ar"] if self.speculating else [])
        runs = []
        for i, prompt in enumerate(self.gate_prompts):
            order = legs[::-1] if i % 2 else legs          # alternate against first-run timing bias
            named = {"serving" if leg == "baseline" else leg: leg for leg in order}
            got = self._run_pair(prompt, self.config.probe_tokens, self.config.seed + 100000 + i, list(named))
            runs.append({named[k]: v for k, v in got.items()})
        baseline = [r["baseline"] for r in runs]
        candidate = [r["candidate"] for r in runs]
        ar = [r.get("ar", r["baseline"]) for r in runs]

        def pooled(results):
            return _rate(sum(len(r.tokens) for r in results), sum(r.seconds for r in results))

        paired = [c.tps / b.tps for b, c in zip(baseline, candidate)]
        against_ar = [c.tps / a.tps for a, c in zip(ar, candidate)]
        margin = self.config.publish_margin
        return {"step": self.learner.steps, "paired_ratios": paired, "ratio": pooled(candidate) / pooled(baseline),
                "candidate_over_ar": pooled(candidate) / pooled(ar),
                "fallback": self.speculating and pooled(baseline) < pooled(ar),
                "passed": min(paired + against_ar) >= margin}

    def _gate_trial_cost(self) -> float:
        legs = 3 if self.speculating else 2
        if self.probe_estimate:
            return self.probe_estimate * legs / 2
        speed = self.tokens / self.budget.service_seconds if self.budget.service_seconds else 1.0
        work = legs * len(self.gate_prompts) * self.config.probe_tokens / speed
        return self.config.initial_probe_factor * work

    # ---- live AR-prefix trials ---------------------------------------------------------------------------------
    def _prefix_trial(self, prompt: Tensor, delivered, seed: int) -> dict:
        """The candidate against the timed prefix of the delivered AR answer (same prompt and seed)."""
        with self.learner.candidate():
            trial = self._answer(prompt, delivered.prefix_tokens, speculative=True, seed=seed)
        row = {"step": self.learner.steps, "reference_tokens": delivered.prefix_tokens,
               "reference_seconds": delivered.prefix_seconds, "candidate_tokens": len(trial.tokens),
               "candidate_seconds": trial.seconds}
        if self.pending_live and self.pending_live[0]["step"] != row["step"]:
            raise RuntimeError("pooled prefix trials must all come from one learning version")
        self.pending_live.append(row)
        pooled = {k: sum(r[k] for r in self.pending_live) for k in row if k != "step"}
        speed_ratio = (_rate(pooled["candidate_tokens"], pooled["candidate_seconds"])
                       / _rate(pooled["reference_tokens"], pooled["reference_seconds"]))
        per_trial = [_rate(r["candidate_tokens"], r["candidate_seconds"])
                     / _rate(r["reference_tokens"], r["reference_seconds"]) for r in self.pending_live]
        complete = len(self.pending_live) == self.config.live_probe_requests
        record = {**row, **pooled, "reference_kind": "delivered_ar_prefix", "paired_ratios": per_trial,
                  "ratio": speed_ratio, "candidate_over_ar": speed_ratio, "probe_requests": len(self.pending_live),
                  "complete": complete, "passed": complete and speed_ratio >= self.config.publish_margin,
                  "fallback": False}
        if complete:
            self.pending_live = []
        return record

    # ---- full-answer screens and confirmations -----------------------------------------------------------------
    def _screen(self, prompt: Tensor, delivered, budget: int, seed: int) -> dict:
        with self.learner.candidate():
            trace = estimate_trace(self.branch, prompt, prompt.new_tensor(delivered.tokens), output_budget=budget,
                                   prefill_seconds=delivered.prefix_seconds, sampler=self.sampler,
                                   sampling=self.sampling, eos_id=self.model.config.eos_token_id,
                                   generator=torch.Generator(device=prompt.device).manual_seed(seed + 300000))
        return {"step": self.learner.steps, "stage": "screen", "reference_kind": self._reference_kind(),
                "reference_step": self.learner.serving_step if self.speculating else 0,
                "reference_tokens": len(delivered.tokens),
                "reference_seconds": delivered.seconds - delivered.prefix_capture_seconds,
                "predicted_seconds": trace.predicted_seconds, "virtual_forwards": float(trace.work.decode_forwards),
                "evaluation_seconds": trace.measured_seconds, "score_seconds": trace.score_seconds,
                "calibration_seconds": trace.calibration_seconds}

    def _confirm(self, prompt: Tensor, delivered, budget: int, seed: int) -> dict:
        legs = ["candidate", "ar"] if self.speculating else ["candidate"]
        if self.requests % 2:
            legs.reverse()
        runs = self._run_pair(prompt, budget, seed, legs)
        trial, ar = runs["candidate"], runs.get("ar", delivered)
        ratio, over_ar = trial.tps / delivered.tps, trial.tps / ar.tps
        return {"step": self.learner.steps, "stage": "confirmation", "reference_kind": self._reference_kind(),
                "ratio": ratio, "candidate_over_ar": over_ar, "paired_ratios": [ratio], "complete": True,
                "passed": min(ratio, over_ar) >= self.config.publish_margin,
                "fallback": self.speculating and delivered.tps < ar.tps, "ar_tps": ar.tps,
                "reference_tokens": len(delivered.tokens), "reference_seconds": delivered.seconds,
                "candidate_tokens": len(trial.tokens), "candidate_seconds": trial.seconds}

    def _live_trial(self, prompt: Tensor, delivered, budget: int, seed: int):
        """One live validation step on the delivered answer when its policy applies and the budget admits it."""
        cfg = self.config
        if cfg.reuse_ar_prefix:
            if self.speculating or not delivered.prefix_tokens:
                return None
            estimate = self.probe_estimate or cfg.initial_probe_factor * delivered.prefix_seconds
            if not self.budget.admits(estimate):
                return None
            record, elapsed = self._charged("validation", lambda: self._prefix_trial(prompt, delivered, seed))
            self.probe_estimate = 1.2 * elapsed
            self._settle_trial(record)
            return record
        gate = self.full_gate
        if (self.speculating and not cfg.reuse_speculative_answers) or not delivered.tokens:
            return None
        if not self.budget.admits(gate.estimate):
            return None
        if gate.ready:
            record, _ = self._charged("validation", lambda: self._confirm(prompt, delivered, budget, seed))
            gate.confirmed(ar_tps=record["ar_tps"] if cfg.reuse_speculative_answers else None)
            self._settle_trial(record)
            return record
        try:
            row, elapsed = self._charged("validation", lambda: self._screen(prompt, delivered, budget, seed))
        except TraceSupportError:
            return None                      # the recomputed target law cannot explain this answer
        record = gate.observe(row, elapsed)
        self.last_probe = record
        if record["complete"]:
            self.next_probe = self.learner.steps + cfg.probe_every
        return record

    # ---- serving -----------------------------------------------------------------------------------------------
    def serve(self, prompt: Tensor, max_new_tokens: int, *, seed: int):
        """Answer one request, then spend admitted maintenance on it; returns (Generation, report)."""
        cfg = self.config
        speculative = self.speculating
        prefix = cfg.probe_tokens if cfg.reuse_ar_prefix and not speculative else None
        _settle(self.model)
        started = time.perf_counter()
        answer = self._answer(prompt, max_new_tokens, speculative=speculative, seed=seed, prefix_tokens=prefix)
        _settle(self.model)
        self.budget.delivered(time.perf_counter() - started)
        self.tokens += len(answer.tokens)
        self.requests += 1

        def keep():
            if answer.tokens:
                full = torch.cat((prompt.detach().to("cpu", torch.long), torch.tensor([answer.tokens])), dim=1)
                self.replay.append(full)

        self._charged("collection", keep)
        due = bool(self.gate_prompts) and self.learner.steps >= self.next_probe
        update = None
        can_learn = self.replay.records and self.learner.steps < self.fit.steps
        if not due and can_learn and self.budget.admits(self.step_estimate):
            micro = self.replay.batch(self.fit.accumulate, self.fit.anchors_per_sequence, batch_size=self.fit.batch_size)
            update, elapsed = self._charged("training", lambda: self.learner.step(micro))
            self.step_estimate = max(1.2 * elapsed, 0.8 * self.step_estimate)
            update["seconds"] = elapsed
        probe = None
        if due:
            if cfg.live and (not self.speculating or cfg.reuse_speculative_answers):
                probe = self._live_trial(prompt, answer, max_new_tokens, seed)
            elif self.budget.admits(self._gate_trial_cost()):
                probe, elapsed = self._charged("validation", self._gate_trial)
                self.probe_estimate = 1.2 * elapsed
                self._settle_trial(probe)
        report = {"request": self.requests, "mode": "speculative" if speculative else "ar", "update": update,
                  "probe": probe, **self.summary()}
        return answer, report

    def summary(self) -> dict:
        wall = self.budget.service_seconds + self.budget.spent
        return {"delivered_tokens": self.tokens, "steps": self.learner.steps,
                "serving_step": self.learner.serving_step, "speculating": self.speculating,
                "net_tps": self.tokens / wall if wall else 0.0, "budget": self.budget.summary()}

    # ---- persistence -------------------------------------------------------------------------------------------
    def state_dict(self) -> dict:
        self.learner.check()
        return {"format": STATE_FORMAT, "fit": asdict(self.fit), "controller": asdict(self.config),
                "sampling": asdict(self.sampling), "model_config": self.model.config.to_dict(),
                "base_fingerprint": frozen_fingerprint(self.model), "master": _to_cpu(self.learner.master),
                "optimizer": _to_cpu(self.learner.optimizer.state_dict()),
                "serving": _to_cpu(self.learner.execution), "step": self.learner.steps,
                "serving_step": self.learner.serving_step, "speculating": self.speculating,
                "gate_prompts": _to_cpu(list(self.gate_prompts)), "replay": _to_cpu(list(self.replay.records)),
                "replay_rng": self.replay.rng.get_state(), "anchors_rng": self.replay.anchors_rng.get_state(),
                "budget": self.budget.summary(), "tokens": self.tokens, "requests": self.requests,
                "next_probe": self.next_probe, "step_estimate": self.step_estimate,
                "probe_estimate": self.probe_estimate, "pending_live": [dict(r) for r in self.pending_live],
                "full_gate": None if self.full_gate is None else self.full_gate.state_dict()}

    def _check_saved(self, state: dict) -> None:
        same_policies = (state.get("format") == STATE_FORMAT
                         and set(state.get("fit", {})) == {f.name for f in fields(FitConfig)}
                         and FitConfig(**state["fit"]) == self.fit
                         and ServiceConfig(**state["controller"]) == self.config
                         and state["sampling"] == asdict(self.sampling)
                         and state["model_config"] == self.model.config.to_dict()
                         and state["base_fingerprint"] == frozen_fingerprint(self.model))
        if not same_policies:
            raise ValueError("the saved service has another format, frozen base, or training/sampling policy")
        prompts = state.get("gate_prompts", [])
        if len(prompts) != len(self.gate_prompts) or not all(torch.equal(a.cpu(), b.cpu())
                                                              for a, b in zip(prompts, self.gate_prompts)):
            raise ValueError("the saved service was gated on other prompts")
        for key, live in (("master", self.learner.master), ("serving", self.learner.execution)):
            saved = state[key]
            if saved.keys() != live.keys() or not all(
                    v.shape == live[n].shape and v.dtype == live[n].dtype and bool(torch.isfinite(v).all())
                    for n, v in saved.items()):
                raise ValueError(f"the saved {key} tensors do not match the draft parameters")
        if not 0 <= state["serving_step"] <= state["step"] <= self.fit.steps:
            raise ValueError("the saved learning and publication counters are inconsistent")
        if state["speculating"] and state["serving_step"] == 0:
            raise ValueError("a speculative service must have published a version")
        if len(state["replay"]) > self.config.replay_records:
            raise ValueError("the saved replay exceeds its capacity")
        pending = state.get("pending_live", [])
        if len(pending) >= self.config.live_probe_requests or any(r["step"] != state["step"] for r in pending):
            raise ValueError("pending live trials must be fewer than a decision and from the saved version")
        if (self.full_gate is None) != (state.get("full_gate") is None):
            raise ValueError("the saved service used another validation policy")

    def load_state_dict(self, state: dict) -> None:
        """Restore into a fresh service over the same frozen model and policies; the restore time is charged."""
        _settle(self.model)
        started = time.perf_counter()
        if self.requests or self.learner.steps or self.replay.records:
            raise ValueError("restore into a fresh service instance")
        self._check_saved(state)
        with torch.no_grad():
            for name, param in self.learner.master.items():
                param.copy_(state["master"][name])
        self.learner._install(state["serving"])
        self.learner.optimizer.load_state_dict(state["optimizer"])
        self.learner.steps, self.learner.serving_step = state["step"], state["serving_step"]
        self.speculating, self.next_probe = state["speculating"], state["next_probe"]
        self.step_estimate, self.probe_estimate = state["step_estimate"], state["probe_estimate"]
        self.pending_live = [dict(r) for r in state.get("pending_live", [])]
        if self.full_gate is not None:
            self.full_gate.load_state_dict(state["full_gate"], step=state["step"], next_probe=state["next_probe"],
                                           speculating=state["speculating"], requests=state["requests"],
                                           serving_step=state["serving_step"])
        self.replay.records.clear()
        self.replay.records.extend(r.clone() for r in state["replay"])
        self.replay.rng.set_state(state["replay_rng"])
        self.replay.anchors_rng.set_state(state["anchors_rng"])
        self.tokens, self.requests = state["tokens"], state["requests"]
        saved = state["budget"]
        restored = TimeBudget(self.config.fraction, saved["service_seconds"], saved["costs"])
        _settle(self.model)
        restored.charge("resume", self.budget.spent + time.perf_counter() - started)
        self.budget = restored


__all__ = ["CleanReplay", "ColdStartService", "FullBlockLearner", "ServiceConfig", "TimeBudget"]
