"""Cold start: serve autoregressively, learn the draft view in a bounded time budget, publish when faster.

A service that starts from a dual-view model whose draft attention has never
been trained:

* ``TimeBudget``: maintenance work (training steps, probes, publication,
  collection) earns credit at ``fraction`` of the delivered generation time; an
  operation is admitted only if its estimated duration fits the credit, and an
  operation that overruns its estimate leaves a debt that later deliveries
  repay.
* ``CleanReplay``: bounded store of completed responses; training batches are
  contiguous crops with random anchors (the offline distillation layout), so
  the draft only ever reads clean positions before its own anchor.
* ``FullBlockLearner``: fp32 masters of every draft attention projection,
  initialised from the AR attention, updated by the offline distillation step
  (full-vocabulary KL to the AR view); the serving copy changes only at
  ``publish`` -- ``candidate()`` installs the masters for a trial and always
  restores the serving weights.
* ``ColdStartService.serve``: answers with the current mode (AR until a version
  is published, speculative afterwards), collects the response, trains when the
  budget admits, and every ``probe_every`` steps runs paired trials on held-out
  gate prompts (same prompt, output cap and seed; alternating order) and
  publishes when every paired throughput ratio clears ``publish_margin``
  (falling back to AR when the published version stops beating AR).

Live validation policies (one at a time) replace the gate-prompt probe while
the service still answers autoregressively:

* ``reuse_ar_prefix``: the delivered AR answer's first ``probe_tokens`` outputs
  are timed as the reference; the candidate answers the same prompt and seed for
  that many tokens; ``live_probe_requests`` such trials of one learning version
  are pooled into one decision;
* ``full_answer_screen``: the candidate is screened on delivered answers with
  the exact conditional work law (``virtual_work.estimate_trace``) against the
  measured answer time (``FullAnswerGate``); a screen that clears its margin
  earns one fresh paired full-request confirmation, which decides publication.
  With ``reuse_speculative_answers`` the screen continues after publication
  against the serving speculative version.

``state_dict`` / ``load_state_dict`` (format ``cold-start-research-v1``) keep the
request-boundary state: masters, optimizer, serving weights, replay with its
random states, counters, pending live evidence and the budget.

Reference behaviour: online-speculation/ablation/src/blockspec_ablation/cold_start.py:42-663.
"""

from __future__ import annotations

import math
import time
from collections import deque
from contextlib import contextmanager
from dataclasses import asdict, dataclass, field

import torch

from .fitting import FitConfig, frozen_fingerprint
from .generation import MaskedAttentionBranch, ProposalSampler, generate, generate_ar
from .sampling import SamplingConfig
from .training import distillation_update, sample_anchors
from .virtual_work import FullAnswerGate, TraceSupportError, estimate_trace


def _sync(model):
    dev = next(model.parameters()).device
    if dev.type == "cuda":
        torch.cuda.synchronize(dev)


@dataclass
class TimeBudget:
    fraction: float = 0.01
    service_seconds: float = 0.0
    costs: dict = field(default_factory=dict)

    def __post_init__(self):
        if not math.isfinite(self.fraction) or not 0 < self.fraction <= 0.1:
            raise ValueError("time fraction must lie in (0, 0.1]")

    @property
    def spent(self) -> float:
        return sum(self.costs.values())

    @property
    def credit(self) -> float:
        return self.fraction * self.service_seconds - self.spent

    def delivered(self, seconds: float) -> None:
        if not math.isfinite(seconds) or seconds < 0:
            raise ValueError("finite nonnegative service duration required")
        self.service_seconds += seconds

    def charge(self, kind: str, seconds: float) -> None:
        if not math.isfinite(seconds) or seconds < 0:
            raise ValueError("finite nonnegative maintenance duration required")
        self.costs[kind] = self.costs.get(kind, 0.0) + seconds

    def admits(self, estimate: float) -> bool:
        if not math.isfinite(estimate) or estimate <= 0:
            raise ValueError("finite positive operation estimate required")
        return self.credit >= estimate

    def summary(self) -> dict:
        return {"fraction": self.fraction, "service_seconds": self.service_seconds, "costs": dict(self.costs),
                "extra_seconds": self.spent,
                "extra_over_service": self.spent / self.service_seconds if self.service_seconds else None,
                "remaining_credit_seconds": self.credit, "debt_seconds": max(0.0, -self.credit)}


class CleanReplay:
    def __init__(self, capacity: int, sequence_length: int, block_size: int, seed: int):
        if (min(capacity, sequence_length, block_size) < 1 or sequence_length < block_size or block_size < 2):
            raise ValueError("positive replay capacity and complete training blocks required")
        self.records: deque = deque(maxlen=capacity)
        self.sequence_length, self.block_size = sequence_length, block_size
        self.rng = torch.Generator().manual_seed(seed)
        self.anchors_rng = torch.Generator().manual_seed(seed + 1)

    def append(self, tokens: torch.Tensor) -> None:
        if tokens.ndim != 2 or tokens.shape[0] != 1 or tokens.dtype != torch.long:
            raise ValueError("one complete integer-token record required")
        if tokens.shape[1] >= self.block_size:
            self.records.append(tokens.detach().cpu().clone())

    def batch(self, count: int, anchors_per_sequence: int, *, batch_size: int = 1):
        if not self.records or count < 1 or batch_size < 1:
            raise ValueError("nonempty replay and positive microbatch/window counts required")
        out = []
        for _ in range(count):
            rows, anchors = [], []
            for _ in range(batch_size):
                rec = self.records[int(torch.randint(len(self.records), (), generator=self.rng))]
                n = min(self.sequence_length, rec.shape[1])
                start = int(torch.randint(rec.shape[1] - n + 1, (), generator=self.rng))
                crop = rec[:, start:start + n].clone()
                rows.append(crop[0])
                anchors.append(sample_anchors(crop, self.block_size, anchors_per_sequence,
                                              generator=self.anchors_rng))
            out.append((torch.nn.utils.rnn.pad_sequence(rows, batch_first=True, padding_value=0),
                        torch.cat(anchors)))
        return out


class FullBlockLearner:
    def __init__(self, model, config: FitConfig):
        if (not isinstance(config, FitConfig) or config.sequence_length < model.config.block_size
                or any(p.requires_grad for p in model.parameters())):
            raise ValueError("a frozen model and a full-block configuration are required")
        self.model, self.config = model, config
        model.initialize_draft_from_ar()
        model.eval()
        self.execution = {n: p for n, p in model.named_parameters() if ".attention.draft." in n}
        self.master = {n: torch.nn.Parameter(p.detach().float().clone()) for n, p in self.execution.items()}
        self.optimizer = config.make_optimizer(list(self.master.values()))
        self.frozen = [(p, p._version) for n, p in model.named_parameters() if n not in self.execution]
        self.steps = self.serving_step = 0

    def check(self) -> None:
        if any(p.requires_grad for p in self.model.parameters()) or any(p._version != v for p, v in self.frozen):
            raise RuntimeError("AR/shared parameters and serving execution must remain fixed")

    def step(self, batches) -> dict:
        self.check()
        if self.steps >= self.config.steps:
            raise ValueError("the learning schedule has finished")
        dev = next(self.model.parameters()).device
        batches = [(t.to(dev), a.to(dev)) for t, a in batches]
        m = distillation_update(self.model, batches, self.optimizer, learning_rate=self.config.rate(self.steps),
                                clip_grad=self.config.clip_grad, chunk_rows=self.config.chunk_rows,
                                master=self.master)
        self.steps += 1
        self.check()
        return {"step": self.steps, **m}

    @torch.no_grad()
    def publish(self) -> None:
        self.check()
        for n, p in self.execution.items():
            p.copy_(self.master[n])
        self.serving_step = self.steps

    @contextmanager
    def candidate(self):
        """Install the latest masters for a trial; restore the serving weights afterwards, even on failure."""
        self.check()
        saved = {n: p.detach().clone() for n, p in self.execution.items()}
        old = self.serving_step
        try:
            self.publish()
            yield
        finally:
            with torch.no_grad():
                for n, p in self.execution.items():
                    p.copy_(saved[n])
            self.serving_step = old


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
        flags = (self.reuse_ar_prefix, self.full_answer_screen, self.reuse_speculative_answers)
        if any(type(f) is not bool for f in flags) or (self.reuse_ar_prefix and self.full_answer_screen):
            raise ValueError("select at most one explicit live validation policy")
        if self.reuse_speculative_answers and not self.full_answer_screen:
            raise ValueError("reusing speculative answers requires full-answer screening")
        FullAnswerGate(self.screen_requests, self.screen_margin, self.initial_screen_estimate)
        if (type(self.live_probe_requests) is not int or self.live_probe_requests < 1
                or (self.live_probe_requests > 1 and not self.reuse_ar_prefix)):
            raise ValueError("several pooled live trials require AR-prefix validation")
        if (min(self.replay_records, self.probe_every, self.probe_tokens) < 1
                or not math.isfinite(self.publish_margin) or self.publish_margin <= 1
                or not math.isfinite(self.initial_step_estimate) or self.initial_step_estimate <= 0
                or not math.isfinite(self.initial_probe_factor) or self.initial_probe_factor < 1):
            raise ValueError("positive replay/probe sizes, cost estimate and publication margin > 1 required")


def _portable(obj):
    if isinstance(obj, torch.Tensor):
        return obj.detach().cpu().clone()
    if isinstance(obj, dict):
        return {k: _portable(v) for k, v in obj.items()}
    if isinstance(obj, (list, tuple)):
        return type(obj)(_portable(v) for v in obj)
    return obj


class ColdStartService:
    """AR service with budget-admitted draft learning and paired publication trials (calls are serialised)."""

    def __init__(self, model, fit: FitConfig, config: ServiceConfig = ServiceConfig(), *, gate_prompts=(),
                 sampling: SamplingConfig = SamplingConfig(1.0)):
        if (config.reuse_ar_prefix or config.full_answer_screen) and not gate_prompts:
            raise ValueError("gate prompts are required for the trials after publication")
        _sync(model)
        t0 = time.perf_counter()
        self.learner = FullBlockLearner(model, fit)
        self.model, self.config, self.fit = model, config, fit
        self.branch = MaskedAttentionBranch(model)
        self.budget = TimeBudget(config.fraction)
        self.replay = CleanReplay(config.replay_records, fit.sequence_length, model.config.block_size, fit.seed)
        self.sampling = sampling
        self.sampler = ProposalSampler(sampling)
        self.gate_prompts = tuple(p.detach().clone() for p in gate_prompts)
        self.speculating = False
        self.next_probe = config.probe_every
        self.step_estimate = config.initial_step_estimate
        self.probe_estimate = 0.0
        self.tokens = self.requests = 0
        self.last_probe = None
        self.pending_live: list[dict] = []
        self.full_gate = (FullAnswerGate(config.screen_requests, config.screen_margin, config.initial_screen_estimate,
                                         reuse_speculative=config.reuse_speculative_answers)
                          if config.full_answer_screen else None)
        _sync(model)
        self.budget.charge("setup", time.perf_counter() - t0)

    def _timed(self, kind, action):
        _sync(self.model)
        t0 = time.perf_counter()
        try:
            return action()
        finally:
            _sync(self.model)
            self.budget.charge(kind, time.perf_counter() - t0)

    def _generate(self, prompt, tokens, *, speculative, seed, prefix_tokens=None):
        g = torch.Generator(device=prompt.device).manual_seed(seed)
        kw = {} if prefix_tokens is None else {"prefix_tokens": prefix_tokens}
        fn = generate if speculative else generate_ar
        return fn(self.branch, prompt, tokens, sampling=self.sampling, eos_id=self.model.config.eos_token_id,
                  generator=g, sampler=self.sampler, **kw)

    # ---- live validation on delivered requests ----
    def _live_prefix(self, prompt, reference, seed) -> dict:
        """Candidate vs the delivered AR answer's timed prefix (same prompt and seed, so the
        candidate's exact sampler reproduces that prefix)."""
        with self.learner.candidate():
            cand = self._generate(prompt, reference.prefix_tokens, speculative=True, seed=seed)
        row = {"step": self.learner.steps, "reference_tokens": reference.prefix_tokens,
               "reference_seconds": reference.prefix_seconds, "candidate_tokens": len(cand.tokens),
               "candidate_seconds": cand.seconds}
        if any(r["step"] != row["step"] for r in self.pending_live):
            raise RuntimeError("pooled prefix trials require one learning version")
        self.pending_live.append(row)
        keys = ("reference_tokens", "reference_seconds", "candidate_tokens", "candidate_seconds")
        tot = {k: sum(r[k] for r in self.pending_live) for k in keys}
        ratio = (tot["candidate_tokens"] / tot["candidate_seconds"]) / (tot["reference_tokens"] /
                                                                          tot["reference_seconds"])
        ratios = [(r["candidate_tokens"] / r["candidate_seconds"]) / (r["reference_tokens"] / r["reference_seconds"])
                  for r in self.pending_live]
        complete = len(self.pending_live) == self.config.live_probe_requests
        out = {**row, **tot, "reference_kind": "delivered_ar_prefix", "paired_ratios": ratios, "ratio": ratio,
               "candidate_over_ar": ratio, "probe_requests": len(self.pending_live), "complete": complete,
               "passed": complete and ratio >= self.config.publish_margin, "fallback": False}
        if complete:
            self.pending_live = []
        return out

    def _screen(self, prompt, reference, tokens, seed) -> dict:
        with self.learner.candidate():
            t = estimate_trace(self.branch, prompt, prompt.new_tensor(reference.tokens), output_budget=tokens,
                               prefill_seconds=reference.prefix_seconds, sampler=self.sampler,
                               sampling=self.sampling, eos_id=self.model.config.eos_token_id,
                               generator=torch.Generator(device=prompt.device).manual_seed(seed + 300000))
        return {"step": self.learner.steps, "stage": "screen",
                "reference_kind": "delivered_speculative_full" if self.speculating else "delivered_ar_full",
                "reference_step": self.learner.serving_step if self.speculating else 0,
                "reference_tokens": len(reference.tokens),
                "reference_seconds": reference.seconds - reference.prefix_capture_seconds,
                "predicted_seconds": t.predicted_seconds, "virtual_forwards": float(t.work.decode_forwards),
                "evaluation_seconds": t.measured_seconds, "score_seconds": t.score_seconds,
                "calibration_seconds": t.calibration_seconds}

    def _confirm(self, prompt, reference, tokens, seed) -> dict:
        pair = {}
        names = ["candidate", "ar"] if self.speculating else ["candidate"]
        if self.requests % 2:
            names.reverse()
        for name in names:
            if name == "candidate":
                with self.learner.candidate():
                    pair[name] = self._generate(prompt, tokens, speculative=True, seed=seed)
            else:
                pair[name] = self._generate(prompt, tokens, speculative=False, seed=seed)
        cand, ar = pair["candidate"], pair.get("ar", reference)
        ratio, vs_ar = cand.tps / reference.tps, cand.tps / ar.tps
        return {"step": self.learner.steps, "stage": "confirmation",
                "reference_kind": "delivered_speculative_full" if self.speculating else "delivered_ar_full",
                "ratio": ratio, "candidate_over_ar": vs_ar, "paired_ratios": [ratio], "complete": True,
                "passed": min(ratio, vs_ar) >= self.config.publish_margin,
                "fallback": self.speculating and reference.tps < ar.tps, "ar_tps": ar.tps,
                "reference_tokens": len(reference.tokens), "reference_seconds": reference.seconds,
                "candidate_tokens": len(cand.tokens), "candidate_seconds": cand.seconds}

    def _decide(self, probe: dict) -> None:
        self.last_probe = probe
        if not probe.get("complete", True):
            return
        if probe["passed"]:
            self._timed("publication", self.learner.publish)
            self.speculating = True
        elif probe.get("fallback", False):
            self.speculating = False
        self.next_probe = self.learner.steps + self.config.probe_every

    def _live(self, prompt, result, max_new_tokens, seed):
        """One live validation step on the delivered request, if its policy applies and the
        budget admits it; returns the trial record or None."""
        cfg = self.config
        if cfg.reuse_ar_prefix and not self.speculating and result.prefix_tokens:
            est = (self.probe_estimate or
                   cfg.initial_probe_factor * result.prefix_seconds)
            if not self.budget.admits(est):
                return None
            before = self.budget.spent
            probe = self._timed("validation", lambda: self._live_prefix(prompt, result, seed))
            self.probe_estimate = 1.2 * (self.budget.spent - before)
            self._decide(probe)
            return probe
        gate = self.full_gate
        if gate is not None and (not self.speculating or cfg.reuse_speculative_answers) and result.tokens:
            if not self.budget.admits(gate.estimate):
                return None
            before = self.budget.spent
            if gate.ready:
                probe = self._timed("validation", lambda: self._confirm(prompt, result, max_new_tokens, seed))
                gate.confirmed(ar_tps=probe["ar_tps"] if cfg.reuse_speculative_answers else None)
                self._decide(probe)
                return probe
            try:
                row = self._timed("validation", lambda: self._screen(prompt, result, max_new_tokens, seed))
            except TraceSupportError:
                return None      # the recomputed target law cannot explain this answer: no evidence
            out = gate.observe(row, self.budget.spent - before)
            self.last_probe = out
            if out["complete"]:
                self.next_probe = self.learner.steps + cfg.probe_every
            return out
        return None

    def _probe(self) -> dict:
        base, cand, ar = [], [], []
        for i, prompt in enumerate(self.gate_prompts):
            seed = self.config.seed + 100000 + i
            names = ["baseline", "candidate"] + (["ar"] if self.speculating else [])
            if i % 2:
                names.reverse()       # alternate the order against first-run timing bias
            pair = {}
            for name in names:
                if name == "candidate":
                    with self.learner.candidate():
                        pair[name] = self._generate(prompt, self.config.probe_tokens, speculative=True, seed=seed)
                else:
                    pair[name] = self._generate(prompt, self.config.probe_tokens,
                                                speculative=self.speculating and name != "ar", seed=seed)
            base.append(pair["baseline"])
            cand.append(pair["candidate"])
            ar.append(pair.get("ar", pair["baseline"]))
        ratios = [c.tps / b.tps for b, c in zip(base, cand)]
        vs_ar = [c.tps / a.tps for a, c in zip(ar, cand)]

        def total(rows):
            return sum(len(r.tokens) for r in rows) / sum(r.seconds for r in rows)

        return {"step": self.learner.steps, "paired_ratios": ratios, "ratio": total(cand) / total(base),
                "candidate_over_ar": total(cand) / total(ar),
                "fallback": self.speculating and total(base) < total(ar),
                "passed": all(r >= self.config.publish_margin for r in ratios + vs_ar)}

    def _probe_cost(self) -> float:
        legs = 3 if self.speculating else 2
        if self.probe_estimate:
            return self.probe_estimate / 2 * legs
        tps = self.tokens / self.budget.service_seconds if self.budget.service_seconds else 1.0
        return self.config.initial_probe_factor * legs * len(self.gate_prompts) * self.config.probe_tokens / tps

    def serve(self, prompt: torch.Tensor, max_new_tokens: int, *, seed: int):
        speculative = self.speculating
        prefix = self.config.probe_tokens if (self.config.reuse_ar_prefix and not speculative) else None
        _sync(self.model)
        t0 = time.perf_counter()
        result = self._generate(prompt, max_new_tokens, speculative=speculative, seed=seed, prefix_tokens=prefix)
        _sync(self.model)
        self.budget.delivered(time.perf_counter() - t0)
        self.tokens += len(result.tokens)
        self.requests += 1
        update = probe = None

        def collect():
            if result.tokens:
                self.replay.append(torch.cat((prompt.detach().cpu().long(),
                                              torch.tensor([result.tokens], dtype=torch.long)), 1))

        self._timed("collection", collect)
        due = bool(self.gate_prompts) and self.learner.steps >= self.next_probe
        if (not due and self.replay.records and self.learner.steps < self.fit.steps
                and self.budget.admits(self.step_estimate)):
            before = self.budget.spent
            update = self._timed("training", lambda: self.learner.step(
                self.replay.batch(self.fit.accumulate, self.fit.anchors_per_sequence, batch_size=self.fit.batch_size)))
            elapsed = self.budget.spent - before
            self.step_estimate = max(1.2 * elapsed, 0.8 * self.step_estimate)
            update["seconds"] = elapsed
        live = self.config.reuse_ar_prefix or self.config.full_answer_screen
        if due and live and (not self.speculating or self.config.reuse_speculative_answers):
            probe = self._live(prompt, result, max_new_tokens, seed)
        elif due and self.budget.admits(self._probe_cost()):
            before = self.budget.spent
            probe = self._timed("validation", self._probe)
            self.probe_estimate = 1.2 * (self.budget.spent - before)
            self._decide(probe)
        return result, {"request": self.requests, "mode": "speculative" if speculative else "ar", "update": update,
                        "probe": probe, **self.summary()}

    def summary(self) -> dict:
        elapsed = self.budget.service_seconds + self.budget.spent
        return {"delivered_tokens": self.tokens, "steps": self.learner.steps,
                "serving_step": self.learner.serving_step, "speculating": self.speculating,
                "net_tps": self.tokens / elapsed if elapsed else 0.0, "budget": self.budget.summary()}

    def state_dict(self) -> dict:
        self.learner.check()
        return {"format": "cold-start-research-v1", "fit": asdict(self.fit), "controller": asdict(self.config),
                "sampling": asdict(self.sampling), "model_config": self.model.config.to_dict(),
                "base_fingerprint": frozen_fingerprint(self.model), "master": _portable(self.learner.master),
                "optimizer": _portable(self.learner.optimizer.state_dict()),
                "serving": _portable(self.learner.execution), "step": self.learner.steps,
                "serving_step": self.learner.serving_step, "speculating": self.speculating,
                "gate_prompts": _portable(list(self.gate_prompts)), "replay": _portable(list(self.replay.records)),
                "replay_rng": self.replay.rng.get_state(), "anchors_rng": self.replay.anchors_rng.get_state(),
                "budget": self.budget.summary(), "tokens": self.tokens, "requests": self.requests,
                "next_probe": self.next_probe, "step_estimate": self.step_estimate,
                "probe_estimate": self.probe_estimate, "pending_live": [dict(r) for r in self.pending_live],
                "full_gate": None if self.full_gate is None else self.full_gate.state_dict()}

    def load_state_dict(self, state: dict) -> None:
        """Restore into a fresh service over the same frozen model and policies (restoring time is charged)."""
        _sync(self.model)
        t0 = time.perf_counter()
        if self.requests or self.learner.steps or self.replay.records:
            raise ValueError("restore into a fresh service instance")
        if (state.get("format") != "cold-start-research-v1" or FitConfig(**state["fit"]) != self.fit
                or ServiceConfig(**state["controller"]) != self.config
                or state["sampling"] != asdict(self.sampling)
                or state["model_config"] != self.model.config.to_dict()
                or state["base_fingerprint"] != frozen_fingerprint(self.model)):
            raise ValueError("saved stream must match its frozen base and training/sampling policies")
        saved_prompts = state.get("gate_prompts", [])
        if len(saved_prompts) != len(self.gate_prompts) or any(
                not torch.equal(a.cpu(), b.cpu()) for a, b in zip(saved_prompts, self.gate_prompts)):
            raise ValueError("restore requires the same publication gate prompts")
        for key, expected in (("master", self.learner.master), ("serving", self.learner.execution)):
            saved = state[key]
            if saved.keys() != expected.keys() or any(
                    v.shape != expected[n].shape or v.dtype != expected[n].dtype or not torch.isfinite(v).all()
                    for n, v in saved.items()):
                raise ValueError("matching finite learning and serving tensors required")
        if not (0 <= state["serving_step"] <= state["step"] <= self.fit.steps) or (
                state["speculating"] and state["serving_step"] == 0):
            raise ValueError("consistent learning and publication counters required")
        records = state["replay"]
        if len(records) > self.config.replay_records:
            raise ValueError("replay exceeds its capacity")
        with torch.no_grad():
            for n, p in self.learner.master.items():
                p.copy_(state["master"][n])
            for n, p in self.learner.execution.items():
                p.copy_(state["serving"][n])
        self.learner.optimizer.load_state_dict(state["optimizer"])
        self.learner.steps, self.learner.serving_step = state["step"], state["serving_step"]
        self.speculating, self.next_probe = state["speculating"], state["next_probe"]
        self.step_estimate, self.probe_estimate = state["step_estimate"], state["probe_estimate"]
        pending = state.get("pending_live", [])
        if len(pending) >= self.config.live_probe_requests or any(r["step"] != state["step"] for r in pending):
            raise ValueError("pending live trials must be fewer than a decision and from the saved version")
        self.pending_live = [dict(r) for r in pending]
        if (self.full_gate is None) != (state.get("full_gate") is None):
            raise ValueError("the saved stream and this service use different validation policies")
        if self.full_gate is not None:
            self.full_gate.load_state_dict(state["full_gate"], step=state["step"], next_probe=state["next_probe"],
                                           speculating=state["speculating"], requests=state["requests"],
                                           serving_step=state["serving_step"])
        self.replay.records.clear()
        self.replay.records.extend(r.clone() for r in records)
        self.replay.rng.set_state(state["replay_rng"])
        self.replay.anchors_rng.set_state(state["anchors_rng"])
        self.tokens, self.requests = state["tokens"], state["requests"]
        b = TimeBudget(self.config.fraction)
        b.delivered(state["budget"]["service_seconds"])
        for k, v in state["budget"]["costs"].items():
            b.charge(k, v)
        setup = self.budget.spent
        _sync(self.model)
        b.charge("resume", setup + time.perf_counter() - t0)
        self.budget = b


__all__ = ["CleanReplay", "ColdStartService", "FullBlockLearner", "ServiceConfig", "TimeBudget"]
