"""Conditional full-answer work of block speculation, and the full-answer screening gate.

Given a delivered autoregressive answer y_1..y_n, exact speculative rejection
correction accepts a drafted token y with probability min(1, q(y) / p(y))
conditional on y being the delivered token.  Integrating those acceptance
flags over the answer gives the expected number of draft rounds, verifier
forwards and AR-tail forwards the speculative decoder spends to deliver *this*
answer -- a per-answer work audit that needs no sampling.

* :func:`expected_work` -- the visit-mass recurrence over round starts
  (differentiable in the acceptance probabilities);
* :func:`inverse_acceptance` -- min(1, q / p) from log probabilities;
* :func:`score_trace` -- every round start of a completed answer scored in
  isolated anchor + mask blocks on the dual-view model (batched, row-chunked
  full-vocabulary normalisation);
* :func:`calibration_starts` / :func:`estimate_trace` -- visit-weighted timing
  of a few real rounds turns the work law into a predicted full-answer time;
* :class:`FullAnswerGate` -- fixed-version screening of a candidate draft
  against measured full-request times before a fresh confirmation trial.

Reference behaviour: online-speculation/ablation/src/blockspec_ablation/
virtual_work.py (work law, trace scoring, timing estimate) and
full_answer_gate.py (screening state).  Round semantics follow
:func:`online_speculation_b200.blockspec.generation.generate`: the first
output token comes from the prefill, a round after j committed tokens drafts
min(block, budget - j + 1) - 1 tokens, and a one-token remainder is an AR
tail step.
"""

from __future__ import annotations

import math
import time
from dataclasses import dataclass

import torch
from torch import Tensor
from torch.nn import functional as F

from .model import trim_cache
from .sampling import SamplingConfig, probabilities


class TraceSupportError(ValueError):
    """A delivered token has zero mass under the recomputed (possibly truncated) target law."""


@dataclass
class VirtualWork:
    """Expected visits per round start j = 1..n-1 (index j - 1)."""

    draft_visits: Tensor
    tail_visits: Tensor
    output_tokens: int

    @property
    def draft_forwards(self) -> Tensor:
        return self.draft_visits.sum()

    @property
    def verifier_forwards(self) -> Tensor:
        return self.draft_visits.sum()

    @property
    def tail_ar_forwards(self) -> Tensor:
        return self.tail_visits.sum()

    @property
    def decode_forwards(self) -> Tensor:
        return 2 * self.draft_forwards + self.tail_ar_forwards

    def cost(self, round_cost=2.0, tail_cost=1.0) -> Tensor:
        """Operation cost of the decode phase (the shared prefill excluded); the
        costs may be scalars or per-start tensors."""
        return (self.draft_visits * round_cost + self.tail_visits * tail_cost).sum()


def expected_work(acceptance: Tensor, *, output_tokens: int, output_budget: int, block_size: int) -> VirtualWork:
    """Visit masses of every round start, conditional on the delivered answer.

    ``acceptance[j - 1, o - 1]`` is the probability that, in a round started
    after j committed tokens, the o-th drafted token is accepted given that the
    delivered token there is y_{j+o}.  A rejection at offset o starts the next
    round after j + o tokens; a fully accepted round of m drafts plus the
    verifier's bonus token starts it after j + m + 1.  Offsets that reach the
    final token cannot change later work.
    """
    n, budget, block = output_tokens, output_budget, block_size
    if (any(type(v) is not int for v in (n, budget, block)) or not 0 <= n <= budget or block < 2
            or tuple(acceptance.shape) != (max(0, n - 1), block - 1) or not acceptance.is_floating_point()
            or not torch.isfinite(acceptance).all() or bool(((acceptance < 0) | (acceptance > 1)).any())):
        raise ValueError("finite acceptance probabilities of shape [n - 1, block - 1] and n <= budget required")
    zero = acceptance.sum() * 0
    if n <= 1:
        empty = acceptance.sum(1)
        return VirtualWork(empty, empty, n)
    mass = [zero] * (n + 1)            # mass[j]: a round starts after j committed tokens
    mass[1] = zero + 1
    draft, tail = [], []
    for j in range(1, n):
        v = mass[j]
        if budget - j == 1:            # one token left: plain AR step
            draft.append(zero)
            tail.append(v)
            continue
        draft.append(v)
        tail.append(zero)
        m = min(block, budget - j + 1) - 1
        alive = v
        for o in range(1, min(m, n - j - 1) + 1):
            a = acceptance[j - 1, o - 1]
            mass[j + o] = mass[j + o] + alive * (1 - a)
            alive = alive * a
        if j + m + 1 < n:
            mass[j + m + 1] = mass[j + m + 1] + alive
    return VirtualWork(torch.stack(draft), torch.stack(tail), n)


def inverse_acceptance(proposal_logp: Tensor, target_logp: Tensor) -> Tensor:
    """P(accept | delivered x) = min(1, q(x) / p(x)); delivered tokens need p(x) > 0."""
    if bool(torch.isneginf(target_logp).any()):
        raise TraceSupportError("delivered tokens require positive recomputed target mass")
    if (proposal_logp.shape != target_logp.shape or not bool(torch.isfinite(target_logp).all())
            or bool(torch.isnan(proposal_logp).any()) or bool(torch.isposinf(proposal_logp).any())
            or bool((proposal_logp > 0).any()) or bool((target_logp > 0).any())):
        raise ValueError("matching log probabilities with positive target mass required")
    return (proposal_logp - target_logp).clamp_max(0).exp()


@dataclass
class TraceScores:
    acceptance: Tensor          # [n - 1, block - 1], 1 where no draft scores the position
    proposal_logp: Tensor
    target_logp: Tensor
    valid: Tensor
    output_budget: int
    output_tokens: int
    block_size: int

    def work(self) -> VirtualWork:
        # the recurrence is scalar-sequential: run it on the host
        return expected_work(self.acceptance.detach().cpu(), output_tokens=self.output_tokens,
                             output_budget=self.output_budget, block_size=self.block_size)


def _token_logp(model, hidden: Tensor, targets: Tensor, sampling: SamplingConfig, chunk_rows: int) -> Tensor:
    out = []
    for s in range(0, hidden.shape[0], chunk_rows):
        logits = F.linear(hidden[s:s + chunk_rows], model.head.weight).float()
        t = targets[s:s + chunk_rows, None]
        if sampling.temperature > 0 and sampling.top_k == 0 and sampling.top_p == 1:
            lp = (logits / sampling.temperature).log_softmax(-1).gather(1, t)
        else:
            lp = probabilities(logits, sampling).gather(1, t).log()
        out.append(lp[:, 0])
    return torch.cat(out) if out else hidden.new_zeros(0, dtype=torch.float32)


def trace_layout(clean: Tensor, anchors: Tensor, length: int, mask_token_id: int):
    """Isolated [anchor, MASK x (length - 1)] blocks for anchor indices into ``clean``.

    Block b sees the clean tokens before its anchor and itself (both directions),
    nothing of the other blocks.  Returns (tokens [1, A L], positions [1, A L],
    allowed [1, 1, A L, len(clean) + A L]).
    """
    if (clean.ndim != 2 or clean.shape[0] != 1 or anchors.ndim != 1 or anchors.numel() < 1 or length < 2
            or bool(((anchors < 0) | (anchors >= clean.shape[1])).any())):
        raise ValueError("batch-one clean tokens, valid anchors and block length >= 2 required")
    dev = clean.device
    A = anchors.numel()
    pos = anchors[:, None] + torch.arange(length, device=dev)
    tok = torch.full((A, length), mask_token_id, dtype=clean.dtype, device=dev)
    tok[:, 0] = clean[0, anchors]
    row_anchor = anchors.repeat_interleave(length)
    hist = torch.arange(clean.shape[1], device=dev)[None] < row_anchor[:, None]
    blk = torch.arange(A, device=dev).repeat_interleave(length)
    own = blk[:, None] == blk[None]
    allowed = torch.cat((hist, own), 1)[None, None]
    return tok.reshape(1, -1), pos.reshape(1, -1), allowed


@torch.no_grad()
def score_trace(model, prompt: Tensor, outputs: Tensor, *, output_budget: int, block_size: int | None = None,
                sampling: SamplingConfig = SamplingConfig(1.0), eos_id: int | None = None, chunk_rows: int = 32,
                anchors_per_pass: int = 64) -> TraceScores:
    """Score every round start of a completed answer with the dual-view model.

    One AR forward over prompt + answer gives the target log-probabilities and
    the history cache; the draft view then scores all round starts of equal
    block length in batched isolated blocks.  Positions no draft reaches keep
    acceptance 1 (neutral) and ``valid`` False.
    """
    block = model.config.block_size if block_size is None else block_size
    n = outputs.numel()
    if (prompt.ndim != 2 or prompt.shape[0] != 1 or prompt.shape[1] < 1 or outputs.ndim != 1
            or outputs.device != prompt.device or type(output_budget) is not int or not 0 <= n <= output_budget
            or block < 2 or min(chunk_rows, anchors_per_pass) < 1
            or bool(((outputs < 0) | (outputs >= model.config.vocab_size)).any())):
        raise ValueError("a batch-one prompt, a completed answer and positive evaluation sizes required")
    if ((n < output_budget and (n == 0 or eos_id is None or int(outputs[-1]) != eos_id))
            or (eos_id is not None and n > 1 and bool((outputs[:-1] == eos_id).any()))):
        raise ValueError("a completed answer ends at its cap or at its first EOS")
    shape = (max(0, n - 1), block - 1)
    q_log = torch.zeros(shape, dtype=torch.float64, device=prompt.device)
    valid = torch.zeros(shape, dtype=torch.bool, device=prompt.device)
    if n <= 1:
        return TraceScores(q_log + 1, q_log, q_log.clone(), valid, output_budget, n, block)
    P = prompt.shape[1]
    clean = torch.cat((prompt, outputs[None]), 1)
    teacher = model(clean, compute_logits=False)
    # p_log[i]: AR log-probability of outputs[i + 1] (predicted at clean index P + i)
    p_log = _token_logp(model, teacher.hidden[0, P:P + n - 1], outputs[1:], sampling, chunk_rows)
    p_full = torch.zeros(shape, dtype=torch.float64, device=prompt.device)
    by_length: dict[int, list[int]] = {}
    for j in range(1, n - 1):
        if output_budget - j > 1:
            by_length.setdefault(min(block, output_budget - j + 1), []).append(j)
    for length, starts in by_length.items():
        for b in range(0, len(starts), anchors_per_pass):
            js = torch.tensor(starts[b:b + anchors_per_pass], device=prompt.device)
            tok, pos, allowed = trace_layout(clean, P + js - 1, length, model.config.mask_token_id)
            out = model(tok, view="draft", cache=teacher.cache, positions=pos, allowed=allowed,
                        compute_logits=False)
            hid = out.hidden.reshape(js.numel(), length, -1)[:, :-1]          # rows predicting y_{j+1..}
            idx = js[:, None] + torch.arange(length - 1, device=prompt.device)[None]   # 0-based output index
            keep = idx < n - 1
            q = _token_logp(model, hid[keep], outputs[idx[keep]], sampling, chunk_rows)
            r = (js - 1)[:, None].expand_as(idx)[keep]
            c = torch.arange(length - 1, device=prompt.device)[None].expand_as(idx)[keep]
            q_log[r, c] = q.double()
            p_full[r, c] = p_log[idx[keep] - 1].double()
            valid[r, c] = True
    acc = torch.ones(shape, dtype=torch.float64, device=prompt.device)
    acc[valid] = inverse_acceptance(q_log[valid], p_full[valid])
    return TraceScores(acc, q_log, p_full, valid, output_budget, n, block)


def calibration_starts(visits: Tensor, count: int) -> list[int]:
    """Round starts (1-based j) at the equal-mass midpoints of the visit distribution."""
    if (visits.ndim != 1 or type(count) is not int or count < 1 or not bool(torch.isfinite(visits).all())
            or bool((visits < 0).any())):
        raise ValueError("finite nonnegative visits and a positive count required")
    total = visits.sum()
    if float(total) == 0:
        return []
    mids = (torch.arange(count, dtype=visits.dtype, device=visits.device) + 0.5) * total / count
    return (torch.searchsorted(visits.cumsum(0), mids) + 1).tolist()


@dataclass
class TraceTiming:
    work: VirtualWork
    predicted_seconds: float
    measured_seconds: float
    score_seconds: float
    calibration_seconds: float
    round_seconds: list
    tail_seconds: float


@torch.no_grad()
def estimate_trace(branch, prompt: Tensor, outputs: Tensor, *, output_budget: int, prefill_seconds: float,
                   sampler, generator: torch.Generator, sampling: SamplingConfig = SamplingConfig(1.0),
                   eos_id: int | None = None, anchors_per_pass: int = 128, chunk_rows: int = 32,
                   calibration_points: int = 3) -> TraceTiming:
    """Predicted full-answer time of the speculative decoder for this answer.

    The work law is exact for the model's p / q; per-round cost comes from
    timing real rounds (draft + verify + correction + cache bookkeeping) at the
    visit-weighted calibration starts, and one AR tail step when the law has
    tail visits.  ``generator`` owns the calibration draws.  All measurement and
    calibration time is reported.
    """
    if (not getattr(branch, "initial_ar_token", False) or getattr(branch, "input_budget_extra", None) != 1
            or sampler.config != sampling or not isinstance(generator, torch.Generator)
            or not 0 <= prefill_seconds < math.inf or type(calibration_points) is not int
            or calibration_points < 1):
        raise ValueError("an anchor-reprocessing branch, matching sampling, finite prefill time and a "
                         "positive calibration count required")

    def sync():
        if prompt.device.type == "cuda":
            torch.cuda.synchronize(prompt.device)

    sync()
    t0 = time.perf_counter()
    scores = score_trace(branch.model, prompt, outputs, output_budget=output_budget, sampling=sampling,
                         eos_id=eos_id, anchors_per_pass=anchors_per_pass, chunk_rows=chunk_rows)
    work = scores.work()
    sync()
    t1 = time.perf_counter()
    starts = calibration_starts(work.draft_visits, calibration_points)
    rounds, tail = [], 0.0
    if starts or float(work.tail_ar_forwards) > 0:
        clean = torch.cat((prompt, outputs[None]), 1)
        teacher = branch.model(clean, compute_logits=False)
        for j in starts:
            a = prompt.shape[1] + j - 1
            cache = trim_cache(teacher.cache, a)
            length = min(branch.default_block_size, output_budget - j + 1)
            sync()
            m = time.perf_counter()
            proposal = branch.draft(clean[:, a:a + 1], cache, length, sampler, generator)
            logits, verified_cache = branch.ar(proposal.verifier_inputs, cache=proposal.cache)
            verified, _ = sampler.verify(proposal, logits[0], generator)
            trim_cache(verified_cache, a + len(verified.tokens))
            sync()
            rounds.append(time.perf_counter() - m)
        if float(work.tail_ar_forwards) > 0:
            a = prompt.shape[1] + outputs.numel() - 2
            cache = trim_cache(teacher.cache, a)
            sync()
            m = time.perf_counter()
            logits, _ = branch.ar(clean[:, a:a + 1], cache=cache, logits_to_keep=1)
            sampler.sample_ar(logits[0, -1], generator)
            sync()
            tail = time.perf_counter() - m
    per_round = sum(rounds) / len(rounds) if rounds else 0.0
    predicted = prefill_seconds + float(work.cost(per_round, tail))
    sync()
    t2 = time.perf_counter()
    return TraceTiming(work, predicted, t2 - t0, t1 - t0, t2 - t1, rounds, tail)


def _positive(x) -> bool:
    return type(x) in (int, float) and math.isfinite(x) and x > 0


class FullAnswerGate:
    """Screening state of one candidate (fixed) draft version before a fresh full-request trial.

    The candidate is screened on ``count`` requests at the same training step:
    each observation carries the measured reference time (``reference_seconds``
    for ``reference_tokens`` tokens) and the candidate's predicted time
    (``predicted_seconds``, e.g. from :func:`estimate_trace`).  When ``count``
    observations are in and sum(reference) / sum(predicted) >= ``margin`` the
    gate becomes ready for a confirmation trial, whose expected cost is then
    1.2 x (mean predicted time + the AR time of the reused speculative reference,
    if any + the switch cost); otherwise the evidence is discarded.  The screen's
    own cost estimate tracks 1.2 x the elapsed screening time (never dropping by
    more than 20 % at once).  With ``reuse_speculative`` the reference may be the
    serving speculative version (``reference_step`` > 0), which needs a measured
    AR rate (:meth:`confirmed`).
    """

    _FIELDS = ("step", "reference_tokens", "reference_seconds", "predicted_seconds")

    def __init__(self, count: int = 2, margin: float = 1.02, initial_cost: float = 0.4, *,
                 reuse_speculative: bool = False):
        if (type(count) is not int or count < 1 or not _positive(margin) or margin < 1
                or not _positive(initial_cost) or type(reuse_speculative) is not bool):
            raise ValueError("positive screening count / cost and a margin >= 1 required")
        self.count, self.margin = count, margin
        self.screen_estimate = float(initial_cost)
        self.confirmation_estimate = 0.0
        self.ready = False
        self.pending: list[dict] = []
        self.reuse_speculative = reuse_speculative
        self.ar_tps = 0.0

    @property
    def estimate(self) -> float:
        return self.confirmation_estimate if self.ready else self.screen_estimate

    def _fields(self):
        return self._FIELDS + (("reference_step",) if self.reuse_speculative else ())

    def observe(self, row: dict, elapsed: float) -> dict:
        ref_step = row.get("reference_step", 0)
        bad = (self.ready or not _positive(elapsed) or type(row.get("step")) is not int or row["step"] < 1
               or type(row.get("reference_tokens")) is not int or row["reference_tokens"] < 1
               or not all(_positive(row.get(k)) for k in ("reference_seconds", "predicted_seconds"))
               or type(ref_step) is not int or not 0 <= ref_step < row["step"]
               or (ref_step and (not self.reuse_speculative or not _positive(self.ar_tps)))
               or any(p["step"] != row["step"] or p.get("reference_step", 0) != ref_step for p in self.pending))
        if bad:
            raise ValueError("positive same-version screening evidence required")
        self.screen_estimate = max(1.2 * elapsed, 0.8 * self.screen_estimate)
        rec = {k: row[k] for k in self._FIELDS}
        if self.reuse_speculative:
            rec["reference_step"] = ref_step
        self.pending.append(rec)
        ref = sum(p["reference_seconds"] for p in self.pending)
        pred = sum(p["predicted_seconds"] for p in self.pending)
        ratio = ref / pred
        k = len(self.pending)
        complete = k == self.count
        self.ready = complete and ratio >= self.margin
        if self.ready:
            switch = max(0.0, elapsed - row.get("evaluation_seconds", 0.0))
            ar = sum(p["reference_tokens"] for p in self.pending) / (k * self.ar_tps) if ref_step else 0.0
            self.confirmation_estimate = 1.2 * (pred / k + ar + switch)
        label = "candidate_over_serving" if ref_step else "candidate_over_ar"
        out = {**row, "ratio": ratio, label: ratio, "screen_requests": k, "screen_passed": self.ready,
               "awaiting_confirmation": self.ready, "passed": False, "complete": complete and not self.ready,
               "fallback": False}
        if out["complete"]:
            self.pending = []
        return out

    def confirmed(self, *, ar_tps: float | None = None) -> None:
        """The confirmation trial ran (whatever its outcome): clear the screen."""
        if ar_tps is not None:
            if not _positive(ar_tps):
                raise ValueError("a positive measured AR throughput is required")
            self.ar_tps = float(ar_tps)
        self.pending = []
        self.ready = False

    def state_dict(self) -> dict:
        st = {"pending": [dict(p) for p in self.pending], "ready": self.ready,
              "screen_estimate": self.screen_estimate, "confirmation_estimate": self.confirmation_estimate}
        if self.reuse_speculative:
            st["ar_tps"] = self.ar_tps
        return st

    def load_state_dict(self, state: dict, *, step: int, next_probe: int, speculating: bool, requests: int,
                        serving_step: int = 0) -> None:
        """Restore a screen; it must be consistent with the service position (``step``,
        ``next_probe``, whether a speculative version serves, ``requests`` seen)."""
        keys = {"pending", "ready", "screen_estimate", "confirmation_estimate"}
        if self.reuse_speculative:
            keys.add("ar_tps")
        if (not isinstance(state, dict) or set(state) != keys or type(state["ready"]) is not bool
                or not _positive(state["screen_estimate"])
                or type(state["confirmation_estimate"]) not in (int, float)
                or not math.isfinite(state["confirmation_estimate"]) or state["confirmation_estimate"] < 0):
            raise ValueError("a finite full-answer gate state is required")
        if self.reuse_speculative:
            r = state["ar_tps"]
            if type(r) not in (int, float) or not math.isfinite(r) or r < 0 or (speculating and r == 0):
                raise ValueError("a finite measured AR rate is required for live speculative trials")
        rows, ready = state["pending"], state["ready"]
        fields = set(self._fields())
        ref_step = serving_step if speculating else 0
        ok = (isinstance(rows, list) and len(rows) <= min(self.count, requests)
              and (not ready or (len(rows) == self.count and state["confirmation_estimate"] > 0))
              and (ready or len(rows) < self.count)
              and (not rows or (step >= 1 and next_probe <= step
                                and (not speculating or (self.reuse_speculative and 0 < serving_step < step)))))
        ok = ok and all(isinstance(p, dict) and set(p) == fields and type(p["step"]) is int and p["step"] == step
                        and type(p["reference_tokens"]) is int and p["reference_tokens"] >= 1
                        and (not self.reuse_speculative
                             or (type(p["reference_step"]) is int and p["reference_step"] == ref_step))
                        and _positive(p["reference_seconds"]) and _positive(p["predicted_seconds"])
                        for p in rows)
        if not ok:
            raise ValueError("bounded same-version full-answer evidence is required")
        if ready and (sum(p["reference_seconds"] for p in rows) / sum(p["predicted_seconds"] for p in rows)
                      < self.margin):
            raise ValueError("a confirmation needs the screening margin")
        self.pending = [dict(p) for p in rows]
        self.ready = ready
        self.screen_estimate = float(state["screen_estimate"])
        self.confirmation_estimate = float(state["confirmation_estimate"])
        self.ar_tps = float(state.get("ar_tps", 0.0))


__all__ = ["FullAnswerGate", "TraceScores", "TraceSupportError", "TraceTiming", "VirtualWork", "calibration_starts",
           "estimate_trace", "expected_work", "inverse_acceptance", "score_trace", "trace_layout"]
