"""Online temperature calibration of a frozen drafter's proposals.

Drafted row d of a block proposes q_d over the vocabulary.  Restricting q_d to its
top-k columns and tempering them (``q^(1/T)``, renormalised) gives a family of
"experts", one per temperature T; the T = 1 expert is the restricted proposal
itself, left unnormalised so that a weight of one on it reproduces the drafter.
:class:`OverlapMix` proposes, per depth, a convex combination of the experts and
learns the combination online from the verified blocks: the total-variation loss
TV(p_d, q_d) = 1 - sum_v min(p_v, q_v) is convex in the weights, its subgradient
with respect to weight e is -sum over {v : q_v < p_v} of expert e at v, and every
``interval`` observed blocks each depth that was reached takes a projected
subgradient step onto the probability simplex with step lr / sqrt(1 + steps taken).

Rows before the first draft (``protected_rows``) pass through.  The exact p / q
correction uses whatever q was proposed, so calibration changes acceptance only,
never the output law.

Behaviour follows online-speculation/ablation/src/blockspec_ablation/calibration.py
(the simplex projection, the tempered-expert mixture and the online weights, with
the same public names).
"""

from __future__ import annotations

import math
import time
from dataclasses import dataclass

import torch
from torch import Tensor


def project_simplex(v: Tensor) -> Tensor:
    """Euclidean projection of every last-axis vector onto {x >= 0, sum x = 1}.

    The projection is max(v - theta, 0) with theta the water level that leaves a
    unit mass above it.  Sorting once fixes the support: with s_j the sum of the j
    largest entries, the support size r is the number of j for which the j-th
    largest entry exceeds (s_j - 1) / j, and theta = (s_r - 1) / r (Held, Wolfe and
    Crowder 1974; Duchi, Shalev-Shwartz, Singer and Chandra 2008).
    """
    top = v.sort(dim=-1, descending=True).values
    sizes = torch.arange(1, v.shape[-1] + 1, device=v.device, dtype=v.dtype)
    levels = (top.cumsum(-1) - 1.0) / sizes
    support = (top > levels).sum(-1, keepdim=True).clamp_min(1)
    theta = levels.gather(-1, support - 1)
    return torch.clamp(v - theta, min=0.0)


@dataclass
class CalibrationFeedback:
    """The pieces of one mixed proposal that its verification needs."""

    indices: Tensor     # [D, k] top-k columns of every drafted row
    experts: Tensor     # [D, E, k] every expert on those columns
    mixed: Tensor       # [D, k] the proposed mixture on those columns
    baseline: Tensor    # [D, k] the drafter's own values on those columns


def _tempered_experts(values: Tensor, powers: Tensor, identity_index: int) -> Tensor:
    """[D, k] top-k values -> [D, E, k]: each power applied and renormalised, identity untouched."""
    raised = values.unsqueeze(1) ** powers.view(1, -1, 1)
    raised = raised / raised.sum(-1, keepdim=True).clamp_min(torch.finfo(raised.dtype).tiny)
    raised[:, identity_index] = values
    return raised


def mix_rows(baseline: Tensor, weights: Tensor, powers: Tensor, identity_index: int, top_k: int,
             protected_rows: int = 1) -> tuple[Tensor, CalibrationFeedback]:
    """The mixed proposal of ``baseline`` [R, V] and the record that verification needs.

    ``weights`` [>= R - protected_rows, E] are per-depth expert weights, ``powers``
    holds 1 / T per expert (any shape with E entries).  Rows before
    ``protected_rows`` are copied unchanged; drafted rows become the weighted sum of
    their experts, zero outside the top-k columns.
    """
    drafted = baseline[protected_rows:]
    values, columns = torch.topk(drafted, min(top_k, baseline.shape[-1]), dim=-1)
    experts = _tempered_experts(values, powers.reshape(-1), identity_index)
    mixture = torch.einsum("dek,de->dk", experts, weights[: values.shape[0]].to(experts.dtype))
    out = torch.zeros_like(baseline)
    out[:protected_rows] = baseline[:protected_rows]
    out[protected_rows:].scatter_(-1, columns, mixture)
    return out, CalibrationFeedback(columns, experts, mixture, values)


_STATE_TENSORS = ("weights", "gradient", "counts", "steps")


class OverlapMix:
    """Per-depth simplex weights over proposal temperatures, learned from verified blocks.

    ``adaptive=False`` keeps the starting weights (all mass on ``fixed_temperature``);
    ``diagnostics=True`` accumulates per-depth TV and support statistics for
    :meth:`metrics`.
    """

    def __init__(self, block_size: int, top_k: int, *, temperatures=(0.5, 0.75, 1.0, 1.25, 1.5),
                 learning_rate: float = 0.5, interval: int = 8, adaptive: bool = True,
                 fixed_temperature: float = 1.0, diagnostics: bool = False, device="cpu",
                 dtype=torch.float32, protected_rows: int = 1):
        temps = tuple(float(t) for t in temperatures)
        problems = []
        if type(block_size) is not int or block_size < 2:
            problems.append("block_size must be an integer >= 2")
        if type(top_k) is not int or top_k < 1:
            problems.append("top_k must be a positive integer")
        if not temps or len(set(temps)) != len(temps) or not all(math.isfinite(t) and t > 0 for t in temps):
            problems.append("temperatures must be distinct, finite and positive")
        elif 1.0 not in temps or float(fixed_temperature) not in temps:
            problems.append("the temperatures must contain 1 and the fixed temperature")
        if not (math.isfinite(learning_rate) and learning_rate > 0):
            problems.append("learning_rate must be finite and positive")
        if type(interval) is not int or interval < 1:
            problems.append("interval must be a positive integer")
        if protected_rows not in (0, 1):
            problems.append("protected_rows is 0 or 1")
        if problems:
            raise ValueError("OverlapMix: " + "; ".join(problems))
        self.block_size, self.top_k, self.temperatures = block_size, top_k, temps
        self.learning_rate, self.interval = float(learning_rate), interval
        self.adaptive, self.diagnostics, self.protected_rows = adaptive, diagnostics, protected_rows
        self.identity_index = temps.index(1.0)
        self.fixed_index = temps.index(float(fixed_temperature))
        depths, n_experts = block_size - 1, len(temps)
        self.powers = torch.tensor([1.0 / t for t in temps], device=device, dtype=dtype)
        self.weights = torch.empty(depths, n_experts, device=device, dtype=dtype)
        self.gradient = torch.empty_like(self.weights)
        self.counts = torch.empty(depths, 1, device=device, dtype=dtype)
        self.steps = torch.empty_like(self.counts)
        # diagnostics columns: observations, TV of the mixture, target mass on the top-k, TV of every expert
        self.totals = torch.empty(depths, 3 + n_experts, device=device, dtype=dtype)
        self.reset()

    @torch.no_grad()
    def reset(self) -> None:
        for t in (self.weights, self.gradient, self.counts, self.steps, self.totals):
            t.zero_()
        self.weights[:, self.fixed_index] = 1.0
        self.updates = 0
        self.feedback_blocks = 0
        self.update_seconds = 0.0

    @torch.no_grad()
    def propose(self, baseline: Tensor) -> tuple[Tensor, CalibrationFeedback]:
        rows = baseline.shape[0] if baseline.ndim == 2 else -1
        if not self.protected_rows < rows <= self.protected_rows + self.block_size - 1:
            raise ValueError(f"a proposal has between {self.protected_rows + 1} and "
                             f"{self.protected_rows + self.block_size - 1} rows of [rows, V]")
        if baseline.device != self.weights.device or baseline.dtype != self.weights.dtype:
            raise ValueError("the proposal must live on the calibration device with its dtype")
        return mix_rows(baseline, self.weights, self.powers, self.identity_index, self.top_k, self.protected_rows)

    @torch.no_grad()
    def observe(self, feedback: CalibrationFeedback, teacher: Tensor) -> None:
        """Record one verified block; ``teacher`` [n, V] is the target law of the n depths it reached."""
        reached = teacher.shape[0]
        if reached == 0 or not (self.adaptive or self.diagnostics):
            return
        if reached > feedback.indices.shape[0]:
            raise ValueError("the target rows must cover a prefix of the proposed depths")
        target = torch.gather(teacher, -1, feedback.indices[:reached])
        experts, mixture = feedback.experts[:reached], feedback.mixed[:reached]
        if self.diagnostics:
            expert_tv = 1.0 - torch.minimum(experts, target.unsqueeze(1)).sum(-1)
            mixture_tv = 1.0 - torch.minimum(mixture, target).sum(-1, keepdim=True)
            seen = torch.ones_like(mixture_tv)
            self.totals[:reached] += torch.cat((seen, mixture_tv, target.sum(-1, keepdim=True), expert_tv), dim=-1)
        self.feedback_blocks += 1
        if not self.adaptive:
            return
        short = (mixture < target).to(experts.dtype)                       # columns where q under-covers p
        self.gradient[:reached] -= torch.einsum("dek,dk->de", experts, short)
        self.counts[:reached] += 1.0
        if self.feedback_blocks % self.interval == 0:
            self.step()

    @torch.no_grad()
    def step(self) -> None:
        """One projected subgradient step on every depth that was observed since the last one."""
        on_gpu = self.weights.is_cuda
        if on_gpu:
            torch.cuda.synchronize(self.weights.device)
        started = time.perf_counter()
        observed = self.counts > 0
        mean_gradient = self.gradient / torch.clamp(self.counts, min=1.0)
        step_size = self.learning_rate * torch.rsqrt(self.steps + 1.0)
        moved = project_simplex(self.weights - step_size * mean_gradient)
        self.weights.copy_(torch.where(observed, moved, self.weights))
        self.steps += observed.to(self.steps.dtype)
        self.gradient.zero_()
        self.counts.zero_()
        self.updates += 1
        if on_gpu:
            torch.cuda.synchronize(self.weights.device)
        self.update_seconds += time.perf_counter() - started

    # ---- persistence -------------------------------------------------------------------------------------------
    def _identity(self) -> dict:
        return {"block_size": self.block_size, "top_k": self.top_k, "temperatures": self.temperatures,
                "learning_rate": self.learning_rate, "interval": self.interval, "dtype": str(self.weights.dtype),
                "protected_rows": self.protected_rows}

    def state_dict(self) -> dict:
        return {"config": self._identity(),
                "tensors": {name: getattr(self, name).detach().to("cpu", copy=True) for name in _STATE_TENSORS},
                "updates": self.updates, "feedback_blocks": self.feedback_blocks,
                "update_seconds": self.update_seconds}

    @torch.no_grad()
    def load_state_dict(self, state: dict) -> None:
        saved = dict(state.get("config") or {})
        saved.setdefault("protected_rows", 1)
        if "temperatures" in saved:
            saved["temperatures"] = tuple(float(t) for t in saved["temperatures"])
        if "learning_rate" in saved:
            saved["learning_rate"] = float(saved["learning_rate"])
        if saved != self._identity():
            raise ValueError("the saved calibration was made with another block, top-k, temperature set, "
                             "learning schedule or dtype")
        tensors = state.get("tensors") or {}
        if sorted(tensors) != sorted(_STATE_TENSORS):
            raise ValueError(f"the saved calibration needs exactly the tensors {', '.join(_STATE_TENSORS)}")
        for name in _STATE_TENSORS:
            mine, theirs = getattr(self, name), tensors[name]
            if (not isinstance(theirs, torch.Tensor) or theirs.shape != mine.shape or theirs.dtype != mine.dtype
                    or not bool(torch.isfinite(theirs).all())):
                raise ValueError(f"saved tensor {name} must be finite with shape {tuple(mine.shape)} and {mine.dtype}")
        weights = tensors["weights"]
        on_simplex = bool((weights >= 0).all()) and torch.allclose(weights.sum(-1), torch.ones(weights.shape[0],
                                                                                                dtype=weights.dtype),
                                                                    atol=1e-6, rtol=1e-6)
        counters_ok = all(type(state.get(k)) is int and state[k] >= 0 for k in ("updates", "feedback_blocks"))
        seconds = state.get("update_seconds", math.nan)
        if (not on_simplex or bool((tensors["counts"] < 0).any()) or bool((tensors["steps"] < 0).any())
                or not counters_ok or not (isinstance(seconds, (int, float)) and math.isfinite(seconds)
                                           and seconds >= 0)):
            raise ValueError("saved weights must lie on the simplex and every counter must be non-negative")
        for name in _STATE_TENSORS:
            getattr(self, name).copy_(tensors[name])
        self.updates = state["updates"]
        self.feedback_blocks = state["feedback_blocks"]
        self.update_seconds = float(seconds)
        self.totals.zero_()

    def metrics(self) -> dict:
        totals = self.totals.detach().cpu()
        seen = totals[:, 0]
        per = totals / seen.clamp_min(1.0).unsqueeze(-1)
        return {"temperatures": self.temperatures, "weights": self.weights.detach().cpu().tolist(),
                "depth_observations": seen.tolist(), "depth_preupdate_tv": per[:, 1].tolist(),
                "depth_support_mass": per[:, 2].tolist(), "depth_expert_tv": per[:, 3:].tolist(),
                "updates": self.updates, "feedback_blocks": self.feedback_blocks,
                "update_seconds": self.update_seconds}


__all__ = ["CalibrationFeedback", "OverlapMix", "mix_rows", "project_simplex"]
