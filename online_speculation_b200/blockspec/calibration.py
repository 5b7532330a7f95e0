"""Online temperature calibration of a frozen drafter's proposals.

A drafted block proposes q_d (depth d = 1..K-1) from the drafter's probabilities.
Tempering q_d (raising its top-k restriction to the power 1/T and renormalising)
can move the proposal closer to the target p_d without retraining the drafter.
:class:`OverlapMix` keeps, per depth, a convex weighting over a small set of
temperatures and proposes the mixture of the tempered experts; after every
verified block it accumulates a subgradient of TV(p_d, q_d) = 1 - sum min(p, q)
with respect to the weights on the depths the block actually reached, and every
``interval`` blocks takes a projected step onto the simplex (step size
lr / sqrt(steps)).  The T = 1 expert is the untempered proposal itself (the
identity), and rows before the first draft (``protected_rows``) pass through.

The target law is untouched: the exact p / q correction uses whatever q was
proposed, so calibration changes speed (acceptance), never the output law.

Reference behaviour: online-speculation/ablation/src/blockspec_ablation/calibration.py
(``project_simplex``, ``mix_rows``, ``OverlapMix`` with its state and metrics).
"""

from __future__ import annotations

import math
import time
from dataclasses import dataclass

import torch


def project_simplex(v: torch.Tensor) -> torch.Tensor:
    """Euclidean projection of every last-axis vector onto {x >= 0, sum x = 1}.

    Sort-based method (Held, Wolfe and Crowder 1974; Duchi et al. 2008): with u the
    values in descending order and c_j = (sum_{i<=j} u_i - 1) / j, the threshold is
    c_rho for the largest rho with u_rho > c_rho, and the projection is max(v - c_rho, 0).
    """
    u = v.sort(dim=-1, descending=True).values
    css = u.cumsum(-1) - 1
    j = torch.arange(1, v.shape[-1] + 1, device=v.device, dtype=v.dtype)
    rho = (u > css / j).sum(-1, keepdim=True).clamp_min(1)
    theta = css.gather(-1, rho - 1) / rho.to(v.dtype)
    return (v - theta).clamp_min(0)


@dataclass
class CalibrationFeedback:
    """What a proposal used, kept until its block is verified."""

    indices: torch.Tensor     # [D, k] top-k columns of each drafted row
    experts: torch.Tensor     # [D, E, k] tempered experts on those columns
    mixed: torch.Tensor       # [D, k] the proposed mixture
    baseline: torch.Tensor    # [D, k] the untempered proposal on those columns


def mix_rows(baseline: torch.Tensor, weights: torch.Tensor, powers: torch.Tensor, identity_index: int, top_k: int,
             protected_rows: int = 1):
    """Mixture proposal of the tempered experts (pure tensor map).

    ``baseline`` [R, V] proposal probabilities; rows ``protected_rows:`` are drafts.
    Each draft row is restricted to its top-k columns; expert e raises them to
    ``powers[e]`` (= 1 / T_e) and renormalises, except the identity expert, which
    keeps the untempered values.  Returns the mixed proposal [R, V] and the
    feedback record.
    """
    vals, idx = baseline[protected_rows:].topk(min(top_k, baseline.shape[-1]), dim=-1)
    ex = vals[:, None, :].pow(powers)
    ex = ex / ex.sum(-1, keepdim=True).clamp_min(torch.finfo(ex.dtype).tiny)
    ex[:, identity_index] = vals
    mixed = (ex * weights[: vals.shape[0], :, None]).sum(1)
    q = torch.zeros_like(baseline)
    q[:protected_rows] = baseline[:protected_rows]
    q[protected_rows:].scatter_(-1, idx, mixed)
    return q, CalibrationFeedback(idx, ex, mixed, vals)


class OverlapMix:
    """Per-depth simplex weights over proposal temperatures, learned online on verified blocks."""

    def __init__(self, block_size: int, top_k: int, *, temperatures=(0.5, 0.75, 1.0, 1.25, 1.5),
                 learning_rate: float = 0.5, interval: int = 8, adaptive: bool = True,
                 fixed_temperature: float = 1.0, diagnostics: bool = False, device="cpu",
                 dtype=torch.float32, protected_rows: int = 1):
        temps = tuple(temperatures)
        if (type(block_size) is not int or block_size < 2 or type(top_k) is not int or top_k < 1 or not temps
                or len(set(temps)) != len(temps) or any(not math.isfinite(t) or t <= 0 for t in temps)
                or 1.0 not in temps or fixed_temperature not in temps or not math.isfinite(learning_rate)
                or learning_rate <= 0 or type(interval) is not int or interval < 1 or protected_rows not in (0, 1)):
            raise ValueError("block >= 2, top_k >= 1, distinct positive temperatures including 1, a positive "
                             "learning rate and interval, and 0 or 1 protected rows are required")
        self.block_size, self.top_k, self.temperatures = block_size, top_k, temps
        self.learning_rate, self.interval, self.adaptive = learning_rate, interval, adaptive
        self.diagnostics, self.protected_rows = diagnostics, protected_rows
        self.fixed_index, self.identity_index = temps.index(fixed_temperature), temps.index(1.0)
        D, E = block_size - 1, len(temps)
        self.weights = torch.zeros(D, E, device=device, dtype=dtype)
        self.powers = self.weights.new_tensor(temps).reciprocal()[None, :, None]
        self.gradient = torch.zeros_like(self.weights)
        self.counts = self.weights.new_zeros(D, 1)
        self.steps = torch.zeros_like(self.counts)
        self.totals = self.weights.new_zeros(D, E + 3)   # count, mixture TV, support mass, expert TVs
        self.reset()

    @torch.no_grad()
    def reset(self) -> None:
        self.weights.zero_()
        self.weights[:, self.fixed_index] = 1
        for t in (self.gradient, self.counts, self.steps, self.totals):
            t.zero_()
        self.updates = self.feedback_blocks = 0
        self.update_seconds = 0.0

    @torch.no_grad()
    def propose(self, baseline: torch.Tensor):
        if (baseline.ndim != 2 or not self.protected_rows < baseline.shape[0] <= self.block_size - 1 + self.protected_rows
                or baseline.device != self.weights.device or baseline.dtype != self.weights.dtype):
            raise ValueError("floating [rows, V] proposals on the calibration device and dtype are required")
        return mix_rows(baseline, self.weights, self.powers, self.identity_index, self.top_k, self.protected_rows)

    @torch.no_grad()
    def observe(self, feedback: CalibrationFeedback, teacher: torch.Tensor) -> None:
        """``teacher`` [n, V]: target probabilities of the first n drafted depths the block reached."""
        n = teacher.shape[0]
        if not n or not (self.adaptive or self.diagnostics):
            return
        if n > feedback.indices.shape[0]:
            raise ValueError("feedback must cover a reached prefix of the proposal")
        p = teacher.gather(-1, feedback.indices[:n])
        ex, q = feedback.experts[:n], feedback.mixed[:n]
        if self.diagnostics:
            ex_tv = 1 - torch.minimum(p[:, None, :], ex).sum(-1)
            tv = 1 - torch.minimum(p, q).sum(-1)
            self.totals[:n] += torch.cat((torch.ones_like(tv[:, None]), tv[:, None], p.sum(-1, keepdim=True), ex_tv),
                                         -1)
        self.feedback_blocks += 1
        if self.adaptive:
            # d/dw_e (1 - sum_v min(p_v, q_v)) = - sum_{v: q_v < p_v} expert_e,v
            self.gradient[:n] -= (ex * (q < p)[:, None, :]).sum(-1)
            self.counts[:n] += 1
            if self.feedback_blocks % self.interval == 0:
                self.step()

    @torch.no_grad()
    def step(self) -> None:
        if self.weights.is_cuda:
            torch.cuda.synchronize(self.weights.device)
        t0 = time.perf_counter()
        seen = self.counts > 0
        g = self.gradient / self.counts.clamp_min(1)
        rate = self.learning_rate / (self.steps + 1).sqrt()
        self.weights.copy_(torch.where(seen, project_simplex(self.weights - rate * g), self.weights))
        self.steps += seen
        self.gradient.zero_()
        self.counts.zero_()
        self.updates += 1
        if self.weights.is_cuda:
            torch.cuda.synchronize(self.weights.device)
        self.update_seconds += time.perf_counter() - t0

    def _config(self) -> dict:
        return {"block_size": self.block_size, "top_k": self.top_k, "temperatures": self.temperatures,
                "learning_rate": self.learning_rate, "interval": self.interval, "dtype": str(self.weights.dtype),
                "protected_rows": self.protected_rows}

    def state_dict(self) -> dict:
        return {"config": self._config(),
                "tensors": {n: getattr(self, n).detach().cpu().clone() for n in ("weights", "gradient", "counts",
                                                                                  "steps")},
                "updates": self.updates, "feedback_blocks": self.feedback_blocks,
                "update_seconds": self.update_seconds}

    @torch.no_grad()
    def load_state_dict(self, state: dict) -> None:
        cfg = dict(state.get("config", {}))
        cfg.setdefault("protected_rows", 1)
        if cfg.get("temperatures") is not None:
            cfg["temperatures"] = tuple(cfg["temperatures"])
        if cfg != self._config():
            raise ValueError("calibration state must match its shape, temperatures, precision and update policy")
        ts = state.get("tensors", {})
        if set(ts) != {"weights", "gradient", "counts", "steps"}:
            raise ValueError("exactly the weights, gradient, counts and steps tensors are required")
        for n, v in ts.items():
            d = getattr(self, n)
            if not isinstance(v, torch.Tensor) or v.shape != d.shape or v.dtype != d.dtype or not torch.isfinite(v).all():
                raise ValueError("finite calibration tensors of matching shape and dtype are required")
        w = ts["weights"]
        if (bool((w < 0).any()) or not torch.allclose(w.sum(-1), torch.ones_like(w[:, 0]), atol=1e-6, rtol=1e-6)
                or bool((ts["counts"] < 0).any()) or bool((ts["steps"] < 0).any())
                or any(type(state.get(k)) is not int or state[k] < 0 for k in ("updates", "feedback_blocks"))
                or not math.isfinite(state.get("update_seconds", math.nan)) or state["update_seconds"] < 0):
            raise ValueError("simplex weights and nonnegative counters are required")
        for n, v in ts.items():
            getattr(self, n).copy_(v)
        self.updates, self.feedback_blocks = state["updates"], state["feedback_blocks"]
        self.update_seconds = float(state["update_seconds"])
        self.totals.zero_()

    def metrics(self) -> dict:
        v = self.totals.detach().cpu()
        c = v[:, :1].clamp_min(1)
        return {"temperatures": self.temperatures, "weights": self.weights.detach().cpu().tolist(),
                "depth_observations": v[:, 0].tolist(), "depth_preupdate_tv": (v[:, 1] / c[:, 0]).tolist(),
                "depth_support_mass": (v[:, 2] / c[:, 0]).tolist(), "depth_expert_tv": (v[:, 3:] / c).tolist(),
                "updates": self.updates, "feedback_blocks": self.feedback_blocks,
                "update_seconds": self.update_seconds}


__all__ = ["CalibrationFeedback", "OverlapMix", "mix_rows", "project_simplex"]
