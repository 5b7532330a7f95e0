"""Request-local continuations mixed into a frozen drafter's proposals.

Generated text repeats itself (lists, code, restated numbers).  An index over the
request's own tokens maps every recent suffix (2..8 tokens) to where it last
occurred, and the tokens that followed that occurrence become a "copy" c_1, c_2, ...
Each drafted row d then proposes

    q_d = (1 - lambda) q0_d + lambda * onehot(c_d)

while the draw follows the copy; the first row whose drawn token leaves the copy,
and every row after it, go back to q0.  The weights lambda live per (suffix-length
group {2, 3, >= 4}, depth) and are learned online from the verified rows by
projected subgradient descent on TV(p_d, q_d), clipped to [0, 1].

All rows are drawn with one set of exponential variates (token = argmax q / E), so
computing the raw and the mixed draw of every row at once and keeping the mixed
one up to the first divergence is the same as the sequential walk.  Row 0 (the
root, drawn from the exact law) is never mixed.

Behaviour follows online-speculation/ablation/src/blockspec_ablation/continuation.py
(the public names ``SuffixLookup``, ``copy_mixture``, ``copy_tv_gradient`` and
``ContinuationMix`` are kept).
"""

from __future__ import annotations

import math
import time
from dataclasses import dataclass

import torch
from torch import Tensor


class SuffixLookup:
    """Most recent continuation of every suffix of ``minimum``..``maximum`` tokens.

    A suffix ending at position s becomes visible once ``lookahead`` tokens have
    followed it, so a match always has at least ``lookahead`` tokens to copy.
    """

    def __init__(self, tokens=(), *, minimum: int = 2, maximum: int = 8, lookahead: int = 2):
        ok = all(type(v) is int for v in (minimum, maximum, lookahead))
        if not ok or minimum < 1 or maximum < minimum or lookahead < 2:
            raise ValueError("suffix lengths need 1 <= minimum <= maximum and a look-ahead of at least 2")
        self.minimum, self.maximum, self.lookahead = minimum, maximum, lookahead
        self.tokens: list[int] = []
        self._after: dict[int, dict[tuple, int]] = {n: {} for n in range(minimum, maximum + 1)}
        self.extend(tokens)

    @property
    def index(self) -> dict[tuple, int]:
        """Every indexed suffix (any length) with the start of its continuation."""
        merged: dict[tuple, int] = {}
        for table in self._after.values():
            merged.update(table)
        return merged

    def extend(self, tokens) -> None:
        for token in tokens:
            self.tokens.append(int(token))
            boundary = len(self.tokens) - self.lookahead          # the suffix ending here now has its look-ahead
            longest = min(self.maximum, boundary)
            for n in range(self.minimum, longest + 1):
                self._after[n][tuple(self.tokens[boundary - n:boundary])] = boundary

    def find(self, length: int) -> tuple[list[int], int]:
        """(up to ``length`` tokens that followed the longest indexed suffix of the text, its length); ([], 0) if none."""
        if type(length) is not int or length < 2:
            raise ValueError("a lookup covers the root and at least one drafted row")
        for n in range(min(self.maximum, len(self.tokens)), self.minimum - 1, -1):
            start = self._after[n].get(tuple(self.tokens[len(self.tokens) - n:]))
            if start is not None:
                return self.tokens[start:start + length], n
        return [], 0


@dataclass
class CopyFeedback:
    baseline: Tensor    # [n, V] drafted rows (1..) before mixing
    copied: Tensor      # [n] copied token per drafted row, -1 where the copy ran out
    weights: Tensor     # [n] lambda applied per drafted row (0 where there is no copy)
    active: Tensor      # [n] the row was drawn from the mixture
    group: int = 0


def _blend(rows: Tensor, lam: Tensor, copied: Tensor) -> Tensor:
    """(1 - lam) rows + lam onehot(copied), row by row (copied < 0 rows need lam = 0)."""
    spike = torch.zeros_like(rows).scatter_(-1, copied.clamp_min(0).unsqueeze(-1), lam.unsqueeze(-1))
    return rows * (1.0 - lam).unsqueeze(-1) + spike


def copy_mixture(baseline: Tensor, weights: Tensor, copied: Tensor, exponential: Tensor):
    """Draw a whole block with the copy-until-divergence rule.

    ``baseline`` [L, V] (row 0 = root), ``weights`` [L - 1] lambdas of rows 1..,
    ``copied`` [L] copied tokens (-1 = none), ``exponential`` [L, V] Exp(1) variates.
    Returns (tokens [L], the law each row was drawn from [L, V], feedback).
    """
    guard = exponential.clamp_min(torch.finfo(baseline.dtype).tiny)
    lam = torch.where(copied[1:] >= 0, weights, torch.zeros_like(weights))
    mixed = torch.cat((baseline[:1], _blend(baseline[1:], lam, copied[1:])), 0)
    plain_draw = torch.argmax(baseline / guard, -1)
    mixed_draw = torch.argmax(mixed / guard, -1)
    # row r (>= 1) is on the copy iff rows 0..r-1 all drew their copied token and row r has one
    on_copy = torch.cummin((mixed_draw[:-1] == copied[:-1]).to(torch.int8), 0).values.bool()
    active = on_copy & (copied[1:] >= 0)
    use_mix = torch.cat((active.new_zeros(1), active))
    law = torch.where(use_mix.unsqueeze(-1), mixed, baseline)
    tokens = torch.where(use_mix, mixed_draw, plain_draw)
    return tokens, law, CopyFeedback(baseline[1:], copied[1:], lam, active)


def copy_tv_gradient(fb: CopyFeedback, teacher: Tensor):
    """(dTV/dlambda on the n reached rows, the mixtures there).

    With q = (1 - lambda) q0 + lambda onehot(c), TV = 1 - sum_v min(p_v, q_v) and dq_v/dlambda
    = [v = c] - q0_v, so dTV/dlambda = sum over {q_v < p_v} of q0_v minus [q_c < p_c].
    Rows that were not drawn from the mixture get zero.
    """
    n = teacher.shape[0]
    base, copy = fb.baseline[:n], fb.copied[:n].clamp_min(0)
    mixture = _blend(base, fb.weights[:n], copy)
    under = mixture < teacher
    at_copy = torch.gather(under, -1, copy.unsqueeze(-1)).squeeze(-1).to(base.dtype)
    slope = torch.where(under, base, torch.zeros_like(base)).sum(-1) - at_copy
    return slope * fb.active[:n].to(base.dtype), mixture


_STATE_TENSORS = ("weights", "gradient", "counts", "steps")


class ContinuationMix:
    """Online lambdas per (suffix-length group, depth); every request builds its own index.

    ``start_depth``: the first drafted depth that may copy (earlier rows are never
    mixed and never learned).
    """

    kind = "continuation"

    def __init__(self, block_size: int, *, learning_rate: float = 0.5, interval: int = 8, adaptive: bool = True,
                 diagnostics: bool = False, device="cpu", dtype=torch.float32, start_depth: int = 1):
        problems = []
        if type(block_size) is not int or block_size < 2:
            problems.append("block_size must be an integer >= 2")
        if not (math.isfinite(learning_rate) and learning_rate > 0):
            problems.append("learning_rate must be finite and positive")
        if type(interval) is not int or interval < 1:
            problems.append("interval must be a positive integer")
        if dtype not in (torch.float32, torch.float64):
            problems.append("dtype is float32 or float64")
        if type(start_depth) is not int or not (type(block_size) is int and 1 <= start_depth < block_size):
            problems.append("start_depth must lie in [1, block_size)")
        if problems:
            raise ValueError("ContinuationMix: " + "; ".join(problems))
        self.block_size, self.learning_rate, self.interval = block_size, float(learning_rate), interval
        self.adaptive, self.diagnostics, self.start_depth = adaptive, diagnostics, start_depth
        shape = (3, block_size - 1)                         # suffix-length groups {2, 3, >= 4} x depth
        self.weights = torch.zeros(shape, device=device, dtype=dtype)
        self.gradient = torch.zeros(shape, device=device, dtype=dtype)
        self.counts = torch.zeros(shape, device=device, dtype=dtype)
        self.steps = torch.zeros(shape, device=device, dtype=dtype)
        self.totals = torch.zeros(block_size - 1, 3, device=device, dtype=dtype)   # rows, TV before, TV after
        self.updates = 0
        self.feedback_blocks = 0
        self.update_seconds = 0.0
        self.memory = SuffixLookup(lookahead=start_depth + 1)
        self.group = 0
        self.copied: list[int] = []

    # ---- request-local text ------------------------------------------------------------------------------------
    def begin_request(self, tokens) -> None:
        self.memory = SuffixLookup(tokens, lookahead=self.start_depth + 1)
        self.copied = []

    def commit(self, tokens) -> None:
        self.memory.extend(tokens)

    def lookup(self, length: int) -> list[int]:
        found, matched = self.memory.find(length)
        self.group = min(matched, 4) - 2 if matched else 0
        self.copied = found if len(found) > self.start_depth else []
        return self.copied

    # ---- drafting and learning -----------------------------------------------------------------------------------
    @torch.no_grad()
    def draft(self, baseline: Tensor, generator=None):
        """(tokens, proposal law, feedback or None) for one block of proposal rows ``baseline`` [L, V]."""
        rows = baseline.shape[0]
        copy = self.lookup(rows)
        variates = torch.empty_like(baseline).exponential_(generator=generator)
        if not copy:
            race = baseline / variates.clamp_min(torch.finfo(baseline.dtype).tiny)
            return race.argmax(-1), baseline, None
        ids = torch.full((rows,), -1, dtype=torch.long, device=baseline.device)
        ids[: len(copy)] = torch.tensor(copy[:rows], dtype=torch.long, device=baseline.device)
        tokens, law, fb = copy_mixture(baseline, self.weights[self.group, : rows - 1], ids, variates)
        fb.group = self.group
        return tokens, law, fb

    @torch.no_grad()
    def observe(self, fb: CopyFeedback | None, teacher: Tensor, *, root: int | None = None) -> None:
        """Learn from the ``teacher`` [n, V] target rows a verified block reached.

        ``root``: the committed root token; a block whose root left the copy taught nothing.
        """
        reached = teacher.shape[0]
        if fb is None or reached < self.start_depth or not (self.adaptive or self.diagnostics):
            return
        if root is not None and self.copied and root != self.copied[0]:
            return
        slope, mixture = copy_tv_gradient(fb, teacher)
        learnable = fb.active[:reached].clone()
        skip = self.start_depth - 1
        learnable[:skip] = False
        slope[:skip] = 0.0
        if self.diagnostics:
            weight = learnable.to(mixture.dtype)
            tv_before = 0.5 * (fb.baseline[:reached] - teacher).abs().sum(-1)
            tv_after = 0.5 * (mixture - teacher).abs().sum(-1)
            self.totals[:reached] += torch.stack((weight, tv_before * weight, tv_after * weight), -1)
        self.feedback_blocks += 1
        if not self.adaptive:
            return
        self.gradient[fb.group, :reached] += slope
        self.counts[fb.group, :reached] += learnable.to(self.counts.dtype)
        if self.feedback_blocks % self.interval == 0:
            self.step()

    @torch.no_grad()
    def step(self) -> None:
        started = time.perf_counter()
        mean = self.gradient / self.counts.clamp_min(1.0)
        size = self.learning_rate * torch.rsqrt(self.steps + 1.0)
        self.weights.copy_((self.weights - size * mean).clamp(0.0, 1.0))
        self.steps += (self.counts > 0).to(self.steps.dtype)
        self.gradient.zero_()
        self.counts.zero_()
        self.updates += 1
        self.update_seconds += time.perf_counter() - started

    # ---- persistence -------------------------------------------------------------------------------------------
    def _identity(self) -> dict:
        return {"block_size": self.block_size, "learning_rate": self.learning_rate, "interval": self.interval,
                "dtype": str(self.weights.dtype), "kind": self.kind, "start_depth": self.start_depth}

    def state_dict(self) -> dict:
        return {"config": self._identity(),
                "tensors": {name: getattr(self, name).detach().to("cpu", copy=True) for name in _STATE_TENSORS},
                "updates": self.updates, "feedback_blocks": self.feedback_blocks,
                "update_seconds": self.update_seconds}

    @torch.no_grad()
    def load_state_dict(self, state: dict) -> None:
        saved = dict(state.get("config") or {})
        if "learning_rate" in saved:
            saved["learning_rate"] = float(saved["learning_rate"])
        if saved != self._identity():
            raise ValueError("the saved continuation mixture was made with another block, schedule, dtype or "
                             "start depth")
        tensors = state.get("tensors") or {}
        if sorted(tensors) != sorted(_STATE_TENSORS):
            raise ValueError(f"the saved continuation mixture needs exactly the tensors {', '.join(_STATE_TENSORS)}")
        for name, value in tensors.items():
            if (not isinstance(value, torch.Tensor) or value.shape != self.weights.shape
                    or value.dtype != self.weights.dtype or not bool(torch.isfinite(value).all())):
                raise ValueError(f"saved tensor {name} must be finite with shape {tuple(self.weights.shape)} "
                                 f"and {self.weights.dtype}")
        w = tensors["weights"]
        frozen_rows_clean = all(not bool(v[:, : self.start_depth - 1].any()) for v in tensors.values())
        counters_ok = all(type(state.get(k)) is int and state[k] >= 0 for k in ("updates", "feedback_blocks"))
        seconds = state.get("update_seconds", math.nan)
        if (bool((w < 0).any()) or bool((w > 1).any()) or not frozen_rows_clean
                or bool((tensors["counts"] < 0).any()) or bool((tensors["steps"] < 0).any()) or not counters_ok
                or not (isinstance(seconds, (int, float)) and math.isfinite(seconds) and seconds >= 0)):
            raise ValueError("saved lambdas must lie in [0, 1] and every counter must be non-negative")
        for name in _STATE_TENSORS:
            getattr(self, name).copy_(tensors[name])
        self.updates = state["updates"]
        self.feedback_blocks = state["feedback_blocks"]
        self.update_seconds = float(seconds)
        self.totals.zero_()

    def metrics(self) -> dict:
        totals = self.totals.cpu()
        rows = totals[:, 0]
        scale = rows.clamp_min(1.0)
        return {"kind": self.kind, "start_depth": self.start_depth, "weights": self.weights.cpu().tolist(),
                "depth_observations": rows.tolist(), "depth_base_tv": (totals[:, 1] / scale).tolist(),
                "depth_mixed_tv": (totals[:, 2] / scale).tolist(), "updates": self.updates,
                "feedback_blocks": self.feedback_blocks, "update_seconds": self.update_seconds}


__all__ = ["ContinuationMix", "CopyFeedback", "SuffixLookup", "copy_mixture", "copy_tv_gradient"]
