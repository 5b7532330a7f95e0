"""Request-local continuations mixed into a frozen drafter's proposals.

Generated text often repeats itself (lists, code, restated numbers).  A
longest-suffix index over the request's tokens finds where the current suffix
occurred before and proposes the tokens that followed it.  Each draft row d is
mixed with a point mass on the copied token c_d,

    q_d = (1 - lambda) q0_d + lambda delta_{c_d},

with lambda learned online per (suffix-length group, depth) by projected
subgradient descent on TV(p_d, q_d) over the reached rows.  The copy applies only
while the proposal walk follows the copy: a row uses the mixture only if every
earlier row's drawn token equalled its copied token.  Drawing all rows with one
set of exponential variates (argmax q / E) makes that parallel computation equal
the sequential copy-until-divergence walk, and row 0 (the root) stays exact.

Reference behaviour: online-speculation/ablation/src/blockspec_ablation/continuation.py
(``SuffixLookup``, ``copy_mixture``, ``copy_tv_gradient``, ``ContinuationMix``).
"""

from __future__ import annotations

import math
import time
from dataclasses import dataclass

import torch


class SuffixLookup:
    """Incremental index: suffix (length ``minimum``..``maximum``) -> where its continuation starts.

    A suffix is indexed once at least ``lookahead`` tokens have followed it."""

    def __init__(self, tokens=(), *, minimum: int = 2, maximum: int = 8, lookahead: int = 2):
        if (type(minimum) is not int or type(maximum) is not int or not 1 <= minimum <= maximum
                or type(lookahead) is not int or lookahead < 2):
            raise ValueError("1 <= minimum <= maximum and lookahead >= 2 are required")
        self.minimum, self.maximum, self.lookahead = minimum, maximum, lookahead
        self.tokens: list[int] = []
        self.index: dict[tuple, int] = {}
        self.extend(tokens)

    def extend(self, tokens) -> None:
        for t in tokens:
            self.tokens.append(int(t))
            start = len(self.tokens) - self.lookahead
            for n in range(self.minimum, min(self.maximum, start) + 1):
                self.index[tuple(self.tokens[start - n:start])] = start

    def find(self, length: int) -> tuple[list[int], int]:
        """The continuation (up to ``length`` tokens) of the longest indexed suffix of the
        text, and that suffix's length (0 when none matches)."""
        if type(length) is not int or length < 2:
            raise ValueError("a root and at least one proposal are required")
        for n in range(min(self.maximum, len(self.tokens)), self.minimum - 1, -1):
            start = self.index.get(tuple(self.tokens[-n:]))
            if start is not None:
                return self.tokens[start:start + length], n
        return [], 0


@dataclass
class CopyFeedback:
    baseline: torch.Tensor    # proposal rows 1.. before mixing [n, V]
    copied: torch.Tensor      # copied token per row 1.. (-1 = none) [n]
    weights: torch.Tensor     # applied lambda per row 1.. [n]
    active: torch.Tensor      # the row used the mixture [n]
    group: int = 0


def copy_mixture(baseline: torch.Tensor, weights: torch.Tensor, copied: torch.Tensor, exponential: torch.Tensor):
    """Copy-until-divergence proposal over all rows at once.

    ``baseline`` [L, V] rows (row 0 = root), ``weights`` [L - 1] lambdas of rows 1..,
    ``copied`` [L] copied tokens (-1 none), ``exponential`` [L, V] Exp(1) variates.
    Returns the drawn tokens [L], the proposal law actually used per row [L, V] and
    the feedback record."""
    tiny = torch.finfo(baseline.dtype).tiny

    def race(q):
        return (q / exponential.clamp_min(tiny)).argmax(-1)

    has_copy = copied[1:] >= 0
    lam = weights * has_copy
    mixed = baseline.clone()
    mixed[1:] *= 1 - lam[:, None]
    mixed[1:].scatter_add_(-1, copied[1:].clamp_min(0)[:, None], lam[:, None])
    raw_tok, mix_tok = race(baseline), race(mixed)
    follows = (mix_tok[:-1] == copied[:-1]).long().cumprod(0).bool()     # rows 0..L-2 stayed on the copy
    active = follows & has_copy
    gate = torch.cat((active.new_zeros(1), active))
    q = torch.where(gate[:, None], mixed, baseline)
    tokens = torch.where(gate, mix_tok, raw_tok)
    return tokens, q, CopyFeedback(baseline[1:], copied[1:], lam, active)


def copy_tv_gradient(fb: CopyFeedback, teacher: torch.Tensor):
    """d TV(p, (1 - lambda) q0 + lambda delta_c) / d lambda on the reached rows, and the mixtures.

    TV = 1 - sum_v min(p, q); on the rows where q_v < p_v the derivative of q_v is
    delta_{v = c} - q0_v, so dTV/dlambda = sum_{q < p} q0_v - [q_c < p_c]."""
    n = teacher.shape[0]
    q0, c = fb.baseline[:n], fb.copied[:n].clamp_min(0)
    lam, active = fb.weights[:n], fb.active[:n]
    q = q0 * (1 - lam[:, None])
    q.scatter_add_(-1, c[:, None], lam[:, None])
    short = q < teacher
    grad = (q0 * short).sum(-1) - short.gather(-1, c[:, None])[:, 0].to(q0.dtype)
    return grad * active, q


class ContinuationMix:
    """Bounded lambdas for suffix matches of length 2, 3 and >= 4, per depth, learned online.

    The coefficients persist across requests; every request builds its own suffix index."""

    kind = "continuation"

    def __init__(self, block_size: int, *, learning_rate: float = 0.5, interval: int = 8, adaptive: bool = True,
                 diagnostics: bool = False, device="cpu", dtype=torch.float32, start_depth: int = 1):
        if (type(block_size) is not int or block_size < 2 or not math.isfinite(learning_rate) or learning_rate <= 0
                or type(interval) is not int or interval < 1 or dtype not in (torch.float32, torch.float64)
                or type(start_depth) is not int or not 1 <= start_depth < block_size):
            raise ValueError("a block >= 2, a positive learning rate and interval, a float dtype and "
                             "1 <= start_depth < block are required")
        self.block_size, self.learning_rate, self.interval = block_size, learning_rate, interval
        self.adaptive, self.diagnostics, self.start_depth = adaptive, diagnostics, start_depth
        self.weights = torch.zeros(3, block_size - 1, device=device, dtype=dtype)
        self.gradient, self.counts, self.steps = (torch.zeros_like(self.weights) for _ in range(3))
        self.totals = self.weights.new_zeros(block_size - 1, 3)   # observations, base TV, mixed TV
        self.updates = self.feedback_blocks = 0
        self.update_seconds = 0.0
        self.memory = SuffixLookup(lookahead=start_depth + 1)
        self.group, self.copied = 0, []

    def begin_request(self, tokens) -> None:
        self.memory = SuffixLookup(tokens, lookahead=self.start_depth + 1)
        self.copied = []

    def commit(self, tokens) -> None:
        self.memory.extend(tokens)

    def lookup(self, length: int) -> list[int]:
        self.copied, match = self.memory.find(length)
        self.group = min(match - 2, 2) if match else 0
        if len(self.copied) <= self.start_depth:
            self.copied = []
        return self.copied

    @torch.no_grad()
    def draft(self, baseline: torch.Tensor, generator=None):
        """Tokens, proposal law and feedback for one block of proposal rows ``baseline`` [L, V]."""
        copied = self.lookup(baseline.shape[0])
        e = torch.empty_like(baseline).exponential_(generator=generator)
        if not copied:
            return (baseline / e.clamp_min(torch.finfo(baseline.dtype).tiny)).argmax(-1), baseline, None
        ids = torch.tensor(copied + [-1] * (baseline.shape[0] - len(copied)), device=baseline.device)
        tokens, q, fb = copy_mixture(baseline, self.weights[self.group, : baseline.shape[0] - 1], ids, e)
        fb.group = self.group
        return tokens, q, fb

    @torch.no_grad()
    def observe(self, fb: CopyFeedback | None, teacher: torch.Tensor, *, root: int | None = None) -> None:
        n = teacher.shape[0]
        if (fb is None or n < self.start_depth or not (self.adaptive or self.diagnostics)
                or (root is not None and self.copied and root != self.copied[0])):
            return
        grad, q = copy_tv_gradient(fb, teacher)
        active = fb.active[:n].clone()
        active[: self.start_depth - 1] = False
        grad[: self.start_depth - 1] = 0
        if self.diagnostics:
            before = 0.5 * (fb.baseline[:n] - teacher).abs().sum(-1)
            after = 0.5 * (q - teacher).abs().sum(-1)
            self.totals[:n] += torch.stack((active.to(q.dtype), before * active, after * active), -1)
        self.feedback_blocks += 1
        if self.adaptive:
            self.gradient[fb.group, :n] += grad
            self.counts[fb.group, :n] += active
            if self.feedback_blocks % self.interval == 0:
                self.step()

    @torch.no_grad()
    def step(self) -> None:
        t0 = time.perf_counter()
        seen = self.counts > 0
        rate = self.learning_rate / (self.steps + 1).sqrt()
        self.weights.sub_(rate * self.gradient / self.counts.clamp_min(1)).clamp_(0, 1)
        self.steps += seen
        self.gradient.zero_()
        self.counts.zero_()
        self.updates += 1
        self.update_seconds += time.perf_counter() - t0

    def _config(self) -> dict:
        return {"block_size": self.block_size, "learning_rate": self.learning_rate, "interval": self.interval,
                "dtype": str(self.weights.dtype), "kind": self.kind, "start_depth": self.start_depth}

    def state_dict(self) -> dict:
        return {"config": self._config(),
                "tensors": {n: getattr(self, n).detach().cpu().clone() for n in ("weights", "gradient", "counts",
                                                                                  "steps")},
                "updates": self.updates, "feedback_blocks": self.feedback_blocks,
                "update_seconds": self.update_seconds}

    @torch.no_grad()
    def load_state_dict(self, state: dict) -> None:
        if state.get("config") != self._config():
            raise ValueError("a matching continuation-mixture configuration is required")
        ts = state.get("tensors", {})
        if set(ts) != {"weights", "gradient", "counts", "steps"}:
            raise ValueError("exactly the weights, gradient, counts and steps tensors are required")
        for v in ts.values():
            if (not isinstance(v, torch.Tensor) or v.shape != self.weights.shape or v.dtype != self.weights.dtype
                    or not bool(torch.isfinite(v).all())):
                raise ValueError("finite continuation tensors of matching shape and dtype are required")
        if (bool((ts["weights"] < 0).any()) or bool((ts["weights"] > 1).any())
                or any(bool((ts[k][:, : self.start_depth - 1] != 0).any()) for k in ts)
                or bool((ts["counts"] < 0).any()) or bool((ts["steps"] < 0).any())
                or any(type(state.get(k)) is not int or state[k] < 0 for k in ("updates", "feedback_blocks"))
                or not math.isfinite(state.get("update_seconds", math.nan)) or state["update_seconds"] < 0):
            raise ValueError("lambdas in [0, 1] and nonnegative counters are required")
        for n, v in ts.items():
            getattr(self, n).copy_(v)
        self.updates, self.feedback_blocks = state["updates"], state["feedback_blocks"]
        self.update_seconds = float(state["update_seconds"])
        self.totals.zero_()

    def metrics(self) -> dict:
        v = self.totals.cpu()
        c = v[:, 0].clamp_min(1)
        return {"kind": self.kind, "start_depth": self.start_depth, "weights": self.weights.cpu().tolist(),
                "depth_observations": v[:, 0].tolist(), "depth_base_tv": (v[:, 1] / c).tolist(),
                "depth_mixed_tv": (v[:, 2] / c).tolist(), "updates": self.updates,
                "feedback_blocks": self.feedback_blocks, "update_seconds": self.update_seconds}


__all__ = ["ContinuationMix", "CopyFeedback", "SuffixLookup", "copy_mixture", "copy_tv_gradient"]
