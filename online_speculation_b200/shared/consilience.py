"""Consilience score of a per-token confidence trajectory.

score = mean(final window) - penalty * mean(initial window), where the initial
window starts after skipping ``skip_fraction`` of the tokens and both windows
span ``window_tokens`` tokens or ``window_fraction`` of the trajectory, clipped to
what remains after the skip.  Window means come from one cumulative sum.
Behavioural contract: src/inference_scaling/shared/consilience.py.
"""

from __future__ import annotations

from collections.abc import Sequence
from dataclasses import dataclass

import numpy as np


@dataclass(frozen=True, slots=True)
class ConfidenceWindows:
    skipped: int
    window: int
    initial: float
    final: float
    score: float


def _check(window_fraction, window_tokens, skip_fraction, initial_penalty) -> None:
    problems = []
    if not (np.isfinite(window_fraction) and 0.0 < window_fraction <= 1.0):
        problems.append("window_fraction must lie in (0, 1]")
    if window_tokens is not None and window_tokens < 1:
        problems.append("window_tokens must be a positive count")
    if not (np.isfinite(skip_fraction) and 0.0 <= skip_fraction < 1.0):
        problems.append("skip_fraction must lie in [0, 1)")
    if not (np.isfinite(initial_penalty) and initial_penalty >= 0.0):
        problems.append("initial_penalty must be finite and non-negative")
    if problems:
        raise ValueError("consilience: " + "; ".join(problems))


def confidence_windows(values: Sequence[float], *, window_fraction: float = 0.2, window_tokens: int | None = None,
                       skip_fraction: float = 0.05, initial_penalty: float = 3.0) -> ConfidenceWindows:
    _check(window_fraction, window_tokens, skip_fraction, initial_penalty)
    x = np.asarray(list(values), dtype=np.float64)
    if x.size == 0 or not np.isfinite(x).all():
        raise ValueError("consilience needs a non-empty trajectory of finite confidences")
    n = x.size
    skip = min(n - 1, int(n * skip_fraction))
    want = window_tokens if window_tokens is not None else max(1, int(n * window_fraction))
    win = min(want, n - skip)
    csum = np.concatenate(([0.0], np.cumsum(x)))
    initial = (csum[skip + win] - csum[skip]) / win
    final = (csum[n] - csum[n - win]) / win
    score = final - initial_penalty * initial
    if not np.isfinite(score):
        raise ValueError("consilience score is not finite")
    return ConfidenceWindows(skip, win, float(initial), float(final), float(score))


__all__ = ["ConfidenceWindows", "confidence_windows"]
