"""Consilience: a confidence-trajectory score, final window mean - penalty x initial window mean.

Reference behaviour: src/inference_scaling/shared/consilience.py:19-49.  The
first ``skip_fraction`` of the trajectory is skipped, windows cover
``window_fraction`` of it (or ``window_tokens``), both clipped to what is left.
"""

from __future__ import annotations

from collections.abc import Sequence
from dataclasses import dataclass
from math import fsum, isfinite


@dataclass(frozen=True, slots=True)
class ConfidenceWindows:
    skipped: int
    window: int
    initial: float
    final: float
    score: float


def confidence_windows(values: Sequence[float], *, window_fraction: float = 0.2, window_tokens: int | None = None,
                       skip_fraction: float = 0.05, initial_penalty: float = 3.0) -> ConfidenceWindows:
    if not (isfinite(window_fraction) and 0 < window_fraction <= 1):
        raise ValueError("Consilience window_fraction must be in (0, 1]")
    if window_tokens is not None and window_tokens <= 0:
        raise ValueError("Consilience window_tokens must be positive")
    if not (isfinite(skip_fraction) and 0 <= skip_fraction < 1):
        raise ValueError("Consilience skip_fraction must be in [0, 1)")
    if not (isfinite(initial_penalty) and initial_penalty >= 0):
        raise ValueError("Consilience initial_penalty must be finite and non-negative")
    if not values or not all(isfinite(v) for v in values):
        raise ValueError("Consilience requires a nonempty finite confidence trajectory")
    n = len(values)
    skip = min(n - 1, int(n * skip_fraction))
    win = min(window_tokens if window_tokens is not None else max(1, int(n * window_fraction)), n - skip)
    ini = fsum(values[skip:skip + win]) / win
    fin = fsum(values[-win:]) / win
    score = fin - initial_penalty * ini
    if not isfinite(score):
        raise ValueError("Consilience score overflowed")
    return ConfidenceWindows(skip, win, ini, fin, score)


__all__ = ["ConfidenceWindows", "confidence_windows"]
