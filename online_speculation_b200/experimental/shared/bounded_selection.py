"""Exact categorical decisions from interval-bounded weights.

The categorical draw with a fixed uniform u picks the first index i whose
normalised cumulative weight exceeds u, i.e. S_<i <= u T < S_<=i with
T = sum(w).  Written as linear forms, S_<i - u T = (1 - u) S_<i - u S_>=i is
largest when the weights before i sit at their upper bounds and the rest at
their lower bounds, and S_<=i - u T is smallest in the opposite corner.  If
both corner conditions hold, every weight vector inside the box selects i;
otherwise ``None`` (the decision is not yet determined; nothing is
approximated).

Reference behaviour: src/inference_scaling/experimental/shared/bounded_selection.py:9-56.
"""

from __future__ import annotations

from collections.abc import Sequence
from math import isfinite

import numpy as np


def invariant_categorical_index(lower_weights: Sequence[float], upper_weights: Sequence[float], *,
                                uniform: float) -> int | None:
    lo = np.asarray([float(v) for v in lower_weights], dtype=np.float64)
    hi = np.asarray([float(v) for v in upper_weights], dtype=np.float64)
    if lo.size == 0 or lo.shape != hi.shape:
        raise ValueError("weight intervals must be non-empty and aligned")
    if not isfinite(uniform) or not 0.0 <= uniform < 1.0:
        raise ValueError("uniform must be finite and lie in [0, 1)")
    if not (np.all(np.isfinite(lo)) and np.all(np.isfinite(hi)) and np.all(lo > 0) and np.all(hi >= lo)):
        raise ValueError("weight intervals must be finite, positive and ordered")
    u = float(uniform)
    hi_before = np.concatenate(([0.0], np.cumsum(hi)[:-1]))      # sum of upper bounds of indices < i
    lo_through = np.cumsum(lo)                                    # sum of lower bounds of indices <= i
    lo_from = lo[::-1].cumsum()[::-1]                             # sum of lower bounds of indices >= i
    hi_after = np.concatenate((hi[::-1].cumsum()[::-1][1:], [0.0]))   # sum of upper bounds of indices > i
    worst_before = (1.0 - u) * hi_before - u * lo_from
    worst_through = (1.0 - u) * lo_through - u * hi_after
    ok = np.nonzero((worst_before <= 0.0) & (worst_through > 0.0))[0]
    return int(ok[0]) if ok.size else None


__all__ = ["invariant_categorical_index"]
