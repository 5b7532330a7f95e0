"""Paired-bootstrap throughput ratios (online-speculation/src/blockspec/measurement.py)."""

from __future__ import annotations

import numpy as np


def paired_ratio(candidate_tokens, candidate_seconds, baseline_tokens, baseline_seconds, *, samples: int = 10000,
                 seed: int = 0, level: float = 0.95) -> dict:
    """Ratio of total throughputs over the same requests, with a paired bootstrap CI."""
    ct, cs = np.asarray(candidate_tokens, float), np.asarray(candidate_seconds, float)
    bt, bs = np.asarray(baseline_tokens, float), np.asarray(baseline_seconds, float)
    if not (len(ct) == len(cs) == len(bt) == len(bs) > 0) or (cs <= 0).any() or (bs <= 0).any():
        raise ValueError("paired, positive per-request measurements required")
    ratio = (ct.sum() / cs.sum()) / (bt.sum() / bs.sum())
    rng = np.random.default_rng(seed)
    idx = rng.integers(0, len(ct), size=(samples, len(ct)))
    boot = (ct[idx].sum(1) / cs[idx].sum(1)) / (bt[idx].sum(1) / bs[idx].sum(1))
    lo, hi = np.quantile(boot, [(1 - level) / 2, (1 + level) / 2])
    return {"ratio": float(ratio), "ci_low": float(lo), "ci_high": float(hi), "level": level, "requests": len(ct)}
