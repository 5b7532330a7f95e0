"""Preference pairs from verifier-scored completions.

Reference behaviour: src/inference_scaling/dllm/preferences.py:11-71.  The
highest- and lowest-reward completions form the pair; a dataset reference
solution may join as one more scored entry but is never preferred without a
score; equal rewards carry no preference and give ``None``.
"""

from __future__ import annotations

from dataclasses import dataclass
from math import isfinite
from typing import Sequence


@dataclass(frozen=True, slots=True)
class PreferencePair:
    chosen: str
    rejected: str
    chosen_source: str
    rejected_source: str


def select_scored_preference_pair(*, candidate_texts: Sequence[str], candidate_rewards: Sequence[float],
                                  reference_text: str | None = None, reference_reward: float | None = None
                                  ) -> PreferencePair | None:
    if not candidate_texts:
        raise ValueError("candidate_texts must be non-empty")
    if len(candidate_texts) != len(candidate_rewards):
        raise ValueError("candidate texts and rewards have different lengths")
    if (reference_text is None) != (reference_reward is None):
        raise ValueError("reference text and reward must be supplied together")
    entries = [(t, float(r), f"candidate:{i}") for i, (t, r) in enumerate(zip(candidate_texts, candidate_rewards))]
    if reference_text is not None:
        entries.append((reference_text, float(reference_reward), "dataset_reference_completion"))
    if not all(isfinite(e[1]) for e in entries):
        raise ValueError("preference rewards must be finite")
    lo = min(e[1] for e in entries)
    hi = max(e[1] for e in entries)
    if lo == hi:
        return None
    best = next(e for e in entries if e[1] == hi)
    worst = next(e for e in entries if e[1] == lo)
    if best[0] == worst[0]:
        raise RuntimeError("verifier assigned different rewards to identical texts")
    return PreferencePair(best[0], worst[0], best[2], worst[2])


__all__ = ["PreferencePair", "select_scored_preference_pair"]
