"""Self-consistency: modal numeric answer, consensus selection, cumulative consensus reward.

Reference behaviour: src/inference_scaling/shared/evaluation/consensus.py:13-57.
Ties between modal answers break to the smallest value (order independent);
among completions with the modal answer the most likely one wins (then the
earliest).
"""

from __future__ import annotations

from collections import Counter
from collections.abc import Callable, Sequence
from fractions import Fraction

from ..types import TokenSequence
from .numeric import extract_numeric_answer


def modal_answer(answers: Sequence[Fraction | None]) -> Fraction | None:
    counts = Counter(a for a in answers if a is not None)
    if not counts:
        return None
    top = max(counts.values())
    return min(a for a, c in counts.items() if c == top)


def consensus_index(texts: Sequence[str], logprobs: Sequence[float]) -> int:
    if not texts or len(texts) != len(logprobs):
        raise ValueError("texts and logprobs must be non-empty and equally sized")
    answers = [extract_numeric_answer(t) for t in texts]
    mode = modal_answer(answers)
    pool = [i for i, a in enumerate(answers) if a == mode] if mode is not None else list(range(len(texts)))
    return max(pool, key=lambda i: (logprobs[i], -i))


class CumulativeConsensusReward:
    """Reward 1 for completions matching the running modal answer across calls."""

    def __init__(self, decoder: Callable[[TokenSequence], str]):
        self._decode = decoder
        self._counts: Counter[Fraction] = Counter()

    @property
    def counts(self) -> Counter[Fraction]:
        return self._counts.copy()

    def __call__(self, _prompt: TokenSequence, generated: Sequence[TokenSequence]) -> tuple[float, ...]:
        answers = [extract_numeric_answer(self._decode(t)) for t in generated]
        self._counts.update(a for a in answers if a is not None)
        mode = modal_answer(list(self._counts.elements()))
        return tuple(1.0 if mode is not None and a == mode else 0.0 for a in answers)


__all__ = ["CumulativeConsensusReward", "consensus_index", "modal_answer"]
