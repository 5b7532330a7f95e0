"""Self-consistency over sampled answers.

* ``modal_answer``: the most frequent parsed answer; ties go to the smallest value,
  so the result does not depend on sample order;
* ``consensus_index``: among completions whose answer is the modal one (all of them
  when nothing parses), the highest log-probability, then the earliest;
* ``CumulativeConsensusReward``: rewards a completion with 1 when its answer equals
  the modal answer of everything seen so far (this call included).

Tie rules follow src/inference_scaling/shared/evaluation/consensus.py so that
consensus choices are comparable with the reference's reports.
"""

from __future__ import annotations

from collections import Counter
from collections.abc import Callable, Sequence
from fractions import Fraction

from ..types import TokenSequence
from .numeric import extract_numeric_answer


def _mode_of_counts(counts: Counter) -> Fraction | None:
    if not counts:
        return None
    return min(counts, key=lambda answer: (-counts[answer], answer))


def modal_answer(answers: Sequence[Fraction | None]) -> Fraction | None:
    return _mode_of_counts(Counter(a for a in answers if a is not None))


def consensus_index(texts: Sequence[str], logprobs: Sequence[float]) -> int:
    if not len(texts) or len(texts) != len(logprobs):
        raise ValueError(f"consensus needs matching non-empty texts and log-probs ({len(texts)} vs {len(logprobs)})")
    answers = [extract_numeric_answer(t) for t in texts]
    mode = modal_answer(answers)
    eligible = range(len(texts)) if mode is None else (i for i, a in enumerate(answers) if a == mode)
    # highest log-prob first; among equal log-probs the earliest index
    return min(eligible, key=lambda i: (-logprobs[i], i))


class CumulativeConsensusReward:
    """Batch reward: 1 for completions that agree with the running modal answer."""

    def __init__(self, decoder: Callable[[TokenSequence], str]):
        self._decode = decoder
        self._seen: Counter[Fraction] = Counter()

    @property
    def counts(self) -> Counter[Fraction]:
        return Counter(self._seen)

    def __call__(self, _prompt: TokenSequence, generated: Sequence[TokenSequence]) -> tuple[float, ...]:
        answers = [extract_numeric_answer(self._decode(tokens)) for tokens in generated]
        self._seen.update(a for a in answers if a is not None)
        mode = _mode_of_counts(self._seen)
        return tuple(float(mode is not None and a == mode) for a in answers)


__all__ = ["CumulativeConsensusReward", "consensus_index", "modal_answer"]
