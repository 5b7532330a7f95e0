"""Rewards defined through the base model's own scores.

``SequenceLogProbabilityReward``: r(y) = c * log p(y | x).  With IS temperature
tau the tilted target p * exp(r / tau) is the power target p^(1 + c / tau)
(reference: src/inference_scaling/arllm/rewards.py:19-57).  Scores come from a
backend's fused full-vocabulary log-softmax scoring.
"""

from __future__ import annotations

from collections.abc import Sequence

from ..shared.types import TokenSequence
from .types import AutoregressiveBackend, ScoreRequest


class SequenceLogProbabilityReward:
    def __init__(self, backend: AutoregressiveBackend, *, coefficient: float = 1.0, normalize: bool = False):
        self.backend = backend
        self.coefficient = float(coefficient)
        self.normalize = normalize

    def __call__(self, prompt: TokenSequence, completion: TokenSequence) -> float:
        return self.batch(prompt, [completion])[0]

    def batch(self, prompt: TokenSequence, completions: Sequence[TokenSequence]) -> list[float]:
        if not completions:
            return []
        scores = self.backend.score_batch([ScoreRequest(tuple(prompt), tuple(tuple(c) for c in completions), None)])
        out = []
        for comp, s in zip(completions, scores):
            total = float(sum(s))
            if self.normalize and comp:
                total /= len(comp)
            out.append(self.coefficient * total)
        return out

    def target_exponent(self, reward_temperature: float) -> float:
        return 1.0 + self.coefficient / reward_temperature
