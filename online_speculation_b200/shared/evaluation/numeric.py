"""Numeric answer extraction and a reference-answer verifier (no generated code is executed).

Extraction order: the last ``#### x``, then the last ``\\boxed{x}``, then the last
"answer is / final answer / answer: x", then the last number anywhere; values
are exact fractions (thousands separators, decimals, exponents and a/b forms).
Reference behaviour: src/inference_scaling/shared/evaluation/numeric.py:40-88.
"""

from __future__ import annotations

import re
from dataclasses import dataclass
from decimal import Decimal, InvalidOperation
from fractions import Fraction

from ..verifier import VerifierContext

_NUM = r"[-+]?(?:\d{1,3}(?:,\d{3})+|\d+)(?:\.\d+)?(?:[eE][-+]?\d+)?"
_FRAC = rf"(?:{_NUM})\s*/\s*(?:{_NUM})"
_VALUE = f"{_FRAC}|{_NUM}"
_PATTERNS = (
    re.compile(rf"####\s*({_VALUE})"),
    re.compile(rf"\\boxed\s*\{{\s*({_VALUE})\s*\}}"),
    re.compile(rf"(?:final\s+answer|answer\s+is|answer)\s*(?:is|:|=)?\s*\$?\s*({_VALUE})", re.IGNORECASE),
)
_ANY = re.compile(_VALUE)


def _fraction(text: str) -> Fraction | None:
    s = text.strip().replace(",", "").replace("$", "")
    try:
        if "/" in s:
            a, b = s.split("/", 1)
            return Fraction(Decimal(a.strip())) / Fraction(Decimal(b.strip()))
        return Fraction(Decimal(s))
    except (InvalidOperation, ValueError, ZeroDivisionError):
        return None


def extract_numeric_answer(text: str) -> Fraction | None:
    for pat in _PATTERNS:
        found = pat.findall(text)
        if found:
            v = _fraction(found[-1])
            if v is not None:
                return v
    found = _ANY.findall(text)
    return _fraction(found[-1]) if found else None


@dataclass(frozen=True, slots=True)
class NumericReferenceVerifier:
    expected: Fraction
    correct_reward: float = 1.0
    incorrect_reward: float = 0.0
    unparseable_reward: float = 0.0

    def score(self, _prompt: str, completion: str) -> float:
        got = extract_numeric_answer(completion)
        if got is None:
            return self.unparseable_reward
        return self.correct_reward if got == self.expected else self.incorrect_reward


def build_numeric_reference_verifier(*, context: VerifierContext, correct_reward: float = 1.0,
                                     incorrect_reward: float = 0.0, unparseable_reward: float = 0.0
                                     ) -> NumericReferenceVerifier:
    """``[verifier]`` factory: reward against the context's bound numeric reference."""
    if context.reference is None:
        raise ValueError("numeric reference verifier requires context.reference")
    expected = extract_numeric_answer(f"#### {context.reference}")
    if expected is None:
        raise ValueError(f"could not parse numeric reference {context.reference!r}")
    return NumericReferenceVerifier(expected, float(correct_reward), float(incorrect_reward), float(unparseable_reward))


__all__ = ["NumericReferenceVerifier", "build_numeric_reference_verifier", "extract_numeric_answer"]
