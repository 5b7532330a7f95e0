"""Exact numeric answers from free text, and a reference-answer verifier.

One scan of the text yields a stream of events: explicit answer markers
(``#### x``, ``\\boxed{x}``, "answer is / final answer / answer: x") and bare
numbers.  The answer is the value of the last event of the most explicit kind
present, in the order ####, boxed, phrase, bare number.  Values are exact
fractions; thousands separators, decimals, exponents and ``a/b`` are read.
Nothing in the text is executed.  The extraction order is the one the reference's
GSM8K scoring uses (src/inference_scaling/shared/evaluation/numeric.py), so
accuracies are comparable.
"""

from __future__ import annotations

import re
from dataclasses import dataclass
from fractions import Fraction

from ..verifier import VerifierContext

_NUMBER = r"[-+]?(?:\d{1,3}(?:,\d{3})+|\d+)(?:\.\d+)?(?:[eE][-+]?\d+)?"
_VALUE = rf"(?:{_NUMBER})\s*/\s*(?:{_NUMBER})|{_NUMBER}"
_EVENTS = re.compile(
    rf"(?P<hash>####\s*(?P<v_hash>{_VALUE}))"
    rf"|(?P<boxed>\\boxed\s*\{{\s*(?P<v_boxed>{_VALUE})\s*\}})"
    rf"|(?P<phrase>(?:final\s+answer|answer\s+is|answer)\s*(?:is|:|=)?\s*\$?\s*(?P<v_phrase>{_VALUE}))"
    rf"|(?P<bare>{_VALUE})",
    re.IGNORECASE)
_PRIORITY = ("hash", "boxed", "phrase", "bare")


def _exact(text: str) -> Fraction | None:
    cleaned = text.replace(",", "").replace("$", "").replace(" ", "")
    try:
        if "/" in cleaned:
            num, den = cleaned.split("/", 1)
            return Fraction(num) / Fraction(den)
        return Fraction(cleaned)
    except (ValueError, ZeroDivisionError):
        return None


def _last_events(text: str) -> dict[str, str]:
    """Last raw value of every event kind; a marker also hides the numbers inside it."""
    last: dict[str, str] = {}
    for match in _EVENTS.finditer(text):
        kind = next(k for k in _PRIORITY if match.group(k) is not None)
        last[kind] = match.group("bare") if kind == "bare" else match.group(f"v_{kind}")
    # bare numbers inside markers count as numbers too
    numbers = re.findall(_VALUE, text)
    if numbers:
        last["bare"] = numbers[-1]
    return last


def extract_numeric_answer(text: str) -> Fraction | None:
    found = _last_events(text)
    for kind in _PRIORITY:
        if kind in found:
            value = _exact(found[kind])
            if value is not None:
                return value
    return None


@dataclass(frozen=True, slots=True)
class NumericReferenceVerifier:
    expected: Fraction
    correct_reward: float = 1.0
    incorrect_reward: float = 0.0
    unparseable_reward: float = 0.0

    def score(self, _prompt: str, completion: str) -> float:
        answer = extract_numeric_answer(completion)
        if answer is None:
            return self.unparseable_reward
        return self.correct_reward if answer == self.expected else self.incorrect_reward


def build_numeric_reference_verifier(*, context: VerifierContext, correct_reward: float = 1.0,
                                     incorrect_reward: float = 0.0, unparseable_reward: float = 0.0
                                     ) -> NumericReferenceVerifier:
    """``[verifier]`` factory: compares completions with the example's numeric reference."""
    if context.reference is None:
        raise ValueError("the numeric verifier scores against context.reference, which is missing")
    expected = _exact(context.reference.strip())
    if expected is None:
        expected = extract_numeric_answer(context.reference)
    if expected is None:
        raise ValueError(f"no number in the reference {context.reference!r}")
    return NumericReferenceVerifier(expected, float(correct_reward), float(incorrect_reward),
                                    float(unparseable_reward))


__all__ = ["NumericReferenceVerifier", "build_numeric_reference_verifier", "extract_numeric_answer"]
