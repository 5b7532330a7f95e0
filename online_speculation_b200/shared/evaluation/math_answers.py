"""MATH-style benchmark problems and answer-only grading of LaTeX answers.

* :func:`load_math500` reads a local MATH-500 JSONL (``unique_id``, ``problem``, ``answer``,
  ``subject``, ``level``); nothing is downloaded.
* :func:`stratified_subset` draws a preregistered development / test split that spreads over
  subject x level strata: the strata are visited round-robin in a seeded order, each stratum
  shuffled on its own, so the subset depends on the identifiers and the seed only (never on
  answers).  The visiting rule is the reference's (experiments/shared/math_benchmark.py) so
  both select the same problems for the same seed.
* :func:`final_answer` takes the last ``\\boxed{...}`` (balanced braces) of a completion, else
  the text after a final "answer is"; :func:`canonical_answer` normalises LaTeX spellings
  (``\\dfrac`` / ``\\frac{a}{b}``, ``\\left`` / ``\\right``, ``\\text{}``, spacing commands,
  degree signs, dollar signs, trailing punctuation); :func:`answers_equivalent` compares two
  answers as exact rationals when both read as numbers, else as canonical strings (tuples and
  intervals element-wise).
* :class:`MathJudge` grades in a separate process with a per-call timeout, so pathological
  inputs cannot stall a run; :func:`build_math_reference_verifier` plugs the grader into the
  verifier interface (factory ``online_speculation_b200.shared.evaluation.math_answers:build_math_reference_verifier``).

The reference grades with the external Math-Verify package; the rules above are this
package's own and cover the answer forms of MATH-500 (integers, fractions, radicals written
in LaTeX, tuples, intervals, text answers).
"""

from __future__ import annotations

import json
import multiprocessing as mp
import random
import re
from collections import defaultdict
from dataclasses import dataclass
from fractions import Fraction
from pathlib import Path
from typing import Any

from ..verifier import VerifierContext


@dataclass(frozen=True)
class MathProblem:
    identifier: str
    question: str
    answer: str
    subject: str
    level: int


def load_math500(path: str | Path) -> list[MathProblem]:
    rows = [json.loads(line) for line in Path(path).read_text(encoding="utf-8").splitlines() if line.strip()]
    problems = [MathProblem(str(r["unique_id"]), str(r["problem"]), str(r["answer"]), str(r["subject"]),
                            int(r["level"])) for r in rows]
    if len({p.identifier for p in problems}) != len(problems):
        raise ValueError("the benchmark repeats a problem identifier")
    return problems


def stratified_subset(problems: list[MathProblem], *, seed: int, minimum_level: int, development_count: int,
                      test_count: int, excluded_ids=()) -> dict[str, list[MathProblem]]:
    if development_count < 0 or test_count <= 0:
        raise ValueError("development_count >= 0 and test_count > 0 are required")
    excluded = set(excluded_ids)
    strata: dict[tuple[str, int], list[MathProblem]] = defaultdict(list)
    for p in sorted(problems, key=lambda q: q.identifier):
        if p.level >= minimum_level and p.identifier not in excluded:
            strata[(p.subject, p.level)].append(p)
    rng = random.Random(seed)
    order = sorted(strata)
    rng.shuffle(order)
    for key in order:
        rng.shuffle(strata[key])
    picked: list[MathProblem] = []
    while any(strata[k] for k in order):
        picked.extend(strata[k].pop() for k in order if strata[k])
    need = development_count + test_count
    if need > len(picked):
        raise ValueError(f"{need} problems requested, {len(picked)} eligible")
    return {"development": picked[:development_count], "test": picked[development_count:need]}


# ------------------------------------------------------------------ answers --
def _balanced(text: str, open_at: int) -> str | None:
    """Content of the brace group that opens at ``open_at`` (None when it never closes)."""
    depth = 0
    for i in range(open_at, len(text)):
        if text[i] == "{":
            depth += 1
        elif text[i] == "}":
            depth -= 1
            if depth == 0:
                return text[open_at + 1:i]
    return None


def final_answer(text: str) -> str | None:
    """The last boxed answer, else what follows the last "answer is" / "answer:"."""
    found = None
    for m in re.finditer(r"\\(?:boxed|fbox)\s*\{", text):
        inner = _balanced(text, m.end() - 1)
        if inner is not None:
            found = inner
    if found is not None:
        return found.strip()
    m = None
    for m in re.finditer(r"answer\s*(?:is|:)\s*", text, re.IGNORECASE):
        pass
    if m is not None:
        tail = text[m.end():].strip().split("\n")[0]
        return tail.rstrip(" .") or None
    return None


def _unfrac(s: str) -> str:
    """``\\frac{a}{b}`` (any nesting) -> ``(a)/(b)``; ``\\frac12`` -> ``(1)/(2)``."""
    while True:
        m = re.search(r"\\[dt]?frac", s)
        if m is None:
            return s
        i = m.end()
        parts = []
        for _ in range(2):
            while i < len(s) and s[i] == " ":
                i += 1
            if i < len(s) and s[i] == "{":
                inner = _balanced(s, i)
                if inner is None:
                    return s
                parts.append(inner)
                i += len(inner) + 2
            elif i < len(s):
                parts.append(s[i])
                i += 1
            else:
                return s
        s = s[:m.start()] + f"({parts[0]})/({parts[1]})" + s[i:]


def canonical_answer(text: str) -> str:
    s = text.strip().strip("$").strip()
    s = re.sub(r"\\text\s*\{([^{}]*)\}", r"\1", s)
    s = re.sub(r"\\mbox\s*\{([^{}]*)\}", r"\1", s)
    s = re.sub(r"\\(left|right|displaystyle|!|,|;|:|quad|qquad)", "", s)
    s = s.replace("^\\circ", "").replace("^{\\circ}", "").replace("\\circ", "").replace("°", "")
    s = s.replace("\\%", "").replace("%", "").replace("\\$", "")
    s = _unfrac(s)
    s = s.replace("\\cdot", "*").replace("\\times", "*")
    s = re.sub(r"\s+", "", s)
    s = s.rstrip(".")
    s = re.sub(r"^(?:[a-zA-Z]\w*)=(?=[^=]+$)", "", s)      # "x=5" -> "5"
    return s


def _as_number(s: str) -> Fraction | None:
    t = s.replace(",", "") if re.fullmatch(r"[-+]?\d{1,3}(,\d{3})+(\.\d+)?", s) else s
    m = re.fullmatch(r"\(?([-+]?\d+(?:\.\d+)?)\)?/\(?([-+]?\d+(?:\.\d+)?)\)?", t)
    try:
        if m:
            return Fraction(m.group(1)) / Fraction(m.group(2))
        if re.fullmatch(r"[-+]?\(?\d+(\.\d+)?\)?", t):
            return Fraction(t.replace("(", "").replace(")", ""))
    except (ValueError, ZeroDivisionError):
        return None
    return None


def _split_top(s: str) -> list[str]:
    depth, out, cur = 0, [], ""
    for ch in s:
        if ch in "([{":
            depth += 1
        elif ch in ")]}":
            depth -= 1
        if ch == "," and depth == 0:
            out.append(cur)
            cur = ""
        else:
            cur += ch
    out.append(cur)
    return out


def answers_equivalent(left: str, right: str) -> bool:
    a, b = canonical_answer(left), canonical_answer(right)
    if a == b:
        return True
    x, y = _as_number(a), _as_number(b)
    if x is not None and y is not None:
        return x == y
    brackets = "([", ")]"
    if a[:1] in brackets[0] and b[:1] == a[:1] and a[-1:] in brackets[1] and b[-1:] == a[-1:]:
        ea, eb = _split_top(a[1:-1]), _split_top(b[1:-1])
        return len(ea) == len(eb) > 1 and all(answers_equivalent(p, q) for p, q in zip(ea, eb))
    return False


def grade(prediction: str, reference: str) -> dict[str, bool]:
    answer = final_answer(prediction)
    return {"correct": answer is not None and answers_equivalent(answer, reference),
            "parseable": answer is not None, "reference_parseable": bool(canonical_answer(reference))}


# ---------------------------------------------------------------- isolation --
def _worker(conn) -> None:
    try:
        while True:
            msg = conn.recv()
            if msg is None:
                return
            op, args = msg
            try:
                if op == "grade":
                    conn.send((True, grade(*args)))
                elif op == "equivalent":
                    conn.send((True, answers_equivalent(*args)))
                else:
                    conn.send((False, f"unknown operation {op!r}"))
            except Exception as err:            # noqa: BLE001 - returned to the caller
                conn.send((False, f"{type(err).__name__}: {err}"))
    except (EOFError, BrokenPipeError):
        pass


class MathJudge:
    """Grades in one persistent child process; a call that exceeds ``timeout_seconds`` restarts it."""

    def __init__(self, timeout_seconds: float = 20.0):
        self.timeout_seconds = float(timeout_seconds)
        self._proc = None
        self._conn = None

    def _call(self, op: str, *args: str) -> Any:
        if self._proc is None:
            ctx = mp.get_context("spawn")
            self._conn, child = ctx.Pipe()
            self._proc = ctx.Process(target=_worker, args=(child,), daemon=True)
            self._proc.start()
            child.close()
        self._conn.send((op, args))
        if not self._conn.poll(self.timeout_seconds):
            self.close()
            raise TimeoutError("math answer grading timed out")
        ok, value = self._conn.recv()
        if not ok:
            raise ValueError(value)
        return value

    def grade(self, prediction: str, reference: str) -> dict[str, bool]:
        return self._call("grade", prediction, reference)

    def equivalent(self, left: str, right: str) -> bool:
        return bool(self._call("equivalent", left, right))

    def close(self) -> None:
        if self._proc is not None:
            try:
                self._conn.send(None)
            except (BrokenPipeError, OSError):
                pass
            self._proc.join(timeout=2)
            if self._proc.is_alive():
                self._proc.terminate()
                self._proc.join(timeout=2)
            self._conn.close()
            self._proc = self._conn = None


@dataclass(frozen=True, slots=True)
class MathReferenceVerifier:
    reference: str
    correct_reward: float = 1.0
    incorrect_reward: float = 0.0
    unparseable_reward: float = 0.0

    def score(self, _prompt: str, completion: str) -> float:
        g = grade(completion, self.reference)
        if not g["parseable"]:
            return self.unparseable_reward
        return self.correct_reward if g["correct"] else self.incorrect_reward


def build_math_reference_verifier(*, context: VerifierContext, correct_reward: float = 1.0,
                                  incorrect_reward: float = 0.0, unparseable_reward: float = 0.0
                                  ) -> MathReferenceVerifier:
    """Verifier factory: 1 for a final answer equivalent to the context's reference answer."""
    if context.reference is None:
        raise ValueError("the math verifier grades against a reference answer")
    return MathReferenceVerifier(str(context.reference), correct_reward, incorrect_reward, unparseable_reward)


__all__ = ["MathJudge", "MathProblem", "MathReferenceVerifier", "answers_equivalent", "build_math_reference_verifier",
           "canonical_answer", "final_answer", "grade", "load_math500", "stratified_subset"]
