"""GSM8K: pinned split files, the shared prompt suffix, preregistered subsets, accuracy.

Each split is identified by its public URL, SHA-256 digest and row count, and the
prompt suffix is the reference's text (src/inference_scaling/shared/evaluation/gsm8k.py):
these are data identities, so they are kept byte for byte, and so is the subset
draw (``random.Random(seed).sample`` over row indices, returned in dataset order),
which makes a preregistered subset name the same questions as in the reference's
reports.  A local file is used only if its digest matches; a download is attempted
only when no matching file exists.
"""

from __future__ import annotations

import hashlib
import json
import random
import urllib.request
from dataclasses import dataclass
from fractions import Fraction
from pathlib import Path
from typing import Iterable, Literal, Sequence

from .numeric import extract_numeric_answer

GSM8K_TRAIN_URL = "https://raw.githubusercontent.com/openai/grade-school-math/master/grade_school_math/data/train.jsonl"
GSM8K_TRAIN_SHA256 = "17f347dc51477c50d4efb83959dbb7c56297aba886e5544ee2aaed3024813465"
GSM8K_TEST_URL = "https://raw.githubusercontent.com/openai/grade-school-math/master/grade_school_math/data/test.jsonl"
GSM8K_TEST_SHA256 = "3730d312f6e3440559ace48831e51066acaca737f6eabec99bccb9e4b3c39d14"
GSM8K_PROMPT_SUFFIX = ("\n\nSolve the problem step by step. End your response with exactly "
                       "`#### <number>`, where <number> is the final numeric answer.")
GSM8KSplit = Literal["train", "test"]


@dataclass(frozen=True)
class _SplitFile:
    url: str
    sha256: str
    rows: int


_SPLITS = {"train": _SplitFile(GSM8K_TRAIN_URL, GSM8K_TRAIN_SHA256, 7473),
           "test": _SplitFile(GSM8K_TEST_URL, GSM8K_TEST_SHA256, 1319)}


@dataclass(frozen=True, slots=True)
class GSM8KProblem:
    index: int
    question: str
    gold_solution: str
    gold_answer: Fraction


def _sha256_of(path: Path) -> str:
    digest = hashlib.sha256()
    with path.open("rb") as handle:
        for block in iter(lambda: handle.read(1 << 20), b""):
            digest.update(block)
    return digest.hexdigest()


def download_gsm8k(path: str | Path, *, split: GSM8KSplit = "test") -> Path:
    spec = _SPLITS[split]
    target = Path(path)
    if target.is_file() and _sha256_of(target) == spec.sha256:
        return target
    target.parent.mkdir(parents=True, exist_ok=True)
    partial = target.parent / (target.name + ".partial")
    try:
        with urllib.request.urlopen(spec.url) as response, partial.open("wb") as out:
            for block in iter(lambda: response.read(1 << 20), b""):
                out.write(block)
        got = _sha256_of(partial)
        if got != spec.sha256:
            raise ValueError(f"GSM8K {split}: downloaded digest {got} is not the pinned {spec.sha256}")
        partial.replace(target)
    finally:
        partial.unlink(missing_ok=True)
    return target


def _rows(path: Path) -> Iterable[tuple[int, dict]]:
    with path.open("r", encoding="utf-8") as handle:
        for i, line in enumerate(handle):
            yield i, json.loads(line)


def load_gsm8k(path: str | Path, *, split: GSM8KSplit = "test", download: bool = True) -> tuple[GSM8KProblem, ...]:
    spec = _SPLITS[split]
    source = download_gsm8k(path, split=split) if download else Path(path)
    if _sha256_of(source) != spec.sha256:
        raise ValueError(f"{source} does not match the pinned GSM8K {split} digest")
    problems = []
    for i, row in _rows(source):
        gold = extract_numeric_answer(str(row["answer"]))
        if gold is None:
            raise ValueError(f"GSM8K {split} row {i}: no numeric gold answer")
        problems.append(GSM8KProblem(i, str(row["question"]), str(row["answer"]), gold))
    if len(problems) != spec.rows:
        raise ValueError(f"GSM8K {split} has {spec.rows} rows; {source} holds {len(problems)}")
    return tuple(problems)


def gsm8k_prompt(question: str) -> str:
    return f"{question}{GSM8K_PROMPT_SUFFIX}"


def select_problems(problems: Sequence[GSM8KProblem], count: int | None, *, seed: int) -> tuple[GSM8KProblem, ...]:
    """Preregistered subset of ``count`` problems (chosen before any inference), in dataset order."""
    n = len(problems)
    if count is None or count == n:
        return tuple(problems)
    if not 1 <= count <= n:
        raise ValueError(f"a subset of {count} problems is not possible from {n}")
    picked = random.Random(seed).sample(range(n), count)
    return tuple(problems[i] for i in sorted(picked))


def accuracy(correct: Iterable[bool]) -> float:
    flags = [bool(c) for c in correct]
    if not flags:
        raise ValueError("accuracy of an empty result set is undefined")
    return sum(flags) / len(flags)


__all__ = ["GSM8KProblem", "GSM8K_PROMPT_SUFFIX", "GSM8K_TEST_SHA256", "GSM8K_TEST_URL", "GSM8K_TRAIN_SHA256",
           "GSM8K_TRAIN_URL", "accuracy", "download_gsm8k", "gsm8k_prompt", "load_gsm8k", "select_problems"]
