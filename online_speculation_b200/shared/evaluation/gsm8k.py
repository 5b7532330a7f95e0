"""GSM8K splits pinned by SHA-256, the shared prompt suffix, preregistered subsets and accuracy.

The split URLs, digests, row counts and prompt suffix are the public GSM8K
files and the reference's prompt text (src/inference_scaling/shared/evaluation/gsm8k.py:45-141):
they identify the data, so they are kept exactly.  A local file is accepted
only if its digest matches; downloading is attempted only when the file is
missing and a network is available.
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

_BASE = "https://raw.githubusercontent.com/openai/grade-school-math/master/grade_school_math/data/"
GSM8K_TRAIN_URL = _BASE + "train.jsonl"
GSM8K_TRAIN_SHA256 = "17f347dc51477c50d4efb83959dbb7c56297aba886e5544ee2aaed3024813465"
GSM8K_TEST_URL = _BASE + "test.jsonl"
GSM8K_TEST_SHA256 = "3730d312f6e3440559ace48831e51066acaca737f6eabec99bccb9e4b3c39d14"
GSM8K_PROMPT_SUFFIX = ("\n\nSolve the problem step by step. End your response with exactly "
                       "`#### <number>`, where <number> is the final numeric answer.")
GSM8KSplit = Literal["train", "test"]
_SPLITS = {"train": (GSM8K_TRAIN_URL, GSM8K_TRAIN_SHA256, 7473), "test": (GSM8K_TEST_URL, GSM8K_TEST_SHA256, 1319)}


@dataclass(frozen=True, slots=True)
class GSM8KProblem:
    index: int
    question: str
    gold_solution: str
    gold_answer: Fraction


def _digest(path: Path) -> str:
    h = hashlib.sha256()
    with path.open("rb") as f:
        while chunk := f.read(1 << 20):
            h.update(chunk)
    return h.hexdigest()


def download_gsm8k(path: str | Path, *, split: GSM8KSplit = "test") -> Path:
    url, sha, _ = _SPLITS[split]
    dst = Path(path)
    if dst.is_file() and _digest(dst) == sha:
        return dst
    dst.parent.mkdir(parents=True, exist_ok=True)
    tmp = dst.with_suffix(dst.suffix + ".download")
    try:
        urllib.request.urlretrieve(url, tmp)
        got = _digest(tmp)
        if got != sha:
            raise ValueError(f"GSM8K {split} checksum mismatch: expected {sha}, downloaded {got}")
        tmp.replace(dst)
    finally:
        tmp.unlink(missing_ok=True)
    return dst


def load_gsm8k(path: str | Path, *, split: GSM8KSplit = "test", download: bool = True) -> tuple[GSM8KProblem, ...]:
    _, sha, rows = _SPLITS[split]
    src = download_gsm8k(path, split=split) if download else Path(path)
    if _digest(src) != sha:
        raise ValueError(f"{src} is not the pinned official GSM8K {split} file")
    out = []
    with src.open("r", encoding="utf-8") as f:
        for i, line in enumerate(f):
            item = json.loads(line)
            ans = extract_numeric_answer(str(item["answer"]))
            if ans is None:
                raise ValueError(f"could not parse GSM8K gold answer at row {i}")
            out.append(GSM8KProblem(i, str(item["question"]), str(item["answer"]), ans))
    if len(out) != rows:
        raise ValueError(f"expected {rows:,} GSM8K {split} rows, found {len(out):,}")
    return tuple(out)


def gsm8k_prompt(question: str) -> str:
    return question + GSM8K_PROMPT_SUFFIX


def select_problems(problems: Sequence[GSM8KProblem], count: int | None, *, seed: int) -> tuple[GSM8KProblem, ...]:
    """A preregistered random subset in dataset order (drawn before any inference)."""
    if count is None or count == len(problems):
        return tuple(problems)
    if not 0 < count <= len(problems):
        raise ValueError(f"count must lie in [1, {len(problems)}]")
    return tuple(problems[i] for i in sorted(random.Random(seed).sample(range(len(problems)), count)))


def accuracy(correct: Iterable[bool]) -> float:
    vals = [bool(v) for v in correct]
    if not vals:
        raise ValueError("accuracy requires at least one result")
    return sum(vals) / len(vals)


__all__ = ["GSM8KProblem", "GSM8K_PROMPT_SUFFIX", "GSM8K_TEST_SHA256", "GSM8K_TEST_URL", "GSM8K_TRAIN_SHA256",
           "GSM8K_TRAIN_URL", "accuracy", "download_gsm8k", "gsm8k_prompt", "load_gsm8k", "select_problems"]
