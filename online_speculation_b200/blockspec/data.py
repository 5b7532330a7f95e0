"""JSONL prompt / token contract shared by the CLI commands
(online-speculation/src/blockspec/data.py, corpus.py).

Each record holds ``input_ids`` (a tokenized prompt or training sequence) and
optionally ``id`` and ``group`` (question-grouped splits keep every record of
one question on the same side).
"""

from __future__ import annotations

import hashlib
import json
from pathlib import Path


def read_records(path) -> list[dict]:
    out = []
    for line in Path(path).read_text().splitlines():
        if line.strip():
            rec = json.loads(line)
            ids = rec.get("input_ids")
            if not isinstance(ids, list) or not ids or any(type(x) is not int or x < 0 for x in ids):
                raise ValueError("each record needs non-negative integer input_ids")
            out.append(rec)
    return out


def write_records(path, records) -> None:
    Path(path).write_text("".join(json.dumps(r) + "\n" for r in records))


def grouped_split(records: list[dict], fraction: float, *, key: str = "group") -> tuple[list, list]:
    """Deterministic split by a hash of the group key (all of a group on one side)."""
    a, b = [], []
    for r in records:
        g = str(r.get(key, r.get("id", json.dumps(r["input_ids"][:16]))))
        (a if int(hashlib.sha256(g.encode()).hexdigest()[:8], 16) / 0xFFFFFFFF < fraction else b).append(r)
    return a, b
