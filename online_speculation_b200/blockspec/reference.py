"""Integrity gate for an optional external numerical reference (a local model directory).

Before any code or weights of a reference implementation are used, the caller's
manifest pins them: ``models.base.reference_lf_sha256`` maps each source / config
file to the SHA-256 of its bytes with CRLF normalised to LF, ``weight_filename`` /
``weight_sha256`` pin the single weight shard.  :func:`checked_reference` refuses
files outside the directory, any digest mismatch, and a shard index that points at
other shards; it returns the manifest's ``base`` entry.  Behaviour of
online-speculation/src/blockspec/reference.py (``checked_reference``).
"""

from __future__ import annotations

import hashlib
import json
from pathlib import Path

CHUNK = 8 << 20


def _text_digest(path: Path) -> str:
    return hashlib.sha256(path.read_bytes().replace(b"\r\n", b"\n")).hexdigest()


def _file_digest(path: Path) -> str:
    digest = hashlib.sha256()
    with path.open("rb") as stream:
        while True:
            block = stream.read(CHUNK)
            if not block:
                break
            digest.update(block)
    return digest.hexdigest()


def checked_reference(directory, manifest) -> dict:
    root = Path(directory).resolve()
    entry = json.loads(Path(manifest).read_text(encoding="utf-8"))["models"]["base"]
    pinned = dict(entry["reference_lf_sha256"])
    weights = entry["weight_filename"]
    for name in list(pinned) + [weights]:
        if (root / name).resolve().parent != root:
            raise ValueError(f"pinned file {name!r} is not directly inside {root}")
    for name, want in pinned.items():
        if _text_digest(root / name) != want:
            raise ValueError(f"{name} does not match its pinned digest")
    if _file_digest(root / weights) != entry["weight_sha256"]:
        raise ValueError(f"{weights} does not match its pinned digest")
    index = root / "model.safetensors.index.json"
    if index.is_file():
        shards = set(json.loads(index.read_text(encoding="utf-8"))["weight_map"].values())
        if shards != {weights}:
            raise ValueError("the weight index names shards other than the pinned one")
    return entry


__all__ = ["checked_reference"]
