"""Stable hashing, atomic JSON, resumable JSONL and dotted-key config overrides.

* ``json_fingerprint``: SHA-256 of canonical JSON (sorted keys, compact
  separators) -- the identity of a command plan, config or record key;
* ``file_sha256`` / ``cached_file_sha256``: content hashes of large immutable
  artifacts, cached by (path, size, mtime, ctime) identity;
* ``write_json_atomic``: write to a temporary file in the same directory,
  fsync, rename -- a crash leaves the previous artifact intact;
* ``load_jsonl`` / ``append_jsonl`` / ``indexed_records``: resumable result
  files keyed by a record identity;
* ``apply_config_overrides``: ``section.key=value`` overrides parsed as TOML
  values that may only replace keys that already exist.

Reference behaviour: experiments/shared/artifacts.py:15-299,
experiments/shared/config_overrides.py:10-48.
"""

from __future__ import annotations

import hashlib
import json
import os
import tempfile
import tomllib
from collections.abc import Callable, Iterable, Mapping, Sequence
from copy import deepcopy
from pathlib import Path
from typing import Any


def json_fingerprint(value: Any) -> str:
    return hashlib.sha256(json.dumps(value, ensure_ascii=False, sort_keys=True,
                                     separators=(",", ":")).encode("utf-8")).hexdigest()


def file_sha256(path: Path, *, chunk_bytes: int = 8 << 20) -> str:
    if chunk_bytes <= 0:
        raise ValueError("chunk_bytes must be positive")
    h = hashlib.sha256()
    with Path(path).open("rb") as f:
        while chunk := f.read(chunk_bytes):
            h.update(chunk)
    return h.hexdigest()


def cached_file_sha256(path: Path, *, cache_directory: Path, expected: str | None = None) -> str:
    p = Path(path).resolve()
    if not p.is_file():
        raise FileNotFoundError(p)
    st = p.stat()
    ident = {"path": str(p), "size": st.st_size, "mtime_ns": st.st_mtime_ns, "ctime_ns": st.st_ctime_ns}
    cache = Path(cache_directory).resolve() / f"{hashlib.sha256(str(p).encode()).hexdigest()}.json"
    digest = None
    if cache.is_file():
        try:
            old = json.loads(cache.read_text(encoding="utf-8"))
        except (OSError, json.JSONDecodeError):
            old = None
        if isinstance(old, dict) and all(old.get(k) == v for k, v in ident.items()):
            cand = old.get("sha256")
            if isinstance(cand, str) and len(cand) == 64:
                digest = cand
    if digest is None:
        digest = file_sha256(p)
        write_json_atomic(cache, {**ident, "sha256": digest}, indent=2)
    if expected is not None and digest != expected:
        raise ValueError(f"artifact hash mismatch for {p}: expected {expected}, got {digest}")
    return digest


def write_json_atomic(path: Path, value: Any, *, indent: int | None = None) -> None:
    path = Path(path)
    path.parent.mkdir(parents=True, exist_ok=True)
    tmp = None
    try:
        with tempfile.NamedTemporaryFile("w", encoding="utf-8", dir=path.parent, prefix=path.name + ".",
                                         suffix=".tmp", delete=False) as f:
            tmp = Path(f.name)
            json.dump(value, f, ensure_ascii=False, indent=indent)
            f.write("\n")
            f.flush()
            os.fsync(f.fileno())
        tmp.replace(path)
        tmp = None
    finally:
        if tmp is not None:
            tmp.unlink(missing_ok=True)


def load_jsonl(path: Path) -> list[dict[str, Any]]:
    """Records of a JSONL file; a torn final line (an interrupted append) is ignored."""
    path = Path(path)
    if not path.is_file():
        return []
    lines = path.read_text(encoding="utf-8").splitlines()
    out = []
    for i, line in enumerate(lines):
        if not line.strip():
            continue
        try:
            rec = json.loads(line)
        except json.JSONDecodeError:
            if i == len(lines) - 1:
                break
            raise ValueError(f"corrupt JSONL record at {path}:{i + 1}") from None
        if not isinstance(rec, dict):
            raise ValueError(f"JSONL record at {path}:{i + 1} is not an object")
        out.append(rec)
    return out


def append_jsonl(path: Path, record: Mapping[str, Any]) -> None:
    path = Path(path)
    path.parent.mkdir(parents=True, exist_ok=True)
    with path.open("a", encoding="utf-8") as f:
        f.write(json.dumps(record, ensure_ascii=False, sort_keys=True) + "\n")
        f.flush()
        os.fsync(f.fileno())


def indexed_records(records: Iterable[Mapping[str, Any]], key: Callable[[Mapping[str, Any]], Any]
                    ) -> dict[Any, dict[str, Any]]:
    """Records by identity; a repeated identity must repeat the same record."""
    out: dict[Any, dict[str, Any]] = {}
    for r in records:
        k = key(r)
        if k in out and out[k] != dict(r):
            raise ValueError(f"conflicting records for {k!r}")
        out[k] = dict(r)
    return out


def parse_override_value(text: str) -> Any:
    if text.strip().lower() in ("none", "null"):
        return None
    try:
        return tomllib.loads(f"value = {text}")["value"]
    except tomllib.TOMLDecodeError:
        return text


def apply_config_overrides(config: Mapping[str, Any], overrides: Sequence[str]) -> dict[str, Any]:
    out = deepcopy(dict(config))
    for item in overrides:
        if "=" not in item:
            raise ValueError(f"config override must contain '=': {item!r}")
        dotted, raw = item.split("=", 1)
        parts = [p.strip() for p in dotted.split(".")]
        if not parts or any(not p for p in parts):
            raise ValueError(f"invalid config override key: {dotted!r}")
        node = out
        for p in parts[:-1]:
            if not isinstance(node.get(p), dict):
                raise KeyError(f"unknown config override path: {dotted!r}")
            node = node[p]
        if parts[-1] not in node:
            raise KeyError(f"unknown config override key: {dotted!r}")
        node[parts[-1]] = parse_override_value(raw.strip())
    return out


__all__ = ["append_jsonl", "apply_config_overrides", "cached_file_sha256", "file_sha256", "indexed_records",
           "json_fingerprint", "load_jsonl", "parse_override_value", "write_json_atomic"]
