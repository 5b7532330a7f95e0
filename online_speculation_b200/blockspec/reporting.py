"""Report helpers: JSON-safe payloads with resource identities removed
(online-speculation/src/blockspec/reporting.py:28-69)."""

from __future__ import annotations

import hashlib
import json
import math
import os
import socket

_SENSITIVE = ("path", "host", "user", "dir", "file")


def parameter_digest(model) -> str:
    h = hashlib.sha256()
    for n, p in model.state_dict().items():
        h.update(n.encode())
        h.update(p.detach().contiguous().cpu().float().numpy().tobytes())
    return h.hexdigest()


def _identity(key: str, value) -> bool:
    """A string or path stored under a location-like key names a local resource; measurements
    under such keys (``actual_path``, ``profiles``) are kept."""
    names = isinstance(value, (str, os.PathLike)) or (
        isinstance(value, (list, tuple)) and bool(value) and all(isinstance(v, (str, os.PathLike)) for v in value))
    return names and any(s in key.lower() for s in _SENSITIVE)


def scrub(value, *, key: str = ""):
    """Drop local resource identities (paths, host names) and non-finite numbers."""
    if isinstance(value, dict):
        return {k: scrub(v, key=k) for k, v in value.items() if not _identity(str(k), v)}
    if isinstance(value, (list, tuple)):
        return [scrub(v, key=key) for v in value]
    if isinstance(value, float) and not math.isfinite(value):
        return None
    if isinstance(value, str):
        home = os.path.expanduser("~")
        value = value.replace(home, "~").replace(socket.gethostname(), "<host>")
    return value


def write_report(path, payload: dict) -> None:
    tmp = f"{path}.tmp"
    with open(tmp, "w") as f:
        json.dump(scrub(payload), f, indent=1, sort_keys=True)
    os.replace(tmp, path)
