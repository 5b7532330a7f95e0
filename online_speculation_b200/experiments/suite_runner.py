"""Resumable, manifested command suites.

A suite is a fixed list of argv commands plus metadata; its plan fingerprint
(canonical JSON hash) is stored in a manifest next to the number of completed
commands.  Re-running the same plan resumes after the last completed command;
a different plan for an existing manifest is refused unless ``restart``.
Commands run with the repository on PYTHONPATH.

Reference behaviour: experiments/shared/suite_runner.py:16-121.
"""

from __future__ import annotations

import json
import os
import shlex
import subprocess
from collections.abc import Mapping, Sequence
from datetime import datetime, timezone
from pathlib import Path
from typing import Any

from .artifacts import json_fingerprint, write_json_atomic


def command_text(command: Sequence[str]) -> str:
    return subprocess.list2cmdline(list(command)) if os.name == "nt" else shlex.join(list(command))


def repository_environment(root: Path, *, base: Mapping[str, str] | None = None) -> dict[str, str]:
    env = dict(os.environ if base is None else base)
    env["PYTHONPATH"] = os.pathsep.join(p for p in (str(root), env.get("PYTHONPATH", "")) if p)
    return env


def _now() -> str:
    return datetime.now(timezone.utc).isoformat()


def run_manifested_commands(*, commands: Sequence[Sequence[str]], root: Path, manifest_path: Path,
                            metadata: Mapping[str, Any], dry_run: bool = False,
                            environment: Mapping[str, str] | None = None, restart: bool = False) -> dict[str, Any]:
    argv = [list(c) for c in commands]
    fp = json_fingerprint({"metadata": dict(metadata), "commands": argv})
    manifest_path = Path(manifest_path)
    done = 0
    if manifest_path.is_file() and not restart:
        manifest = json.loads(manifest_path.read_text(encoding="utf-8"))
        if manifest.get("plan_fingerprint") != fp:
            raise ValueError(f"existing suite manifest has a different command plan: {manifest_path}")
        done = int(manifest.get("completed_commands", 0))
        if not 0 <= done <= len(argv):
            raise ValueError("suite manifest has an invalid completed command count")
        manifest.pop("finished_at_utc", None)
        manifest["resumed_at_utc"] = _now()
    else:
        manifest = {"schema_version": 2, **dict(metadata), "commands": [command_text(c) for c in argv],
                    "command_argv": argv, "command_sha256": [json_fingerprint(c) for c in argv],
                    "plan_fingerprint": fp, "started_at_utc": _now(), "completed_commands": 0}
    manifest["status"] = "dry_run" if dry_run else "running"
    write_json_atomic(manifest_path, manifest, indent=2)
    for i, c in enumerate(argv):
        print(f"{'SKIP' if i < done else 'RUN'} {command_text(c)}", flush=True)
    if dry_run:
        return manifest
    env = repository_environment(Path(root), base=environment)
    try:
        for i in range(done, len(argv)):
            subprocess.run(argv[i], cwd=root, env=env, check=True)
            manifest["completed_commands"] = i + 1
            write_json_atomic(manifest_path, manifest, indent=2)
    except BaseException:
        manifest["status"] = "failed"
        manifest["finished_at_utc"] = _now()
        write_json_atomic(manifest_path, manifest, indent=2)
        raise
    manifest["status"] = "complete"
    manifest["finished_at_utc"] = _now()
    write_json_atomic(manifest_path, manifest, indent=2)
    return manifest


__all__ = ["command_text", "repository_environment", "run_manifested_commands"]
