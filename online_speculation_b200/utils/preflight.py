"""Environment preflight: can this machine run a stage of the framework?

Checks are grouped by stage -- ``inference`` (one B200 and the compiled extension),
``multi_gpu`` (NCCL, symmetric memory and peer access between every device pair),
``training`` (the fused optimizer and training kernels) and ``checkpoints`` (safetensors,
the HF tokenizer stack) -- and each returns (name, passed, detail).  Nothing here changes a
device setting: the checks read versions, device properties and peer-access capability.

    python -m online_speculation_b200.utils.preflight --stages inference,multi_gpu

prints one JSON report and exits non-zero when a requested stage fails.  Role-specific
dependency checks of experiments/shared/environment.py, restated for this framework's own
requirements (a CUDA build of torch >= 2.9, compute capability 10.0, the in-tree extension).
"""

from __future__ import annotations

import argparse
import importlib
import json
import sys
from collections.abc import Callable, Sequence
from typing import Any

STAGES = ("inference", "multi_gpu", "training", "checkpoints")
Check = tuple[str, bool, str]


def _version_at_least(version: str, minimum: tuple[int, ...]) -> bool:
    parts = []
    for piece in version.split("+")[0].split(".")[:len(minimum)]:
        digits = "".join(ch for ch in piece if ch.isdigit())
        parts.append(int(digits) if digits else 0)
    return tuple(parts) >= minimum


def _module(name: str) -> tuple[bool, str]:
    try:
        mod = importlib.import_module(name)
    except Exception as err:                    # noqa: BLE001 - reported, not raised
        return False, f"{type(err).__name__}: {err}"
    return True, str(getattr(mod, "__version__", "present"))


def inference_checks(torch_mod=None) -> list[Check]:
    import torch

    t = torch_mod or torch
    out: list[Check] = [("torch >= 2.9", _version_at_least(t.__version__, (2, 9)), t.__version__),
                        ("torch built with CUDA", t.version.cuda is not None, str(t.version.cuda))]
    cuda = bool(t.cuda.is_available())
    out.append(("a CUDA device is visible", cuda, f"{t.cuda.device_count()} device(s)" if cuda else "none"))
    if cuda:
        caps = [t.cuda.get_device_capability(i) for i in range(t.cuda.device_count())]
        out.append(("every device is compute capability 10.0 (sm_100a)", all(c == (10, 0) for c in caps), str(caps)))
    try:
        from ..ops import _ext

        ext = _ext.load()
        out.append(("in-tree extension loads", ext is not None, "loaded" if ext is not None else str(_ext._error)))
    except Exception as err:                    # noqa: BLE001
        out.append(("in-tree extension loads", False, f"{type(err).__name__}: {err}"))
    return out


def multi_gpu_checks(torch_mod=None) -> list[Check]:
    import torch

    t = torch_mod or torch
    dist = t.distributed
    out: list[Check] = [("torch.distributed with NCCL", bool(dist.is_available() and dist.is_nccl_available()), ""),
                        ("symmetric memory module", *_module("torch.distributed._symmetric_memory"))]
    n = t.cuda.device_count() if t.cuda.is_available() else 0
    out.append(("at least two devices", n >= 2, f"{n} device(s)"))
    if n >= 2:
        missing = [(i, j) for i in range(n) for j in range(n) if i != j and not t.cuda.can_device_access_peer(i, j)]
        out.append(("peer access between every device pair", not missing, f"missing {missing}" if missing else "all"))
    return out


def training_checks() -> list[Check]:
    out: list[Check] = []
    try:
        from ..ops import _ext

        ext = _ext.load()
        for fn in ("adamw", "grad_sq_norm", "grpo_loss", "dp_reduce_scatter", "dp_all_gather"):
            out.append((f"extension exports {fn}", ext is not None and hasattr(ext, fn), ""))
    except Exception as err:                    # noqa: BLE001
        out.append(("extension exports the training kernels", False, f"{type(err).__name__}: {err}"))
    return out


def checkpoint_checks() -> list[Check]:
    return [(f"python package {name}", *_module(name)) for name in ("safetensors", "tokenizers", "transformers")]


RUNNERS: dict[str, Callable[[], list[Check]]] = {"inference": inference_checks, "multi_gpu": multi_gpu_checks,
                                                 "training": training_checks, "checkpoints": checkpoint_checks}


def preflight(stages: Sequence[str] = STAGES, runners: dict[str, Callable[[], list[Check]]] | None = None
              ) -> dict[str, Any]:
    runners = runners or RUNNERS
    unknown = sorted(set(stages) - set(runners))
    if unknown:
        raise ValueError(f"unknown preflight stages {unknown}; choose from {sorted(runners)}")
    report: dict[str, Any] = {"python": sys.version.split()[0], "stages": {}}
    for stage in stages:
        checks = runners[stage]()
        report["stages"][stage] = {"passed": all(ok for _, ok, _ in checks),
                                   "checks": [{"check": n, "passed": ok, "detail": d} for n, ok, d in checks]}
    report["passed"] = all(s["passed"] for s in report["stages"].values())
    return report


def main(argv=None) -> int:
    p = argparse.ArgumentParser(prog="python -m online_speculation_b200.utils.preflight")
    p.add_argument("--stages", default="inference,checkpoints", help=f"comma-separated subset of {','.join(STAGES)}")
    a = p.parse_args(argv)
    report = preflight([s for s in a.stages.split(",") if s])
    print(json.dumps(report, indent=2))
    return 0 if report["passed"] else 1


if __name__ == "__main__":
    raise SystemExit(main())
