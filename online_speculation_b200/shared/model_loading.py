"""Model roles, loading options, checkpoint resolution and the identity string used by caches.

Reference behaviour: src/inference_scaling/shared/model_loading.py:18-133.
``model_identity`` produces the same string format (``model[+adapter:a][;key=value...]``)
so generation, re-scoring and replay caches agree across runs.
"""

from __future__ import annotations

import json
from collections.abc import Mapping
from pathlib import Path
from typing import Any

MODEL_ROLES = ("base", "proposal", "rl")
_OPTIONS = frozenset({"revision", "tokenizer_name_or_path", "tokenizer_revision", "adapter_revision", "cache_dir",
                      "local_files_only", "trust_remote_code", "device_map", "attn_implementation", "model_kwargs",
                      "tokenizer_kwargs"})


def model_role(path: str, config: Mapping[str, Any], *, adapter_base: str | None = None) -> str:
    for role in MODEL_ROLES:
        got = config.get("models", {}).get(role)
        if got is not None and (str(got) == path or Path(str(got)).resolve() == Path(path).resolve()):
            return role
    return "rl" if adapter_base is not None else "base"


def model_loading_options(config: Mapping[str, Any], role: str = "base") -> dict[str, Any]:
    """Common ``[model_loading]`` options overlaid with the role's own table."""
    if role not in MODEL_ROLES:
        raise ValueError(f"unknown model role: {role}")
    table = config.get("model_loading", {})
    if not isinstance(table, Mapping) or not isinstance(table.get(role, {}), Mapping):
        raise TypeError("model_loading and its role settings must be tables")
    common = {k: v for k, v in table.items() if k not in MODEL_ROLES}
    own = dict(table.get(role, {}))
    out = {**common, **own}
    bad = set(out) - _OPTIONS
    if bad:
        raise ValueError("unknown model_loading settings: " + ", ".join(sorted(bad)))
    for name in ("model_kwargs", "tokenizer_kwargs"):
        a, b = common.get(name, {}), own.get(name, {})
        if not isinstance(a, Mapping) or not isinstance(b, Mapping):
            raise TypeError(f"model_loading.{name} must be a table")
        if a or b:
            out[name] = {**a, **b}
    runtime = config.get("runtime", {})
    for name, default in (("local_files_only", True), ("trust_remote_code", False)):
        out.setdefault(name, runtime.get(name, default))
        if not isinstance(out[name], bool):
            raise TypeError(f"model_loading.{name} must be boolean")
    models = config.get("models", {})
    adapter = role == "rl" and models.get("rl_kind") == "peft_adapter"
    key = "base_revision" if adapter else f"{role}_revision"
    if "revision" not in out and key in models and not adapter:
        out["revision"] = str(models[key])
    if adapter and "revision" not in out:
        out["revision"] = model_loading_options(config, "base").get("revision")
    return out


def resolve_checkpoint_path(name_or_path: str, *, revision: str | None = None, cache_dir: str | None = None,
                            local_files_only: bool = True) -> Path:
    """A local checkpoint directory, or a Hub snapshot (offline unless ``local_files_only`` is False)."""
    p = Path(name_or_path).expanduser()
    if p.is_dir():
        return p.resolve()
    if p.is_absolute() or name_or_path.startswith(("./", "../", ".\\", "..\\")):
        raise FileNotFoundError(p)
    from huggingface_hub import snapshot_download

    return Path(snapshot_download(name_or_path, revision=revision, cache_dir=cache_dir,
                                  local_files_only=local_files_only,
                                  ignore_patterns=["*.h5", "*.msgpack", "*.onnx", "*.gguf", "*.ot", "original/*"]))


def model_identity(model: str, adapter: str | None = None, *, revision: str | None = None,
                   adapter_revision: str | None = None, tokenizer: str | None = None,
                   tokenizer_revision: str | None = None) -> str:
    s = model if adapter is None else f"{model}+adapter:{adapter}"
    for k, v in (("revision", revision), ("adapter_revision", adapter_revision), ("tokenizer", tokenizer),
                 ("tokenizer_revision", tokenizer_revision)):
        if v is not None:
            s += f";{k}={v}"
    return s


def checkpoint_weight_files(path: Path) -> tuple[Path, ...]:
    """Weight files of a safetensors / PyTorch checkpoint (single file or sharded index), without loading."""
    d = Path(path).resolve()
    for single, index in (("model.safetensors", "model.safetensors.index.json"),
                          ("pytorch_model.bin", "pytorch_model.bin.index.json")):
        if (d / single).is_file():
            return (d / single,)
        if not (d / index).is_file():
            continue
        data = json.loads((d / index).read_text(encoding="utf-8"))
        wm = data.get("weight_map") if isinstance(data, dict) else None
        if not isinstance(wm, dict) or not wm:
            raise ValueError(f"invalid checkpoint weight_map: {d / index}")
        if not all(isinstance(v, str) for v in wm.values()):
            raise ValueError("checkpoint shard names must be strings")
        files = []
        for name in sorted(set(wm.values())):
            sp = Path(name)
            if sp.is_absolute() or sp.drive or ".." in sp.parts or "\\" in name:
                raise ValueError(f"checkpoint shard must be relative to its directory: {name}")
            if not (d / name).is_file():
                raise FileNotFoundError(d / name)
            files.append(d / name)
        return tuple(files)
    raise FileNotFoundError(f"no supported checkpoint weights or shard index in {d}")


__all__ = ["MODEL_ROLES", "checkpoint_weight_files", "model_identity", "model_loading_options", "model_role",
           "resolve_checkpoint_path"]
