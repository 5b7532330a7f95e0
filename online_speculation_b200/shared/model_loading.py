"""Model roles, loading options, checkpoint files and the identity string that keys caches.

Options come from ``[model_loading]``: top-level keys apply to every role and a
per-role sub-table (``base`` / ``proposal`` / ``rl``) overrides them, with the two
keyword-argument tables merged key by key.  ``local_files_only`` and
``trust_remote_code`` fall back to ``[runtime]``.  Revisions fall back to
``[models] <role>_revision`` (an RL PEFT adapter loads on the base revision).

``model_identity`` renders ``model[+adapter:a][;key=value...]`` in a fixed key
order: generation, re-scoring and replay caches written by the reference
(src/inference_scaling/shared/model_loading.py) key on that string, so the format
is kept.
"""

from __future__ import annotations

import json
from collections.abc import Mapping
from pathlib import Path, PurePath
from typing import Any

MODEL_ROLES = ("base", "proposal", "rl")
_ALLOWED = frozenset({"revision", "tokenizer_name_or_path", "tokenizer_revision", "adapter_revision", "cache_dir",
                      "local_files_only", "trust_remote_code", "device_map", "attn_implementation", "model_kwargs",
                      "tokenizer_kwargs"})
_MERGED_TABLES = ("model_kwargs", "tokenizer_kwargs")
_RUNTIME_DEFAULTS = (("local_files_only", True), ("trust_remote_code", False))
_IDENTITY_KEYS = ("revision", "adapter_revision", "tokenizer", "tokenizer_revision")


def _same_path(a: str, b: str) -> bool:
    return a == b or Path(a).resolve() == Path(b).resolve()


def model_role(path: str, config: Mapping[str, Any], *, adapter_base: str | None = None) -> str:
    models = config.get("models", {})
    matches = [role for role in MODEL_ROLES if models.get(role) is not None and _same_path(str(models[role]), path)]
    if matches:
        return matches[0]
    return "base" if adapter_base is None else "rl"


def _table(value: object, what: str) -> Mapping[str, Any]:
    if not isinstance(value, Mapping):
        raise TypeError(f"{what} must be a TOML table")
    return value


def model_loading_options(config: Mapping[str, Any], role: str = "base") -> dict[str, Any]:
    """Shared ``[model_loading]`` settings overlaid with the role's table."""
    if role not in MODEL_ROLES:
        raise ValueError(f"role {role!r} is not one of {MODEL_ROLES}")
    root = _table(config.get("model_loading", {}), "model_loading")
    own = dict(_table(root.get(role, {}), f"model_loading.{role}"))
    shared = {k: v for k, v in root.items() if k not in MODEL_ROLES}
    options = {**shared, **own}
    unknown = sorted(set(options) - _ALLOWED)
    if unknown:
        raise ValueError(f"unsupported model_loading settings {unknown}")
    for name in _MERGED_TABLES:
        merged = {**_table(shared.get(name, {}), f"model_loading.{name}"),
                  **_table(own.get(name, {}), f"model_loading.{role}.{name}")}
        if merged:
            options[name] = merged
    runtime = config.get("runtime", {})
    for name, fallback in _RUNTIME_DEFAULTS:
        value = options.setdefault(name, runtime.get(name, fallback))
        if not isinstance(value, bool):
            raise TypeError(f"model_loading.{name} has to be true or false")
    models = config.get("models", {})
    adapter_rl = role == "rl" and models.get("rl_kind") == "peft_adapter"
    if "revision" not in options:
        if adapter_rl:
            options["revision"] = model_loading_options(config, "base").get("revision")
        elif f"{role}_revision" in models:
            options["revision"] = str(models[f"{role}_revision"])
    return options


def resolve_checkpoint_path(name_or_path: str, *, revision: str | None = None, cache_dir: str | None = None,
                            local_files_only: bool = True) -> Path:
    """A local checkpoint directory, or the Hub snapshot of a repository id (offline by default)."""
    candidate = Path(name_or_path).expanduser()
    if candidate.is_dir():
        return candidate.resolve()
    looks_local = candidate.is_absolute() or name_or_path.split("/", 1)[0] in (".", "..") or \
        name_or_path.startswith((".\\", "..\\"))
    if looks_local:
        raise FileNotFoundError(candidate)
    from huggingface_hub import snapshot_download

    skip = ["*.h5", "*.msgpack", "*.onnx", "*.gguf", "*.ot", "original/*"]
    return Path(snapshot_download(name_or_path, revision=revision, cache_dir=cache_dir,
                                  local_files_only=local_files_only, ignore_patterns=skip))


def model_identity(model: str, adapter: str | None = None, *, revision: str | None = None,
                   adapter_revision: str | None = None, tokenizer: str | None = None,
                   tokenizer_revision: str | None = None) -> str:
    values = dict(zip(_IDENTITY_KEYS, (revision, adapter_revision, tokenizer, tokenizer_revision)))
    head = model if adapter is None else f"{model}+adapter:{adapter}"
    return "".join([head] + [f";{k}={values[k]}" for k in _IDENTITY_KEYS if values[k] is not None])


def _shard_files(directory: Path, index_file: Path) -> tuple[Path, ...]:
    try:
        weight_map = json.loads(index_file.read_text(encoding="utf-8"))["weight_map"]
    except (KeyError, TypeError) as error:
        raise ValueError(f"{index_file} has no weight_map") from error
    if not isinstance(weight_map, dict) or not weight_map or \
            not all(isinstance(v, str) for v in weight_map.values()):
        raise ValueError(f"{index_file}: weight_map must map tensor names to shard file names")
    files = []
    for shard in sorted(set(weight_map.values())):
        parts = PurePath(shard)
        if parts.is_absolute() or parts.drive or ".." in parts.parts or "\\" in shard:
            raise ValueError(f"{index_file}: shard {shard!r} is not a plain relative file name")
        path = directory / shard
        if not path.is_file():
            raise FileNotFoundError(path)
        files.append(path)
    return tuple(files)


def checkpoint_weight_files(path: Path) -> tuple[Path, ...]:
    """The weight files of a safetensors or PyTorch checkpoint directory, single file or sharded."""
    directory = Path(path).resolve()
    layouts = (("model.safetensors", "model.safetensors.index.json"),
               ("pytorch_model.bin", "pytorch_model.bin.index.json"))
    for single, index in layouts:
        if (directory / single).is_file():
            return (directory / single,)
        if (directory / index).is_file():
            return _shard_files(directory, directory / index)
    raise FileNotFoundError(f"{directory} holds no safetensors / PyTorch weights or shard index")


__all__ = ["MODEL_ROLES", "checkpoint_weight_files", "model_identity", "model_loading_options", "model_role",
           "resolve_checkpoint_path"]
