"""Configuration-driven construction of the autoregressive backends of an experiment.

TOML layout (the reference's sections, ``src/inference_scaling/arllm/backends/loader.py:196-340``,
with the engine of this package behind every role)::

    [models]
    base = "Qwen/Qwen2.5-1.5B-Instruct"      # local dir / Hub snapshot, or "random:<preset>"
    proposal = "..."                         # optional; roles with the same path share one engine

    [runtime]
    backend = "b200"                         # "transformers" / "vllm" / "vllm-sync" map to the same engine
    kv_cache_gb = 16
    max_batch_size = 64
    reference_temperature = 1.0              # optional ReferencePolicyBackend wrapper
    score_cache_entries = 100000             # optional ScoreCachingBackend wrapper
    continuous_batching = false              # optional ContinuousBatchingBackend wrapper

    [model_loading]                          # shared.model_loading options (per-role tables allowed)

    [acceleration.speculation]               # optional rollout-reuse speculation in the engine backend
    enabled = true
    tiers = [[4, 8], [16, 4], [512, 0]]      # [maximum active batch, draft tokens]
    stochastic_tree = false                  # plus min_context_tokens, min_token_probability, tree_max_*

Checkpoints are read from safetensors in the HF Qwen2 / Qwen3 layout
(``config.json`` + ``model*.safetensors``); the tokenizer is loaded with
``transformers.AutoTokenizer`` when present (for ``encode`` / ``decode``).
"""

from __future__ import annotations

import json
from collections.abc import Mapping
from pathlib import Path
from typing import Any

import torch

from ...shared.model_loading import (MODEL_ROLES, checkpoint_weight_files, model_identity, model_loading_options,
                                     resolve_checkpoint_path)

BACKEND_CHOICES = ("b200", "transformers", "vllm", "vllm-sync")


def _table(value: Any, name: str) -> dict[str, Any]:
    if value is None:
        return {}
    if not isinstance(value, Mapping):
        raise TypeError(f"{name} must be a table")
    return dict(value)


_SPECULATION_KEYS = ("min_context_tokens", "min_token_probability", "tree_max_context_tokens", "tree_max_contexts",
                     "vllm_max_cached_requests", "stochastic_tree")


def speculation_from_config(config: Mapping[str, Any]):
    """``[acceleration.speculation]`` as an ``ActiveBatchSpeculationConfig`` (None when absent or disabled).

    Keys of src/inference_scaling/arllm/backends/loader.py:81-116; ``dynamic_vllm`` is accepted
    and has no effect here (the engine has no separate vLLM speculation mode).
    """
    from ..acceleration import ActiveBatchSpeculationConfig, SpeculationTier

    table = _table(_table(config.get("acceleration"), "acceleration").get("speculation"), "acceleration.speculation")
    if not table or not bool(table.pop("enabled", False)):
        return None
    table.pop("dynamic_vllm", None)
    tiers = table.pop("tiers", None)
    unknown = sorted(set(table) - set(_SPECULATION_KEYS))
    if unknown:
        raise ValueError("unknown speculation settings: " + ", ".join(unknown))
    if tiers is not None:
        if not isinstance(tiers, (list, tuple)):
            raise TypeError("acceleration.speculation.tiers must be an array")
        try:
            table["tiers"] = tuple(SpeculationTier(int(t[0]), int(t[1])) for t in tiers)
        except (TypeError, ValueError, IndexError) as err:
            raise ValueError("each speculation tier is [maximum_active_batch, draft_tokens]") from err
    return ActiveBatchSpeculationConfig(**table)


def load_state_dict(path: Path, device="cpu") -> dict[str, torch.Tensor]:
    from safetensors.torch import load_file

    sd: dict[str, torch.Tensor] = {}
    for f in checkpoint_weight_files(path):
        if f.suffix == ".safetensors":
            sd.update(load_file(str(f), device=str(device)))
        else:
            sd.update(torch.load(f, map_location=device, weights_only=True))
    return sd


class LoadedModel:
    """One engine backend per distinct model path, with optional tokenizer."""

    def __init__(self, path: str, config: Mapping[str, Any], role: str, *, tp_group=None):
        from ...api import build_runner
        from ...engine.backend import EngineBackend
        from ...models.decoder import PRESETS, DecoderConfig, build_weights

        rt = _table(config.get("runtime"), "runtime")
        opts = model_loading_options(config, role)
        self.tokenizer = None
        if path.startswith("random:"):
            cfg = PRESETS[path.split(":", 1)[1]]
            weights = None
            self.model_id = path
        else:
            ckpt = resolve_checkpoint_path(path, revision=opts.get("revision"), cache_dir=opts.get("cache_dir"),
                                           local_files_only=opts.get("local_files_only", True))
            cfg = DecoderConfig.from_hf(json.loads((ckpt / "config.json").read_text()), name=path)
            sd = load_state_dict(ckpt)
            dev = torch.device("cuda", torch.cuda.current_device())
            tp = 1 if tp_group is None else torch.distributed.get_world_size(tp_group)
            rank = 0 if tp_group is None else torch.distributed.get_rank(tp_group)
            weights = build_weights(cfg, sd, tp=tp, rank=rank, device=dev)
            del sd
            self.model_id = model_identity(path, revision=opts.get("revision"))
            try:
                from transformers import AutoTokenizer

                self.tokenizer = AutoTokenizer.from_pretrained(str(ckpt), **_table(opts.get("tokenizer_kwargs"),
                                                                                     "tokenizer_kwargs"))
            except Exception:   # noqa: BLE001 - a checkpoint without tokenizer files is still usable by id
                self.tokenizer = None
        kv = int(float(rt.get("kv_cache_gb", 16)) * 2 ** 30)
        runner = build_runner(cfg, tp_group=tp_group, seed=int(rt.get("seed", 0)), kv_bytes=kv, weights=weights,
                              max_tokens=int(rt.get("max_prefill_tokens", 8192)))
        self.backend = EngineBackend(runner, model_id=self.model_id, max_batch=int(rt.get("max_batch_size", 64)),
                                     max_seq_tokens=int(rt.get("max_sequence_tokens", 8192)),
                                     bos_token_id=getattr(self.tokenizer, "bos_token_id", None),
                                     speculation=speculation_from_config(config))
        self.backend.tokenizer = self.tokenizer


def _wrap(backend, config: Mapping[str, Any]):
    from .batching import ContinuousBatchingBackend
    from .cache import ScoreCachingBackend
    from .reference import ReferencePolicyBackend

    rt = _table(config.get("runtime"), "runtime")
    out = backend
    if rt.get("reference_temperature") not in (None, 1, 1.0):
        out = ReferencePolicyBackend(out, temperature=float(rt["reference_temperature"]))
    if rt.get("score_cache_entries"):
        out = ScoreCachingBackend(out, maximum_entries=int(rt["score_cache_entries"]))
    if rt.get("continuous_batching"):
        out = ContinuousBatchingBackend(out, max_batch_size=int(rt.get("max_batch_size", 64)),
                                        max_batch_tokens=int(rt.get("max_batch_tokens", 65536)))
    return out


def load_backend_from_config(config: Mapping[str, Any], *, role: str = "base", tp_group=None,
                             _cache: dict | None = None) -> Any:
    """The (wrapped) backend of ``role``; roles naming the same model path share one engine."""
    if role not in MODEL_ROLES:
        raise ValueError(f"unknown model role {role!r}")
    rt = _table(config.get("runtime"), "runtime")
    kind = str(rt.get("backend", "b200"))
    if kind not in BACKEND_CHOICES:
        raise ValueError(f"runtime.backend must be one of {BACKEND_CHOICES}")
    models = _table(config.get("models"), "models")
    path = models.get(role) or models.get("base")
    if not path:
        raise ValueError(f"[models] defines neither {role!r} nor 'base'")
    cache = _cache if _cache is not None else {}
    if path not in cache:
        cache[path] = LoadedModel(str(path), config, role, tp_group=tp_group)
    return _wrap(cache[path].backend, config)


def load_backends_from_config(config: Mapping[str, Any], *, tp_group=None) -> dict[str, Any]:
    """Every configured role -> backend (one engine per distinct path)."""
    models = _table(config.get("models"), "models")
    shared: dict = {}
    return {r: load_backend_from_config(config, role=r, tp_group=tp_group, _cache=shared)
            for r in MODEL_ROLES if models.get(r) or r == "base"}


def close_backends(backends: Mapping[str, Any]) -> None:
    seen = set()
    for b in backends.values():
        while b is not None and id(b) not in seen:
            seen.add(id(b))
            if hasattr(b, "close"):
                b.close()
            b = getattr(b, "backend", getattr(b, "_backend", None))


__all__ = ["BACKEND_CHOICES", "close_backends", "load_backend_from_config", "load_backends_from_config",
           "load_state_dict"]
