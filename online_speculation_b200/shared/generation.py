"""Generation budget: the effective max_new_tokens given the model's context window.

The context limit is the smallest advertised limit found anywhere on the
backend object graph (``max_position_embeddings``, ``n_positions``,
``max_model_len``, ``model_max_length`` on the backend, its model, config,
tokenizer or engine), ignoring "unlimited" sentinels.  Reference behaviour:
src/inference_scaling/shared/generation.py:9-63.
"""

from __future__ import annotations

from collections.abc import Mapping, Sequence
from copy import deepcopy
from typing import Any

DEFAULT_MAX_NEW_TOKENS = 32768
_LIMIT_KEYS = ("max_position_embeddings", "n_positions", "max_model_len", "model_max_length")
_CHILD_KEYS = ("backend", "model", "config", "text_config", "tokenizer", "engine", "_engine", "_runtime", "llm_engine",
               "model_config", "vllm_config", "runner", "cfg", "w")


def _get(obj, key):
    return obj.get(key) if isinstance(obj, Mapping) else getattr(obj, key, None)


def context_limit(backend: Any) -> int | None:
    limits, seen, stack = [], set(), [backend]
    while stack:
        obj = stack.pop()
        if obj is None or id(obj) in seen:
            continue
        seen.add(id(obj))
        for k in _LIMIT_KEYS:
            v = _get(obj, k)
            if isinstance(v, int) and not isinstance(v, bool) and 0 < v < 10 ** 9:
                limits.append(v)
        for k in _CHILD_KEYS:
            child = _get(obj, k)
            if child is not obj:
                stack.append(child)
    return min(limits) if limits else None


def generation_config_for_prompt(config: Mapping[str, Any], prompt_length: int, backends: Sequence[Any]
                                 ) -> tuple[dict[str, Any], dict[str, Any]]:
    """Clip ``generation.max_new_tokens`` (and algorithm block sizes) to the context window."""
    out = deepcopy(dict(config))
    requested = out.get("generation", {}).get("max_new_tokens", DEFAULT_MAX_NEW_TOKENS)
    if isinstance(requested, bool) or not isinstance(requested, int) or requested <= 0:
        raise ValueError("generation.max_new_tokens must be a positive integer")
    if prompt_length < 0:
        raise ValueError("prompt_length must be non-negative")
    limits = [v for b in backends if b is not None and (v := context_limit(b)) is not None]
    explicit = out.get("runtime", {}).get("context_window")
    if explicit is not None:
        if isinstance(explicit, bool) or not isinstance(explicit, int) or explicit <= 0:
            raise ValueError("runtime.context_window must be a positive integer")
        limits.append(explicit)
    available = min(limits) - max(1, prompt_length) if limits else requested
    if available <= 0:
        raise ValueError("prompt fills the model context window; shorten the prompt or select a longer-context model")
    eff = min(requested, available)
    out.setdefault("generation", {})["max_new_tokens"] = eff
    for section in ("mh", "conditional_is", "iterated_is"):
        t = out.get(section, {})
        if "block_size" in t:
            t["block_size"] = min(int(t["block_size"]), eff)
    return out, {"requested_max_new_tokens": requested, "effective_max_new_tokens": eff,
                 "context_limit": min(limits) if limits else None, "prompt_tokens": prompt_length,
                 "length_limited_by_context": eff < requested}


__all__ = ["DEFAULT_MAX_NEW_TOKENS", "context_limit", "generation_config_for_prompt"]
