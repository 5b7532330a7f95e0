"""Model-derived rewards from configuration (``[reward]`` with legacy ``[conditional_is]`` keys).

Reference behaviour: src/inference_scaling/arllm/reward_factory.py:16-77.
"""

from __future__ import annotations

from collections.abc import Mapping
from typing import Any

from .config import SamplingConfig
from .output import output_settings_from_config, thinking_format_from_backend
from .rewards import ConsilienceReward, SequenceLogProbabilityReward

MODEL_REWARD_SOURCES = ("consilience", "sequence_log_probability")


def model_reward_from_config(backend: Any, config: Mapping[str, Any], *, source: str,
                             sampling: SamplingConfig | None = None):
    common, legacy = config.get("reward", {}), config.get("conditional_is", {})
    if source == "sequence_log_probability":
        return SequenceLogProbabilityReward(backend, sampling, scale=float(common.get(
            "logprob_scale", legacy.get("logprob_reward_scale", 1.0))))
    if source != "consilience":
        raise ValueError(f"unknown model reward source: {source}")
    opts = common.get("consilience", {})

    def setting(name, default):
        old = "reward_scale" if name == "scale" else name
        return opts.get(name, legacy.get(f"consilience_{old}", default))

    out_opts = output_settings_from_config(config)
    if legacy.get("consilience_reasoning_end_text") is not None:
        out_opts.setdefault("thinking_end_text", legacy["consilience_reasoning_end_text"])
    scope = str(opts.get("scope", "thinking"))
    if scope not in ("thinking", "full"):
        raise ValueError("Consilience scope must be thinking or full")
    wt = setting("window_tokens", None)
    return ConsilienceReward(
        backend, SamplingConfig(temperature=float(opts.get("score_temperature", 1.0))),
        top_k=int(setting("top_k", 5)), window_fraction=float(setting("window_fraction", 0.2)),
        window_tokens=None if wt is None else int(wt), skip_fraction=float(setting("skip_fraction", 0.05)),
        initial_penalty=float(setting("initial_penalty", 3.0)), scale=float(setting("scale", 1.0)),
        thinking_format=thinking_format_from_backend(backend, out_opts) if scope == "thinking" else None,
        scope=scope)


def reward_temperature_from_config(config: Mapping[str, Any], *, source: str, default: float = 1.0) -> float:
    if "temperature" in config.get("reward", {}):
        return float(config["reward"]["temperature"])
    if source == "consilience":
        return 2.0
    return float(config.get("conditional_is", {}).get("reward_temperature", default))


__all__ = ["MODEL_REWARD_SOURCES", "model_reward_from_config", "reward_temperature_from_config"]
