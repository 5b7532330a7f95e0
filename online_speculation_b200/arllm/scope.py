"""Sampling scope: sample only the thinking phase with the algorithm, then complete the answer directly.

With ``scope = "thinking"`` the algorithm's backend is wrapped so generation
stops at the end of the first complete thinking block (absorbing EOS
padding); ``finish`` then samples the final content from the base policy and
reports how the output was segmented.  Formats that cannot give a
prefix-stable stop (JSON / XML, disabled thinking, unknown delimiters) fall
back to the full sequence with the reason recorded.
Reference behaviour: src/inference_scaling/arllm/scope.py:18-136.
"""

from __future__ import annotations

from collections.abc import Mapping
from dataclasses import dataclass, replace
from typing import Any, Literal

from ..shared.output import OutputParser, full_sequence_segments
from ..shared.types import TokenSequence
from .backends.stopping import StoppedSequenceBackend
from .config import SamplingConfig
from .output import output_settings_from_config, thinking_format_from_backend
from .types import GenerationRequest


@dataclass(frozen=True, slots=True)
class SamplingScope:
    scope: Literal["full", "thinking"] = "full"
    thinking_format: OutputParser | None = None
    generation_chunk_size: int = 256
    requested_scope: Literal["full", "thinking"] | None = None
    fallback_reason: str | None = None

    def __post_init__(self) -> None:
        if self.scope not in ("full", "thinking"):
            raise ValueError("sampling scope must be full or thinking")
        if self.requested_scope is None:
            object.__setattr__(self, "requested_scope", self.scope)
        fmt = self.thinking_format
        if self.scope == "thinking":
            reason = None
            if getattr(fmt, "mode", None) == "disabled":
                reason = "disabled"
            elif fmt is None or not getattr(fmt, "supports_early_stop", True):
                reason = ("structured_format_requires_full_sequence" if getattr(fmt, "kind", None) in ("json", "xml")
                          else "unrecognized_format")
            if reason is not None:
                object.__setattr__(self, "scope", "full")
                object.__setattr__(self, "fallback_reason", reason)
        if self.generation_chunk_size <= 0:
            raise ValueError("generation_chunk_size must be positive")

    @classmethod
    def from_config(cls, backend: Any, config: Mapping[str, Any], *, active: bool = True) -> "SamplingScope":
        opts = output_settings_from_config(config)
        scope = opts.get("sampling_scope", "full") if active else "full"
        if scope not in ("full", "thinking"):
            raise ValueError("sampling scope must be full or thinking")
        return cls(scope, thinking_format_from_backend(backend, opts), int(opts.get("generation_chunk_size", 256)))

    def full_fallback(self, reason: str) -> "SamplingScope":
        return replace(self, scope="full", fallback_reason=reason)

    def for_prompt(self, prompt: TokenSequence) -> "SamplingScope":
        cb = getattr(self.thinking_format, "prompt_mode", None)
        if self.scope == "thinking" and cb is not None and cb(prompt) == "disabled":
            return self.full_fallback("disabled")
        return self

    def wrap(self, backend: Any, prompt: TokenSequence) -> Any:
        if self.scope == "full":
            return backend
        eos = getattr(backend.tokenizer, "eos_token_id", None)
        if eos is None:
            raise ValueError("thinking sampling requires an EOS padding token")
        return StoppedSequenceBackend(backend, stop_token_sequences=(), thinking_parser=self.thinking_format,
                                      thinking_prompt=prompt, eos_token_id=eos, protected_prefix_length=len(prompt),
                                      generation_chunk_size=self.generation_chunk_size)

    def finish(self, backend: Any, prompt: TokenSequence, tokens: TokenSequence, *, max_new_tokens: int,
               sampling: SamplingConfig, seed: int) -> tuple[TokenSequence, dict[str, Any]]:
        seq = tuple(tokens)
        extra = 0
        if self.scope == "thinking":
            seg = self.thinking_format.split(prompt, seq, eos_token_id=backend.tokenizer.eos_token_id)
            if seg.has_complete_thinking and seg.boundary_end is not None:
                seq = seq[:seg.boundary_end]
                left = max_new_tokens - len(seq)
                if left > 0:
                    s = backend.sample_batch([GenerationRequest(prompt + seq, left, sampling, seed,
                                                                "scope:final-content")])[0]
                    extra = len(s.token_ids)
                    seq += s.token_ids
        info = self.describe_output(backend, prompt, seq)
        eff, reason = self.scope, self.fallback_reason
        if self.scope == "thinking" and info["thinking_status"] != "complete":
            eff, reason = "full", info["thinking_status"]
        elif self.requested_scope == "thinking" and info.get("thinking_format_name") in ("json", "xml"):
            eff, reason = "full", "structured_format_requires_full_sequence"
        info.update(requested_sampling_scope=self.requested_scope, sampling_scope=eff, sampling_fallback_reason=reason,
                    sampling_policy_scope="thinking_with_full_sequence_fallback" if self.scope == "thinking" else "full",
                    final_content_generated_tokens=extra,
                    generation_budget_exhausted=len(seq) >= max_new_tokens and not info["ended_by_eos"])
        return seq, info

    def describe_output(self, backend: Any, prompt: TokenSequence, tokens: TokenSequence) -> dict[str, Any]:
        eos = getattr(getattr(backend, "tokenizer", None), "eos_token_id", None)
        if self.thinking_format is None:
            seg = full_sequence_segments(tokens, eos_token_id=eos, reason="unrecognized_format")
        else:
            seg = self.thinking_format.split(prompt, tuple(tokens), eos_token_id=eos)
            if not seg.has_complete_thinking:
                seg = full_sequence_segments(tokens, eos_token_id=eos, reason=seg.status)
        return {**seg.describe(), "thinking_token_ids": seg.thinking_token_ids,
                "thinking_text": seg.thinking_text if seg.thinking_text is not None else backend.decode(
                    seg.thinking_token_ids),
                "content_token_ids": seg.content_token_ids,
                "content_text": seg.content_text if seg.content_text is not None else backend.decode(
                    seg.content_token_ids),
                "thinking_format": self.thinking_format.describe() if self.thinking_format is not None else None}


__all__ = ["SamplingScope"]
