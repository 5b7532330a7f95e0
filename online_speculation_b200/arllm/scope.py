"""Sampling scope: run the algorithm on the thinking phase only, then answer directly.

With ``scope = "thinking"`` the algorithm's backend is wrapped so generation stops at
the end of the first complete thinking block (EOS padding after it); ``finish``
then samples the final content from the base policy and reports how the output was
segmented.  Formats without a prefix-stable stop (JSON / XML, thinking switched off,
unknown delimiters) fall back to the full sequence with the reason recorded.  The
report keys follow src/inference_scaling/arllm/scope.py, which experiment records use.
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

_SCOPES = ("full", "thinking")


def _no_early_stop_reason(fmt: OutputParser | None) -> str | None:
    """Why a thinking-only scope cannot be honoured with this format (None: it can)."""
    if getattr(fmt, "mode", None) == "disabled":
        return "disabled"
    if fmt is not None and getattr(fmt, "supports_early_stop", True):
        return None
    if getattr(fmt, "kind", None) in ("json", "xml"):
        return "structured_format_requires_full_sequence"
    return "unrecognized_format"


@dataclass(frozen=True, slots=True)
class SamplingScope:
    scope: Literal["full", "thinking"] = "full"
    thinking_format: OutputParser | None = None
    generation_chunk_size: int = 256
    requested_scope: Literal["full", "thinking"] | None = None
    fallback_reason: str | None = None

    def __post_init__(self) -> None:
        if self.scope not in _SCOPES:
            raise ValueError(f"sampling scope {self.scope!r} is not one of {_SCOPES}")
        if self.generation_chunk_size < 1:
            raise ValueError("generation_chunk_size has to be positive")
        if self.requested_scope is None:
            object.__setattr__(self, "requested_scope", self.scope)
        if self.scope == "thinking":
            reason = _no_early_stop_reason(self.thinking_format)
            if reason is not None:
                object.__setattr__(self, "scope", "full")
                object.__setattr__(self, "fallback_reason", reason)

    @classmethod
    def from_config(cls, backend: Any, config: Mapping[str, Any], *, active: bool = True) -> "SamplingScope":
        settings = output_settings_from_config(config)
        scope = settings.get("sampling_scope", "full") if active else "full"
        if scope not in _SCOPES:
            raise ValueError(f"output.sampling_scope {scope!r} is not one of {_SCOPES}")
        return cls(scope, thinking_format_from_backend(backend, settings),
                   int(settings.get("generation_chunk_size", 256)))

    def full_fallback(self, reason: str) -> "SamplingScope":
        return replace(self, scope="full", fallback_reason=reason)

    def for_prompt(self, prompt: TokenSequence) -> "SamplingScope":
        prompt_mode = getattr(self.thinking_format, "prompt_mode", None)
        if self.scope == "thinking" and prompt_mode is not None and prompt_mode(prompt) == "disabled":
            return self.full_fallback("disabled")
        return self

    def wrap(self, backend: Any, prompt: TokenSequence) -> Any:
        if self.scope == "full":
            return backend
        eos = getattr(backend.tokenizer, "eos_token_id", None)
        if eos is None:
            raise ValueError("stopping after the thinking block pads with EOS, and the tokenizer has none")
        return StoppedSequenceBackend(backend, stop_token_sequences=(), eos_token_id=eos,
                                      protected_prefix_length=len(prompt), thinking_parser=self.thinking_format,
                                      thinking_prompt=prompt, generation_chunk_size=self.generation_chunk_size)

    def _append_answer(self, backend, prompt, tokens, max_new_tokens, sampling, seed) -> tuple[tuple, int]:
        seg = self.thinking_format.split(prompt, tokens, eos_token_id=backend.tokenizer.eos_token_id)
        if not seg.has_complete_thinking or seg.boundary_end is None:
            return tokens, 0
        head = tokens[:seg.boundary_end]
        budget = max_new_tokens - len(head)
        if budget <= 0:
            return head, 0
        answer = backend.sample_batch([GenerationRequest(prompt + head, budget, sampling, seed,
                                                         "scope:final-content")])[0]
        return head + tuple(answer.token_ids), len(answer.token_ids)

    def finish(self, backend: Any, prompt: TokenSequence, tokens: TokenSequence, *, max_new_tokens: int,
               sampling: SamplingConfig, seed: int) -> tuple[TokenSequence, dict[str, Any]]:
        sequence, answered = tuple(tokens), 0
        if self.scope == "thinking":
            sequence, answered = self._append_answer(backend, prompt, sequence, max_new_tokens, sampling, seed)
        report = self.describe_output(backend, prompt, sequence)
        effective, reason = self.scope, self.fallback_reason
        if self.scope == "thinking" and report["thinking_status"] != "complete":
            effective, reason = "full", report["thinking_status"]
        elif self.requested_scope == "thinking" and report.get("thinking_format_name") in ("json", "xml"):
            effective, reason = "full", "structured_format_requires_full_sequence"
        report.update(
            requested_sampling_scope=self.requested_scope, sampling_scope=effective,
            sampling_fallback_reason=reason,
            sampling_policy_scope="thinking_with_full_sequence_fallback" if self.scope == "thinking" else "full",
            final_content_generated_tokens=answered,
            generation_budget_exhausted=len(sequence) >= max_new_tokens and not report["ended_by_eos"])
        return sequence, report

    def describe_output(self, backend: Any, prompt: TokenSequence, tokens: TokenSequence) -> dict[str, Any]:
        eos = getattr(getattr(backend, "tokenizer", None), "eos_token_id", None)
        fmt = self.thinking_format
        seg = None if fmt is None else fmt.split(prompt, tuple(tokens), eos_token_id=eos)
        if seg is None or not seg.has_complete_thinking:
            seg = full_sequence_segments(tokens, eos_token_id=eos,
                                         reason="unrecognized_format" if seg is None else seg.status)

        def text(given, ids):
            return given if given is not None else backend.decode(ids)

        return {**seg.describe(),
                "thinking_token_ids": seg.thinking_token_ids,
                "thinking_text": text(seg.thinking_text, seg.thinking_token_ids),
                "content_token_ids": seg.content_token_ids,
                "content_text": text(seg.content_text, seg.content_token_ids),
                "thinking_format": None if fmt is None else fmt.describe()}


__all__ = ["SamplingScope"]
