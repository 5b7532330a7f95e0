"""Token-level thinking / content segmentation of a completion.

A :class:`ThinkingFormat` is one thinking phase delimited by token markers
(an optional opening marker, a closing marker), possibly already open in the
prompt (chat templates that prefill ``<think>``).  :class:`ThinkingParser`
accepts the first complete, non-empty thinking block among its formats and
otherwise returns the whole completion as content with the reason
(``absent``, ``incomplete``, ``empty``, ``malformed``, ``leading_content``,
``disabled``, ``unrecognized_format``).  The first complete block is a
prefix-stable boundary, so it doubles as a generation stop rule.

Reference behaviour: src/inference_scaling/shared/output.py:25-253.
"""

from __future__ import annotations

from collections.abc import Callable
from dataclasses import dataclass, field, replace
from typing import Literal, Protocol

from .types import TokenSequence


def find_token_sequence(tokens: TokenSequence, marker: TokenSequence, *, start: int = 0) -> int | None:
    if not marker:
        raise ValueError("a token marker must be nonempty")
    m = tuple(marker)
    n = len(m)
    for i in range(start, len(tokens) - n + 1):
        if tuple(tokens[i:i + n]) == m:
            return i
    return None


def _last(tokens: TokenSequence, marker: TokenSequence, end: int | None = None) -> int:
    n = len(marker)
    stop = len(tokens) if end is None else end
    found = -1
    for i in range(0, stop):
        if tuple(tokens[i:i + n]) == tuple(marker):
            found = i
    return found


@dataclass(frozen=True, slots=True)
class OutputSegments:
    thinking_token_ids: TokenSequence
    content_token_ids: TokenSequence
    thinking_start: int | None
    thinking_end: int | None
    boundary_end: int | None
    status: str
    ended_by_eos: bool
    format_name: str | None = None
    thinking_text: str | None = None
    content_text: str | None = None

    @property
    def has_complete_thinking(self) -> bool:
        return self.status == "complete"

    def describe(self) -> dict[str, object]:
        mode = ("thinking" if self.status in ("complete", "incomplete")
                else "content" if self.status in ("empty", "absent", "disabled") else "unknown")
        return {"thinking_status": self.status, "thinking_tokens": len(self.thinking_token_ids),
                "content_tokens": len(self.content_token_ids), "thinking_start": self.thinking_start,
                "thinking_end": self.thinking_end, "thinking_boundary_end": self.boundary_end,
                "ended_by_eos": self.ended_by_eos, "thinking_format_name": self.format_name,
                "detected_output_mode": mode,
                "segmentation_mode": "thinking_and_content" if self.has_complete_thinking else "full",
                "segmentation_fallback_reason": None if self.has_complete_thinking else self.status}


class OutputParser(Protocol):
    def split(self, prompt: TokenSequence, completion: TokenSequence, *, eos_token_id: int | None = None
              ) -> OutputSegments: ...

    def describe(self) -> dict[str, object]: ...


def _strip_eos(completion: TokenSequence, eos: int | None) -> tuple[TokenSequence, bool]:
    toks = tuple(completion)
    if eos is not None and eos in toks:
        return toks[:toks.index(eos)], True
    return toks, False


@dataclass(frozen=True, slots=True)
class ThinkingFormat:
    """One thinking phase followed by content; ``start_token_ids=None`` means generation starts thinking."""

    end_token_ids: TokenSequence
    start_token_ids: TokenSequence | None = None
    starts_in_thinking: bool | None = None
    name: str = "custom"

    def __post_init__(self) -> None:
        if self.starts_in_thinking is not None and not isinstance(self.starts_in_thinking, bool):
            raise ValueError("starts_in_thinking must be a boolean or None")
        for attr in ("end_token_ids", "start_token_ids"):
            m = getattr(self, attr)
            if m is None and attr == "start_token_ids":
                continue
            if not m or any(not isinstance(t, int) or t < 0 for t in m):
                raise ValueError(f"{attr} must contain non-negative token IDs")
            object.__setattr__(self, attr, tuple(m))
        if self.start_token_ids == self.end_token_ids:
            raise ValueError("thinking start and end markers must differ")

    def prompt_is_thinking(self, prompt: TokenSequence) -> bool:
        """Whether generation begins inside the thinking phase (the prompt's last structural marker opens it)."""
        if self.starts_in_thinking is not None:
            return self.starts_in_thinking
        if self.start_token_ids is None:
            return True
        return _last(prompt, self.start_token_ids) > _last(prompt, self.end_token_ids)

    def split(self, prompt: TokenSequence, completion: TokenSequence, *, eos_token_id: int | None = None
              ) -> OutputSegments:
        toks, ended = _strip_eos(completion, eos_token_id)
        if self.prompt_is_thinking(tuple(prompt)):
            start = 0
        elif self.start_token_ids is not None:
            at = find_token_sequence(toks, self.start_token_ids)
            start = None if at is None else at + len(self.start_token_ids)
        else:
            start = None
        if start is None:
            return OutputSegments((), toks, None, None, None, "absent", ended)
        end = find_token_sequence(toks, self.end_token_ids, start=start)
        if end is None:
            return OutputSegments(toks[start:], (), start, None, None, "incomplete", ended)
        b = end + len(self.end_token_ids)
        think = toks[start:end]
        return OutputSegments(think, toks[b:], start, end, b, "complete" if think else "empty", ended)

    def describe(self) -> dict[str, object]:
        return {"name": self.name, "start_token_ids": self.start_token_ids, "end_token_ids": self.end_token_ids,
                "starts_in_thinking": self.starts_in_thinking}


def full_sequence_segments(completion: TokenSequence, *, eos_token_id: int | None = None, reason: str
                           ) -> OutputSegments:
    toks, ended = _strip_eos(completion, eos_token_id)
    return OutputSegments((), toks, None, None, None, reason, ended)


@dataclass(frozen=True, slots=True)
class ThinkingParser:
    """The first complete non-empty thinking block among ``formats``; otherwise the full output."""

    formats: tuple[ThinkingFormat, ...] = ()
    mode: Literal["auto", "enabled", "disabled"] = "auto"
    is_blank: Callable[[TokenSequence], bool] | None = field(default=None, compare=False, repr=False)

    def __post_init__(self) -> None:
        if self.mode not in ("auto", "enabled", "disabled"):
            raise ValueError("thinking mode must be auto, enabled or disabled")

    def prompt_mode(self, prompt: TokenSequence) -> str:
        """``disabled`` when the prompt already holds a blank, closed thinking block (thinking switched off)."""
        if self.mode != "auto" or self.is_blank is None:
            return self.mode
        for f in self.formats:
            if f.start_token_ids is None or f.starts_in_thinking is not None:
                continue
            end = _last(prompt, f.end_token_ids)
            if end < 0:
                continue
            start = _last(prompt, f.start_token_ids, end)
            if start >= 0 and self.is_blank(prompt[end + len(f.end_token_ids):]) and self.is_blank(
                    prompt[start + len(f.start_token_ids):end]):
                return "disabled"
        return "auto"

    def split(self, prompt: TokenSequence, completion: TokenSequence, *, eos_token_id: int | None = None
              ) -> OutputSegments:
        def fallback(reason):
            return full_sequence_segments(completion, eos_token_id=eos_token_id, reason=reason)

        if self.prompt_mode(prompt) == "disabled":
            return fallback("disabled")
        if not self.formats:
            return fallback("unrecognized_format")
        found = []
        for f in self.formats:
            g = f
            if (self.is_blank is not None and f.starts_in_thinking is None and f.start_token_ids is not None
                    and f.prompt_is_thinking(prompt)):
                # a prefilled opening marker counts only when followed by whitespace (not a quoted tag)
                opened = _last(prompt, f.start_token_ids)
                g = replace(f, starts_in_thinking=self.is_blank(prompt[opened + len(f.start_token_ids):]))
            seg = g.split(prompt, completion, eos_token_id=eos_token_id)
            if seg.thinking_start is not None:
                found.append((seg, g))
        if not found:
            return fallback("absent")
        seg, f = min(found, key=lambda m: m[0].thinking_start or 0)
        if seg.thinking_start and f.start_token_ids is not None:
            lead = completion[:seg.thinking_start - len(f.start_token_ids)]
            if lead and self.is_blank is not None and not self.is_blank(lead):
                return fallback("leading_content")
        for other in self.formats:
            if other.start_token_ids is not None:
                nested = find_token_sequence(completion, other.start_token_ids, start=seg.thinking_start)
                if nested is not None and (seg.thinking_end is None or nested < seg.thinking_end):
                    return fallback("malformed")
        if seg.status != "complete":
            return fallback(seg.status)
        if self.is_blank is not None and self.is_blank(seg.thinking_token_ids):
            return fallback("empty")
        return replace(seg, format_name=f.name)

    def describe(self) -> dict[str, object]:
        return {"mode": self.mode, "formats": [f.describe() for f in self.formats], "fallback": "full_sequence",
                "boundary_rule": "first_complete_nonempty_thinking_block"}


__all__ = ["OutputParser", "OutputSegments", "ThinkingFormat", "ThinkingParser", "find_token_sequence",
           "full_sequence_segments"]
