"""Splitting a completion's tokens into a thinking block and the content after it.

A :class:`ThinkingFormat` describes one thinking phase: an optional opening marker,
a closing marker, and whether generation starts inside it (a chat template may put
the opening marker in the prompt).  :class:`ThinkingParser` takes the earliest
thinking block that any of its formats finds and keeps it only if it passes every
check below; otherwise the whole completion is content and the segments carry the
reason:

    disabled             the prompt holds a blank, closed block (thinking switched off)
    unrecognized_format  the parser has no formats
    absent               no format finds an opening
    leading_content      non-blank tokens precede the opening marker
    malformed            another opening marker appears before the block closes
    incomplete / empty   the block never closes / holds nothing

Because the first complete block cannot change as tokens are appended, its end is
also a valid generation stop point.  Status names and the ``describe()`` keys are
those of src/inference_scaling/shared/output.py, which experiment reports read.
Marker search runs on numpy sliding windows of the token ids.
"""

from __future__ import annotations

from collections.abc import Callable
from dataclasses import dataclass, field, replace
from typing import Literal, Protocol

import numpy as np

from .types import TokenSequence


def _hits(tokens: TokenSequence, marker: TokenSequence) -> np.ndarray:
    """Start offsets of every occurrence of ``marker`` in ``tokens`` (increasing)."""
    m = np.asarray(marker, dtype=np.int64)
    t = np.asarray(tokens, dtype=np.int64)
    if m.size == 0:
        raise ValueError("a token marker cannot be empty")
    if t.size < m.size:
        return np.zeros(0, dtype=np.int64)
    windows = np.lib.stride_tricks.sliding_window_view(t, m.size)
    return np.flatnonzero((windows == m).all(axis=1))


def find_token_sequence(tokens: TokenSequence, marker: TokenSequence, *, start: int = 0) -> int | None:
    """First occurrence of ``marker`` at or after ``start``."""
    hits = _hits(tokens, marker)
    hits = hits[hits >= start]
    return int(hits[0]) if hits.size else None


def _last_before(tokens: TokenSequence, marker: TokenSequence, end: int | None = None) -> int:
    """Last occurrence starting before ``end`` (default: anywhere), or -1."""
    hits = _hits(tokens, marker)
    if end is not None:
        hits = hits[hits < end]
    return int(hits[-1]) if hits.size else -1


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
        if self.status in ("complete", "incomplete"):
            detected = "thinking"
        elif self.status in ("empty", "absent", "disabled"):
            detected = "content"
        else:
            detected = "unknown"
        complete = self.has_complete_thinking
        return {"thinking_status": self.status, "thinking_tokens": len(self.thinking_token_ids),
                "content_tokens": len(self.content_token_ids), "thinking_start": self.thinking_start,
                "thinking_end": self.thinking_end, "thinking_boundary_end": self.boundary_end,
                "ended_by_eos": self.ended_by_eos, "thinking_format_name": self.format_name,
                "detected_output_mode": detected,
                "segmentation_mode": "thinking_and_content" if complete else "full",
                "segmentation_fallback_reason": None if complete else self.status}


class OutputParser(Protocol):
    def split(self, prompt: TokenSequence, completion: TokenSequence, *, eos_token_id: int | None = None
              ) -> OutputSegments: ...

    def describe(self) -> dict[str, object]: ...


def _cut_at_eos(completion: TokenSequence, eos: int | None) -> tuple[tuple[int, ...], bool]:
    tokens = tuple(completion)
    if eos is None:
        return tokens, False
    try:
        return tokens[:tokens.index(eos)], True
    except ValueError:
        return tokens, False


def _valid_marker(marker, what: str) -> tuple[int, ...]:
    ids = tuple(marker)
    if not ids or not all(isinstance(t, int) and t >= 0 for t in ids):
        raise ValueError(f"{what} has to be a non-empty sequence of non-negative token ids")
    return ids


@dataclass(frozen=True, slots=True)
class ThinkingFormat:
    """One thinking phase followed by content; ``start_token_ids=None`` means generation starts thinking."""

    end_token_ids: TokenSequence
    start_token_ids: TokenSequence | None = None
    starts_in_thinking: bool | None = None
    name: str = "custom"

    def __post_init__(self) -> None:
        if self.starts_in_thinking not in (None, True, False):
            raise ValueError("starts_in_thinking is True, False or None")
        object.__setattr__(self, "end_token_ids", _valid_marker(self.end_token_ids, "end_token_ids"))
        if self.start_token_ids is not None:
            object.__setattr__(self, "start_token_ids", _valid_marker(self.start_token_ids, "start_token_ids"))
            if self.start_token_ids == self.end_token_ids:
                raise ValueError("the opening and closing markers have to differ")

    def prompt_is_thinking(self, prompt: TokenSequence) -> bool:
        """Does generation begin inside the thinking phase?  Fixed by ``starts_in_thinking``,
        else true when the prompt's last opening marker comes after its last closing one."""
        if self.starts_in_thinking is not None:
            return self.starts_in_thinking
        if self.start_token_ids is None:
            return True
        return _last_before(prompt, self.start_token_ids) > _last_before(prompt, self.end_token_ids)

    def _opening(self, prompt: TokenSequence, tokens: tuple[int, ...]) -> int | None:
        if self.prompt_is_thinking(tuple(prompt)):
            return 0
        if self.start_token_ids is None:
            return None
        at = find_token_sequence(tokens, self.start_token_ids)
        return None if at is None else at + len(self.start_token_ids)

    def split(self, prompt: TokenSequence, completion: TokenSequence, *, eos_token_id: int | None = None
              ) -> OutputSegments:
        tokens, ended = _cut_at_eos(completion, eos_token_id)
        start = self._opening(prompt, tokens)
        if start is None:
            return OutputSegments((), tokens, None, None, None, "absent", ended)
        close = find_token_sequence(tokens, self.end_token_ids, start=start)
        if close is None:
            return OutputSegments(tokens[start:], (), start, None, None, "incomplete", ended)
        after = close + len(self.end_token_ids)
        block = tokens[start:close]
        return OutputSegments(block, tokens[after:], start, close, after, "complete" if block else "empty", ended)

    def describe(self) -> dict[str, object]:
        return {"name": self.name, "start_token_ids": self.start_token_ids, "end_token_ids": self.end_token_ids,
                "starts_in_thinking": self.starts_in_thinking}


def full_sequence_segments(completion: TokenSequence, *, eos_token_id: int | None = None, reason: str
                           ) -> OutputSegments:
    tokens, ended = _cut_at_eos(completion, eos_token_id)
    return OutputSegments((), tokens, None, None, None, reason, ended)


@dataclass(frozen=True, slots=True)
class ThinkingParser:
    """Earliest thinking block among ``formats`` that passes the checks; else the full output."""

    formats: tuple[ThinkingFormat, ...] = ()
    mode: Literal["auto", "enabled", "disabled"] = "auto"
    is_blank: Callable[[TokenSequence], bool] | None = field(default=None, compare=False, repr=False)

    def __post_init__(self) -> None:
        if self.mode not in ("auto", "enabled", "disabled"):
            raise ValueError(f"thinking mode {self.mode!r} is not auto, enabled or disabled")

    def _blank(self, tokens: TokenSequence) -> bool:
        return self.is_blank is not None and self.is_blank(tokens)

    def prompt_mode(self, prompt: TokenSequence) -> str:
        """``disabled`` when the prompt ends with a blank, closed thinking block; else the configured mode."""
        if self.mode != "auto" or self.is_blank is None:
            return self.mode
        for f in self.formats:
            if f.start_token_ids is None or f.starts_in_thinking is not None:
                continue
            close = _last_before(prompt, f.end_token_ids)
            if close < 0:
                continue
            open_ = _last_before(prompt, f.start_token_ids, close)
            if open_ < 0:
                continue
            inside = prompt[open_ + len(f.start_token_ids):close]
            after = prompt[close + len(f.end_token_ids):]
            if self._blank(inside) and self._blank(after):
                return "disabled"
        return "auto"

    def _resolved(self, f: ThinkingFormat, prompt: TokenSequence) -> ThinkingFormat:
        """A prefilled opening marker counts only when followed by blank tokens (not a quoted tag)."""
        if self.is_blank is None or f.starts_in_thinking is not None or f.start_token_ids is None:
            return f
        if not f.prompt_is_thinking(prompt):
            return f
        opened = _last_before(prompt, f.start_token_ids)
        return replace(f, starts_in_thinking=self.is_blank(prompt[opened + len(f.start_token_ids):]))

    def _earliest(self, prompt, completion, eos) -> tuple[OutputSegments, ThinkingFormat] | None:
        best = None
        for f in self.formats:
            g = self._resolved(f, prompt)
            seg = g.split(prompt, completion, eos_token_id=eos)
            if seg.thinking_start is not None and (best is None or seg.thinking_start < best[0].thinking_start):
                best = (seg, g)
        return best

    def _rejection(self, seg: OutputSegments, f: ThinkingFormat, completion: TokenSequence) -> str | None:
        if seg.thinking_start and f.start_token_ids is not None:
            lead = completion[:seg.thinking_start - len(f.start_token_ids)]
            if lead and self.is_blank is not None and not self.is_blank(lead):
                return "leading_content"
        for other in self.formats:
            if other.start_token_ids is None:
                continue
            again = find_token_sequence(completion, other.start_token_ids, start=seg.thinking_start)
            if again is not None and (seg.thinking_end is None or again < seg.thinking_end):
                return "malformed"
        if seg.status != "complete":
            return seg.status
        if self._blank(seg.thinking_token_ids):
            return "empty"
        return None

    def split(self, prompt: TokenSequence, completion: TokenSequence, *, eos_token_id: int | None = None
              ) -> OutputSegments:
        if self.prompt_mode(prompt) == "disabled":
            reason = "disabled"
        elif not self.formats:
            reason = "unrecognized_format"
        else:
            best = self._earliest(prompt, completion, eos_token_id)
            if best is None:
                reason = "absent"
            else:
                seg, f = best
                reason = self._rejection(seg, f, completion)
                if reason is None:
                    return replace(seg, format_name=f.name)
        return full_sequence_segments(completion, eos_token_id=eos_token_id, reason=reason)

    def describe(self) -> dict[str, object]:
        return {"mode": self.mode, "formats": [f.describe() for f in self.formats], "fallback": "full_sequence",
                "boundary_rule": "first_complete_nonempty_thinking_block"}


__all__ = ["OutputParser", "OutputSegments", "ThinkingFormat", "ThinkingParser", "find_token_sequence",
           "full_sequence_segments"]
