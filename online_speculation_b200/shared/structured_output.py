"""Thinking / answer fields of JSON or XML completions, aligned to the generated tokens.

A structured completion is one JSON object or an XML document (optionally inside a
```json / ```xml fence).  Its reasoning lives in a field named ``thinking``,
``reasoning``, ``analysis`` or ``think`` (or at an explicit path) and its answer,
optionally, in ``answer`` / ``content`` / ``final``.  The character span of each
field is located in the decoded text and then mapped to token boundaries of the
original completion by comparing decoded prefixes (never by re-tokenising); a span
inside a token is reported as unaligned and the whole completion is used instead.

JSON is read by a small iterative lexer that records the span of every value while
tracking the key path; XML spans come from expat's byte offsets.  Status strings and
``describe()`` keys follow src/inference_scaling/shared/structured_output.py, which
the experiment reports read.
"""

from __future__ import annotations

import json
import re
from collections.abc import Callable, Mapping
from dataclasses import dataclass
from typing import Any
from xml.parsers import expat

from .output import OutputSegments, ThinkingParser, full_sequence_segments
from .types import TokenSequence

Span = tuple[Any, int, int]       # (value, first char, end char)
_AMBIGUOUS = object()
_MAX_DEPTH = 64
_THINKING_NAMES = ("thinking", "reasoning", "analysis", "think")
_CONTENT_NAMES = ("answer", "content", "final")

_JSON_TOKEN = re.compile(r"""
    (?P<ws>[ \t\r\n]+)
  | (?P<string>"(?:[^"\\\x00-\x1f]|\\(?:["\\/bfnrt]|u[0-9a-fA-F]{4}))*")
  | (?P<number>-?(?:0|[1-9]\d*)(?:\.\d+)?(?:[eE][-+]?\d+)?)
  | (?P<literal>true|false|null)
  | (?P<punct>[{}\[\]:,])
""", re.VERBOSE)


def _json_tokens(text: str):
    pos = 0
    while pos < len(text):
        m = _JSON_TOKEN.match(text, pos)
        if m is None:
            raise ValueError(f"unexpected character {text[pos]!r} in JSON at {pos}")
        pos = m.end()
        if m.lastgroup != "ws":
            yield m.lastgroup, m.group(), m.start(), m.end()


class _Frame:
    __slots__ = ("kind", "value", "start", "path", "key", "expect")

    def __init__(self, kind, start, path):
        self.kind = kind            # "object" or "array"
        self.value = {} if kind == "object" else []
        self.start = start
        self.path = path
        self.key = None
        self.expect = "key_or_end" if kind == "object" else "value_or_end"


def json_fields(text: str) -> dict[tuple[str, ...], Span]:
    """Every value of a single JSON object keyed by its key path, with its span
    (string values: the characters between the quotes).  Arrays are leaves."""
    spans: dict[tuple[str, ...], Span] = {}
    stack: list[_Frame] = []
    top: list = []

    def place(value, path, start, end):
        # values inside arrays are part of the array's value, not addressable fields
        if not any(f.kind == "array" for f in stack):
            spans[path] = (value, start, end)
        if not stack:
            top.append(value)
            return
        frame = stack[-1]
        if frame.kind == "object":
            frame.value[frame.key] = value
        else:
            frame.value.append(value)
        frame.expect = "comma_or_end"

    def child_path():
        frame = stack[-1] if stack else None
        if frame is None:
            return ()
        return frame.path + ((frame.key,) if frame.kind == "object" else ())

    for kind, raw, start, end in _json_tokens(text):
        frame = stack[-1] if stack else None
        if top:
            raise ValueError("text continues after the JSON object")
        if frame is not None and frame.expect in ("key_or_end", "key"):
            if kind == "punct" and raw == "}" and frame.expect == "key_or_end":
                pass
            elif kind == "string":
                key = json.loads(raw)
                if key in frame.value:
                    raise ValueError(f"repeated JSON key {key!r}")
                frame.key = key
                frame.expect = "colon"
                continue
            else:
                raise ValueError("a JSON object key has to be a string")
        if frame is not None and frame.expect == "colon":
            if raw != ":":
                raise ValueError("missing ':' after a JSON key")
            frame.expect = "value"
            continue
        if frame is not None and frame.expect == "comma_or_end":
            if raw == ",":
                frame.expect = "key" if frame.kind == "object" else "value"
                continue
            if raw not in "}]":
                raise ValueError("missing ',' between JSON members")
        if kind == "punct" and raw in "}]":
            if frame is None or (raw == "}") != (frame.kind == "object") or frame.expect in ("key", "value"):
                raise ValueError(f"unbalanced {raw!r} in JSON")
            stack.pop()
            place(frame.value, frame.path, frame.start, end)
            continue
        if kind == "punct" and raw in "{[":
            if len(stack) >= _MAX_DEPTH:
                raise ValueError(f"JSON nested deeper than {_MAX_DEPTH} levels")
            stack.append(_Frame("object" if raw == "{" else "array", start, child_path()))
            continue
        if kind == "punct":
            raise ValueError(f"unexpected {raw!r} in JSON")
        path = child_path()
        if kind == "string":
            place(json.loads(raw), path, start + 1, end - 1)
        elif kind == "number":
            place(json.loads(raw), path, start, end)
        else:
            place({"true": True, "false": False, "null": None}[raw], path, start, end)
    if stack or not top or not isinstance(top[0], dict):
        raise ValueError("the output is not exactly one complete JSON object")
    return spans


class _XmlSpans:
    """Collects the text content and character span of every element path (expat)."""

    def __init__(self, raw: bytes):
        self.raw = raw
        self.parser = expat.ParserCreate()
        self.open: list[tuple[str, int, list[str]]] = []      # (name, content start byte, text pieces)
        self.spans: dict[tuple[str, ...], Span] = {}
        p = self.parser
        p.StartElementHandler = self._start
        p.EndElementHandler = self._end
        p.CharacterDataHandler = self._text
        p.StartDoctypeDeclHandler = self._refuse
        p.ExternalEntityRefHandler = self._refuse

    def _refuse(self, *_):
        raise ValueError("document types and external entities are not accepted")

    def _tag_end(self, at: int) -> int:
        """Byte just after the '>' closing the start tag at ``at`` (quoted '>' skipped)."""
        quote = None
        for i in range(at, len(self.raw)):
            c = self.raw[i]
            if quote is not None:
                quote = None if c == quote else quote
            elif c in b"\"'":
                quote = c
            elif c == ord(">"):
                return i + 1
        return len(self.raw)

    def _start(self, name, _attributes):
        if len(self.open) >= _MAX_DEPTH:
            raise ValueError(f"XML nested deeper than {_MAX_DEPTH} levels")
        self.open.append((name, self._tag_end(self.parser.CurrentByteIndex), []))

    def _text(self, data):
        for _, _, pieces in self.open:
            pieces.append(data)

    def _chars(self, nbytes: int) -> int:
        return len(self.raw[:nbytes].decode("utf-8"))

    def _end(self, _name):
        path = tuple(name for name, _, _ in self.open)
        _, begin, pieces = self.open.pop()
        stop = max(begin, self.parser.CurrentByteIndex)
        value = _AMBIGUOUS if path in self.spans else "".join(pieces)
        self.spans[path] = (value, self._chars(begin), self._chars(stop))

    def parse(self) -> dict[tuple[str, ...], Span]:
        self.parser.Parse(self.raw, True)
        return self.spans


def xml_fields(text: str, *, _fragment: bool = False) -> dict[tuple[str, ...], Span]:
    """Text content of every XML element by path, with its span; repeated paths are ambiguous."""
    try:
        return _XmlSpans(text.encode("utf-8")).parse()
    except expat.ExpatError as error:
        junk = expat.errors.codes[expat.errors.XML_ERROR_JUNK_AFTER_DOC_ELEMENT]
        if _fragment or error.code != junk:
            raise
    # several top-level elements: parse them under a synthetic root and shift the spans back
    root = "<_output_fragment>"
    inner = xml_fields(root + text + "</_output_fragment>", _fragment=True)
    return {path[1:]: (value, a - len(root), b - len(root)) for path, (value, a, b) in inner.items() if len(path) > 1}


def _field(fields: Mapping[tuple[str, ...], Span], path, names, *, required: bool) -> Span | None:
    if path is not None:
        hits = [span for key, span in fields.items() if key == tuple(path)]
    else:
        hits = [span for key, span in fields.items() if key and key[-1] in names]
    if len(hits) > 1:
        raise ValueError("several fields match; give an explicit path")
    if hits and hits[0][0] is _AMBIGUOUS:
        raise ValueError("the field is repeated")
    if required and not hits:
        raise ValueError("no thinking field")
    return hits[0] if hits else None


def token_boundary(tokens: TokenSequence, text: str, pos: int, decode: Callable[[TokenSequence], str]) -> int | None:
    """Token count k with decode(tokens[:k]) == text[:pos], or None if pos is inside a token."""
    target = text[:pos]
    cache: dict[int, str] = {}

    def prefix(k: int) -> str:
        if k not in cache:
            cache[k] = decode(tokens[:k])
        return cache[k]

    lo, hi = 0, len(tokens)
    while lo <= hi:                         # prefix lengths grow with k: bisect on them
        mid = (lo + hi) // 2
        got = prefix(mid)
        if got == target:
            return mid
        lo, hi = (mid + 1, hi) if len(got) < pos else (lo, mid - 1)
    # byte-level tokens can decode to replacement characters part-way: look around the bisection point
    for k in range(max(0, hi - 8), min(len(tokens), lo + 8) + 1):
        if prefix(k) == target:
            return k
    return None


_FENCE = re.compile(r"(\s*```(?:json|xml)?[ \t]*\r?\n)(.*?)(\r?\n```\s*)", re.DOTALL)


@dataclass(frozen=True, slots=True)
class StructuredThinkingParser:
    kind: str
    decode: Callable[[TokenSequence], str]
    thinking_path: tuple[str, ...] | None = None
    content_path: tuple[str, ...] | None = None

    def __post_init__(self):
        if self.kind not in ("json", "xml"):
            raise ValueError(f"structured kind {self.kind!r} is not json or xml")

    def _spans(self, text: str) -> tuple[Span, Span | None]:
        body, shift = text, 0
        if text.lstrip().startswith("```"):
            fenced = _FENCE.fullmatch(text)
            if fenced is None:
                raise ValueError("unterminated or malformed code fence")
            body, shift = fenced.group(2), len(fenced.group(1))
        found = json_fields(body) if self.kind == "json" else xml_fields(body)
        fields = {k: (v, a + shift, b + shift) for k, (v, a, b) in found.items()}
        thinking = _field(fields, self.thinking_path, _THINKING_NAMES, required=True)
        content = _field(fields, self.content_path, _CONTENT_NAMES, required=self.content_path is not None)
        for span in (thinking, content):
            if span is not None and isinstance(span[0], str):
                span[0].encode("utf-8")
        return thinking, content

    def split(self, prompt, completion, *, eos_token_id=None) -> OutputSegments:
        tokens = tuple(completion)
        ended = eos_token_id is not None and eos_token_id in tokens
        if ended:
            tokens = tokens[:tokens.index(eos_token_id)]
        text = self.decode(tokens)

        def whole(reason: str) -> OutputSegments:
            return full_sequence_segments(completion, eos_token_id=eos_token_id, reason=reason)

        try:
            thinking, content = self._spans(text)
        except (ValueError, UnicodeError, expat.ExpatError, RecursionError):
            return whole("malformed_" + self.kind)
        if not isinstance(thinking[0], str):
            return whole("non_text_thinking_field")
        if not thinking[0].strip():
            return whole("empty")
        first = token_boundary(tokens, text, thinking[1], self.decode)
        last = token_boundary(tokens, text, thinking[2], self.decode)
        if first is None or last is None or last <= first:
            return whole("unaligned_thinking_tokens")
        content_tokens: TokenSequence = ()
        content_text = ""
        if content is not None:
            c0 = token_boundary(tokens, text, content[1], self.decode)
            c1 = token_boundary(tokens, text, content[2], self.decode)
            if c0 is None or c1 is None:
                return whole("unaligned_content_tokens")
            content_tokens = tokens[c0:c1]
            content_text = content[0] if isinstance(content[0], str) else json.dumps(content[0], ensure_ascii=False)
        return OutputSegments(tokens[first:last], content_tokens, first, last, None, "complete", ended, self.kind,
                              thinking[0], content_text)

    def describe(self) -> dict[str, object]:
        return {"kind": self.kind, "thinking_path": self.thinking_path, "content_path": self.content_path,
                "requires_complete_output": True, "token_alignment": "original_token_boundaries"}


@dataclass(frozen=True, slots=True)
class UnifiedOutputParser:
    """Marker formats first; JSON / XML parsing when the decoded text looks structured."""

    markers: ThinkingParser
    decode: Callable[[TokenSequence], str] | None = None
    kind: str = "auto"
    thinking_path: tuple[str, ...] | None = None
    content_path: tuple[str, ...] | None = None

    @property
    def formats(self):
        return self.markers.formats

    @property
    def mode(self):
        return self.markers.mode

    @property
    def supports_early_stop(self) -> bool:
        return bool(self.formats) and self.kind in ("auto", "tags")

    def prompt_mode(self, prompt):
        return self.markers.prompt_mode(prompt)

    def _structured_kind(self, text: str, marker_status: str) -> str | None:
        if self.kind != "auto":
            return self.kind
        if text.startswith(("{", "```json")):
            return "json"
        if text.startswith("```xml"):
            return "xml"
        if text.startswith("<") and marker_status in ("leading_content", "absent", "unrecognized_format"):
            return "xml"
        return None

    def split(self, prompt, completion, *, eos_token_id=None) -> OutputSegments:
        by_markers = self.markers.split(prompt, completion, eos_token_id=eos_token_id)
        if by_markers.status == "disabled" or self.decode is None or self.kind == "tags":
            return by_markers
        tokens = tuple(completion)
        if eos_token_id is not None and eos_token_id in tokens:
            tokens = tokens[:tokens.index(eos_token_id)]
        kind = self._structured_kind(self.decode(tokens).lstrip(), by_markers.status)
        if kind is None:
            return by_markers
        return StructuredThinkingParser(kind, self.decode, self.thinking_path, self.content_path).split(
            prompt, completion, eos_token_id=eos_token_id)

    def stop_boundary(self, prompt, completion, *, eos_token_id=None) -> int | None:
        """Where generation may stop: the end of the first complete marker thinking block."""
        if not self.supports_early_stop:
            return None
        if self.decode is not None and self.decode(completion).lstrip().startswith("{"):
            return None
        seg = self.markers.split(prompt, completion, eos_token_id=eos_token_id)
        return seg.boundary_end if seg.has_complete_thinking else None

    def describe(self) -> dict[str, object]:
        return {**self.markers.describe(), "format": self.kind, "thinking_path": self.thinking_path,
                "content_path": self.content_path, "structured_sampling": "full"}


__all__ = ["StructuredThinkingParser", "UnifiedOutputParser", "json_fields", "token_boundary", "xml_fields"]
