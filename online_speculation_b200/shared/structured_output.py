"""JSON / XML thinking and answer fields aligned to the original generated tokens.

A structured completion (one JSON object, or XML, optionally inside a
```json / ```xml fence) carries its reasoning in a field (``thinking`` /
``reasoning`` / ``analysis`` / ``think`` unless a path is given) and optionally
its answer (``answer`` / ``content`` / ``final``).  Character spans of those
fields are mapped back to token boundaries of the original completion by
comparing decoded prefixes (never by re-tokenising); a span that does not fall
on token boundaries is reported as unaligned and the whole completion is used.

Reference behaviour: src/inference_scaling/shared/structured_output.py:166-289.
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

Span = tuple[Any, int, int]       # (value, start char, end char)
_REPEATED = object()
_WS = " \r\n\t"


def json_fields(text: str) -> dict[tuple[str, ...], Span]:
    """Every value of a single JSON object with its character span (strings: inside the quotes)."""

    def no_constants(v):
        raise ValueError(f"invalid JSON constant: {v}")

    dec = json.JSONDecoder(parse_constant=no_constants)
    out: dict[tuple[str, ...], Span] = {}

    def skip(i):
        while i < len(text) and text[i] in _WS:
            i += 1
        return i

    def value(i, path):
        if len(path) > 64:
            raise ValueError("JSON nesting exceeds 64 levels")
        s = skip(i)
        if s >= len(text):
            raise ValueError("incomplete JSON value")
        if text[s] == "{":
            obj: dict[str, Any] = {}
            i = skip(s + 1)
            if i < len(text) and text[i] == "}":
                out[path] = (obj, s, i + 1)
                return obj, i + 1
            while True:
                key, e = dec.raw_decode(text, i)
                if not isinstance(key, str) or key in obj:
                    raise ValueError("JSON keys must be distinct strings")
                i = skip(e)
                if i >= len(text) or text[i] != ":":
                    raise ValueError("missing JSON colon")
                obj[key], i = value(i + 1, path + (key,))
                i = skip(i)
                if i < len(text) and text[i] == "}":
                    i += 1
                    break
                if i >= len(text) or text[i] != ",":
                    raise ValueError("missing JSON object delimiter")
                i = skip(i + 1)
            out[path] = (obj, s, i)
            return obj, i
        v, e = dec.raw_decode(text, s)
        out[path] = (v, s + 1, e - 1) if isinstance(v, str) else (v, s, e)
        return v, e

    top, end = value(0, ())
    if not isinstance(top, dict) or skip(end) != len(text):
        raise ValueError("output must contain exactly one JSON object")
    return out


def xml_fields(text: str, *, _fragment: bool = False) -> dict[tuple[str, ...], Span]:
    """Text content of every XML element with its character span; repeated paths are marked ambiguous."""
    raw = text.encode("utf-8")
    p = expat.ParserCreate()
    stack: list[list] = []                   # [name, content start byte, pieces]
    out: dict[tuple[str, ...], Span] = {}

    def chars(nbytes: int) -> int:
        return len(raw[:nbytes].decode("utf-8"))

    def on_start(name, _attrs):
        if len(stack) >= 64:
            raise ValueError("XML nesting exceeds 64 levels")
        i, quote = p.CurrentByteIndex, None
        while i < len(raw):                  # end of the opening tag (skipping quoted attribute values)
            c = raw[i]
            if quote is not None:
                if c == quote:
                    quote = None
            elif c in (34, 39):
                quote = c
            elif c == 62:
                break
            i += 1
        stack.append([name, i + 1, []])

    def on_data(d):
        for entry in stack:
            entry[2].append(d)

    def on_end(_name):
        path = tuple(e[0] for e in stack)
        _, begin, pieces = stack.pop()
        stop = max(begin, p.CurrentByteIndex)
        out[path] = (_REPEATED if path in out else "".join(pieces), chars(begin), chars(stop))

    def refuse(*_):
        raise ValueError("XML document types and external entities are unsupported")

    p.StartElementHandler, p.EndElementHandler, p.CharacterDataHandler = on_start, on_end, on_data
    p.StartDoctypeDeclHandler = p.ExternalEntityRefHandler = refuse
    try:
        p.Parse(raw, True)
    except expat.ExpatError as err:
        if not _fragment and err.code == expat.errors.codes[expat.errors.XML_ERROR_JUNK_AFTER_DOC_ELEMENT]:
            wrap = "<_output_fragment>"
            inner = xml_fields(wrap + text + "</_output_fragment>", _fragment=True)
            return {k[1:]: (v, a - len(wrap), b - len(wrap)) for k, (v, a, b) in inner.items() if len(k) > 1}
        raise
    return out


def _pick(fields: Mapping[tuple[str, ...], Span], path, names, *, required: bool) -> Span | None:
    hits = [v for k, v in fields.items() if k and (k == path if path is not None else k[-1] in names)]
    if len(hits) > 1:
        raise ValueError("ambiguous structured output fields; specify a path")
    if hits and hits[0][0] is _REPEATED:
        raise ValueError("ambiguous repeated structured output field")
    if not hits and required:
        raise ValueError("missing thinking field")
    return hits[0] if hits else None


def token_boundary(tokens: TokenSequence, text: str, pos: int, decode: Callable[[TokenSequence], str]) -> int | None:
    """Index k with decode(tokens[:k]) == text[:pos], or None when pos falls inside a token."""
    want = text[:pos]
    lo, hi = 0, len(tokens)
    while lo <= hi:
        mid = (lo + hi) // 2
        pre = decode(tokens[:mid])
        if pre == want:
            return mid
        if len(pre) < pos:
            lo = mid + 1
        else:
            hi = mid - 1
    # byte-fallback tokens may decode to replacement characters mid-sequence: probe the neighbourhood
    for k in range(max(0, hi - 8), min(len(tokens), lo + 8) + 1):
        if decode(tokens[:k]) == want:
            return k
    return None


@dataclass(frozen=True, slots=True)
class StructuredThinkingParser:
    kind: str
    decode: Callable[[TokenSequence], str]
    thinking_path: tuple[str, ...] | None = None
    content_path: tuple[str, ...] | None = None

    def __post_init__(self):
        if self.kind not in ("json", "xml"):
            raise ValueError("structured output kind must be json or xml")

    def split(self, prompt, completion, *, eos_token_id=None) -> OutputSegments:
        toks = tuple(completion)
        ended = eos_token_id is not None and eos_token_id in toks
        if ended:
            toks = toks[:toks.index(eos_token_id)]
        text = self.decode(toks)

        def fallback(reason):
            return full_sequence_segments(completion, eos_token_id=eos_token_id, reason=reason)

        try:
            body, off = text, 0
            if text.lstrip().startswith("```"):
                m = re.fullmatch(r"(\s*```(?:json|xml)?[ \t]*\r?\n)(.*?)(\r?\n```\s*)", text, re.DOTALL)
                if m is None:
                    raise ValueError("malformed structured output fence")
                body, off = m.group(2), len(m.group(1))
            raw = json_fields(body) if self.kind == "json" else xml_fields(body)
            fields = {k: (v, a + off, b + off) for k, (v, a, b) in raw.items()}
            think = _pick(fields, self.thinking_path, ("thinking", "reasoning", "analysis", "think"), required=True)
            content = _pick(fields, self.content_path, ("answer", "content", "final"),
                            required=self.content_path is not None)
        except (ValueError, expat.ExpatError, RecursionError):
            return fallback("malformed_" + self.kind)
        if not isinstance(think[0], str):
            return fallback("non_text_thinking_field")
        try:
            think[0].encode("utf-8")
            if content is not None and isinstance(content[0], str):
                content[0].encode("utf-8")
        except UnicodeError:
            return fallback("malformed_" + self.kind)
        if not think[0].strip():
            return fallback("empty")
        s = token_boundary(toks, text, think[1], self.decode)
        e = token_boundary(toks, text, think[2], self.decode)
        if s is None or e is None or e <= s:
            return fallback("unaligned_thinking_tokens")
        c_toks: TokenSequence = ()
        c_text = ""
        if content is not None:
            cs = token_boundary(toks, text, content[1], self.decode)
            ce = token_boundary(toks, text, content[2], self.decode)
            if cs is None or ce is None:
                return fallback("unaligned_content_tokens")
            c_toks = toks[cs:ce]
            c_text = content[0] if isinstance(content[0], str) else json.dumps(content[0], ensure_ascii=False)
        return OutputSegments(toks[s:e], c_toks, s, e, None, "complete", ended, self.kind, think[0], c_text)

    def describe(self) -> dict[str, object]:
        return {"kind": self.kind, "thinking_path": self.thinking_path, "content_path": self.content_path,
                "requires_complete_output": True, "token_alignment": "original_token_boundaries"}


@dataclass(frozen=True, slots=True)
class UnifiedOutputParser:
    """Marker formats first; JSON / XML structured outputs when the decoded text looks structured."""

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

    def split(self, prompt, completion, *, eos_token_id=None) -> OutputSegments:
        seg = self.markers.split(prompt, completion, eos_token_id=eos_token_id)
        if seg.status == "disabled" or self.decode is None or self.kind == "tags":
            return seg
        toks = (completion[:completion.index(eos_token_id)]
                if eos_token_id is not None and eos_token_id in completion else completion)
        text = self.decode(toks).lstrip()
        kind = self.kind
        if kind == "auto":
            if text.startswith(("{", "```json")):
                kind = "json"
            elif text.startswith("```xml") or (text.startswith("<") and seg.status in (
                    "leading_content", "absent", "unrecognized_format")):
                kind = "xml"
            else:
                return seg
        return StructuredThinkingParser(kind, self.decode, self.thinking_path, self.content_path).split(
            prompt, completion, eos_token_id=eos_token_id)

    def stop_boundary(self, prompt, completion, *, eos_token_id=None) -> int | None:
        """Token index where generation may stop (the end of the first complete thinking block)."""
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
