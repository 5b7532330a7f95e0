"""Thinking-format resolution from explicit settings and tokenizer metadata.

Known delimiter pairs are taken when both markers are in the tokenizer's
vocabulary or chat template (``<think>``, ``<thinking>``, ``[THINK]``,
``<reasoning>``); explicit ``thinking_start_text`` / ``thinking_end_text`` or a
``thinking_formats`` list override.  Unknown formats fall back to the full
sequence.  Reference behaviour: src/inference_scaling/arllm/output.py:20-134.
"""

from __future__ import annotations

from collections.abc import Mapping
from typing import Any

from ..shared.output import ThinkingFormat, ThinkingParser
from ..shared.structured_output import UnifiedOutputParser

THINKING_MARKERS = (("think", "<think>", "</think>"), ("thinking", "<thinking>", "</thinking>"),
                    ("bracket_think", "[THINK]", "[/THINK]"), ("reasoning", "<reasoning>", "</reasoning>"))


def output_settings_from_config(config: Mapping[str, Any]) -> dict[str, Any]:
    opts = dict(config.get("output", {}))
    tmpl = config.get("prompt", {}).get("chat_template_kwargs", {})
    if opts.get("thinking_mode", "auto") == "auto" and "enable_thinking" in tmpl:
        if not isinstance(tmpl["enable_thinking"], bool):
            raise ValueError("prompt.chat_template_kwargs.enable_thinking must be boolean")
        opts["thinking_mode"] = "enabled" if tmpl["enable_thinking"] else "disabled"
    return opts


def _path(opts, name):
    v = opts.get(name)
    if v is None:
        return None
    parts = v.split(".") if isinstance(v, str) else v
    if not isinstance(parts, (list, tuple)) or not parts or not all(isinstance(p, str) and p for p in parts):
        raise ValueError(f"{name} must be a dotted path or nonempty array of field names")
    return tuple(parts)


def thinking_format_from_backend(backend: Any, settings: Mapping[str, Any] | None = None, *,
                                 required: bool = False) -> UnifiedOutputParser:
    opts = settings or {}
    kind = str(opts.get("thinking_format", "auto"))
    if kind not in ("auto", "tags", "json", "xml"):
        raise ValueError("thinking_format must be auto, tags, json or xml")
    mode = opts.get("thinking_mode", "auto")
    if mode not in ("auto", "enabled", "disabled"):
        raise ValueError("thinking_mode must be auto, enabled or disabled")
    start_t, end_t = opts.get("thinking_start_text"), opts.get("thinking_end_text")
    tok = getattr(backend, "tokenizer", None)
    vocab = tok.get_vocab() if callable(getattr(tok, "get_vocab", None)) else {}
    template = str(getattr(tok, "chat_template", "") or "")
    listed = opts.get("thinking_formats")
    if listed is not None and (start_t is not None or end_t is not None):
        raise ValueError("provide thinking_formats or one thinking_start/end_text pair")
    if listed is not None:
        if not isinstance(listed, (list, tuple)) or not listed:
            raise ValueError("thinking_formats must be a nonempty array of tables")
        defs = list(listed)
    elif end_t is not None:
        defs = [{"name": "configured", "start_text": start_t, "end_text": end_t,
                 "starts_in_thinking": opts.get("starts_in_thinking")}]
    elif start_t is not None:
        raise ValueError("thinking_start_text requires thinking_end_text")
    else:
        defs = [{"name": n, "start_text": s, "end_text": e, "starts_in_thinking": opts.get("starts_in_thinking")}
                for n, s, e in THINKING_MARKERS if (s in vocab and e in vocab) or (s in template and e in template)]
    encode = getattr(backend, "encode", None) or getattr(tok, "encode", None)
    formats = []
    for d in defs:
        if not isinstance(d, Mapping):
            raise ValueError("each thinking format must be a table")
        s, e = d.get("start_text"), d.get("end_text")
        if not isinstance(e, str) or not e:
            raise ValueError("thinking end_text must be a nonempty string")
        if s is not None and (not isinstance(s, str) or not s):
            raise ValueError("thinking start_text must be a nonempty string")
        if encode is None:
            raise ValueError("resolving thinking markers requires a tokenizer encoder")
        formats.append(ThinkingFormat(tuple(encode(e, add_special_tokens=False)),
                                      None if s is None else tuple(encode(s, add_special_tokens=False)),
                                      d.get("starts_in_thinking", opts.get("starts_in_thinking")),
                                      str(d.get("name", "configured"))))
    if required and not formats:
        raise ValueError("thinking requires a configured format or recognized tokenizer delimiters")
    tdec, bdec = getattr(tok, "decode", None), getattr(backend, "decode", None)

    def decode(ids):
        if tdec is not None:
            return str(tdec(ids, skip_special_tokens=False, clean_up_tokenization_spaces=False))
        if bdec is None:
            raise ValueError("structured output parsing requires a token decoder")
        return str(bdec(ids, skip_special_tokens=False))

    has_dec = tdec is not None or bdec is not None
    markers = ThinkingParser(tuple(formats), mode=mode,
                             is_blank=(lambda ids: not ids or decode(ids).strip() == "") if has_dec else None)
    return UnifiedOutputParser(markers, decode if has_dec else None, kind, _path(opts, "thinking_path"),
                               _path(opts, "content_path"))


__all__ = ["THINKING_MARKERS", "output_settings_from_config", "thinking_format_from_backend"]
