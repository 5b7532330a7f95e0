"""Which thinking format a backend's outputs use, from explicit settings or the tokenizer.

Resolution order: an explicit ``thinking_formats`` list of tables; else one
``thinking_start_text`` / ``thinking_end_text`` pair; else every known delimiter
pair whose two markers both occur in the tokenizer vocabulary or chat template
(``<think>``, ``<thinking>``, ``[THINK]``, ``<reasoning>``).  Marker texts are
encoded with the backend's tokenizer; JSON / XML outputs are handled by the
structured parser behind the same object.  Setting names follow the ``[output]``
table of src/inference_scaling/arllm/output.py (config compatibility).
"""

from __future__ import annotations

from collections.abc import Mapping
from typing import Any

from ..shared.output import ThinkingFormat, ThinkingParser
from ..shared.structured_output import UnifiedOutputParser

THINKING_MARKERS = (("think", "<think>", "</think>"), ("thinking", "<thinking>", "</thinking>"),
                    ("bracket_think", "[THINK]", "[/THINK]"), ("reasoning", "<reasoning>", "</reasoning>"))
_KINDS = ("auto", "tags", "json", "xml")
_MODES = ("auto", "enabled", "disabled")


def output_settings_from_config(config: Mapping[str, Any]) -> dict[str, Any]:
    """``[output]`` settings; a chat template's ``enable_thinking`` decides an "auto" mode."""
    settings = dict(config.get("output", {}))
    template_kwargs = config.get("prompt", {}).get("chat_template_kwargs", {})
    if settings.get("thinking_mode", "auto") == "auto" and "enable_thinking" in template_kwargs:
        flag = template_kwargs["enable_thinking"]
        if not isinstance(flag, bool):
            raise ValueError("prompt.chat_template_kwargs.enable_thinking has to be true or false")
        settings["thinking_mode"] = "enabled" if flag else "disabled"
    return settings


def _field_path(settings: Mapping[str, Any], key: str) -> tuple[str, ...] | None:
    raw = settings.get(key)
    if raw is None:
        return None
    parts = tuple(raw.split(".")) if isinstance(raw, str) else tuple(raw) if isinstance(raw, (list, tuple)) else ()
    if not parts or not all(isinstance(p, str) and p for p in parts):
        raise ValueError(f"{key} is a dotted path or a non-empty list of field names")
    return parts


def _format_tables(settings: Mapping[str, Any], vocab, template: str) -> list[Mapping[str, Any]]:
    listed = settings.get("thinking_formats")
    start, end = settings.get("thinking_start_text"), settings.get("thinking_end_text")
    default_start = settings.get("starts_in_thinking")
    if listed is not None:
        if start is not None or end is not None:
            raise ValueError("give either thinking_formats or a thinking_start/end_text pair, not both")
        if not isinstance(listed, (list, tuple)) or not listed:
            raise ValueError("thinking_formats has to be a non-empty list of tables")
        return list(listed)
    if end is not None:
        return [{"name": "configured", "start_text": start, "end_text": end, "starts_in_thinking": default_start}]
    if start is not None:
        raise ValueError("thinking_start_text needs a thinking_end_text")

    def known(marker: str) -> bool:
        return marker in vocab or marker in template

    return [{"name": name, "start_text": s, "end_text": e, "starts_in_thinking": default_start}
            for name, s, e in THINKING_MARKERS if known(s) and known(e)]


def thinking_format_from_backend(backend: Any, settings: Mapping[str, Any] | None = None, *,
                                 required: bool = False) -> UnifiedOutputParser:
    settings = settings or {}
    kind = str(settings.get("thinking_format", "auto"))
    mode = settings.get("thinking_mode", "auto")
    if kind not in _KINDS:
        raise ValueError(f"thinking_format {kind!r} is not one of {_KINDS}")
    if mode not in _MODES:
        raise ValueError(f"thinking_mode {mode!r} is not one of {_MODES}")
    tokenizer = getattr(backend, "tokenizer", None)
    vocab = tokenizer.get_vocab() if callable(getattr(tokenizer, "get_vocab", None)) else {}
    template = str(getattr(tokenizer, "chat_template", "") or "")
    encode = getattr(backend, "encode", None) or getattr(tokenizer, "encode", None)

    def ids(text: str) -> tuple[int, ...]:
        if encode is None:
            raise ValueError("thinking markers are text: encoding them needs a tokenizer")
        return tuple(encode(text, add_special_tokens=False))

    formats = []
    for table in _format_tables(settings, vocab, template):
        if not isinstance(table, Mapping):
            raise ValueError("every entry of thinking_formats is a table")
        start, end = table.get("start_text"), table.get("end_text")
        if not (isinstance(end, str) and end):
            raise ValueError("a thinking format needs a non-empty end_text")
        if start is not None and not (isinstance(start, str) and start):
            raise ValueError("start_text, when given, is a non-empty string")
        formats.append(ThinkingFormat(ids(end), None if start is None else ids(start),
                                      table.get("starts_in_thinking", settings.get("starts_in_thinking")),
                                      str(table.get("name", "configured"))))
    if required and not formats:
        raise ValueError("no thinking format: configure one or use a tokenizer with known delimiters")

    token_decode = getattr(tokenizer, "decode", None)
    backend_decode = getattr(backend, "decode", None)
    decode = None
    if token_decode is not None:
        def decode(t):
            return str(token_decode(t, skip_special_tokens=False, clean_up_tokenization_spaces=False))
    elif backend_decode is not None:
        def decode(t):
            return str(backend_decode(t, skip_special_tokens=False))
    is_blank = None if decode is None else (lambda t: not t or not decode(t).strip())
    markers = ThinkingParser(tuple(formats), mode=mode, is_blank=is_blank)
    return UnifiedOutputParser(markers, decode, kind, _field_path(settings, "thinking_path"),
                               _field_path(settings, "content_path"))


__all__ = ["THINKING_MARKERS", "output_settings_from_config", "thinking_format_from_backend"]
