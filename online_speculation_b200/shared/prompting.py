"""Prompt rendering: the tokenizer's chat template, or plain ``role: content`` text.

``prompt.format`` = auto (chat template when the tokenizer has one) | chat | plain;
``output.thinking_mode`` (enabled / disabled) sets ``enable_thinking`` for
templates that understand it.  Reference behaviour: src/inference_scaling/shared/prompting.py:9-32.
"""

from __future__ import annotations

from collections.abc import Mapping, Sequence
from typing import Any


def render_prompt(tokenizer: Any, messages: Sequence[Mapping[str, str]], config: Mapping[str, Any]) -> str:
    opts = config.get("prompt", {})
    fmt = opts.get("format", "auto")
    if fmt not in ("auto", "chat", "plain"):
        raise ValueError("prompt.format must be auto, chat or plain")
    template = getattr(tokenizer, "chat_template", None)
    has_template = bool(template) or (not hasattr(tokenizer, "chat_template")
                                      and callable(getattr(tokenizer, "apply_chat_template", None)))
    if fmt == "plain" or (fmt == "auto" and not has_template):
        if len(messages) == 1 and messages[0]["role"] == "user":
            return messages[0]["content"]
        return "\n\n".join(f"{m['role']}: {m['content']}" for m in messages) + "\n\nassistant:"
    if not has_template:
        raise ValueError("prompt.format=chat requires a tokenizer chat template")
    kwargs = dict(opts.get("chat_template_kwargs", {}))
    if {"tokenize", "add_generation_prompt", "return_tensors"} & kwargs.keys():
        raise ValueError("chat_template_kwargs must preserve text rendering and the generation prompt")
    mode = config.get("output", {}).get("thinking_mode", "auto")
    if mode != "auto" and "enable_thinking" in str(template):
        want = mode == "enabled"
        if "enable_thinking" in kwargs and kwargs["enable_thinking"] != want:
            raise ValueError("thinking_mode conflicts with chat_template_kwargs.enable_thinking")
        kwargs["enable_thinking"] = want
    return str(tokenizer.apply_chat_template(messages, tokenize=False, add_generation_prompt=True, **kwargs))


__all__ = ["render_prompt"]
