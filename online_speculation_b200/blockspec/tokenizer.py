"""Tokenizer from a local model directory: ``tokenizer.json`` only, no model or remote code.

:class:`LocalTokenizer` encodes and decodes with the fast ``tokenizers`` library and
renders chat messages with the directory's own template (``chat_template.jinja`` or
the ``chat_template`` field of ``tokenizer_config.json``).  A missing template is an
error rather than a silent default, so prompts never depend on a library's implicit
template.  Interface of online-speculation/src/blockspec/tokenizer.py
(``encode`` / ``decode`` / ``render_chat``).
"""

from __future__ import annotations

import json
from pathlib import Path

SPECIAL_TOKEN_FIELDS = ("bos_token", "eos_token", "pad_token", "unk_token")


def _special_tokens(config: dict) -> dict[str, str]:
    found = {}
    for field in SPECIAL_TOKEN_FIELDS:
        value = config.get(field)
        if isinstance(value, dict):                       # AddedToken serialisation
            value = value.get("content")
        if isinstance(value, str):
            found[field] = value
    return found


class LocalTokenizer:
    def __init__(self, directory):
        from tokenizers import Tokenizer

        self.directory = Path(directory)
        self.backend = Tokenizer.from_file(str(self.directory / "tokenizer.json"))
        self._template_renderer = None

    def encode(self, text: str, add_special_tokens: bool = False) -> list[int]:
        return self.backend.encode(text, add_special_tokens=add_special_tokens).ids

    def decode(self, ids, skip_special_tokens: bool = False) -> str:
        return self.backend.decode(list(ids), skip_special_tokens=skip_special_tokens)

    def _template(self) -> tuple[str, dict]:
        config_path = self.directory / "tokenizer_config.json"
        config = json.loads(config_path.read_text(encoding="utf-8")) if config_path.is_file() else {}
        jinja = self.directory / "chat_template.jinja"
        template = jinja.read_text(encoding="utf-8") if jinja.is_file() else config.get("chat_template")
        if not isinstance(template, str) or not template.strip():
            raise ValueError(f"{self.directory} has no local chat template (chat_template.jinja or "
                             "tokenizer_config.json:chat_template)")
        return template, _special_tokens(config)

    def render_chat(self, messages, *, add_generation_prompt: bool = False) -> str:
        """The conversation as text under the directory's template (template handling only)."""
        if self._template_renderer is None:
            from transformers import PreTrainedTokenizerFast

            template, special = self._template()
            self._template_renderer = PreTrainedTokenizerFast(
                tokenizer_file=str(self.directory / "tokenizer.json"), chat_template=template, **special)
        return self._template_renderer.apply_chat_template(list(messages), tokenize=False,
                                                           add_generation_prompt=add_generation_prompt)


__all__ = ["LocalTokenizer"]
