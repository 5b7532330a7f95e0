"""CPU tests of the sampling scope: run the algorithm on the thinking phase only, then sample
the final content from the base policy (behaviour of src/inference_scaling/arllm/scope.py,
covered in the reference by tests/test_sampling_scope.py)."""

from __future__ import annotations

from types import SimpleNamespace

import numpy as np
import pytest

from online_speculation_b200.arllm.backends.tabular import TabularBackend
from online_speculation_b200.arllm.config import SamplingConfig
from online_speculation_b200.arllm.scope import SamplingScope
from online_speculation_b200.arllm.types import GenerationRequest
from online_speculation_b200.shared.output import ThinkingFormat

EOS, END = 0, 6
PROMPT = (1, 2)
# deterministic continuation by position after the two-token prompt: thinking 3 4, marker 6, answer 7 8 9 ...
SCRIPT = (3, 4, END, 7, 8, 9, 10, 11, 12, 13, 14, 15)


class _ScriptedBackend(TabularBackend):
    """One-hot next-token law by position, with the tokenizer surface the scope needs."""

    def __init__(self):
        def row(prefix):
            p = np.full(16, 1e-12)
            p[SCRIPT[len(prefix) - len(PROMPT)]] = 1.0
            return p / p.sum()

        super().__init__(row, 16)
        self.tokenizer = SimpleNamespace(eos_token_id=EOS)

    def decode(self, ids):
        return " ".join(str(t) for t in ids)


def _sample(backend, n, seed=0):
    req = GenerationRequest(PROMPT, n, SamplingConfig(eos_token_id=EOS), seed, "t")
    return tuple(backend.sample_batch([req])[0].token_ids)


def test_full_scope_is_a_pass_through():
    base = _ScriptedBackend()
    scope = SamplingScope("full", ThinkingFormat(end_token_ids=(END,)))
    assert scope.wrap(base, PROMPT) is base
    seq, report = scope.finish(base, PROMPT, _sample(base, 6), max_new_tokens=6, sampling=SamplingConfig(),
                               seed=1)
    assert seq == SCRIPT[:6]
    assert report["sampling_scope"] == "full" and report["final_content_generated_tokens"] == 0


def test_thinking_scope_stops_after_the_block_and_appends_the_answer():
    base = _ScriptedBackend()
    scope = SamplingScope("thinking", ThinkingFormat(end_token_ids=(END,)), generation_chunk_size=4)
    wrapped = scope.wrap(base, PROMPT)
    tokens = _sample(wrapped, 8)
    assert tokens == (3, 4, END) + (EOS,) * 5                   # EOS padding after the thinking block
    seq, report = scope.finish(base, PROMPT, tokens, max_new_tokens=8, sampling=SamplingConfig(), seed=1)
    assert seq == (3, 4, END, 7, 8, 9, 10, 11)                  # answer drawn from the base policy
    assert report["sampling_scope"] == "thinking" and report["sampling_fallback_reason"] is None
    assert report["final_content_generated_tokens"] == 5
    assert report["thinking_token_ids"] == (3, 4) and report["content_token_ids"] == (7, 8, 9, 10, 11)
    assert report["generation_budget_exhausted"]


def test_thinking_scope_falls_back_when_the_block_never_closes():
    base = _ScriptedBackend()
    scope = SamplingScope("thinking", ThinkingFormat(end_token_ids=(END,)))
    seq, report = scope.finish(base, PROMPT, (3, 4), max_new_tokens=2, sampling=SamplingConfig(), seed=1)
    assert seq == (3, 4) and report["sampling_scope"] == "full"
    assert report["requested_sampling_scope"] == "thinking" and report["sampling_fallback_reason"]


def test_scope_validation_and_fallbacks():
    with pytest.raises(ValueError):
        SamplingScope("partial")
    with pytest.raises(ValueError):
        SamplingScope("full", generation_chunk_size=0)
    s = SamplingScope("thinking", None)                          # no usable format: full sequence
    assert s.scope == "full" and s.requested_scope == "thinking" and s.fallback_reason == "unrecognized_format"
    f = SamplingScope("thinking", ThinkingFormat(end_token_ids=(END,))).full_fallback("disabled")
    assert f.scope == "full" and f.fallback_reason == "disabled"
    no_eos = _ScriptedBackend()
    no_eos.tokenizer = SimpleNamespace(eos_token_id=None)
    with pytest.raises(ValueError):
        SamplingScope("thinking", ThinkingFormat(end_token_ids=(END,))).wrap(no_eos, PROMPT)
