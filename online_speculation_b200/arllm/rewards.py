"""Rewards defined through the base model's own scores.

* ``SequenceLogProbabilityReward``: r(y) = c log p(y | x) under ``sampling``.
  With IS temperature tau the tilted target p exp(r / tau) is the power target
  p^(1 + c / tau) (reference: src/inference_scaling/arllm/rewards.py:19-57).
* ``ConsilienceReward``: a verifier-free confidence-trajectory reward.  Token
  t's confidence is -(mean of the top-K next-token log-probabilities); the
  sequence reward is final-window mean - penalty x initial-window mean
  (shared.consilience), over the thinking span when one is found, else the
  full sequence (reference: src/inference_scaling/arllm/rewards.py:60-236).
  The statistics come from the backend's fused per-row scoring kernel.
"""

from __future__ import annotations

from collections import Counter
from collections.abc import Sequence
from math import isfinite
from threading import Lock
from typing import Any, Literal

from ..shared.consilience import confidence_windows
from ..shared.output import OutputParser, ThinkingFormat, ThinkingParser
from ..shared.types import TokenSequence
from .config import SamplingConfig
from .types import AutoregressiveBackend, ScoreRequest


class SequenceLogProbabilityReward:
    def __init__(self, backend: AutoregressiveBackend, sampling: SamplingConfig | None = None, *, scale: float = 1.0,
                 coefficient: float | None = None, normalize: bool = False):
        self.backend = backend
        self.sampling = sampling
        self.scale = float(coefficient if coefficient is not None else scale)
        if not isfinite(self.scale):
            raise ValueError("log-probability reward scale must be finite")
        self.normalize = normalize

    @property
    def coefficient(self) -> float:
        return self.scale

    def __call__(self, prompt: TokenSequence, completion: TokenSequence) -> float:
        return self.batch(prompt, (completion,))[0]

    def batch(self, prompt: TokenSequence, completions: Sequence[TokenSequence]) -> tuple[float, ...]:
        if not completions:
            return ()
        scored = self.backend.score_batch([ScoreRequest(tuple(prompt), tuple(tuple(c) for c in completions),
                                                        self.sampling)])
        if len(scored) != len(completions):
            raise RuntimeError("backend returned an invalid log-probability score batch")
        out = []
        for comp, s in zip(completions, scored):
            if len(s) != len(comp):
                raise RuntimeError("backend returned an invalid token score shape")
            total = float(sum(s))
            if self.normalize and comp:
                total /= len(comp)
            out.append(self.scale * total)
        return tuple(out)

    def target_exponent(self, reward_temperature: float) -> float:
        return 1.0 + self.scale / reward_temperature


class ConsilienceReward:
    def __init__(self, backend: Any, sampling: SamplingConfig | None = None, *, top_k: int = 5,
                 window_fraction: float = 0.2, window_tokens: int | None = None, skip_fraction: float = 0.05,
                 initial_penalty: float = 3.0, scale: float = 1.0,
                 reasoning_end_token_ids: TokenSequence | None = None, thinking_format: OutputParser | None = None,
                 scope: Literal["thinking", "full"] = "thinking"):
        if top_k <= 0:
            raise ValueError("Consilience top_k must be positive")
        if not (isfinite(scale) and scale > 0):
            raise ValueError("Consilience scale must be finite and positive")
        if reasoning_end_token_ids is not None and not reasoning_end_token_ids:
            raise ValueError("reasoning_end_token_ids must be nonempty when provided")
        if scope not in ("thinking", "full"):
            raise ValueError("Consilience scope must be thinking or full")
        if thinking_format is not None and reasoning_end_token_ids is not None:
            raise ValueError("provide thinking_format or reasoning_end_token_ids, not both")
        self.backend, self.sampling, self.top_k = backend, sampling, int(top_k)
        self.window_fraction, self.window_tokens = window_fraction, window_tokens
        self.skip_fraction, self.initial_penalty, self.scale = skip_fraction, initial_penalty, float(scale)
        self.reasoning_end_token_ids, self.scope = reasoning_end_token_ids, scope
        self._score((0.0,))                                   # validates the window settings
        if scope == "thinking" and thinking_format is None:
            if reasoning_end_token_ids is not None:
                thinking_format = ThinkingFormat(end_token_ids=tuple(reasoning_end_token_ids))
            else:
                from .output import thinking_format_from_backend

                thinking_format = thinking_format_from_backend(backend)
        if isinstance(thinking_format, ThinkingFormat):
            thinking_format = ThinkingParser((thinking_format,))
        self.thinking_format = thinking_format
        self._counts: Counter = Counter()
        self._lock = Lock()

    def _score(self, values: Sequence[float]) -> float:
        w = confidence_windows(values, window_fraction=self.window_fraction, window_tokens=self.window_tokens,
                               skip_fraction=self.skip_fraction, initial_penalty=self.initial_penalty)
        s = self.scale * w.score
        if not isfinite(s):
            raise ValueError("Consilience scaled score must be finite")
        return s

    def _input(self, prompt: TokenSequence, completion: TokenSequence):
        prefix, toks = tuple(prompt), tuple(completion)
        eos = getattr(getattr(self.backend, "tokenizer", None), "eos_token_id", None)
        if eos is not None and eos in toks:
            toks = toks[:toks.index(eos) + 1]        # the generated EOS counts, absorbing padding does not
        used, reason = "full", None
        if self.scope == "thinking":
            seg = self.thinking_format.split(prefix, toks, eos_token_id=eos)
            if seg.has_complete_thinking:
                prefix += toks[:seg.thinking_start]
                toks = seg.thinking_token_ids
                used = "thinking"
            else:
                reason = seg.status
        return prefix, toks, {"requested_reward_scope": self.scope, "reward_scope": used,
                              "reward_mode": "consilience_" + used, "reward_fallback_reason": reason}

    def describe_completion(self, prompt, completion) -> dict[str, object]:
        return self._input(prompt, completion)[2]

    def scope_statistics(self) -> dict[str, object]:
        with self._lock:
            c = dict(self._counts)
        return {"evaluated_sequences": sum(c.values()),
                "thinking_sequences": sum(v for (m, _), v in c.items() if m == "thinking"),
                "full_sequences": sum(v for (m, _), v in c.items() if m == "full"),
                "fallback_reasons": {r: v for (_, r), v in c.items() if r is not None}}

    def __call__(self, prompt: TokenSequence, completion: TokenSequence) -> float:
        return self.batch(prompt, (completion,))[0]

    def batch(self, prompt: TokenSequence, completions: Sequence[TokenSequence]) -> tuple[float, ...]:
        if not completions:
            return ()
        rewards = [0.0] * len(completions)
        groups: dict[TokenSequence, list] = {}
        modes = []
        for i, c in enumerate(completions):
            pre, toks, d = self._input(prompt, c)
            modes.append((d["reward_scope"], d["reward_fallback_reason"]))
            if toks:
                groups.setdefault(pre, []).append((i, toks))
        if groups:
            fn = getattr(self.backend, "score_statistics_batch", None)
            if fn is None:
                raise ValueError("Consilience reward requires a backend with top-K score statistics")
            reqs = [ScoreRequest(p, tuple(t for _, t in g), self.sampling) for p, g in groups.items()]
            flat = [x for g in groups.values() for x in g]
            stats = fn(reqs, confidence_top_k=self.top_k)
            if len(stats) != len(flat):
                raise RuntimeError("backend returned an invalid Consilience score batch")
            for (i, toks), st in zip(flat, stats):
                vals = tuple(float(v) for v in st.token_topk_confidences)
                if len(vals) != len(toks):
                    raise RuntimeError("backend returned an invalid Consilience trajectory")
                rewards[i] = self._score(vals)
        with self._lock:
            self._counts.update(modes)
        return tuple(rewards)

    def describe(self) -> dict[str, object]:
        return {"source": "model_consilience", "model_id": self.backend.model_id,
                "policy_id": self.sampling.policy_id if self.sampling is not None else None, "top_k": self.top_k,
                "window_fraction": self.window_fraction, "window_tokens": self.window_tokens,
                "skip_fraction": self.skip_fraction, "initial_penalty": self.initial_penalty, "scale": self.scale,
                "reasoning_end_token_ids": self.reasoning_end_token_ids, "scope": self.scope,
                "fallback": "full_sequence",
                "thinking_format": self.thinking_format.describe() if self.thinking_format is not None else None}


__all__ = ["ConsilienceReward", "SequenceLogProbabilityReward"]
