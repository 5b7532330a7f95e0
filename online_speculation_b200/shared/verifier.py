"""Configurable verifier rewards behind the token-level reward interface.

A verifier scores decoded (prompt, completion) text; adapters expose it as
``reward(prompt_tokens, completion_tokens) -> float`` (and a batched form) for
the AR and dLLM algorithms, and as a GRPO-style batched training callback.
Configuration is one TOML ``[verifier]`` table:

    provider = "python" | "constant"
    factory  = "package.module:factory"      # python: called as factory(context=..., **options)
    name, options = {...}, requires_reference = bool, value = <float>  # constant

The table format, the factory call convention and the ``version`` replay key
(``name:`` + the first 16 hex digits of the SHA-256 of the sorted compact JSON
description) are those of src/inference_scaling/shared/verifier.py:69-451, so
existing configs and replay caches stay valid.
"""

from __future__ import annotations

import hashlib
import importlib
import json
import tomllib
from collections.abc import Callable, Mapping, Sequence
from dataclasses import dataclass, field
from math import isfinite
from pathlib import Path
from typing import Any, Protocol, runtime_checkable

from .types import TokenSequence


@dataclass(frozen=True, slots=True)
class VerifierInput:
    prompt: str
    completion: str


@dataclass(frozen=True, slots=True)
class VerifierContext:
    """What a verifier instance may see at construction (reference only if it opts in)."""

    prompt: str
    reference: str | None = None
    metadata: Mapping[str, object] = field(default_factory=dict)


@runtime_checkable
class TextVerifier(Protocol):
    def score(self, prompt: str, completion: str) -> float: ...


class BatchTextVerifier(TextVerifier, Protocol):
    def score_batch(self, inputs: Sequence[VerifierInput]) -> Sequence[float]: ...


VerifierCallable = Callable[[str, str], float]
VerifierBatchCallable = Callable[[Sequence[VerifierInput]], Sequence[float]]
TokenReward = Callable[[TokenSequence, TokenSequence], float]
TokenBatchReward = Callable[[TokenSequence, Sequence[TokenSequence]], Sequence[float]]

_FIELDS = {"provider", "name", "factory", "options", "requires_reference", "value"}


@dataclass(frozen=True, slots=True)
class VerifierSpec:
    provider: str
    name: str
    factory: str | None = None
    options: Mapping[str, object] = field(default_factory=dict)
    requires_reference: bool = False

    @classmethod
    def from_mapping(cls, values: Mapping[str, object]) -> "VerifierSpec":
        extra = sorted(set(values) - _FIELDS)
        if extra:
            raise ValueError(f"unknown verifier configuration fields: {extra}")
        provider = values.get("provider", "python")
        if not isinstance(provider, str) or not provider:
            raise TypeError("verifier.provider must be a non-empty string")
        if provider not in ("python", "constant"):
            raise ValueError(f"unsupported verifier provider {provider!r}")
        factory = values.get("factory")
        if factory is not None and (not isinstance(factory, str) or not factory):
            raise TypeError("verifier.factory must be a non-empty string")
        if provider == "python" and not factory:
            raise ValueError("a Python verifier requires verifier.factory")
        if provider == "constant" and factory is not None:
            raise ValueError("a constant verifier cannot define verifier.factory")
        opts = values.get("options", {})
        if not isinstance(opts, Mapping):
            raise TypeError("verifier.options must be a table")
        opts = dict(opts)
        if "context" in opts:
            raise ValueError("verifier.options.context is reserved by the runtime")
        if "value" in values:
            if provider != "constant":
                raise ValueError("verifier.value is valid only for provider='constant'")
            opts["value"] = values["value"]
        if provider == "constant" and "value" not in opts:
            raise ValueError("a constant verifier requires verifier.value")
        name = values.get("name", factory or provider)
        if not isinstance(name, str) or not name:
            raise TypeError("verifier.name must be a non-empty string")
        req = values.get("requires_reference", False)
        if not isinstance(req, bool):
            raise TypeError("verifier.requires_reference must be a boolean")
        return cls(provider, name, factory, opts, req)

    def as_dict(self) -> dict[str, object]:
        return {"provider": self.provider, "name": self.name, "factory": self.factory, "options": dict(self.options),
                "requires_reference": self.requires_reference}


def verifier_spec_from_config(config: Mapping[str, object]) -> VerifierSpec:
    table = config.get("verifier")
    if not isinstance(table, Mapping):
        raise ValueError("a verifier-assisted method requires a [verifier] table")
    return VerifierSpec.from_mapping(table)


def load_verifier_table(path: str | Path) -> dict[str, object]:
    """A standalone TOML file holding exactly one ``[verifier]`` table (validated eagerly)."""
    src = Path(path)
    with src.open("rb") as f:
        doc = tomllib.load(f)
    if set(doc) != {"verifier"}:
        raise ValueError(f"{src} must contain one top-level [verifier] table and no other sections")
    if not isinstance(doc["verifier"], dict):
        raise TypeError("[verifier] must be a TOML table")
    VerifierSpec.from_mapping(doc["verifier"])
    return dict(doc["verifier"])


def replace_verifier_from_file(config: dict[str, Any], path: str | Path | None) -> None:
    if path is not None:
        config["verifier"] = load_verifier_table(path)


def _load_factory(ref: str) -> Callable[..., object]:
    module, sep, attr = ref.partition(":")
    if not sep or not module or not attr:
        raise ValueError("verifier.factory must use the form 'package.module:factory_name'")
    fn = getattr(importlib.import_module(module), attr, None)
    if not callable(fn):
        raise TypeError(f"verifier factory {ref!r} is not callable")
    return fn


def _finite(value: object, name: str) -> float:
    try:
        v = float(value)  # type: ignore[arg-type]
    except (TypeError, ValueError) as e:
        raise TypeError(f"verifier {name!r} returned a non-numeric reward {value!r}") from e
    if not isfinite(v):
        raise ValueError(f"verifier {name!r} returned a non-finite reward {v!r}")
    return v


class ConfiguredVerifier:
    """A validated verifier instance with its reproducibility metadata."""

    def __init__(self, spec: VerifierSpec, score: VerifierCallable, score_batch: VerifierBatchCallable | None = None):
        self.spec, self._score, self._batch = spec, score, score_batch

    def score(self, prompt: str, completion: str) -> float:
        return _finite(self._score(prompt, completion), self.spec.name)

    def score_batch(self, inputs: Sequence[VerifierInput]) -> tuple[float, ...]:
        if self._batch is None:
            return tuple(self.score(i.prompt, i.completion) for i in inputs)
        vals = tuple(self._batch(inputs))
        if len(vals) != len(inputs):
            raise ValueError(f"verifier {self.spec.name!r} returned {len(vals)} rewards for {len(inputs)} inputs")
        return tuple(_finite(v, self.spec.name) for v in vals)

    def describe(self) -> dict[str, object]:
        return self.spec.as_dict()

    @property
    def version(self) -> str:
        blob = json.dumps(self.spec.as_dict(), ensure_ascii=False, sort_keys=True, separators=(",", ":"))
        return f"{self.spec.name}:{hashlib.sha256(blob.encode('utf-8')).hexdigest()[:16]}"


def build_verifier(spec: VerifierSpec, *, context: VerifierContext) -> ConfiguredVerifier:
    if spec.requires_reference and context.reference is None:
        raise ValueError(f"verifier {spec.name!r} requires a reference value")
    if spec.provider == "constant":
        v = _finite(spec.options["value"], spec.name)
        return ConfiguredVerifier(spec, lambda _p, _c: v)
    made = _load_factory(spec.factory)(context=context, **dict(spec.options))
    if isinstance(made, TextVerifier):
        batch = getattr(made, "score_batch", None)
        return ConfiguredVerifier(spec, made.score, batch if callable(batch) else None)
    if callable(made):
        return ConfiguredVerifier(spec, made)
    raise TypeError(f"verifier factory {spec.factory!r} returned unsupported value {type(made).__name__}")


class TokenVerifierReward:
    """Token-level adapter: decodes ids and forwards to the text verifier."""

    def __init__(self, verifier: ConfiguredVerifier, decoder: Callable[[TokenSequence], str]):
        self.verifier, self._decode = verifier, decoder

    def __call__(self, prompt: TokenSequence, completion: TokenSequence) -> float:
        return self.verifier.score(self._decode(prompt), self._decode(completion))

    def batch(self, prompt: TokenSequence, completions: Sequence[TokenSequence]) -> tuple[float, ...]:
        p = self._decode(prompt)
        return self.verifier.score_batch(tuple(VerifierInput(p, self._decode(c)) for c in completions))

    def describe(self) -> dict[str, object]:
        return self.verifier.describe()

    @property
    def version(self) -> str:
        return self.verifier.version


def _text(value: object) -> str:
    if isinstance(value, str):
        return value
    if isinstance(value, Mapping):
        if "content" not in value:
            raise TypeError("a training message must contain a content field")
        return str(value["content"])
    if isinstance(value, Sequence) and not isinstance(value, (bytes, bytearray)):
        return "\n".join(_text(v) for v in value)
    raise TypeError(f"unsupported training text value: {type(value).__name__}")


class ConfiguredTrainingVerifierReward:
    """Batched training-reward callback (prompts, completions, ...) -> rewards, one verifier per prompt."""

    def __init__(self, spec: VerifierSpec, *, reference_field: str = "reference"):
        if not reference_field:
            raise ValueError("reference_field must be non-empty")
        self.spec, self.reference_field = spec, reference_field
        self._cache: dict[tuple[str, str | None], ConfiguredVerifier] = {}
        self.calls = self.completions = self.completion_tokens = 0
        self.reward_sum = 0.0
        self.reward_minimum: float | None = None
        self.reward_maximum: float | None = None

    def __call__(self, prompts: Sequence[object], completions: Sequence[object],
                 completion_ids: Sequence[Sequence[int]] | None = None, **columns: object) -> list[float]:
        if len(prompts) != len(completions):
            raise ValueError("training prompts and completions have different lengths")
        if self.spec.requires_reference:
            refs = columns.get(self.reference_field)
            if not isinstance(refs, Sequence) or isinstance(refs, (str, bytes, bytearray)):
                raise ValueError(f"training verifier requires column {self.reference_field!r}")
            if len(refs) != len(completions):
                raise ValueError("training references and completions have different lengths")
        else:
            refs = (None,) * len(completions)
        ptxt = [_text(p) for p in prompts]
        ctxt = [_text(c) for c in completions]
        groups: dict[tuple[str, str | None], list[int]] = {}
        for i, (p, r) in enumerate(zip(ptxt, refs)):
            groups.setdefault((p, None if r is None else str(r)), []).append(i)
        out = [0.0] * len(completions)
        for key, idx in groups.items():
            v = self._cache.get(key)
            if v is None:
                v = self._cache[key] = build_verifier(self.spec, context=VerifierContext(key[0], key[1]))
            for i, val in zip(idx, v.score_batch(tuple(VerifierInput(key[0], ctxt[i]) for i in idx))):
                out[i] = val
        self.calls += 1
        self.completions += len(completions)
        if completion_ids is not None:
            if len(completion_ids) != len(completions):
                raise ValueError("training completion token ids and completions have different lengths")
            self.completion_tokens += sum(len(t) for t in completion_ids)
        if out:
            self.reward_sum += sum(out)
            lo, hi = min(out), max(out)
            self.reward_minimum = lo if self.reward_minimum is None else min(self.reward_minimum, lo)
            self.reward_maximum = hi if self.reward_maximum is None else max(self.reward_maximum, hi)
        return out

    def snapshot(self, *, num_generations: int) -> dict[str, int | float | None]:
        if num_generations <= 0:
            raise ValueError("num_generations must be positive")
        return {"reward_calls": self.calls, "generated_completions": self.completions,
                "generated_prompt_groups": self.completions // num_generations,
                "generated_completion_tokens": self.completion_tokens, "reward_sum": self.reward_sum,
                "observed_mean_reward": self.reward_sum / self.completions if self.completions else None,
                "observed_minimum_reward": self.reward_minimum, "observed_maximum_reward": self.reward_maximum}


def build_token_verifier_reward(config: Mapping[str, object], *, context: VerifierContext,
                                decoder: Callable[[TokenSequence], str]) -> TokenVerifierReward:
    return TokenVerifierReward(build_verifier(verifier_spec_from_config(config), context=context), decoder)


__all__ = ["BatchTextVerifier", "ConfiguredTrainingVerifierReward", "ConfiguredVerifier", "TextVerifier",
           "TokenBatchReward", "TokenReward", "TokenVerifierReward", "VerifierContext", "VerifierInput",
           "VerifierSpec", "build_token_verifier_reward", "build_verifier", "load_verifier_table",
           "replace_verifier_from_file", "verifier_spec_from_config"]
