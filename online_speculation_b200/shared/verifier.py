"""Verifier rewards: text scorers configured by a ``[verifier]`` TOML table and exposed as
token-level rewards (single and batched) or as a batched training-reward callback.

Table fields (validated against one schema, all problems reported together):

    provider           "python" (default) or "constant"
    factory            "package.module:callable"; called as factory(context=..., **options)
    name               label used in the replay version key (default: factory, else provider)
    options            keyword arguments of the factory ("context" is reserved)
    requires_reference the verifier needs the example's reference answer
    value              the reward of a constant verifier

The table format, the factory call convention and the replay version string
(``name:`` + 16 hex digits of the SHA-256 of the compact, key-sorted JSON of the
spec) are the plugin contract of src/inference_scaling/shared/verifier.py: configs
and replay caches written for it keep working here.
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
    """What a verifier sees when it is built (the reference only if it asks for one)."""

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

_PROVIDERS = ("python", "constant")
_KNOWN_FIELDS = frozenset({"provider", "name", "factory", "options", "requires_reference", "value"})


def _nonempty_str(v: object) -> bool:
    return isinstance(v, str) and bool(v)


def _table_problems(t: Mapping[str, object]) -> tuple[list[str], list[str]]:
    """(type problems, value problems) of one [verifier] table."""
    types: list[str] = []
    values: list[str] = []
    unknown = sorted(set(t) - _KNOWN_FIELDS)
    if unknown:
        values.append(f"unknown fields {unknown}")
    provider = t.get("provider", "python")
    if not _nonempty_str(provider):
        types.append("provider must be a non-empty string")
    elif provider not in _PROVIDERS:
        values.append(f"provider {provider!r} is not one of {_PROVIDERS}")
    if "factory" in t and t["factory"] is not None and not _nonempty_str(t["factory"]):
        types.append("factory must be a non-empty string")
    if "options" in t and not isinstance(t["options"], Mapping):
        types.append("options must be a table")
    elif isinstance(t.get("options"), Mapping) and "context" in t["options"]:
        values.append("options.context is reserved for the runtime")
    if "name" in t and not _nonempty_str(t["name"]):
        types.append("name must be a non-empty string")
    if not isinstance(t.get("requires_reference", False), bool):
        types.append("requires_reference must be true or false")
    factory = t.get("factory")
    has_value = "value" in t or (isinstance(t.get("options"), Mapping) and "value" in t["options"])
    if provider == "python":
        if not factory:
            values.append("a python verifier needs a factory")
        if "value" in t:
            values.append("value belongs to constant verifiers")
    elif provider == "constant":
        if factory is not None:
            values.append("a constant verifier takes no factory")
        if not has_value:
            values.append("a constant verifier needs a value")
    return types, values


@dataclass(frozen=True, slots=True)
class VerifierSpec:
    provider: str
    name: str
    factory: str | None = None
    options: Mapping[str, object] = field(default_factory=dict)
    requires_reference: bool = False

    @classmethod
    def from_mapping(cls, values: Mapping[str, object]) -> "VerifierSpec":
        type_problems, value_problems = _table_problems(values)
        if type_problems:
            raise TypeError("invalid [verifier] table: " + "; ".join(type_problems + value_problems))
        if value_problems:
            raise ValueError("invalid [verifier] table: " + "; ".join(value_problems))
        provider = values.get("provider", "python")
        factory = values.get("factory")
        options = dict(values.get("options", {}))
        if "value" in values:
            options["value"] = values["value"]
        return cls(provider, values.get("name", factory or provider), factory, options,
                   values.get("requires_reference", False))

    def as_dict(self) -> dict[str, object]:
        return {"provider": self.provider, "name": self.name, "factory": self.factory, "options": dict(self.options),
                "requires_reference": self.requires_reference}

    def version(self) -> str:
        blob = json.dumps(self.as_dict(), ensure_ascii=False, sort_keys=True, separators=(",", ":"))
        return self.name + ":" + hashlib.sha256(blob.encode("utf-8")).hexdigest()[:16]


def verifier_spec_from_config(config: Mapping[str, object]) -> VerifierSpec:
    table = config.get("verifier")
    if not isinstance(table, Mapping):
        raise ValueError("this method scores with a verifier: the config needs a [verifier] table")
    return VerifierSpec.from_mapping(table)


def load_verifier_table(path: str | Path) -> dict[str, object]:
    """Read a TOML file that holds exactly one ``[verifier]`` table, validating it."""
    path = Path(path)
    document = tomllib.loads(path.read_text(encoding="utf-8"))
    if list(document) != ["verifier"]:
        raise ValueError(f"{path}: expected a single [verifier] table, found sections {sorted(document)}")
    table = document["verifier"]
    if not isinstance(table, dict):
        raise TypeError(f"{path}: [verifier] is not a table")
    VerifierSpec.from_mapping(table)
    return dict(table)


def replace_verifier_from_file(config: dict[str, Any], path: str | Path | None) -> None:
    if path is not None:
        config["verifier"] = load_verifier_table(path)


def _resolve(reference: str) -> Callable[..., object]:
    module_name, _, attribute = reference.partition(":")
    if not module_name or not attribute:
        raise ValueError(f"factory {reference!r} is not of the form 'package.module:callable'")
    target = getattr(importlib.import_module(module_name), attribute, None)
    if not callable(target):
        raise TypeError(f"factory {reference!r} does not name a callable")
    return target


def _as_reward(raw: object, who: str) -> float:
    try:
        value = float(raw)  # type: ignore[arg-type]
    except (TypeError, ValueError):
        raise TypeError(f"verifier {who!r} produced {raw!r}, which is not a number") from None
    if not isfinite(value):
        raise ValueError(f"verifier {who!r} produced the non-finite reward {value}")
    return value


class ConfiguredVerifier:
    """A built verifier: checked scalar and batched scoring plus its replay identity."""

    def __init__(self, spec: VerifierSpec, score: VerifierCallable, score_batch: VerifierBatchCallable | None = None):
        self.spec = spec
        self._one = score
        self._many = score_batch

    def score(self, prompt: str, completion: str) -> float:
        return _as_reward(self._one(prompt, completion), self.spec.name)

    def score_batch(self, inputs: Sequence[VerifierInput]) -> tuple[float, ...]:
        items = tuple(inputs)
        raw = tuple(self._many(items)) if self._many is not None else tuple(
            self._one(i.prompt, i.completion) for i in items)
        if len(raw) != len(items):
            raise ValueError(f"verifier {self.spec.name!r}: {len(raw)} rewards for {len(items)} inputs")
        return tuple(_as_reward(r, self.spec.name) for r in raw)

    def describe(self) -> dict[str, object]:
        return self.spec.as_dict()

    @property
    def version(self) -> str:
        return self.spec.version()


def build_verifier(spec: VerifierSpec, *, context: VerifierContext) -> ConfiguredVerifier:
    if spec.requires_reference and context.reference is None:
        raise ValueError(f"verifier {spec.name!r} scores against a reference, and none was given")
    if spec.provider == "constant":
        constant = _as_reward(spec.options["value"], spec.name)
        return ConfiguredVerifier(spec, lambda prompt, completion: constant)
    product = _resolve(spec.factory)(context=context, **dict(spec.options))
    if isinstance(product, TextVerifier):
        batch = getattr(product, "score_batch", None)
        return ConfiguredVerifier(spec, product.score, batch if callable(batch) else None)
    if callable(product):
        return ConfiguredVerifier(spec, product)
    raise TypeError(f"factory {spec.factory!r} returned a {type(product).__name__}, neither a verifier nor a callable")


class TokenVerifierReward:
    """reward(prompt_tokens, completion_tokens): decode, then score the text."""

    def __init__(self, verifier: ConfiguredVerifier, decoder: Callable[[TokenSequence], str]):
        self.verifier = verifier
        self.decoder = decoder

    def __call__(self, prompt: TokenSequence, completion: TokenSequence) -> float:
        return self.verifier.score(self.decoder(prompt), self.decoder(completion))

    def batch(self, prompt: TokenSequence, completions: Sequence[TokenSequence]) -> tuple[float, ...]:
        text = self.decoder(prompt)
        return self.verifier.score_batch([VerifierInput(text, self.decoder(c)) for c in completions])

    def describe(self) -> dict[str, object]:
        return self.verifier.describe()

    @property
    def version(self) -> str:
        return self.verifier.version


def _message_text(value: object) -> str:
    """Training columns hold strings, chat messages ({"content": ...}) or lists of either."""
    if isinstance(value, str):
        return value
    if isinstance(value, Mapping):
        try:
            return str(value["content"])
        except KeyError:
            raise TypeError("a chat message without a 'content' field") from None
    if isinstance(value, Sequence) and not isinstance(value, (bytes, bytearray)):
        return "\n".join(map(_message_text, value))
    raise TypeError(f"cannot read text from a {type(value).__name__}")


@dataclass
class _RewardTally:
    calls: int = 0
    completions: int = 0
    completion_tokens: int = 0
    total: float = 0.0
    low: float | None = None
    high: float | None = None

    def add(self, rewards: Sequence[float]) -> None:
        self.calls += 1
        self.completions += len(rewards)
        if rewards:
            self.total += sum(rewards)
            self.low = min(rewards) if self.low is None else min(self.low, *rewards)
            self.high = max(rewards) if self.high is None else max(self.high, *rewards)


class ConfiguredTrainingVerifierReward:
    """Batched training reward (prompts, completions, ...) -> rewards.  One verifier is built
    per distinct (prompt, reference) pair and cached; every completion of that pair is
    scored in one batch."""

    def __init__(self, spec: VerifierSpec, *, reference_field: str = "reference"):
        if not reference_field:
            raise ValueError("reference_field has to name a dataset column")
        self.spec = spec
        self.reference_field = reference_field
        self._verifiers: dict[tuple[str, str | None], ConfiguredVerifier] = {}
        self._tally = _RewardTally()

    # read-only counters of the calls so far
    calls = property(lambda self: self._tally.calls)
    completions = property(lambda self: self._tally.completions)
    completion_tokens = property(lambda self: self._tally.completion_tokens)
    reward_sum = property(lambda self: self._tally.total)
    reward_minimum = property(lambda self: self._tally.low)
    reward_maximum = property(lambda self: self._tally.high)

    def _references(self, n: int, columns: Mapping[str, object]) -> Sequence[str | None]:
        if not self.spec.requires_reference:
            return [None] * n
        refs = columns.get(self.reference_field)
        if isinstance(refs, (str, bytes, bytearray)) or not isinstance(refs, Sequence):
            raise ValueError(f"the verifier needs the column {self.reference_field!r} (one reference per row)")
        if len(refs) != n:
            raise ValueError(f"{len(refs)} references for {n} completions")
        return [str(r) for r in refs]

    def _verifier(self, prompt: str, reference: str | None) -> ConfiguredVerifier:
        key = (prompt, reference)
        if key not in self._verifiers:
            self._verifiers[key] = build_verifier(self.spec, context=VerifierContext(prompt, reference))
        return self._verifiers[key]

    def __call__(self, prompts: Sequence[object], completions: Sequence[object],
                 completion_ids: Sequence[Sequence[int]] | None = None, **columns: object) -> list[float]:
        n = len(completions)
        if len(prompts) != n:
            raise ValueError(f"{len(prompts)} prompts for {n} completions")
        if completion_ids is not None and len(completion_ids) != n:
            raise ValueError(f"{len(completion_ids)} token-id rows for {n} completions")
        refs = self._references(n, columns)
        prompt_text = [_message_text(p) for p in prompts]
        completion_text = [_message_text(c) for c in completions]
        rows_of: dict[tuple[str, str | None], list[int]] = {}
        for i, key in enumerate(zip(prompt_text, refs)):
            rows_of.setdefault(key, []).append(i)
        rewards = [0.0] * n
        for (prompt, reference), rows in rows_of.items():
            scored = self._verifier(prompt, reference).score_batch(
                [VerifierInput(prompt, completion_text[i]) for i in rows])
            for i, r in zip(rows, scored):
                rewards[i] = r
        self._tally.add(rewards)
        if completion_ids is not None:
            self._tally.completion_tokens += sum(map(len, completion_ids))
        return rewards

    def snapshot(self, *, num_generations: int) -> dict[str, int | float | None]:
        if num_generations < 1:
            raise ValueError("num_generations has to be at least 1")
        t = self._tally
        return {"reward_calls": t.calls, "generated_completions": t.completions,
                "generated_prompt_groups": t.completions // num_generations,
                "generated_completion_tokens": t.completion_tokens, "reward_sum": t.total,
                "observed_mean_reward": t.total / t.completions if t.completions else None,
                "observed_minimum_reward": t.low, "observed_maximum_reward": t.high}


def build_token_verifier_reward(config: Mapping[str, object], *, context: VerifierContext,
                                decoder: Callable[[TokenSequence], str]) -> TokenVerifierReward:
    return TokenVerifierReward(build_verifier(verifier_spec_from_config(config), context=context), decoder)


__all__ = ["BatchTextVerifier", "ConfiguredTrainingVerifierReward", "ConfiguredVerifier", "TextVerifier",
           "TokenBatchReward", "TokenReward", "TokenVerifierReward", "VerifierContext", "VerifierInput",
           "VerifierSpec", "build_token_verifier_reward", "build_verifier", "load_verifier_table",
           "replace_verifier_from_file", "verifier_spec_from_config"]
