"""Order-independent random streams.

A :class:`SeedStream` maps a root seed and a path of names/indices to a 63-bit
seed, so every stochastic decision of an algorithm (a chain's cut, a proposal,
an accept draw) has its own stream and batching or asynchronous scheduling
cannot change any random number.

The derivation (blake2b-64 keyed by the 16-byte little-endian root, over a
compact JSON encoding of typed path parts) is kept bit-compatible with the
reference (src/inference_scaling/shared/rng.py:43-57) so that seeds, and hence
sampled trajectories of the CPU tabular oracle, agree across the two projects.
"""

from __future__ import annotations

import hashlib
import json
from dataclasses import dataclass
from math import isfinite

import numpy as np


def _encode(part: object) -> list:
    if part is None:
        return ["none", None]
    if isinstance(part, bool):
        return ["bool", part]
    if isinstance(part, int):
        return ["int", str(part)]
    if isinstance(part, float):
        if not isfinite(part):
            raise ValueError("seed path floats must be finite")
        return ["float", part.hex()]
    if isinstance(part, str):
        return ["str", part]
    if isinstance(part, bytes):
        return ["bytes", part.hex()]
    raise TypeError("seed path entries must be None, bool, int, float, str, or bytes")


@dataclass(frozen=True, slots=True)
class SeedStream:
    root_seed: int

    def __post_init__(self) -> None:
        if isinstance(self.root_seed, bool) or not isinstance(self.root_seed, int):
            raise TypeError("root_seed must be an integer")
        if not 0 <= self.root_seed < 2**128:
            raise ValueError("root_seed must lie in [0, 2**128)")

    def derive(self, *path: object) -> int:
        payload = json.dumps([_encode(p) for p in path], ensure_ascii=False, separators=(",", ":")).encode("utf-8")
        key = self.root_seed.to_bytes(16, "little", signed=False)
        digest = hashlib.blake2b(payload, digest_size=8, key=key).digest()
        return int.from_bytes(digest, "little") & ((1 << 63) - 1)

    def generator(self, *path: object) -> np.random.Generator:
        return np.random.default_rng(self.derive(*path))

    def child(self, *path: object) -> "SeedStream":
        return SeedStream(self.derive(*path))
