"""EOS-absorbing fixed-length view (the stopped-sequence backend with EOS as the only stop).

Reference behaviour: src/inference_scaling/arllm/backends/absorbing.py:11-30.
"""

from __future__ import annotations

from collections.abc import Sequence

from ..types import AutoregressiveBackend, GenerationRequest, SequenceSample
from .stopping import StoppedSequenceBackend


class AbsorbingEOSBackend(StoppedSequenceBackend):
    def __init__(self, backend: AutoregressiveBackend, eos_token_id: int, *, absorbing_after: int = 0):
        super().__init__(backend, stop_token_sequences=(), eos_token_id=eos_token_id,
                         protected_prefix_length=absorbing_after, generation_chunk_size=None)
        self.absorbing_after = absorbing_after
        self.model_id = f"{backend.model_id}|absorbing-eos={eos_token_id};after={absorbing_after}"

    def sample_batch(self, requests: Sequence[GenerationRequest]) -> list[SequenceSample]:
        if any(r.sampling.eos_token_id is not None for r in requests):
            raise ValueError("the outer fixed-length policy must leave eos_token_id unset; "
                             "the adapter supplies absorbing EOS semantics")
        return super().sample_batch(requests)


__all__ = ["AbsorbingEOSBackend"]
