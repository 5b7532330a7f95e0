"""Fixed-length generation with EOS absorbing: once EOS is emitted every later token is
EOS with probability one, so an outer fixed-length policy sees sequences of the length
it asked for.  Implemented as a stop-sequence backend whose only stop is EOS; tokens
before ``absorbing_after`` may not stop.  The model-id suffix is part of the cache and
replay identity (src/inference_scaling/arllm/backends/absorbing.py).
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
        owners = [r.request_id for r in requests if r.sampling.eos_token_id is not None]
        if owners:
            raise ValueError(f"requests {owners[:3]} set eos_token_id; with an absorbing-EOS backend the "
                             "outer policy is fixed-length and EOS handling belongs to this adapter")
        return super().sample_batch(requests)


__all__ = ["AbsorbingEOSBackend"]
