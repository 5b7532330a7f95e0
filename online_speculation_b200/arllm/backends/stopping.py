"""Fixed-length view of generation that stops at token-sequence boundaries.

A stop (a configured marker, EOS, or the end of the first complete thinking block)
keeps its model probability and every later position is EOS padding with
probability one.  So a stopped sequence has the fixed length the caller asked for,
its padding scores log 1, and any non-EOS token after a stop scores log 0; the same
contract then serves conditional IS, replay and fixed-length MH.

Generation runs in chunks (``generation_chunk_size``) so a request that stops early
does not spend its whole budget; every chunk after the first draws from the seed
stream ``(seed, "stop-chunk", offset)`` under the request id
``<id>:stop-chunk:<offset>``.  Those names, and the model-id suffix that records
the stop configuration, are the cache and random-stream identities of
src/inference_scaling/arllm/backends/stopping.py.
"""

from __future__ import annotations

from collections.abc import Sequence
from dataclasses import dataclass, field, replace

from ...shared.output import OutputParser, find_token_sequence
from ...shared.rng import SeedStream
from ...shared.types import TokenSequence
from ..config import SamplingConfig
from ..types import AutoregressiveBackend, GenerationRequest, ScoreRequest, SequenceSample

_NEG_INF = float("-inf")


@dataclass
class _Progress:
    """What one request has generated so far."""

    request: GenerationRequest
    tokens: list[int] = field(default_factory=list)
    logprobs: list[float] = field(default_factory=list)
    reference: list[float] | None = field(default_factory=list)
    stopped: bool = False

    @property
    def remaining(self) -> int:
        return self.request.max_new_tokens - len(self.tokens)


class StoppedSequenceBackend:
    def __init__(self, backend: AutoregressiveBackend, *, stop_token_sequences: Sequence[TokenSequence],
                 eos_token_id: int, protected_prefix_length: int, generation_chunk_size: int | None = 256,
                 thinking_parser: OutputParser | None = None, thinking_prompt: TokenSequence = ()):
        stops = tuple(tuple(marker) for marker in stop_token_sequences)
        if not all(stops_ok := [bool(m) and min(m) >= 0 for m in stops]):
            raise ValueError(f"stop markers must be non-empty token-id sequences ({stops_ok.count(False)} are not)")
        if eos_token_id < 0:
            raise ValueError("eos_token_id must be a token id")
        if protected_prefix_length < 0:
            raise ValueError("protected_prefix_length cannot be negative")
        if generation_chunk_size is not None and generation_chunk_size < 1:
            raise ValueError("generation_chunk_size must be positive (or None for one chunk)")
        if thinking_parser is not None and len(thinking_prompt) != protected_prefix_length:
            raise ValueError("the thinking prompt is the protected prefix: their lengths must agree")
        self.backend = backend
        self.stop_token_sequences = stops
        self.eos_token_id = eos_token_id
        self.protected_prefix_length = protected_prefix_length
        self.generation_chunk_size = generation_chunk_size
        self.thinking_parser = thinking_parser
        self.thinking_prompt = tuple(thinking_prompt)
        ident = f"{backend.model_id}|stops={stops};eos={eos_token_id};after={protected_prefix_length};" \
                f"chunk={generation_chunk_size}"
        self.model_id = ident if thinking_parser is None else f"{ident};thinking={thinking_parser.describe()}"
        self._markers = (*stops, (eos_token_id,))

    # ---- pass-through metadata of the wrapped backend
    @property
    def tokenizer(self):
        return getattr(self.backend, "tokenizer")

    @property
    def parameter_count(self):
        return getattr(self.backend, "parameter_count")

    def encode(self, text: str, *, add_special_tokens: bool = True):
        return self.backend.encode(text, add_special_tokens=add_special_tokens)

    def decode(self, tokens: TokenSequence, *, skip_special_tokens: bool = True):
        return self.backend.decode(tokens, skip_special_tokens=skip_special_tokens)

    def snapshot(self):
        return self.backend.snapshot()

    def score_statistics_batch(self, requests, *, confidence_top_k=None):
        return self.backend.score_statistics_batch(requests, confidence_top_k=confidence_top_k)

    # ---- stop rule
    def _thinking_end(self, generated: TokenSequence) -> int | None:
        parser = self.thinking_parser
        if parser is None:
            return None
        boundary = getattr(parser, "stop_boundary", None)
        if boundary is not None:
            return boundary(self.thinking_prompt, generated, eos_token_id=self.eos_token_id)
        seg = parser.split(self.thinking_prompt, generated, eos_token_id=self.eos_token_id)
        return seg.boundary_end if seg.has_complete_thinking else None

    def _stop_end(self, generated: TokenSequence) -> int | None:
        """Length of the generated tokens up to and including the first stop, if any."""
        candidates = [self._thinking_end(generated)]
        for marker in self._markers:
            at = find_token_sequence(generated, marker)
            candidates.append(None if at is None else at + len(marker))
        found = [c for c in candidates if c is not None]
        return min(found) if found else None

    def _generated_part(self, prefix: TokenSequence) -> TokenSequence:
        if len(prefix) < self.protected_prefix_length:
            raise ValueError(f"the prefix ({len(prefix)} tokens) is shorter than the protected prompt")
        generated = tuple(prefix[self.protected_prefix_length:])
        end = self._stop_end(generated)
        if end is not None and any(t != self.eos_token_id for t in generated[end:]):
            raise ValueError("the prefix continues with non-EOS tokens after a stop")
        return generated

    def _inner_policy(self, sampling: SamplingConfig | None) -> SamplingConfig:
        policy = sampling if sampling is not None else SamplingConfig()
        if policy.eos_token_id not in (None, self.eos_token_id):
            raise ValueError(f"the request's EOS {policy.eos_token_id} is not this backend's {self.eos_token_id}")
        return replace(policy, eos_token_id=self.eos_token_id)

    def _padding_scores(self, tail: TokenSequence) -> tuple[float, ...]:
        return tuple(0.0 if t == self.eos_token_id else _NEG_INF for t in tail)

    # ---- generation
    def _chunk_request(self, p: _Progress) -> GenerationRequest:
        r = p.request
        offset = len(p.tokens)
        whole = r.arithmetic_uniform is not None or self.generation_chunk_size is None
        size = p.remaining if whole else min(p.remaining, self.generation_chunk_size)
        seed = r.seed if offset == 0 else SeedStream(r.seed).derive("stop-chunk", offset)
        uniforms = None if r.uniforms is None else r.uniforms[offset:offset + size]
        return GenerationRequest(r.prefix + tuple(p.tokens), size, self._inner_policy(r.sampling), seed,
                                 f"{r.request_id}:stop-chunk:{offset}", uniforms, r.arithmetic_uniform)

    def _absorb(self, p: _Progress, chunk: GenerationRequest, sample: SequenceSample, ref_policy: str) -> None:
        if (sample.prefix != chunk.prefix or sample.policy_id != chunk.sampling.policy_id
                or sample.model_id != self.backend.model_id or not 0 < len(sample.token_ids) <= chunk.max_new_tokens):
            raise RuntimeError("the wrapped backend's sample does not answer its request")
        before = self._generated_part(chunk.prefix)
        end = self._stop_end(before + tuple(sample.token_ids))
        keep = len(sample.token_ids) if end is None else end - len(before)
        p.tokens.extend(sample.token_ids[:keep])
        p.logprobs.extend(sample.token_logprobs[:keep])
        if sample.reference_policy_id != ref_policy:
            p.reference = None
        elif p.reference is not None:
            p.reference.extend(sample.reference_token_logprobs[:keep])
        if end is not None:
            p.stopped = True
        elif len(sample.token_ids) != chunk.max_new_tokens:
            raise RuntimeError("a chunk ended early without EOS or a stop marker")

    def _finished(self, p: _Progress) -> SequenceSample:
        r = p.request
        pad = p.remaining
        reference = None if p.reference is None else tuple(p.reference) + (0.0,) * pad
        return SequenceSample(r.prefix, tuple(p.tokens) + (self.eos_token_id,) * pad,
                              tuple(p.logprobs) + (0.0,) * pad, r.sampling.policy_id, self.model_id, r.request_id,
                              "stop" if p.stopped else "length", reference,
                              None if reference is None else SamplingConfig(eos_token_id=r.sampling.eos_token_id
                                                                            ).policy_id)

    def sample_batch(self, requests: Sequence[GenerationRequest]) -> list[SequenceSample]:
        progress = [_Progress(r) for r in requests]
        for p in progress:
            p.stopped = self._stop_end(self._generated_part(p.request.prefix)) is not None
        ref_policy = SamplingConfig(eos_token_id=self.eos_token_id).policy_id
        while True:
            active = [p for p in progress if not p.stopped and p.remaining > 0]
            if not active:
                break
            chunks = [self._chunk_request(p) for p in active]
            samples = self.backend.sample_batch(chunks)
            if len(samples) != len(chunks):
                raise RuntimeError(f"{len(samples)} samples came back for {len(chunks)} chunk requests")
            for p, chunk, sample in zip(active, chunks, samples):
                self._absorb(p, chunk, sample, ref_policy)
        return [self._finished(p) for p in progress]

    # ---- scoring
    def score_batch(self, requests: Sequence[ScoreRequest]) -> list[tuple[float, ...]]:
        results: list[tuple[float, ...] | None] = []
        forwarded: list[ScoreRequest] = []
        slots: list[tuple[int, TokenSequence]] = []        # (result index, padding tail)
        for r in requests:
            generated = self._generated_part(r.prefix)
            already_stopped = self._stop_end(generated) is not None
            for continuation in r.continuations:
                if already_stopped or not continuation:
                    results.append(self._padding_scores(continuation))
                    continue
                end = self._stop_end(generated + tuple(continuation))
                keep = len(continuation) if end is None else end - len(generated)
                slots.append((len(results), continuation[keep:]))
                results.append(None)
                forwarded.append(ScoreRequest(r.prefix, (continuation[:keep],), self._inner_policy(r.sampling)))
        scored = self.backend.score_batch(forwarded) if forwarded else []
        if len(scored) != len(forwarded):
            raise RuntimeError(f"{len(scored)} scores came back for {len(forwarded)} requests")
        for (index, tail), request, score in zip(slots, forwarded, scored):
            if len(score) != len(request.continuations[0]):
                raise RuntimeError("a score does not have one entry per scored token")
            results[index] = tuple(score) + self._padding_scores(tail)
        return results  # type: ignore[return-value]


__all__ = ["StoppedSequenceBackend"]
