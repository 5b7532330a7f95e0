"""Fixed-length absorbing view of generation stopped at token-sequence boundaries.

A stop marker (a configured token sequence, EOS, or the end of a complete
thinking block) keeps its model probability; every position after it is EOS
padding with probability one.  Sampling proceeds in chunks so a stop found
early ends the request; scoring truncates at the stop and scores the padding
as log 1 (EOS) or log 0 (anything else).  The same contract then serves
conditional IS, replay and fixed-length MH.
Reference behaviour: src/inference_scaling/arllm/backends/stopping.py:20-218.
"""

from __future__ import annotations

from collections.abc import Sequence
from dataclasses import replace

from ...shared.output import OutputParser, find_token_sequence
from ...shared.rng import SeedStream
from ...shared.types import TokenSequence
from ..config import SamplingConfig
from ..types import AutoregressiveBackend, GenerationRequest, ScoreRequest, SequenceSample


class StoppedSequenceBackend:
    def __init__(self, backend: AutoregressiveBackend, *, stop_token_sequences: Sequence[TokenSequence],
                 eos_token_id: int, protected_prefix_length: int, generation_chunk_size: int | None = 256,
                 thinking_parser: OutputParser | None = None, thinking_prompt: TokenSequence = ()):
        stops = tuple(tuple(m) for m in stop_token_sequences)
        if any(not m or any(t < 0 for t in m) for m in stops):
            raise ValueError("stop_token_sequences must contain nonempty token markers")
        if eos_token_id < 0 or protected_prefix_length < 0 or (generation_chunk_size is not None
                                                               and generation_chunk_size <= 0):
            raise ValueError("invalid EOS, protected prefix length or generation chunk size")
        if thinking_parser is not None and len(thinking_prompt) != protected_prefix_length:
            raise ValueError("thinking_prompt must match the protected prefix length")
        self.backend = backend
        self.stop_token_sequences, self.eos_token_id = stops, eos_token_id
        self.protected_prefix_length, self.generation_chunk_size = protected_prefix_length, generation_chunk_size
        self.thinking_parser, self.thinking_prompt = thinking_parser, tuple(thinking_prompt)
        self.model_id = (f"{backend.model_id}|stops={stops};eos={eos_token_id};after={protected_prefix_length};"
                         f"chunk={generation_chunk_size}")
        if thinking_parser is not None:
            self.model_id += f";thinking={thinking_parser.describe()}"

    # metadata passthrough
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

    # stop semantics
    def _stop_end(self, generated: TokenSequence) -> int | None:
        ends = []
        if self.thinking_parser is not None:
            cb = getattr(self.thinking_parser, "stop_boundary", None)
            if cb is not None:
                b = cb(self.thinking_prompt, generated, eos_token_id=self.eos_token_id)
            else:
                seg = self.thinking_parser.split(self.thinking_prompt, generated, eos_token_id=self.eos_token_id)
                b = seg.boundary_end if seg.has_complete_thinking else None
            if b is not None:
                ends.append(b)
        for m in (*self.stop_token_sequences, (self.eos_token_id,)):
            i = find_token_sequence(generated, m)
            if i is not None:
                ends.append(i + len(m))
        return min(ends) if ends else None

    def _generated(self, prefix: TokenSequence) -> TokenSequence:
        if len(prefix) < self.protected_prefix_length:
            raise ValueError("prefix is shorter than the protected prompt")
        gen = prefix[self.protected_prefix_length:]
        end = self._stop_end(gen)
        if end is not None and any(t != self.eos_token_id for t in gen[end:]):
            raise ValueError("a stopped prefix contains non-padding tokens after its boundary")
        return gen

    def _inner(self, sampling: SamplingConfig | None) -> SamplingConfig:
        s = sampling or SamplingConfig()
        if s.eos_token_id not in (None, self.eos_token_id):
            raise ValueError("sampling uses a different EOS token")
        return replace(s, eos_token_id=self.eos_token_id)

    def _pad_scores(self, tail: TokenSequence) -> tuple[float, ...]:
        return tuple(0.0 if t == self.eos_token_id else float("-inf") for t in tail)

    def sample_batch(self, requests: Sequence[GenerationRequest]) -> list[SequenceSample]:
        n = len(requests)
        toks: list[list[int]] = [[] for _ in range(n)]
        logs: list[list[float]] = [[] for _ in range(n)]
        refs: list[list[float] | None] = [[] for _ in range(n)]
        done = [self._stop_end(self._generated(r.prefix)) is not None for r in requests]
        ref_id = SamplingConfig(eos_token_id=self.eos_token_id).policy_id
        while True:
            pending, owner = [], []
            for i, r in enumerate(requests):
                off = len(toks[i])
                if done[i] or off >= r.max_new_tokens:
                    continue
                rest = r.max_new_tokens - off
                # an arithmetic-coded request keeps one interval: never split it
                chunk = rest if r.arithmetic_uniform is not None or self.generation_chunk_size is None else min(
                    rest, self.generation_chunk_size)
                pending.append(GenerationRequest(
                    r.prefix + tuple(toks[i]), chunk, self._inner(r.sampling),
                    r.seed if off == 0 else SeedStream(r.seed).derive("stop-chunk", off),
                    f"{r.request_id}:stop-chunk:{off}",
                    None if r.uniforms is None else r.uniforms[off:off + chunk], r.arithmetic_uniform))
                owner.append(i)
            if not pending:
                break
            got = self.backend.sample_batch(pending)
            if len(got) != len(pending):
                raise RuntimeError("wrapped backend returned an invalid sample count")
            for i, req, s in zip(owner, pending, got):
                if (s.prefix != req.prefix or s.policy_id != req.sampling.policy_id
                        or s.model_id != self.backend.model_id or not 0 < len(s.token_ids) <= req.max_new_tokens):
                    raise RuntimeError("wrapped backend violated the generation contract")
                before = self._generated(req.prefix)
                end = self._stop_end(before + s.token_ids)
                keep = len(s.token_ids) if end is None else end - len(before)
                toks[i].extend(s.token_ids[:keep])
                logs[i].extend(s.token_logprobs[:keep])
                if s.reference_policy_id != ref_id:
                    refs[i] = None
                elif refs[i] is not None:
                    refs[i].extend(s.reference_token_logprobs[:keep])
                if end is not None:
                    done[i] = True
                elif len(s.token_ids) != req.max_new_tokens:
                    raise RuntimeError("generation ended without EOS or a configured stop marker")
        out = []
        for i, r in enumerate(requests):
            miss = r.max_new_tokens - len(toks[i])
            ref = refs[i]
            out.append(SequenceSample(
                r.prefix, tuple(toks[i]) + (self.eos_token_id,) * miss, tuple(logs[i]) + (0.0,) * miss,
                r.sampling.policy_id, self.model_id, r.request_id, "stop" if done[i] else "length",
                None if ref is None else tuple(ref) + (0.0,) * miss,
                None if ref is None else SamplingConfig(eos_token_id=r.sampling.eos_token_id).policy_id))
        return out

    def score_batch(self, requests: Sequence[ScoreRequest]) -> list[tuple[float, ...]]:
        pending, meta, res = [], [], []
        for r in requests:
            gen = self._generated(r.prefix)
            terminal = self._stop_end(gen) is not None
            for c in r.continuations:
                k = len(res)
                res.append(None)
                if terminal or not c:
                    res[k] = self._pad_scores(c)
                    continue
                end = self._stop_end(gen + c)
                keep = len(c) if end is None else end - len(gen)
                pending.append(ScoreRequest(r.prefix, (c[:keep],), self._inner(r.sampling)))
                meta.append((k, c[keep:]))
        scored = self.backend.score_batch(pending) if pending else []
        if len(scored) != len(pending):
            raise RuntimeError("wrapped backend returned an invalid score count")
        for (k, tail), req, sc in zip(meta, pending, scored):
            if len(sc) != len(req.continuations[0]):
                raise RuntimeError("wrapped backend returned an invalid score shape")
            res[k] = tuple(sc) + self._pad_scores(tail)
        return res  # type: ignore[return-value]


__all__ = ["StoppedSequenceBackend"]
