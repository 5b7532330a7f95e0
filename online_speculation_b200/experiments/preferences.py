"""Verified preference pairs for VRPO training, built resumably from a diffusion backend.

For every problem of a preregistered subset (``select_problems`` over the problem file,
chosen before any inference) the run draws ``num_generations`` completions from the
diffusion backend in one batch, scores them -- and, when asked, the dataset's reference
solution -- with the configured verifier, and keeps the highest- and the lowest-scored text
as a pair (:func:`~online_speculation_b200.dllm.preferences.select_scored_preference_pair`).
Equal scores carry no preference: the problem is recorded as skipped.

The output is a JSONL file with one record per visited problem, appended and flushed as
soon as the problem is done.  Every record carries the run fingerprint (a digest of the
configuration, the problem subset, the counts and this package's source files that decide
the pairs), so an interrupted run resumes after its last record and a changed run is
refused instead of mixing two record sets.  A manifest beside it holds the inputs, the
status (``running`` / ``complete``) and the generation counters of the backend.
:func:`load_preference_pairs` turns the records into the token triples that
:class:`~online_speculation_b200.training.vrpo.VRPOTrainer` consumes.

    python -m online_speculation_b200.experiments.preferences --config vrpo.toml \\
        --problems data/gsm8k/train.jsonl [--max-pairs N] [--candidate-pool-size M] \\
        [--output pairs.jsonl] [--manifest pairs.manifest.json] [--verifier-config v.toml]

Behaviour of experiments/dllm/prepare_gsm8k_vrpo.py (record fields, the
``vrpo-preference`` seed stream and request ids, fingerprint refusal, the shortfall
error); the execution-profile layer and LLaDA checkpoint hashing of that script are
replaced by this package's config tables and weight loader.
"""

from __future__ import annotations

import argparse
import hashlib
import json
import time
from collections.abc import Callable, Sequence
from dataclasses import asdict, dataclass, is_dataclass
from pathlib import Path
from typing import Any

from ..dllm.preferences import select_scored_preference_pair
from ..shared.evaluation.gsm8k import GSM8KProblem, gsm8k_prompt, load_gsm8k, select_problems
from ..shared.evaluation.numeric import extract_numeric_answer
from ..shared.rng import SeedStream
from ..shared.verifier import (VerifierContext, VerifierInput, VerifierSpec, build_verifier,
                               replace_verifier_from_file, verifier_spec_from_config)

# sources whose behaviour decides the pairs (part of the fingerprint)
SOURCE_FILES = ("experiments/preferences.py", "dllm/preferences.py", "dllm/backend.py", "shared/verifier.py",
                "shared/evaluation/numeric.py", "shared/evaluation/gsm8k.py")
_PACKAGE = Path(__file__).resolve().parents[1]


@dataclass(frozen=True, slots=True)
class PreferenceRun:
    max_pairs: int
    candidate_pool_size: int
    num_generations: int
    seed: int
    include_reference_completion: bool = True

    def __post_init__(self) -> None:
        for name in ("max_pairs", "candidate_pool_size", "num_generations"):
            if getattr(self, name) <= 0:
                raise ValueError(f"{name} must be positive")
        if self.max_pairs > self.candidate_pool_size:
            raise ValueError("max_pairs cannot exceed candidate_pool_size")


def source_digests() -> dict[str, str]:
    return {name: hashlib.sha256((_PACKAGE / name).read_bytes()).hexdigest() for name in SOURCE_FILES}


def fingerprint_of(effective: dict[str, Any]) -> str:
    blob = json.dumps(effective, ensure_ascii=False, sort_keys=True, separators=(",", ":"), default=str)
    return hashlib.sha256(blob.encode("utf-8")).hexdigest()


def load_problem_file(path: str | Path, *, split: str = "train", pinned: bool = True) -> tuple[GSM8KProblem, ...]:
    """Problems of a JSONL file with ``question`` / ``answer`` fields.

    ``pinned`` requires the official GSM8K split (checked by digest); otherwise any file of
    that layout is read, each answer's final number becoming the gold answer.
    """
    if pinned:
        return load_gsm8k(path, split=split, download=False)
    out = []
    for i, line in enumerate(Path(path).read_text(encoding="utf-8").splitlines()):
        if not line.strip():
            continue
        row = json.loads(line)
        gold = extract_numeric_answer(str(row["answer"]))
        if gold is None:
            raise ValueError(f"{path} row {i}: no numeric gold answer")
        out.append(GSM8KProblem(len(out), str(row["question"]), str(row["answer"]), gold))
    if not out:
        raise ValueError(f"{path} holds no problems")
    return tuple(out)


def _counters(snapshot: Any) -> dict | None:
    if is_dataclass(snapshot) and not isinstance(snapshot, type):
        snapshot = asdict(snapshot)
    return snapshot if isinstance(snapshot, dict) else None


def _read_records(path: Path) -> list[dict]:
    if not path.is_file():
        return []
    return [json.loads(line) for line in path.read_text(encoding="utf-8").splitlines() if line.strip()]


def build_preference_pairs(backend: Any, problems: Sequence[GSM8KProblem], run: PreferenceRun,
                           verifier_spec: VerifierSpec, *, encode_prompt: Callable[[str], Sequence[int]],
                           decode: Callable[[Sequence[int]], str], make_request: Callable[..., Any],
                           output: Path, manifest: Path, effective: dict[str, Any],
                           log: Callable[[str], None] = print) -> dict[str, Any]:
    """Visit the preregistered problems until ``run.max_pairs`` pairs exist; returns the manifest.

    ``make_request(prefix, seed, request_id)`` builds one generation request of the
    backend; ``effective`` holds what else defines the run (config, model) for the
    fingerprint.
    """
    subset = select_problems(problems, run.candidate_pool_size, seed=run.seed)
    effective = {**effective, **asdict(run), "problem_indices": [p.index for p in subset],
                 "verifier": verifier_spec.as_dict(), "sources": source_digests()}
    fp = fingerprint_of(effective)
    output.parent.mkdir(parents=True, exist_ok=True)
    manifest.parent.mkdir(parents=True, exist_ok=True)
    if manifest.is_file():
        if json.loads(manifest.read_text(encoding="utf-8")).get("fingerprint") != fp:
            raise ValueError(f"{manifest} belongs to a run with another fingerprint")
    else:
        manifest.write_text(json.dumps({"fingerprint": fp, "status": "running", **effective}, indent=2,
                                       ensure_ascii=False, default=str), encoding="utf-8")
    records = _read_records(output)
    if any(r.get("fingerprint") != fp for r in records):
        raise ValueError(f"{output} holds records of a run with another fingerprint")
    done = {int(r["problem_index"]) for r in records}
    pairs = sum(r.get("status") == "pair" for r in records)
    seeds = SeedStream(run.seed)
    snapshot = getattr(backend, "snapshot", None)
    before = _counters(snapshot()) if callable(snapshot) else None
    started = time.perf_counter()
    with output.open("a", encoding="utf-8", buffering=1) as sink:
        for prob in subset:
            if pairs >= run.max_pairs:
                break
            if prob.index in done:
                continue
            prompt_text = gsm8k_prompt(prob.question)
            prefix = tuple(encode_prompt(prompt_text))
            reqs = [make_request(prefix, seeds.derive("vrpo-preference", prob.index, d),
                                 f"vrpo-preference:{prob.index}:{d}") for d in range(run.num_generations)]
            texts = [decode(s.token_ids) for s in backend.sample_batch(reqs)]
            verifier = build_verifier(verifier_spec, context=VerifierContext(
                prompt=prompt_text, reference=str(prob.gold_answer) if verifier_spec.requires_reference else None,
                metadata={"benchmark": "gsm8k", "problem_index": prob.index}))
            with_ref = run.include_reference_completion
            scored = tuple(texts) + ((prob.gold_solution,) if with_ref else ())
            rewards = list(verifier.score_batch([VerifierInput(prompt_text, t) for t in scored]))
            cand = rewards[:len(texts)]
            pair = select_scored_preference_pair(candidate_texts=texts, candidate_rewards=cand,
                                                 reference_text=prob.gold_solution if with_ref else None,
                                                 reference_reward=rewards[-1] if with_ref else None)
            preds = [extract_numeric_answer(t) for t in texts]
            rec: dict[str, Any] = {
                "fingerprint": fp, "problem_index": prob.index, "question": prob.question,
                "gold_answer": str(prob.gold_answer),
                "reference_completion_verifier_reward": rewards[-1] if with_ref else None,
                "candidates": [{"draw": d, "text": t, "prediction": None if p is None else str(p),
                                "correct": p == prob.gold_answer, "verifier_reward": r}
                               for d, (t, p, r) in enumerate(zip(texts, preds, cand))]}
            if pair is None:
                rec["status"] = "skipped_equal_verifier_rewards"
            else:
                rec.update(status="pair", prompt=prompt_text, chosen=pair.chosen, rejected=pair.rejected,
                           chosen_source=pair.chosen_source, rejected_source=pair.rejected_source)
                pairs += 1
            sink.write(json.dumps(rec, ensure_ascii=False) + "\n")
            records.append(rec)
            done.add(prob.index)
            log(f"preferences rows={len(done)}/{len(subset)} pairs={pairs}/{run.max_pairs}")
    if pairs < run.max_pairs:
        raise RuntimeError(f"the candidate pool gave {pairs} pairs, fewer than the {run.max_pairs} requested")
    after = _counters(snapshot()) if callable(snapshot) else None
    compute = None
    if before is not None and after is not None:
        compute = {k: after[k] - before.get(k, 0) for k in after if isinstance(after[k], (int, float))}
    result = {"fingerprint": fp, "status": "complete", **effective, "records": len(records),
              "preference_pairs": pairs, "elapsed_seconds": time.perf_counter() - started,
              "generation_compute": compute}
    manifest.write_text(json.dumps(result, indent=2, ensure_ascii=False, default=str), encoding="utf-8")
    return result


def load_preference_pairs(path: str | Path, encode: Callable[[str], Sequence[int]], *,
                          fingerprint: str | None = None) -> list[tuple[tuple[int, ...], tuple[int, ...],
                                                                         tuple[int, ...]]]:
    """(prompt, chosen, rejected) token triples of the ``pair`` records, in file order."""
    out = []
    for rec in _read_records(Path(path)):
        if fingerprint is not None and rec.get("fingerprint") != fingerprint:
            raise ValueError(f"{path} holds records of another run")
        if rec.get("status") != "pair":
            continue
        out.append((tuple(encode(rec["prompt"])), tuple(encode(rec["chosen"])), tuple(encode(rec["rejected"]))))
    return out


def _byte_codec(vocab: int) -> tuple[Callable[[str], list[int]], Callable[[Sequence[int]], str]]:
    """UTF-8 bytes as token ids (offset 2, below ``vocab``): a stand-in for weights without a tokenizer."""
    if vocab < 258:
        raise ValueError("the byte codec needs a vocabulary of at least 258 tokens")

    def enc(text: str) -> list[int]:
        return [b + 2 for b in text.encode("utf-8")]

    def dec(ids: Sequence[int]) -> str:
        return bytes(int(t) - 2 for t in ids if 2 <= int(t) < 258).decode("utf-8", errors="replace")

    return enc, dec


def main(argv=None) -> int:
    import tomllib

    from ..dllm.config import DiffusionSamplingConfig
    from ..dllm.loader import load_diffusion_backend
    from ..dllm.types import DiffusionGenerationRequest

    p = argparse.ArgumentParser(prog="python -m online_speculation_b200.experiments.preferences")
    p.add_argument("--config", type=Path, required=True)
    p.add_argument("--problems", type=Path, required=True, help="JSONL with question / answer fields")
    p.add_argument("--unpinned", action="store_true", help="accept a problem file other than the pinned GSM8K split")
    p.add_argument("--output", type=Path)
    p.add_argument("--manifest", type=Path)
    p.add_argument("--max-pairs", type=int)
    p.add_argument("--candidate-pool-size", type=int)
    p.add_argument("--verifier-config", type=Path)
    p.add_argument("--include-reference-completion", action=argparse.BooleanOptionalAction, default=None)
    a = p.parse_args(argv)
    config = tomllib.loads(a.config.read_text(encoding="utf-8"))
    replace_verifier_from_file(config, a.verifier_config)
    spec = verifier_spec_from_config(config)
    tr = dict(config["vrpo_training"])
    run = PreferenceRun(
        max_pairs=int(a.max_pairs or tr["preference_pairs"]),
        candidate_pool_size=int(a.candidate_pool_size or tr["candidate_pool_size"]),
        num_generations=int(tr["num_generations"]), seed=int(tr["seed"]),
        include_reference_completion=(bool(tr.get("include_reference_completion", True))
                                      if a.include_reference_completion is None else a.include_reference_completion))
    output = a.output or Path(str(tr["preference_data"]))
    manifest = a.manifest or Path(str(tr["preference_manifest"]))
    gen = dict(config["generation"])
    length = int(gen.pop("max_new_tokens"))
    sampling = DiffusionSamplingConfig(**gen)
    problems = load_problem_file(a.problems, pinned=not a.unpinned)
    backend = load_diffusion_backend(config, "base")
    tok_dir = Path(str(config["model"]["path"]))
    if (tok_dir / "tokenizer.json").is_file():
        from ..blockspec.tokenizer import LocalTokenizer

        tok = LocalTokenizer(tok_dir)
        encode, decode = tok.encode, tok.decode
    else:
        encode, decode = _byte_codec(int(backend.model.cfg.vocab_size))
    length = max(sampling.block_length, length - length % sampling.block_length)

    def make_request(prefix, seed, rid):
        return DiffusionGenerationRequest(prefix, length, sampling, seed, rid)

    effective = {"config": config, "problems_file": str(a.problems), "generation_length": length}
    try:
        result = build_preference_pairs(backend, problems, run, spec, encode_prompt=encode, decode=decode,
                                        make_request=make_request, output=output, manifest=manifest,
                                        effective=effective)
    finally:
        close = getattr(backend, "close", None)
        if callable(close):
            close()
    print(json.dumps({"output": str(output), "pairs": result["preference_pairs"], "records": result["records"]}))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
