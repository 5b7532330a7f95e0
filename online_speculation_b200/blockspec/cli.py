"""Command line for the dual-view speculation stack.

    python -m online_speculation_b200.blockspec evaluate {benchmark,audit} ...
    python -m online_speculation_b200.blockspec online --model M --prompts P.jsonl ...
    python -m online_speculation_b200.blockspec fit {train,resume,demo} ...

Mirrors the reference command groups (online-speculation/src/blockspec/cli.py,
commands/{evaluate,continue_training,fit}.py).  ``--model`` is a
``blockspec-dual-view-v1`` checkpoint, a published dual-view directory, or
``random:<preset>`` for random weights (``tiny``, ``qwen3-1.7b``).  With
``--engine kernel`` (CUDA, head_dim 128) decoding runs on the sm_100a kernels.
"""

from __future__ import annotations

import argparse
import json
import sys
import time
from pathlib import Path

import torch

from .data import read_records
from .fitting import FitConfig, TokenDataset, Trainer
from .generation import MaskedAttentionBranch, generate, generate_ar
from .measurement import paired_ratio
from .model import DualViewConfig, DualViewDecoder
from .online import OnlineFeedback, SuffixConfig, SuffixLearner
from .reporting import write_report
from .sampling import SamplingConfig
from .training import sample_anchors
from .weights import load_checkpoint, load_public

PRESETS = {
    "tiny": DualViewConfig(vocab_size=64, hidden_size=32, intermediate_size=64, num_hidden_layers=2,
                           num_attention_heads=4, num_key_value_heads=2, head_dim=8, block_size=4, mask_token_id=1),
    "small128": DualViewConfig(vocab_size=2048, hidden_size=512, intermediate_size=1024, num_hidden_layers=4,
                               num_attention_heads=4, num_key_value_heads=2, head_dim=128, block_size=4,
                               mask_token_id=1),
    "qwen3-1.7b": DualViewConfig(vocab_size=151936, hidden_size=2048, intermediate_size=6144, num_hidden_layers=28,
                                 num_attention_heads=16, num_key_value_heads=8, head_dim=128, block_size=32,
                                 mask_token_id=151669, tie_word_embeddings=True),
}


def load_model(spec: str, device: str, dtype=torch.float32) -> DualViewDecoder:
    if spec.startswith("random:"):
        torch.manual_seed(0)
        m = DualViewDecoder(PRESETS[spec.split(":", 1)[1]])
        return m.to(device=device, dtype=dtype).eval().requires_grad_(False)
    p = Path(spec)
    if p.is_dir():
        return load_public(p, device=device, dtype=dtype)
    model, _ = load_checkpoint(p, device=device)
    return model.to(dtype=dtype).eval().requires_grad_(False)


def _branch(model, engine: str):
    if engine == "kernel":
        from .kernel_branch import KernelBranch

        return KernelBranch(model, device=model.embedding.weight.device)
    return MaskedAttentionBranch(model)


def _prompts(path, limit, device, vocab):
    if path is None:
        g = torch.Generator().manual_seed(0)
        return [torch.randint(2, vocab, (1, 16), generator=g).to(device) for _ in range(limit)]
    recs = read_records(path)[:limit]
    return [torch.tensor([r["input_ids"]], device=device) for r in recs]


def cmd_benchmark(a) -> dict:
    model = load_model(a.model, a.device)
    branch = _branch(model, a.engine)
    sampling = SamplingConfig(temperature=a.temperature)
    ar, sp = [], []
    for i, prompt in enumerate(_prompts(a.prompts, a.limit, a.device, model.config.vocab_size)):
        g1 = torch.Generator(device=a.device).manual_seed(i)
        g2 = torch.Generator(device=a.device).manual_seed(i)
        ar.append(generate_ar(branch, prompt, a.max_new_tokens, sampling=sampling, generator=g1))
        sp.append(generate(branch, prompt, a.max_new_tokens, sampling=sampling, generator=g2))
    ratio = paired_ratio([len(x.tokens) for x in sp], [x.seconds for x in sp], [len(x.tokens) for x in ar],
                         [x.seconds for x in ar])
    tpf = sum(len(x.tokens) - x.prefill_output_tokens for x in sp) / max(1, sum(x.decode_forwards for x in sp))
    return {"ar_tps": sum(len(x.tokens) for x in ar) / sum(x.seconds for x in ar),
            "spec_tps": sum(len(x.tokens) for x in sp) / sum(x.seconds for x in sp), "speedup": ratio,
            "decode_tpf": tpf, "requests": len(sp), "engine": a.engine, "temperature": a.temperature}


def cmd_audit(a) -> dict:
    from .audit import audit

    original = load_model(a.model, a.device)
    learned = load_model(a.learned or a.model, a.device)
    if a.online_state:
        learner = SuffixLearner(learned, SuffixConfig(**torch.load(a.online_state, weights_only=True)["config"]))
        learner.load_state_dict(torch.load(a.online_state, weights_only=True))
    recs = _prompts(a.prompts, a.limit, a.device, original.config.vocab_size)
    L = min(x.shape[1] for x in recs)
    seqs = torch.cat([x[:, :L] for x in recs])
    anchors = sample_anchors(seqs, original.config.block_size, 2, generator=torch.Generator(device=a.device).manual_seed(0))
    return audit(original, learned, seqs, anchors)


def cmd_online(a) -> dict:
    model = load_model(a.model, a.device)
    learner = SuffixLearner(model, SuffixConfig(last_layers=a.last_layers, stride=a.stride,
                                                replay_blocks=a.replay_blocks, learning_rate=a.lr, loss=a.loss))
    branch = MaskedAttentionBranch(model)
    sampling = SamplingConfig(temperature=a.temperature)
    runs = []
    for i, prompt in enumerate(_prompts(a.prompts, a.limit, a.device, model.config.vocab_size)):
        g = torch.Generator(device=a.device).manual_seed(i)
        runs.append(generate(branch, prompt, a.max_new_tokens, sampling=sampling, generator=g,
                             feedback=OnlineFeedback(learner=learner)))
    if a.save_state:
        torch.save(learner.state_dict(), a.save_state)
    tokens = sum(len(r.tokens) for r in runs)
    secs = sum(r.seconds for r in runs)
    return {"tps": tokens / secs if secs else 0.0, "requests": len(runs), "updates": learner.updates,
            "update_seconds": learner.update_seconds, "last_loss": learner.last_loss,
            "mean_accepted": sum(sum(r.accepted_per_round) for r in runs) / max(1, sum(len(r.accepted_per_round)
                                                                                    for r in runs))}


def cmd_fit(a) -> dict:
    if a.action == "demo":
        import json as _json
        import tempfile

        tmp = Path(tempfile.mkdtemp())
        g = torch.Generator().manual_seed(0)
        (tmp / "d.jsonl").write_text("".join(_json.dumps({"input_ids": torch.randint(2, 64, (40,), generator=g)
                                                         .tolist()}) + "\n" for _ in range(16)))
        a.data, a.model = str(tmp / "d.jsonl"), "random:tiny"
        a.action = "train"
        a.steps = a.steps or 5
    if a.action == "resume":
        trainer = Trainer.resume(a.checkpoint, a.data, device=a.device)
    else:
        model = load_model(a.model, a.device)
        cfg = FitConfig(steps=a.steps or 100, sequence_length=a.sequence_length, anchors_per_sequence=a.anchors,
                        learning_rate=a.lr, warmup_steps=min(a.warmup, (a.steps or 100) - 1))
        trainer = Trainer(model.float().requires_grad_(False), TokenDataset(a.data, model.config.vocab_size,
                                                                            cfg.sequence_length), cfg)
    t0 = time.perf_counter()
    records = trainer.run(until=a.stop_after)
    if a.checkpoint and a.action != "resume" or (a.action == "resume" and a.save):
        out = a.save or a.checkpoint
        if Path(out).exists():
            Path(out).unlink()
        trainer.save(out)
    return {"steps": trainer.step, "final_loss": records[-1]["loss"] if records else None,
            "seconds": time.perf_counter() - t0}


def main(argv=None) -> int:
    p = argparse.ArgumentParser(prog="python -m online_speculation_b200.blockspec")
    sub = p.add_subparsers(dest="group", required=True)
    ev = sub.add_parser("evaluate")
    ev.add_argument("mode", choices=("benchmark", "audit"))
    on = sub.add_parser("online")
    fi = sub.add_parser("fit")
    fi.add_argument("action", choices=("train", "resume", "demo"))
    for q in (ev, on, fi):
        q.add_argument("--model", default="random:tiny")
        q.add_argument("--device", default="cuda" if torch.cuda.is_available() else "cpu")
        q.add_argument("--prompts", default=None)
        q.add_argument("--limit", type=int, default=4)
        q.add_argument("--max-new-tokens", type=int, default=64)
        q.add_argument("--temperature", type=float, default=0.0)
        q.add_argument("--report", default=None)
    ev.add_argument("--engine", choices=("module", "kernel"), default="module")
    ev.add_argument("--learned", default=None)
    ev.add_argument("--online-state", default=None)
    on.add_argument("--last-layers", type=int, default=1)
    on.add_argument("--stride", type=int, default=16)
    on.add_argument("--replay-blocks", type=int, default=1)
    on.add_argument("--lr", type=float, default=1e-5)
    on.add_argument("--loss", choices=("forward_kl", "tv"), default="tv")
    on.add_argument("--save-state", default=None)
    fi.add_argument("--data", default=None)
    fi.add_argument("--checkpoint", default=None)
    fi.add_argument("--save", default=None)
    fi.add_argument("--steps", type=int, default=0)
    fi.add_argument("--stop-after", type=int, default=None)
    fi.add_argument("--sequence-length", type=int, default=32)
    fi.add_argument("--anchors", type=int, default=4)
    fi.add_argument("--lr", type=float, default=1e-4)
    fi.add_argument("--warmup", type=int, default=10)
    a = p.parse_args(argv)
    if a.group == "evaluate":
        out = cmd_benchmark(a) if a.mode == "benchmark" else cmd_audit(a)
    elif a.group == "online":
        out = cmd_online(a)
    else:
        out = cmd_fit(a)
    if a.report:
        write_report(a.report, out)
    print(json.dumps(out))
    return 0


if __name__ == "__main__":
    sys.exit(main())
