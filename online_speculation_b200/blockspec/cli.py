"""Command line for the dual-view speculation stack.

    python -m online_speculation_b200.blockspec evaluate {benchmark,audit,trace,profile} ...
    python -m online_speculation_b200.blockspec online --model M --prompts P.jsonl ...
    python -m online_speculation_b200.blockspec fit {train,resume,demo} ...
    python -m online_speculation_b200.blockspec lowrank {demo,train,benchmark} ...

Mirrors the reference command groups (online-speculation/src/blockspec/cli.py,
commands/{evaluate,continue_training,fit}.py; the ``lowrank`` group follows
online-speculation/ablation/src/blockspec_ablation/cli.py demo/train/benchmark).  ``--model`` is a
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
from .generation import MaskedAttentionBranch, ProposalSampler, generate, generate_ar
from .measurement import paired_ratio
from .model import DualViewConfig, DualViewDecoder, cache_length
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


def _compare(a: torch.Tensor, b: torch.Tensor) -> dict:
    """Max logit error, total variation of the two softmaxes and argmax agreement of [N, V] rows."""
    a, b = a.float(), b.float()
    tv = 0.5 * (a.softmax(-1) - b.softmax(-1)).abs().sum(-1)
    return {"max_logit_error": float((a - b).abs().max()), "max_tv": float(tv.max()),
            "argmax_equal": bool(torch.equal(a.argmax(-1), b.argmax(-1)))}


@torch.inference_mode()
def cmd_trace(a) -> dict:
    """Explain one greedy decision: the AR and speculative logits for output token ``token_index``
    of request ``request_index``, and a same-cache replay of that row alone against the row inside
    a full masked block (online-speculation/src/blockspec/commands/evaluate.py trace_decision)."""
    model = load_model(a.model, a.device)
    prompts = _prompts(a.prompts, a.request_index + 1, a.device, model.config.vocab_size)
    if a.request_index >= len(prompts) or not 0 <= a.token_index < a.max_new_tokens:
        raise ValueError("trace needs a valid request index and a token index below --max-new-tokens")
    prompt = prompts[a.request_index]
    block = a.block_size or model.config.block_size
    branch, captures, outputs = MaskedAttentionBranch(model), {}, {}
    for mode in ("ar", "speculative"):
        got = {}

        def hook(module, args, kwargs, out, got=got):
            if kwargs.get("view", "ar") == "draft":
                return
            tokens = args[0] if args else kwargs["tokens"]
            first = cache_length(kwargs.get("cache")) + tokens.shape[1] - out.logits.shape[1] + 1
            row = prompt.shape[1] + a.token_index - first
            if 0 <= row < out.logits.shape[1]:
                got.update(logits=out.logits[0, row].float().clone(), cache=kwargs.get("cache"),
                           inputs=tokens.clone())

        h = model.register_forward_hook(hook, with_kwargs=True)
        try:
            res = (generate_ar(branch, prompt, a.max_new_tokens) if mode == "ar" else
                   generate(branch, prompt, a.max_new_tokens, block_size=block))
        finally:
            h.remove()
        outputs[mode], captures[mode] = res.tokens, got
    if not all(captures.values()):
        raise ValueError("the traced token lies outside the generated range")
    ar, sp = captures["ar"]["logits"], captures["speculative"]["logits"]
    ar_id, sp_id = int(ar.argmax()), int(sp.argmax())
    saved = captures["ar"]
    future = prompt.new_full((1, block), model.config.mask_token_id)
    future[:, :1] = saved["inputs"][:, -1:]
    single = model(future[:, :1], cache=saved["cache"]).logits[0, 0]
    whole = model(future, cache=saved["cache"]).logits[0, 0]
    diff = next((i for i, (x, y) in enumerate(zip(outputs["ar"], outputs["speculative"])) if x != y), None)
    return {"request_index": a.request_index, "token_index": a.token_index, "first_difference": diff,
            "prefix_identical": outputs["ar"][:a.token_index] == outputs["speculative"][:a.token_index],
            "actual_path": _compare(ar[None], sp[None]), "ar_choice": ar_id, "speculative_choice": sp_id,
            "ar_gap_between_choices": float(ar[ar_id] - ar[sp_id]),
            "block_gap_between_choices": float(sp[ar_id] - sp[sp_id]),
            "same_cache_single_vs_block": _compare(single[None], whole[None]),
            "same_cache_single_choice": int(single.argmax()), "same_cache_block_choice": int(whole.argmax())}


class _ScopedSampler(ProposalSampler):
    """A sampler whose three decisions run inside named profiler regions."""

    def sample_ar(self, logits, generator):
        with torch.profiler.record_function("blockspec.sample_ar"):
            return super().sample_ar(logits, generator)

    def propose(self, logits, generator):
        with torch.profiler.record_function("blockspec.propose"):
            return super().propose(logits, generator)

    def verify(self, proposal, target_logits, generator):
        with torch.profiler.record_function("blockspec.correct"):
            return super().verify(proposal, target_logits, generator)


def cmd_profile(a) -> dict:
    """Operator attribution for AR and speculative decoding of one request, kept apart from the
    throughput numbers: an uninstrumented run fixes the expected tokens and round counters, the
    profiled run must reproduce them, and no parameter may change
    (online-speculation/src/blockspec/commands/evaluate.py profile_generation)."""
    if a.max_new_tokens > 256:
        raise ValueError("profile takes at most 256 new tokens")
    model = load_model(a.model, a.device)          # outside inference mode: parameters keep versions
    with torch.inference_mode():
        return _profile(a, model)


def _profile(a, model) -> dict:
    prompt = _prompts(a.prompts, 1, a.device, model.config.vocab_size)[0]
    block = a.block_size or model.config.block_size
    sampling = SamplingConfig(temperature=a.temperature)
    activities = [torch.profiler.ProfilerActivity.CPU]
    if prompt.is_cuda:
        activities.append(torch.profiler.ProfilerActivity.CUDA)
    versions = {n: p._version for n, p in model.named_parameters()}
    branch, records = MaskedAttentionBranch(model), []

    def run(method, sampler):
        g = torch.Generator(device=prompt.device).manual_seed(0)
        kw = {"sampler": sampler, "sampling": sampling, "generator": g}
        return (generate_ar(branch, prompt, a.max_new_tokens, **kw) if method == "ar" else
                generate(branch, prompt, a.max_new_tokens, block_size=block, **kw))

    for method in ("ar", "speculative"):
        expected = run(method, ProposalSampler(sampling))
        open_scopes = []

        def enter(module, args, kwargs, stack=open_scopes):
            stage = ("draft" if kwargs.get("view") == "draft" else
                     "prefill" if kwargs.get("cache") is None else "ar_forward")
            scope = torch.profiler.record_function(f"blockspec.{stage}")
            scope.__enter__()
            stack.append(scope)

        def leave(module, args, out, stack=open_scopes):
            stack.pop().__exit__(None, None, None)

        pre = model.register_forward_pre_hook(enter, with_kwargs=True)
        post = model.register_forward_hook(leave, always_call=True)
        try:
            with torch.profiler.profile(activities=activities, acc_events=True) as prof:
                actual = run(method, _ScopedSampler(sampling))
        finally:
            pre.remove()
            post.remove()
        events = [{"name": e.key, "count": e.count, "self_cpu_us": e.self_cpu_time_total,
                   "self_device_us": e.self_device_time_total, "inclusive_device_us": e.device_time_total}
                  for e in prof.key_averages() if e.device_type == torch.autograd.DeviceType.CPU]
        records.append({
            "method": method, "tokens": len(actual.tokens), "decode_forwards": actual.decode_forwards,
            "tokens_unchanged": actual.tokens == expected.tokens,
            "counters_unchanged": (actual.accepted_per_round == expected.accepted_per_round
                                   and actual.decode_forwards == expected.decode_forwards),
            "regions": [e for e in events if e["name"].startswith("blockspec.")],
            "operators": sorted((e for e in events if not e["name"].startswith("blockspec.")),
                                key=lambda e: (e["self_device_us"], e["self_cpu_us"]), reverse=True)[:20]})
    unchanged = versions == {n: p._version for n, p in model.named_parameters()}
    return {"profiles": records, "parameters_unchanged": unchanged,
            "pass": unchanged and all(r["tokens_unchanged"] and r["counters_unchanged"] for r in records)}


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


def _lowrank_model(spec: str, device: str, dtype):
    from . import lowrank as lr

    if spec.startswith("random:"):
        torch.manual_seed(0)
        presets = {"tiny": lr.LowRankConfig(vocab_size=64),
                   "small": lr.LowRankConfig(vocab_size=2048, hidden_size=256, intermediate_size=512,
                                             num_hidden_layers=4, head_dim=64, adapter_rank=16, adapter_alpha=16.0)}
        return lr.LowRankDecoder(presets[spec.split(":", 1)[1]]).to(device).set_base_dtype(dtype).eval()
    if Path(spec).is_dir():
        return lr.from_hf(spec, device=device, dtype=dtype)
    return lr.load(spec, device=device).set_base_dtype(dtype).eval()


def _sequences(path, vocab: int, length: int, device):
    if path is None:
        g = torch.Generator().manual_seed(0)
        base = torch.randint(2, vocab, (4, 8), generator=g)
        return base.repeat(4, length // 8 + 1)[:, :length].to(device)     # repetitive text a draft can learn
    rows = [r["input_ids"][:length] for r in read_records(path) if len(r["input_ids"]) >= length]
    if not rows:
        raise ValueError("no sequence in the data is long enough")
    return torch.tensor(rows, device=device)


def cmd_lowrank(a) -> dict:
    from . import lowrank as lr
    from .lowrank_exec import GraphNoiseBranch

    dtype = {"float32": torch.float32, "bfloat16": torch.bfloat16}[a.dtype]
    out = {"action": a.action}
    model = _lowrank_model(a.model, a.device, dtype)
    if a.action in ("train", "demo"):
        data = _sequences(a.data, model.config.vocab_size, a.sequence_length, a.device)
        model.train_adapters_only()
        opt = torch.optim.AdamW(model.adapter_parameters(), lr=a.lr)
        g = torch.Generator(device=a.device).manual_seed(0)
        t0, losses = time.perf_counter(), []
        for step in range(a.steps):
            kind = a.warmup_loss if step < a.warmup else a.loss
            rows = torch.randint(0, data.shape[0], (min(a.batch, data.shape[0]),), generator=g, device=a.device)
            losses.append(lr.offline_step(model, opt, data[rows], a.block_size, kind=kind, generator=g)["loss"])
        out.update(steps=a.steps, first_loss=losses[0] if losses else None, final_loss=losses[-1] if losses else None,
                   train_seconds=time.perf_counter() - t0)
        if a.save:
            lr.save(model, a.save)
        if a.save_peft:
            lr.save_peft(model, a.save_peft)
        if a.action == "train":
            return out
        model = model.eval().requires_grad_(False)
    sampling = SamplingConfig(temperature=a.temperature)
    graph = a.execution == "cuda_graph"
    branch = (GraphNoiseBranch(model, block_size=a.block_size, capacity=a.capacity) if graph
              else lr.NoiseBranch(model, block_size=a.block_size))
    if graph:
        branch.prepare()
    prompts = _prompts(a.prompts, a.limit, a.device, model.config.vocab_size)
    runs = {"ar": [], "static": [], "online": []}
    learner = lr.LowRankLearner(model, learning_rate=a.online_lr, interval=a.interval) if a.online else None
    for i, prompt in enumerate(prompts):
        def gen():
            return torch.Generator(device=a.device).manual_seed(i)

        runs["ar"].append(generate_ar(branch, prompt, a.max_new_tokens, sampling=sampling, generator=gen()))
        runs["static"].append(generate(branch, prompt, a.max_new_tokens, sampling=sampling, generator=gen()))
        if learner is not None:
            runs["online"].append(generate(branch, prompt, a.max_new_tokens, sampling=sampling, generator=gen(),
                                           feedback=lr.LowRankFeedback(learner)))
    for name, rs in runs.items():
        if rs:
            secs = sum(r.seconds for r in rs)
            rounds = sum(len(r.accepted_per_round) for r in rs)
            out[name] = {"tps": sum(len(r.tokens) for r in rs) / secs if secs else 0.0,
                         "decode_forwards": sum(r.decode_forwards for r in rs),
                         "mean_accepted": sum(sum(r.accepted_per_round) for r in rs) / rounds if rounds else None,
                         "updates": sum(r.updates for r in rs)}
    out.update(execution=a.execution, block_size=a.block_size, requests=len(prompts),
               setup_seconds=getattr(branch, "setup_seconds", 0.0))
    return out


def main(argv=None) -> int:
    p = argparse.ArgumentParser(prog="python -m online_speculation_b200.blockspec")
    sub = p.add_subparsers(dest="group", required=True)
    ev = sub.add_parser("evaluate")
    ev.add_argument("mode", choices=("benchmark", "audit", "trace", "profile"))
    on = sub.add_parser("online")
    fi = sub.add_parser("fit")
    fi.add_argument("action", choices=("train", "resume", "demo"))
    lo = sub.add_parser("lowrank")
    lo.add_argument("action", choices=("demo", "train", "benchmark"))
    for q in (ev, on, fi, lo):
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
    ev.add_argument("--request-index", type=int, default=0)
    ev.add_argument("--token-index", type=int, default=0)
    ev.add_argument("--block-size", type=int, default=None)
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
    lo.add_argument("--dtype", choices=("float32", "bfloat16"), default="float32")
    lo.add_argument("--data", default=None)
    lo.add_argument("--steps", type=int, default=30)
    lo.add_argument("--warmup", type=int, default=0)
    lo.add_argument("--batch", type=int, default=8)
    lo.add_argument("--sequence-length", type=int, default=32)
    lo.add_argument("--block-size", type=int, default=4)
    lo.add_argument("--lr", type=float, default=1e-2)
    lo.add_argument("--loss", choices=("l1", "tv", "forward_kl", "reverse_kl", "reverse_kl_l1"), default="l1")
    lo.add_argument("--warmup-loss", choices=("forward_kl", "reverse_kl", "reverse_kl_l1"), default="reverse_kl_l1")
    lo.add_argument("--save", default=None)
    lo.add_argument("--save-peft", default=None)
    lo.add_argument("--execution", choices=("eager", "cuda_graph"), default="eager")
    lo.add_argument("--capacity", type=int, default=4096)
    lo.add_argument("--online", action="store_true")
    lo.add_argument("--online-lr", type=float, default=1e-3)
    lo.add_argument("--interval", type=int, default=2)
    a = p.parse_args(argv)
    if a.group == "evaluate":
        out = {"benchmark": cmd_benchmark, "audit": cmd_audit, "trace": cmd_trace,
               "profile": cmd_profile}[a.mode](a)
    elif a.group == "online":
        out = cmd_online(a)
    elif a.group == "lowrank":
        out = cmd_lowrank(a)
    else:
        out = cmd_fit(a)
    if a.report:
        write_report(a.report, out)
    print(json.dumps(out))
    return 1 if a.group == "evaluate" and a.mode == "profile" and not out["pass"] else 0


if __name__ == "__main__":
    sys.exit(main())
