"""Headline benchmark: suffix-MH rollouts on a Qwen2.5-7B-shaped decoder with
block-bidirectional speculative drafting and an online draft learner.

Workload (random-init bf16 weights, synthetic uniform-random prompt ids):
  64 chains over one shared 512-token uniform-random prompt (the shape of the
  reference's batched MH API, which takes one prompt for all chains; both arms
  run it) and 512 generated tokens each, power target p^4 (proposal temperature
  1/4); every MH update regenerates the suffix after a uniformly drawn cut while
  reusing the prefix KV.  Drafting uses a
  1-layer block-4 draft head; the online learner updates every 64 verified blocks.
  The engine drafts in the rounds where the measured acceptance makes speculation
  faster than plain decoding, and at least every 8th round so the learner keeps
  training (``--spec-policy always`` drafts every round; ``--no-draft`` runs plain
  decoding only).  Every emitted token follows the proposal policy exactly either way.
  Tensor parallel over N GPUs of one node (one process per GPU, NCCL).

A "step" is one MH update of every chain (64 proposals).  W warm-up steps run
first (after the initial extension of every chain), then exactly K steps are
timed with CUDA events on every rank between a barrier and a synchronize; the
reported time is the maximum over ranks.  ``value`` = generated tokens per second
for the whole job.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

With --impl reference the same workload runs on the unmodified reference
package installed under baseline/_ref (its TransformersBackend and
run_mh_chains_batched); under N ranks each rank runs 64/N chains on its own GPU.
"""

from __future__ import annotations

import argparse
import dataclasses
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

BASELINE_TOKENS_PER_SECOND = None  # BASELINE.md publishes no number for this metric and config
METRIC = "generated tok/s per box, Qwen2.5-7B-shape TP=1..8 (max over ranks); spec accept len"


def parse():
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=4)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", choices=("ours", "reference"), default="ours")
    p.add_argument("--workload", choices=("mh-spec", "grpo", "dllm", "is"), default="mh-spec",
                   help="mh-spec: suffix-MH rollouts with speculative drafting (headline); "
                        "grpo: GRPO training on the Qwen2.5-1.5B shape, data parallel; "
                        "dllm: LLaDA-MoE-shaped block diffusion, expert parallel")
    p.add_argument("--requests-per-rank", type=int, default=4)
    p.add_argument("--ep-impl", choices=("fused", "nccl"), default="fused")
    p.add_argument("--group-size", type=int, default=8)
    p.add_argument("--prompts-per-rank", type=int, default=1)
    p.add_argument("--model", default="qwen2.5-7b")
    p.add_argument("--chains", type=int, default=64)
    p.add_argument("--prompt-len", type=int, default=512)
    p.add_argument("--gen-len", type=int, default=512)
    p.add_argument("--alpha", type=float, default=4.0)
    p.add_argument("--block", type=int, default=4)
    p.add_argument("--stride", type=int, default=64)
    p.add_argument("--no-learner", action="store_true")
    p.add_argument("--no-draft", action="store_true",
                   help="plain one-token decoding without the draft head (shows what speculation adds)")
    p.add_argument("--spec-policy", choices=("adaptive", "always", "never"), default="adaptive",
                   help="draft every round (always) or where the measured acceptance makes it pay (adaptive)")
    p.add_argument("--probe-every", type=int, default=8,
                   help="adaptive policy: at least one speculative round per this many rounds")
    p.add_argument("--plain-steps", type=int, default=4, help="decode steps chained in one plain round")
    p.add_argument("--json-out", help="also write the result line to this file (rank 0)")
    p.add_argument("--distinct-prompts", action="store_true",
                   help="a different uniform-random prompt per chain (no shared prefix pages)")
    p.add_argument("--no-graphs", action="store_true")
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--kv-gb", type=float, default=24.0)
    # conditional importance sampling (Qwen2.5-1.5B shape): one decision block per prompt per step
    p.add_argument("--is-prompts", type=int, default=64, help="prompts per step, whole job")
    p.add_argument("--is-ref-prompts", type=int, default=8,
                   help="prompts per step of the reference arm (it decodes prompt groups one batch at a time)")
    p.add_argument("--is-prompt-len", type=int, default=256)
    p.add_argument("--is-candidates", type=int, default=16)
    p.add_argument("--is-block", type=int, default=32)
    p.add_argument("--is-rollouts", type=int, default=8)
    p.add_argument("--is-rollout-len", type=int, default=256)
    p.add_argument("--is-workers", type=int, default=16,
                   help="prompt threads of the repo arm (more threads than needed to fill 256-wide "
                        "batches only add interpreter contention)")
    return p.parse_args()


class ClockSampler:
    """Samples SM clocks and throttle reasons with nvidia-smi during the timed region."""

    def __init__(self, index: int):
        self.index = index
        self.samples: list[tuple[float, float, str]] = []
        self._proc = None
        self._thread = None

    def __enter__(self):
        cmd = ["nvidia-smi", "-i", str(self.index),
               "--query-gpu=clocks.sm,clocks.max.sm,clocks_event_reasons.active,"
               "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
               "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap",
               "--format=csv,noheader,nounits", "-lms", "200"]
        try:
            self._proc = subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self._proc = None
            return self

        def reader():
            for line in self._proc.stdout:
                self.samples.append(tuple(x.strip() for x in line.split(",")))

        self._thread = threading.Thread(target=reader, daemon=True)
        self._thread.start()
        return self

    def __exit__(self, *exc):
        if self._proc is not None:
            self._proc.terminate()
            try:
                self._proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self._proc.kill()
        if self._thread is not None:
            self._thread.join(timeout=5)

    def summary(self) -> dict:
        sm, mx, reasons = [], None, set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for s in self.samples:
            try:
                sm.append(float(s[0]))
                mx = float(s[1])
            except (ValueError, IndexError):
                continue
            for name, flag in zip(names, s[3:7]):
                if flag.strip().lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def dist_setup(n: int):
    import torch

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", str(n)))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != n:
        raise SystemExit(f"--gpus {n} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    group = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                device_id=torch.device("cuda", local))
        group = dist.group.WORLD
    return rank, world, local, group


def max_over_ranks(value: float, world: int) -> float:
    import torch

    if world == 1:
        return value
    import torch.distributed as dist

    t = torch.tensor([value], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def sum_over_ranks(value: float, world: int) -> float:
    import torch

    if world == 1:
        return value
    import torch.distributed as dist

    t = torch.tensor([value], dtype=torch.float64, device="cuda")
    dist.all_reduce(t)
    return float(t.item())


def barrier(world: int):
    import torch

    if world > 1:
        import torch.distributed as dist

        dist.barrier()
    torch.cuda.synchronize()


def run_ours(args, rank, world, local, group) -> dict:
    import numpy as np
    import torch

    from online_speculation_b200.api import build_mh_engine
    from online_speculation_b200.ops import _ext

    engine = build_mh_engine(args.model, tp_group=group, seed=args.seed, alpha=args.alpha, length=args.gen_len,
                             block_size=args.block, learner_stride=None if args.no_learner else args.stride,
                             use_graphs=not args.no_graphs, kv_bytes=int(args.kv_gb * 2**30),
                             max_seq_tokens=args.prompt_len + args.gen_len + 2 * args.block,
                             draft=not args.no_draft, spec_policy=args.spec_policy, probe_every=args.probe_every,
                             plain_steps=args.plain_steps)
    rng = np.random.default_rng(args.seed + 17)
    vocab = engine.runner.cfg.vocab_size
    # one uniform-random prompt shared by the chains (the reference API's shape)
    rows = args.chains if args.distinct_prompts else 1
    prompt_host = torch.from_numpy(rng.integers(0, vocab - 2, size=(rows, args.prompt_len)).astype(np.int32))
    prompt_host = prompt_host.pin_memory()
    prompt_dev = prompt_host.to("cuda", non_blocking=True)
    prompts = prompt_dev.cpu().tolist()
    engine.add_chains(prompts if args.distinct_prompts else prompts * args.chains)
    engine.run_until_idle()                       # initial extension of every chain to 512 tokens
    # Chains run asynchronously: a chain starts its next update as soon as its
    # proposal is decided.  A step is `chains` completed updates (in any order).
    engine.set_quota(args.warmup + args.steps + 64)
    per_step = args.chains
    while engine.stats["mh_updates"] < args.warmup * per_step:
        engine.round()
    barrier(world)
    stats0 = dict(engine.stats)
    launches0 = _ext.launches()
    learner0 = engine.learner.updates if engine.learner else 0
    sampler = ClockSampler(local)
    with sampler:
        barrier(world)
        wall0 = time.perf_counter()
        start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        state_host = torch.empty(args.chains, args.gen_len, dtype=torch.int32).pin_memory()
        goal = stats0["mh_updates"]
        for _ in range(args.steps):
            goal += per_step
            while engine.stats["mh_updates"] < goal:
                engine.round()
            # end-to-end: read back every chain's current state (tokens) each step
            state_dev = torch.tensor([c.tokens for c in engine.chains], dtype=torch.int32, device="cuda")
            state_host.copy_(state_dev, non_blocking=True)
        stop.record()
        torch.cuda.synchronize()
        wall = time.perf_counter() - wall0
        barrier(world)
    ms = start.elapsed_time(stop)
    ms = max_over_ranks(ms, world)
    wall = max_over_ranks(wall, world)
    st = engine.stats
    generated = st["generated"] - stats0["generated"]   # identical on every rank (TP)
    blocks = st["blocks"] - stats0["blocks"]
    emitted = st["emitted"] - stats0["emitted"]
    launches = (_ext.launches() - launches0) + (st["graph_kernel_launches"] - stats0["graph_kernel_launches"])
    h2d = (st["h2d_bytes"] - stats0["h2d_bytes"]) / args.steps + args.chains * args.gen_len * 4 * 0
    d2h = (st["d2h_bytes"] - stats0["d2h_bytes"]) / args.steps + args.chains * args.gen_len * 4
    value = generated / (ms / 1e3)
    accept_len = emitted / blocks if blocks else None       # over the speculative rounds
    out = {
        "metric": METRIC,
        "value": value,
        "unit": "tok/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms / args.steps,
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None if BASELINE_TOKENS_PER_SECOND is None else value / BASELINE_TOKENS_PER_SECOND,
        "dtype": "bf16",
        "data": "synthetic (uniform-random prompt ids, random-init weights)",
        "config": {"model": f"{args.model} (random init)", "global_batch": args.chains, "seq_len": args.prompt_len + args.gen_len,
                   "prompt": ("a distinct uniform-random prompt per chain" if args.distinct_prompts
                              else "one uniform-random prompt shared by all chains"),
                   "prompt_len": args.prompt_len, "gen_len": args.gen_len, "parallelism": f"tp{world}",
                   "mh_alpha": args.alpha,
                   "draft": "none (plain decoding)" if args.no_draft else f"1-layer block-{args.block} draft head",
                   "learner_stride_blocks": None if (args.no_learner or args.no_draft) else args.stride,
                   "spec_policy": "none" if args.no_draft else args.spec_policy,
                   "probe_every": args.probe_every if args.spec_policy == "adaptive" else None,
                   "plain_steps": args.plain_steps,
                   "l2": "weights (15 GB) streamed every round exceed the 126 MB L2",
                   "step": "64 completed MH updates; chains run asynchronously (no lock-step barrier)"},
        "spec_accept_len": accept_len,
        "generated_tokens": generated,
        "mh_acceptance_rate": (st["mh_accepted"] - stats0["mh_accepted"]) / max(1, st["mh_updates"] - stats0["mh_updates"]),
        "learner_updates": (engine.learner.updates - learner0) if engine.learner else 0,
        "spec_rounds": st["spec_rounds"] - stats0["spec_rounds"],
        "plain_rounds": st["plain_rounds"] - stats0["plain_rounds"],
        "clocks": sampler.summary(),
        "e2e": {"value": generated / wall, "unit": "tok/s", "h2d_bytes_per_step": int(h2d),
                "d2h_bytes_per_step": int(d2h)},
        "gpu_launches": int(launches),
    }
    engine.close()
    del engine
    return out


DLLM_METRIC = "block-diffusion generated tok/s (LLaDA-MoE-7B-A1B shape, expert parallel, whole job)"


def run_dllm(args, rank, world, local, group) -> dict:
    """256 generated tokens after a 256-token prompt, 32-token blocks, 32 reverse steps per block.

    Every rank serves its own requests (data parallel outside the MoE layers);
    the 64 experts are split over the ranks and tokens cross NVLink in every
    MoE layer.  One step = one complete generation of every rank's requests.
    """
    import numpy as np
    import torch

    from online_speculation_b200.dllm.backend import DiffusionEngineBackend
    from online_speculation_b200.dllm.config import DiffusionSamplingConfig
    from online_speculation_b200.dllm.types import DiffusionGenerationRequest
    from online_speculation_b200.models.moe import PRESETS, MoEDiffusionModel, build_weights, random_state_dict
    from online_speculation_b200.ops import _ext

    cfg = PRESETS["llada-moe-7b-a1b"]
    E = cfg.num_experts
    lo, hi = (rank * E // world, (rank + 1) * E // world)
    sd = random_state_dict(cfg, seed=args.seed, device="cuda")
    weights = build_weights(cfg, sd, device="cuda", expert_range=(lo, hi))
    del sd
    torch.cuda.empty_cache()
    prompt_len, gen_len, B = 256, 256, args.requests_per_rank
    ep = None
    if world > 1:
        from online_speculation_b200.parallel.ep import ExpertParallelMoE, NcclExpertParallelMoE

        cls = ExpertParallelMoE if args.ep_impl == "fused" else NcclExpertParallelMoE
        ep = cls(group, experts=E, top_k=cfg.num_experts_per_tok, hidden=cfg.hidden_size,
                 ffn=cfg.moe_intermediate_size, max_tokens=B * (prompt_len + gen_len), device="cuda")
    model = MoEDiffusionModel(weights, ep=ep)
    backend = DiffusionEngineBackend(model, model_id="llada-moe-7b-a1b (random init)")
    sampling = DiffusionSamplingConfig(block_length=32, steps_per_block=32, temperature=1.0)
    rng = np.random.default_rng(args.seed + 101 * rank)
    prompts_host = torch.from_numpy(rng.integers(0, cfg.mask_token_id - 1, size=(B, prompt_len)).astype(np.int32))
    prompts_host = prompts_host.pin_memory()

    def step(i):
        # end to end: the prompts come from pinned host memory every step; tokens come back to the host
        dev = prompts_host.to("cuda", non_blocking=True)
        reqs = [DiffusionGenerationRequest(tuple(dev[b].tolist()), gen_len, sampling, seed=1000 * i + b + 7 * rank,
                                           request_id=f"r{rank}:{i}:{b}") for b in range(B)]
        out = backend.sample_batch(reqs)
        return sum(len(o.token_ids) for o in out)

    for i in range(args.warmup):
        step(i)
    barrier(world)
    launches0 = _ext.launches()
    sampler = ClockSampler(local)
    with sampler:
        barrier(world)
        wall0 = time.perf_counter()
        start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        generated = 0
        for i in range(args.steps):
            generated += step(args.warmup + i)
        stop.record()
        torch.cuda.synchronize()
        wall = time.perf_counter() - wall0
        barrier(world)
    ms = max_over_ranks(start.elapsed_time(stop), world)
    wall = max_over_ranks(wall, world)
    total = sum_over_ranks(generated, world)
    value = total / (ms / 1e3)
    return {
        "metric": DLLM_METRIC, "value": value, "unit": "tok/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic (uniform-random prompt ids, random-init weights)",
        "config": {"model": "llada-moe-7b-a1b (random init)", "global_batch": B * world,
                   "seq_len": prompt_len + gen_len, "parallelism": f"ep{world}" if world > 1 else "single",
                   "ep_exchange": args.ep_impl if world > 1 else None, "block_length": 32, "steps_per_block": 32,
                   "l2": "expert weights (13 GB) streamed every reverse step exceed the 126 MB L2"},
        "clocks": sampler.summary(),
        "e2e": {"value": total / wall, "unit": "tok/s", "h2d_bytes_per_step": int(B * prompt_len * 4),
                "d2h_bytes_per_step": int(B * gen_len * 8)},
        "gpu_launches": int(_ext.launches() - launches0),
    }


GRPO_METRIC = "GRPO tokens/s (prompt + completion tokens trained per second, whole job)"


def run_grpo(args, rank, world, local, group) -> dict:
    """GRPO steps: rollouts with the current policy, reference log-probs, loss, backward, sharded AdamW."""
    import torch

    from online_speculation_b200.models.decoder import PRESETS
    from online_speculation_b200.ops import _ext
    from online_speculation_b200.training.grpo import GRPOConfig, GRPOTrainer

    model = args.model if args.model != "qwen2.5-7b" else "qwen2.5-1.5b"
    prompt_len = args.prompt_len if args.prompt_len != 512 else 256
    conf = GRPOConfig(group_size=args.group_size, prompts_per_rank=args.prompts_per_rank, prompt_length=prompt_len,
                      completion_length=args.gen_len, seed=args.seed)
    tr = GRPOTrainer(PRESETS[model], conf, group=group, seed=args.seed, kv_bytes=int(min(args.kv_gb, 8) * 2**30),
                     use_graphs=not args.no_graphs)
    for _ in range(args.warmup):
        tr.step()
    barrier(world)
    launches0 = _ext.launches()
    graph0 = tr.backend.stats.get("graph_kernel_launches", 0)
    sampler = ClockSampler(local)
    tokens = completion = 0
    parts = {"rollout_s": 0.0, "train_s": 0.0}
    with sampler:
        barrier(world)
        wall0 = time.perf_counter()
        start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        for _ in range(args.steps):
            st = tr.step()
            tokens += st["tokens"]
            completion += st["completion_tokens"]
            for k in parts:
                parts[k] += st[k]
        stop.record()
        torch.cuda.synchronize()
        wall = time.perf_counter() - wall0
        barrier(world)
    ms = max_over_ranks(start.elapsed_time(stop), world)
    wall = max_over_ranks(wall, world)
    total = sum_over_ranks(float(tokens), world)
    launches = _ext.launches() - launches0 + tr.backend.stats.get("graph_kernel_launches", 0) - graph0
    B = conf.group_size * conf.prompts_per_rank
    seq = conf.prompt_length + conf.completion_length
    out = {
        "metric": GRPO_METRIC, "value": total / (ms / 1e3), "unit": "tok/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16 (fp32 master weights and AdamW state)",
        "data": "synthetic (uniform-random prompt ids, Bernoulli(0.5) rewards, random-init weights)",
        "config": {"model": f"{model} (random init)", "global_batch": B * world, "seq_len": seq,
                   "prompt_len": conf.prompt_length, "completion_len": conf.completion_length,
                   "group_size": conf.group_size, "parallelism": f"dp{world}", "lr": conf.learning_rate,
                   "beta": conf.beta, "epsilon": conf.epsilon,
                   "l2": "weights, optimizer state and activations (tens of GB) exceed the 126 MB L2"},
        "completion_tokens": sum_over_ranks(float(completion), world),
        "rollout_fraction": parts["rollout_s"] / max(1e-9, parts["rollout_s"] + parts["train_s"]),
        "trainable_parameters": tr.params.trainable,
        "clocks": sampler.summary(),
        "e2e": {"value": total / wall, "unit": "tok/s", "h2d_bytes_per_step": B * (seq * 8 + conf.completion_length + 4),
                "d2h_bytes_per_step": B * conf.completion_length * 4 + 4},
        "gpu_launches": int(launches),
    }
    tr.close()
    return out


def run_reference(args, rank, world, local, group) -> dict:
    if args.distinct_prompts:
        return {"impl": "reference", "unavailable": "the reference's batched MH API (run_mh_chains_batched) "
                                                    "takes one prompt for all chains"}
    ref = os.path.join(ROOT, "baseline", "_ref")
    if not os.path.isdir(os.path.join(ref, "inference_scaling")):
        return {"impl": "reference", "unavailable": "reference package not installed under baseline/_ref"}
    sys.path.insert(0, ref)
    import numpy as np
    import torch
    from transformers import Qwen2Config, Qwen2ForCausalLM

    from inference_scaling.arllm.algorithms.mh import run_mh_chains_batched
    from inference_scaling.arllm.backends.transformers_backend import TransformersBackend
    from inference_scaling.arllm.config import MHConfig, SamplingConfig
    from inference_scaling.shared.rng import SeedStream

    from online_speculation_b200.models.decoder import PRESETS

    c = PRESETS[args.model]
    hf = Qwen2Config(vocab_size=c.vocab_size, hidden_size=c.hidden_size, intermediate_size=c.intermediate_size,
                     num_hidden_layers=c.num_hidden_layers, num_attention_heads=c.num_attention_heads,
                     num_key_value_heads=c.num_key_value_heads, rope_theta=c.rope_theta, rms_norm_eps=c.rms_norm_eps,
                     tie_word_embeddings=c.tie_word_embeddings, max_position_embeddings=4096,
                     torch_dtype="bfloat16")
    torch.manual_seed(args.seed)
    with torch.device("cuda"):
        model = Qwen2ForCausalLM(hf).to(torch.bfloat16)
    model.eval()

    class Tok:
        pad_token_id = 0
        eos_token_id = None
        bos_token_id = 1

    backend = TransformersBackend(model, Tok(), model_id="qwen2.5-7b-random", device="cuda")
    per_rank = args.chains // world
    rng = np.random.default_rng(args.seed + 17 + rank)
    prompt = tuple(int(x) for x in rng.integers(0, c.vocab_size - 2, size=args.prompt_len))

    class Timed:
        """Records CUDA events around the sample calls of the timed MH updates."""

        def __init__(self, inner):
            self.inner = inner
            self.calls = 0
            self.start = torch.cuda.Event(enable_timing=True)
            self.stop = torch.cuda.Event(enable_timing=True)
            self.timed_tokens = 0

        @property
        def model_id(self):
            return self.inner.model_id

        def sample_batch(self, requests):
            # call 0 = extension, 1..W = warm-up updates, W+1..W+K = timed updates
            timed = 1 + args.warmup <= self.calls < 1 + args.warmup + args.steps
            if self.calls == 1 + args.warmup:
                barrier(world)
                self.wall0 = time.perf_counter()
                self.start.record()
            out = self.inner.sample_batch(requests)
            if timed:
                self.timed_tokens += sum(len(s.token_ids) for s in out)
            self.calls += 1
            if self.calls == 1 + args.warmup + args.steps:
                self.stop.record()
                torch.cuda.synchronize()
                self.wall = time.perf_counter() - self.wall0
            return out

        def score_batch(self, requests):
            return self.inner.score_batch(requests)

    timed = Timed(backend)
    cfg = MHConfig(alpha=args.alpha, total_length=args.gen_len, block_size=args.gen_len, iterations=args.warmup + args.steps)
    sampler = ClockSampler(local)
    with sampler:
        run_mh_chains_batched(timed, prompt, cfg, SamplingConfig(temperature=1.0 / args.alpha),
                              [SeedStream(args.seed)] * per_rank, chain_ids=list(range(rank * per_rank, (rank + 1) * per_rank)))
    ms = max_over_ranks(timed.start.elapsed_time(timed.stop), world)
    tokens = sum_over_ranks(timed.timed_tokens, world)
    wall = max_over_ranks(timed.wall, world)
    return {
        "impl": "reference", "metric": METRIC, "value": tokens / (ms / 1e3), "unit": "tok/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (uniform-random prompt ids, random-init weights)",
        "config": {"model": f"{args.model} (random init, HF Qwen2ForCausalLM)", "global_batch": args.chains,
                   "seq_len": args.prompt_len + args.gen_len, "parallelism": f"dp{world}",
                   "path": "inference_scaling TransformersBackend + run_mh_chains_batched (unmodified)"},
        "clocks": sampler.summary(),
        "e2e": {"value": tokens / wall, "unit": "tok/s", "h2d_bytes_per_step": None, "d2h_bytes_per_step": None},
    }


IS_METRIC = "conditional-IS generated tok/s (Qwen2.5-1.5B shape, whole job)"


def _is_workload(args, rank, world, prompts_total):
    """Per-rank prompts (distinct uniform-random ids) and the shared IS settings."""
    import numpy as np

    from online_speculation_b200.models.decoder import PRESETS

    vocab = PRESETS["qwen2.5-1.5b"].vocab_size
    per_rank = max(1, prompts_total // world)
    rng = np.random.default_rng(args.seed + 101 + rank)
    prompts = [tuple(int(x) for x in rng.integers(0, vocab - 2, size=args.is_prompt_len)) for _ in range(per_rank)]
    tokens_per_prompt = (args.is_candidates * args.is_block
                         + args.is_candidates * args.is_rollouts * args.is_rollout_len)
    return prompts, tokens_per_prompt


def _is_result(args, world, impl, ms, wall, tokens, prompts_per_step, clocks, extra):
    out = {
        "metric": IS_METRIC, "value": tokens / (ms / 1e3), "unit": "tok/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic (uniform-random prompt ids, random-init weights)",
        "config": {"model": "qwen2.5-1.5b (random init)", "global_batch": prompts_per_step,
                   "seq_len": args.is_prompt_len + args.is_block + args.is_rollout_len,
                   "parallelism": f"dp{world}", "candidates": args.is_candidates, "block": args.is_block,
                   "rollouts_per_candidate": args.is_rollouts, "rollout_len": args.is_rollout_len,
                   "reward": "sequence log-probability, c=0.5, tau=0.5", "temperature": 1.0,
                   "step": "one conditional-IS decision block (first block) of every prompt",
                   "prompt_threads_per_rank": (min(args.is_workers, prompts_per_step // world) if impl is None
                                               else prompts_per_step // world),
                   "l2": "weights (3 GB) and KV streamed every decode step exceed the 126 MB L2"},
        "clocks": clocks,
    }
    if impl:
        out["impl"] = impl
    out.update(extra)
    return out


def run_is(args, rank, world, local, group) -> dict:
    """Conditional IS on the engine backend: prompts run as threads whose sample/score
    calls are merged by the continuous-batching wrapper into wide engine batches."""
    from concurrent.futures import ThreadPoolExecutor

    import torch

    from online_speculation_b200.api import build_runner
    from online_speculation_b200.arllm.algorithms.conditional_is import conditional_is_step
    from online_speculation_b200.arllm.backends.batching import ContinuousBatchingBackend
    from online_speculation_b200.arllm.config import ConditionalISConfig, SamplingConfig
    from online_speculation_b200.arllm.rewards import SequenceLogProbabilityReward
    from online_speculation_b200.engine.backend import EngineBackend
    from online_speculation_b200.ops import _ext
    from online_speculation_b200.shared.rng import SeedStream

    prompts, tokens_per_prompt = _is_workload(args, rank, world, args.is_prompts)
    runner = build_runner("qwen2.5-1.5b", seed=args.seed, kv_bytes=int(args.kv_gb * 2**30), max_tokens=8192)
    seq_max = args.is_prompt_len + args.is_block + args.is_rollout_len
    engine = EngineBackend(runner, model_id="qwen2.5-1.5b-random", max_batch=256, max_seq_tokens=seq_max,
                           prefill_tokens=8192, decode_chunk=16, score_pack=256)
    backend = ContinuousBatchingBackend(engine, max_batch_size=256, max_batch_tokens=1 << 22,
                                        batch_wait_seconds=0.002)
    reward = SequenceLogProbabilityReward(backend, coefficient=0.5)
    cfg = ConditionalISConfig(candidate_count=args.is_candidates, rollout_count=args.is_rollouts,
                              block_size=args.is_block, total_length=args.is_block + args.is_rollout_len,
                              reward_temperature=0.5)
    policy = SamplingConfig(temperature=1.0)

    def one(step, i):
        st = conditional_is_step(base_backend=backend, rollout_backend=backend, prompt=prompts[i], generated_prefix=(),
                                 config=cfg, base_sampling=policy, rollout_sampling=policy, reward=None,
                                 seeds=SeedStream(args.seed * 1_000_003 + step * 10_007 + rank * 101 + i),
                                 step_index=0, reward_batch=reward.batch)
        return st.selected.token_ids

    pool = ThreadPoolExecutor(max_workers=max(1, min(args.is_workers, len(prompts))))

    def step(k):
        return list(pool.map(lambda i: one(k, i), range(len(prompts))))

    for k in range(args.warmup):
        step(k)
    torch.cuda.synchronize()
    barrier(world)
    launches0 = _ext.launches() + engine.stats["graph_kernel_launches"]
    gen0 = engine.stats["generated_tokens"]
    sampler = ClockSampler(local)
    with sampler:
        barrier(world)
        wall0 = time.perf_counter()
        start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        chosen = []
        for k in range(args.steps):
            chosen.append(step(args.warmup + k))
        stop.record()
        torch.cuda.synchronize()
        wall = time.perf_counter() - wall0
        barrier(world)
    pool.shutdown()
    ms = max_over_ranks(start.elapsed_time(stop), world)
    wall = max_over_ranks(wall, world)
    generated = sum_over_ranks(engine.stats["generated_tokens"] - gen0, world)
    expected = tokens_per_prompt * len(prompts) * args.steps * world
    launches = _ext.launches() + engine.stats["graph_kernel_launches"] - launches0
    out = _is_result(args, world, None, ms, wall, generated, len(prompts) * world, sampler.summary(), {
        "generated_tokens": generated, "expected_tokens": expected,
        "batching": dataclasses.asdict(backend.snapshot()),
        "e2e": {"value": generated / wall, "unit": "tok/s",
                "h2d_bytes_per_step": len(prompts) * world * args.is_prompt_len * 4,
                "d2h_bytes_per_step": len(prompts) * world * args.is_block * 4},
        "gpu_launches": int(launches),
    })
    backend.close()
    engine.close()
    return out


def run_is_reference(args, rank, world, local, group) -> dict:
    """The same IS decision blocks on the unmodified reference: its TransformersBackend behind its
    own continuous-batching wrapper, prompts as threads, reward batches as in the repo arm."""
    ref = os.path.join(ROOT, "baseline", "_ref")
    if not os.path.isdir(os.path.join(ref, "inference_scaling")):
        return {"impl": "reference", "unavailable": "reference package not installed under baseline/_ref"}
    sys.path.insert(0, ref)
    from concurrent.futures import ThreadPoolExecutor

    import torch
    from transformers import Qwen2Config, Qwen2ForCausalLM

    from inference_scaling.arllm.algorithms.conditional_is import conditional_is_step
    from inference_scaling.arllm.backends.batching import ContinuousBatchingBackend
    from inference_scaling.arllm.backends.transformers_backend import TransformersBackend
    from inference_scaling.arllm.config import ConditionalISConfig, SamplingConfig
    from inference_scaling.arllm.rewards import SequenceLogProbabilityReward
    from inference_scaling.shared.rng import SeedStream

    from online_speculation_b200.models.decoder import PRESETS

    c = PRESETS["qwen2.5-1.5b"]
    hf = Qwen2Config(vocab_size=c.vocab_size, hidden_size=c.hidden_size, intermediate_size=c.intermediate_size,
                     num_hidden_layers=c.num_hidden_layers, num_attention_heads=c.num_attention_heads,
                     num_key_value_heads=c.num_key_value_heads, rope_theta=c.rope_theta, rms_norm_eps=c.rms_norm_eps,
                     tie_word_embeddings=c.tie_word_embeddings, max_position_embeddings=4096,
                     torch_dtype="bfloat16")
    torch.manual_seed(args.seed)
    with torch.device("cuda"):
        model = Qwen2ForCausalLM(hf).to(torch.bfloat16)
    model.eval()

    class Tok:
        pad_token_id = 0
        eos_token_id = None
        bos_token_id = 1

    inner = TransformersBackend(model, Tok(), model_id="qwen2.5-1.5b-random", device="cuda")
    backend = ContinuousBatchingBackend(inner, max_batch_size=256, max_batch_tokens=1 << 22, batch_wait_seconds=0.002)
    prompts, tokens_per_prompt = _is_workload(args, rank, world, args.is_ref_prompts)
    reward = SequenceLogProbabilityReward(backend, scale=0.5)
    cfg = ConditionalISConfig(candidate_count=args.is_candidates, rollout_count=args.is_rollouts,
                              block_size=args.is_block, total_length=args.is_block + args.is_rollout_len,
                              reward_temperature=0.5)
    policy = SamplingConfig(temperature=1.0)
    counted = {"tokens": 0}
    lock = threading.Lock()

    class Counting:
        def __init__(self, b):
            self.b = b

        @property
        def model_id(self):
            return self.b.model_id

        def sample_batch(self, requests):
            out = self.b.sample_batch(requests)
            with lock:
                counted["tokens"] += sum(len(s.token_ids) for s in out)
            return out

        def score_batch(self, requests):
            return self.b.score_batch(requests)

    counting = Counting(backend)

    def one(step, i):
        st = conditional_is_step(base_backend=counting, rollout_backend=counting, prompt=prompts[i],
                                 generated_prefix=(), config=cfg, base_sampling=policy, rollout_sampling=policy,
                                 reward=None, seeds=SeedStream(args.seed * 1_000_003 + step * 10_007 + rank * 101 + i),
                                 step_index=0, reward_batch=reward.batch)
        return st.selected.token_ids

    pool = ThreadPoolExecutor(max_workers=len(prompts))

    def step(k):
        return list(pool.map(lambda i: one(k, i), range(len(prompts))))

    for k in range(args.warmup):
        step(k)
    torch.cuda.synchronize()
    barrier(world)
    counted["tokens"] = 0
    sampler = ClockSampler(local)
    with sampler:
        barrier(world)
        wall0 = time.perf_counter()
        start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        for k in range(args.steps):
            step(args.warmup + k)
        stop.record()
        torch.cuda.synchronize()
        wall = time.perf_counter() - wall0
        barrier(world)
    pool.shutdown()
    ms = max_over_ranks(start.elapsed_time(stop), world)
    wall = max_over_ranks(wall, world)
    generated = sum_over_ranks(counted["tokens"], world)
    return _is_result(args, world, "reference", ms, wall, generated, len(prompts) * world, sampler.summary(), {
        "generated_tokens": generated,
        "path": "inference_scaling TransformersBackend + ContinuousBatchingBackend + conditional_is_step (unmodified)",
        "e2e": {"value": generated / wall, "unit": "tok/s", "h2d_bytes_per_step": None, "d2h_bytes_per_step": None},
    })


# reference arms that cannot run in this image, whatever the hardware (reported before any device setup)
REFERENCE_UNAVAILABLE = {
    "dllm": "the reference LLaDA-MoE path loads remote model code from the Hugging Face hub, which this machine "
            "cannot reach",
    "grpo": "the reference GRPO path needs trl and peft, which are not installed in this image",
}


def main():
    args = parse()
    if args.impl == "reference" and args.workload in REFERENCE_UNAVAILABLE:
        if int(os.environ.get("RANK", "0")) == 0:
            out = {"impl": "reference", "unavailable": REFERENCE_UNAVAILABLE[args.workload]}
            print(json.dumps(out), flush=True)
            if args.json_out:
                os.makedirs(os.path.dirname(os.path.abspath(args.json_out)), exist_ok=True)
                with open(args.json_out, "w", encoding="utf-8") as handle:
                    handle.write(json.dumps(out) + "\n")
        return
    rank, world, local, group = dist_setup(args.gpus)
    try:
        if args.workload == "dllm":
            out = run_dllm(args, rank, world, local, group)
        elif args.workload == "is":
            out = (run_is(args, rank, world, local, group) if args.impl == "ours"
                   else run_is_reference(args, rank, world, local, group))
        elif args.workload == "grpo":
            out = run_grpo(args, rank, world, local, group)
        else:
            out = (run_ours(args, rank, world, local, group) if args.impl == "ours"
                   else run_reference(args, rank, world, local, group))
    finally:
        pass
    if rank == 0:
        print(json.dumps(out), flush=True)
        if args.json_out:
            os.makedirs(os.path.dirname(os.path.abspath(args.json_out)), exist_ok=True)
            with open(args.json_out, "w", encoding="utf-8") as handle:
                handle.write(json.dumps(out) + "\n")
    if world > 1:
        import gc

        import torch
        import torch.distributed as dist

        gc.collect()
        torch.cuda.synchronize()
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
