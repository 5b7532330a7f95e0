"""Worker for tests/test_tp_gpu.py (launched with torch.distributed.run).

Every rank builds its shard of the same random weights, runs prefill, decode
and a verify block through the tensor-parallel runner (NCCL baseline and the
fused peer-memory collective), and checks the logits against the fp32 oracle;
then it runs the speculative MH engine and checks the emitted log-probabilities.
"""

import datetime
import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from online_speculation_b200.api import build_mh_engine  # noqa: E402
from online_speculation_b200.engine.kv_cache import KVCache  # noqa: E402
from online_speculation_b200.engine.runner import Collectives, ModelRunner, build_meta  # noqa: E402
from online_speculation_b200.models.decoder import DecoderConfig, build_weights, random_state_dict, reference_forward  # noqa: E402
from online_speculation_b200.ops import workspace  # noqa: E402

# 14 query heads over 2 KV heads: at 4 and 8 ranks the query heads are padded to 16
# (zero heads) and every KV head is replicated on the ranks that share it.
CFG = DecoderConfig(vocab_size=1024, hidden_size=1792, intermediate_size=1024, num_hidden_layers=3,
                    num_attention_heads=14, num_key_value_heads=2, name="small")


def rel(a, b):
    return float((a.float() - b.float()).norm() / b.float().norm())


def main():
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    rank, world = dist.get_rank(), dist.get_world_size()
    dev = torch.device("cuda", local)
    sd = random_state_dict(CFG, seed=0, std=0.05, device=dev)
    torch.manual_seed(0)
    seq = torch.randint(0, CFG.vocab_size, (70,))
    ref = reference_forward(CFG, {k: v.cpu() for k, v in sd.items()}, seq)
    # NCCL baseline, fused pull all-reduce (both algorithms at every world size), and
    # GEMM push + local reduction (up to four ranks)
    variants = [(False, None, "auto"), (True, False, "oneshot"), (True, False, "twoshot")]
    if world <= 4:
        variants.append((True, True, "auto"))
    for fused, push, algorithm in variants:
        w = build_weights(CFG, sd, tp=world, rank=rank, device=dev)
        if world > 2:
            assert w.heads.q_slots * world > CFG.num_attention_heads   # padded query heads
        cache = KVCache(CFG.num_hidden_layers, w.heads.kv_slots, 64, dev)
        comm = Collectives(dist.group.WORLD, hidden=CFG.hidden_size, max_tokens=1024, device=dev, fused=fused,
                           push=push, algorithm=algorithm)
        if fused:
            assert comm.impl.push == bool(push and world <= 4)
        r = ModelRunner(w, cache, collectives=comm, max_tokens=1024)
        G = r.q_slots // r.kv_slots
        s = cache.create()
        table = torch.zeros(1, 8, dtype=torch.int32)
        slots = cache.append(s, 60)
        cache.fill_table([s], table)
        out = r.forward(build_meta(dev, table, seq[:60].tolist(), list(range(60)), slots, [60], [60], [0], G))
        assert rel(out.cpu(), ref[:60]) < 5e-2, ("prefill", fused, push, algorithm, rel(out.cpu(), ref[:60]))
        slots = cache.append(s, 4)
        cache.fill_table([s], table)
        out = r.forward(build_meta(dev, table, seq[60:64].tolist(), list(range(60, 64)), slots, [4], [64], [0], G))
        assert rel(out.cpu(), ref[60:64]) < 5e-2, ("verify", fused, push, algorithm)
        torch.cuda.synchronize()
        workspace.check_status(dev)
    # vocabulary-parallel samplers draw exactly what the unsharded kernels draw on full rows
    from online_speculation_b200.ops import kernels as K  # noqa: E402

    V, width = 1024, 1024 // world
    shard = K.VocabShard(rank * width, width, V, dist.group.WORLD, world)
    g = torch.Generator(device=dev).manual_seed(7)
    B, n = 5, 3
    full_t = torch.randn(B * (n + 1), V, device=dev, generator=g) * 3
    full_d = full_t[torch.arange(B * (n + 1), device=dev).view(B, n + 1)[:, :n].reshape(-1)] + \
        torch.randn(B * n, V, device=dev, generator=g)
    seeds = torch.arange(11, 11 + B, dtype=torch.int64, device=dev)
    it = torch.full((B,), 0.7, device=dev)
    rows_it = it.repeat_interleave(n)
    si = torch.arange(B, dtype=torch.int32, device=dev).repeat_interleave(n)
    streams = torch.zeros(B * n, dtype=torch.int32, device=dev)
    rin = torch.arange(n, dtype=torch.int32, device=dev).repeat(B)
    want = K.gumbel_sample(full_d, rows_it, seeds, seed_index=si, streams=streams, row_in_seq=rin, salt=5)
    got = K.gumbel_sample(full_d[:, rank * width:(rank + 1) * width].contiguous(), rows_it, seeds, seed_index=si,
                          streams=streams, row_in_seq=rin, salt=5, shard=shard)
    assert torch.equal(want, got), ("sharded gumbel", want, got)
    cand = want.view(B, n)
    ref = K.spec_verify(full_t, full_d, cand, it, seeds, salt=9)
    res = K.spec_verify(full_t[:, rank * width:(rank + 1) * width].contiguous(),
                        full_d[:, rank * width:(rank + 1) * width].contiguous(), cand, it, seeds, salt=9, shard=shard)
    for key in ("count", "tail", "valid"):
        assert torch.equal(ref[key], res[key]), (key, ref[key], res[key])
    for b in range(B):
        c = int(ref["count"][b]) + 1
        assert torch.equal(ref["emitted"][b, :c], res["emitted"][b, :c])
        assert torch.allclose(ref["logq"][b, :c], res["logq"][b, :c], atol=1e-4)
        assert torch.allclose(ref["logp"][b, :c], res["logp"][b, :c], atol=1e-4)
    eng = build_mh_engine(CFG, tp_group=dist.group.WORLD, seed=3, alpha=2.0, length=24, block_size=4,
                          learner_stride=8, use_graphs=False, kv_bytes=64 << 20, max_seq_tokens=64, max_batch=8)
    prompt = list(range(5, 21))
    eng.add_chains([prompt] * 6)
    eng.run_until_idle()
    eng.set_quota(2)
    eng.run_until_idle()
    assert eng.stats["mh_updates"] == 12 and eng.learner.updates >= 1
    oracle = {k: v.cpu() for k, v in random_state_dict(CFG, seed=3, std=0.02, device=dev).items()}
    for ch in eng.chains:
        full = torch.tensor(ch.prompt + ch.tokens)
        logits = reference_forward(CFG, oracle, full)[len(prompt) - 1:-1]
        lp = logits.log_softmax(-1).gather(-1, torch.tensor(ch.tokens)[:, None]).squeeze(-1)
        assert torch.allclose(torch.tensor(ch.logp), lp, atol=0.05)
    # every rank must hold identical chains (replicated sampling decisions)
    toks = torch.tensor([ch.tokens for ch in eng.chains], device=dev)
    gathered = [torch.empty_like(toks) for _ in range(world)]
    dist.all_gather(gathered, toks)
    assert all(torch.equal(gathered[0], g) for g in gathered)
    workspace.check_status(dev)
    dist.barrier()
    if rank == 0:
        print("TP_OK", world, flush=True)
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
