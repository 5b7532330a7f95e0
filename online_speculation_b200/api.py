"""Public entry points that assemble the B200 engine.

``build_mh_engine`` creates (per tensor-parallel rank) the random-init or
loaded decoder weights, the paged KV cache, the batched runner, the
block-bidirectional draft head and its online learner, and returns an
:class:`~online_speculation_b200.engine.mh_engine.MHEngine` ready for
``add_chains`` / ``set_quota`` / ``run_until_idle``.
"""

from __future__ import annotations

import torch

from .engine.draft import DraftHead, SuffixConfig, SuffixLearner, init_draft
from .engine.kv_cache import KVCache
from .engine.mh_engine import MHEngine
from .engine.runner import Collectives, ModelRunner
from .models.decoder import PRESETS, DecoderConfig, random_weights


def resolve_config(model: str | DecoderConfig) -> DecoderConfig:
    if isinstance(model, DecoderConfig):
        return model
    try:
        return PRESETS[model]
    except KeyError:
        raise ValueError(f"unknown model preset {model!r}; choose from {sorted(PRESETS)}") from None


def build_runner(model: str | DecoderConfig, *, tp_group=None, seed: int = 0, kv_bytes: int = 8 << 30,
                 max_tokens: int = 8192, max_logit_rows: int = 512, weights=None,
                 fused_collectives: bool = True) -> ModelRunner:
    cfg = resolve_config(model)
    device = torch.device("cuda", torch.cuda.current_device())
    comm = Collectives(tp_group, hidden=cfg.hidden_size, max_tokens=max_tokens, device=device, fused=fused_collectives)
    w = weights if weights is not None else random_weights(cfg, tp=comm.world, rank=comm.rank, seed=seed,
                                                           device=device)
    pages = KVCache.pages_for_budget(kv_bytes, cfg.num_hidden_layers, w.heads.kv_slots)
    cache = KVCache(cfg.num_hidden_layers, w.heads.kv_slots, pages, device)
    return ModelRunner(w, cache, collectives=comm, max_tokens=max_tokens, max_logit_rows=max_logit_rows)


def build_mh_engine(model: str | DecoderConfig = "qwen2.5-7b", *, tp_group=None, seed: int = 0, alpha: float = 4.0,
                    length: int = 512, block_size: int = 4, learner_stride: int | None = 64,
                    learner_loss: str = "tv", learning_rate: float = 1e-5, use_graphs: bool = True,
                    kv_bytes: int = 24 << 30, max_seq_tokens: int = 1040, max_batch: int = 64,
                    fused_collectives: bool = True, draft: bool = True, spec_policy: str = "adaptive",
                    probe_every: int = 8, plain_steps: int = 4, share_prefix: bool = False) -> MHEngine:
    """Suffix-MH engine.

    ``draft=False`` decodes one token per round without a draft head (the baseline
    that shows what block speculation adds).  ``spec_policy``: ``adaptive`` drafts
    in the rounds where the measured acceptance makes speculation faster than plain
    decoding, with a speculative round at least every ``probe_every`` rounds so the
    online learner keeps training; ``always`` drafts every round; ``never`` never.
    A plain round chains ``plain_steps`` decode steps in one graph replay.  ``share_prefix``:
    two-pass attention over the prompt pages every chain shares (measured slower on the 7B
    headline workload, so off by default).
    """
    runner = build_runner(model, tp_group=tp_group, seed=seed, kv_bytes=kv_bytes,
                          max_logit_rows=max(512, max_batch * block_size), fused_collectives=fused_collectives)
    if not draft:
        return MHEngine(runner, None, alpha=alpha, length=length, root_seed=seed, learner=None,
                        use_graphs=use_graphs, max_pages_per_seq=-(-(max_seq_tokens + plain_steps) // 32) + 1,
                        plain_steps=plain_steps, share_prefix=share_prefix)
    draft_weights = init_draft(runner.w, seed=seed + 1)
    head = DraftHead(runner, draft_weights, block_size=block_size)
    learner = None
    if learner_stride:
        learner = SuffixLearner(head, SuffixConfig(stride=learner_stride, loss=learner_loss,
                                                   learning_rate=learning_rate), use_graphs=use_graphs)
    max_pages = -(-(max_seq_tokens + plain_steps) // 32) + 1
    return MHEngine(runner, head, alpha=alpha, length=length, root_seed=seed, learner=learner,
                    use_graphs=use_graphs, max_pages_per_seq=max_pages, spec_policy=spec_policy,
                    probe_every=probe_every, plain_steps=plain_steps, share_prefix=share_prefix)
