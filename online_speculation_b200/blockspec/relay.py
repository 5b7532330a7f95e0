"""PrefixRelay: a trainable Markov correction of parallel draft rows, with prefix admission.

The dual-view drafter proposes every depth of a block in parallel, so depth d
does not know which token was drawn at depth d - 1.  A relay head adds that
dependence cheaply: candidate d is drawn from

    q_d = transform(draft_logits_d + P E[token_{d-1}])

with a low-rank token embedding E [V, r] and projection P [r -> V] (P starts at
zero, so the relay starts as the plain parallel proposal), sequentially from
the anchor.  A confidence head sigma(c([rmsnorm(h_d), E[token_{d-1}]])) predicts
whether depth d will be accepted; with ``threshold`` > 0 the block stops once the
product of those survival probabilities falls below it (the first candidate is
always drawn).  Verification is the exact p / q correction on the saved
corrected rows, so the output law is the target's.

:class:`RelayLearner` trains the head online (AdamW, clipped) on verified blocks:
TV(p_d, q_d) on the supervised depths plus a binary cross-entropy that teaches the
confidence head 1 - TV.  :class:`RelayBranch` plugs the relay into
:func:`online_speculation_b200.blockspec.generation.generate`; pass its
``feedback()`` as the ``feedback`` argument to train while decoding.

Reference behaviour: online-speculation/ablation/src/blockspec_ablation/relay.py
(``RelayHead``, ``relay_candidates``, ``relay_loss``, ``RelayLearner``, ``generate_relay``).
"""

from __future__ import annotations

import math
import time
from dataclasses import asdict, dataclass

import torch
from torch import nn
from torch.nn import functional as F

from .generation import DraftBatch, MaskedAttentionBranch, ProposalSampler
from .sampling import SamplingConfig, draw, probabilities


@dataclass(frozen=True)
class RelayConfig:
    vocab_size: int
    hidden_size: int
    rank: int = 64

    def __post_init__(self):
        if any(type(v) is not int or v < 1 for v in asdict(self).values()):
            raise ValueError("positive integer head dimensions are required")


class RelayHead(nn.Module):
    def __init__(self, config: RelayConfig):
        super().__init__()
        self.config = config
        self.embedding = nn.Embedding(config.vocab_size, config.rank)
        self.projection = nn.Linear(config.rank, config.vocab_size, bias=False)
        self.confidence = nn.Linear(config.hidden_size + config.rank, 1)
        nn.init.normal_(self.embedding.weight, std=config.rank ** -0.5)
        nn.init.zeros_(self.projection.weight)
        nn.init.zeros_(self.confidence.weight)
        nn.init.zeros_(self.confidence.bias)

    def forward(self, logits: torch.Tensor, previous: torch.Tensor) -> torch.Tensor:
        return logits.to(self.projection.weight.dtype) + self.projection(self.embedding(previous))

    def confidence_logits(self, hidden: torch.Tensor, previous: torch.Tensor) -> torch.Tensor:
        h = hidden.to(self.confidence.weight.dtype)
        h = h * (h.square().mean(-1, keepdim=True) + 1e-6).rsqrt()
        return self.confidence(torch.cat((h, self.embedding(previous)), -1)).squeeze(-1)

    @torch.no_grad()
    def initialize_from_embedding(self, embedding: torch.Tensor, *, seed: int = 271828) -> None:
        """Token features from the frozen base embedding through a fixed Gaussian projection
        (row-normalised; a private generator keeps rollouts' randomness untouched)."""
        if (embedding.ndim != 2 or tuple(embedding.shape) != (self.config.vocab_size, self.config.hidden_size)
                or not bool(torch.isfinite(embedding).all()) or int(self.projection.weight.count_nonzero())):
            raise ValueError("finite base embeddings of matching shape and a zero projection are required")
        dev = self.embedding.weight.device
        g = torch.Generator(device=dev).manual_seed(seed)
        proj = torch.randn(self.config.hidden_size, self.config.rank, device=dev, generator=g) / math.sqrt(
            self.config.rank)
        feats = F.normalize(embedding.detach().to(dev, torch.float32) @ proj, dim=-1)
        self.embedding.weight.copy_(feats.to(self.embedding.weight.dtype))


@dataclass
class RelayDraft:
    tokens: torch.Tensor      # drawn candidates (depths 1..n)
    q: torch.Tensor | None    # their corrected proposal laws [n, V] (None when greedy)


@torch.no_grad()
def relay_candidates(head: RelayHead, logits: torch.Tensor, hidden: torch.Tensor, anchor: int, *,
                     sampling: SamplingConfig = SamplingConfig(), threshold: float = 0.0,
                     generator=None) -> RelayDraft:
    """Draw candidates for depths 1..len(logits) sequentially from the corrected rows."""
    if not math.isfinite(threshold) or not 0 <= threshold <= 1:
        raise ValueError("the admission threshold must lie in [0, 1]")
    if (logits.ndim != 2 or not len(logits) or tuple(hidden.shape) != (len(logits), head.config.hidden_size)
            or logits.shape[-1] != head.config.vocab_size):
        raise ValueError("one logit row and one hidden row per draft depth are required")
    prev = torch.tensor(anchor, device=logits.device)
    toks, rows = [], []
    survival = 1.0
    for d in range(len(logits)):
        if threshold and d > 0:
            survival *= float(head.confidence_logits(hidden[d], prev).sigmoid())
            if survival < threshold:
                break
        corrected = head(logits[d], prev)
        if sampling.temperature == 0:
            tok = corrected.argmax(-1)
        else:
            q = probabilities(corrected, sampling)
            rows.append(q)
            tok = draw(q, generator)
        toks.append(tok)
        prev = tok
    return RelayDraft(torch.stack(toks), torch.stack(rows) if rows else None)


@dataclass
class RelayFeedback:
    logits: torch.Tensor      # draft rows [n, V]
    hidden: torch.Tensor      # draft hidden rows [n, H]
    previous: torch.Tensor    # token before each depth [n]
    teacher: torch.Tensor     # target logits of those depths [n, V]


def relay_loss(head: RelayHead, fb: RelayFeedback, *, sampling: SamplingConfig = SamplingConfig(1.0),
               confidence_weight: float = 0.1):
    """TV(p, q) of the corrected rows plus the confidence head's BCE towards 1 - TV (inputs detached)."""
    if sampling.temperature <= 0 or not math.isfinite(confidence_weight) or confidence_weight < 0:
        raise ValueError("a positive training temperature and a finite nonnegative confidence weight are required")
    q = probabilities(head(fb.logits.detach(), fb.previous.detach()), sampling)
    p = probabilities(fb.teacher.detach(), sampling)
    tv = 0.5 * (p - q).abs().sum(-1)
    conf = F.binary_cross_entropy_with_logits(head.confidence_logits(fb.hidden.detach(), fb.previous.detach()),
                                              (1 - tv).detach())
    return tv.mean() + confidence_weight * conf, tv.mean().detach(), conf.detach()


class RelayLearner:
    """Head-only online updates every ``interval`` verified blocks (feedback is bounded per update)."""

    def __init__(self, head: RelayHead, *, lr: float = 1e-3, interval: int = 8,
                 sampling: SamplingConfig = SamplingConfig(1.0), confidence_weight: float = 0.1):
        if type(interval) is not int or interval < 1 or not math.isfinite(lr) or lr <= 0:
            raise ValueError("a positive update interval and learning rate are required")
        if sampling.temperature <= 0 or not math.isfinite(confidence_weight) or confidence_weight < 0:
            raise ValueError("a positive training temperature and a nonnegative confidence weight are required")
        self.head, self.interval, self.sampling, self.confidence_weight = head, interval, sampling, confidence_weight
        self.optimizer = torch.optim.AdamW(head.parameters(), lr=lr, weight_decay=0.0)
        self.pending: list[RelayFeedback] = []
        self.updates = self.feedback_blocks = self.examples = 0
        self.update_seconds = 0.0
        self.last_metrics: dict = {}

    def observe(self, fb: RelayFeedback, *, may_update: bool = True) -> None:
        if not len(fb.previous):
            return
        self.feedback_blocks += 1
        self.pending.append(RelayFeedback(*(t.detach().clone() for t in (fb.logits, fb.hidden, fb.previous,
                                                                         fb.teacher))))
        if len(self.pending) >= self.interval:
            if may_update:
                self.step()
            else:
                self.pending.clear()

    @torch.enable_grad()
    def step(self) -> None:
        if not self.pending:
            return
        t0 = time.perf_counter()
        fb = RelayFeedback(*(torch.cat([getattr(r, k) for r in self.pending]) for k in
                             ("logits", "hidden", "previous", "teacher")))
        self.optimizer.zero_grad(set_to_none=True)
        loss, tv, conf = relay_loss(self.head, fb, sampling=self.sampling, confidence_weight=self.confidence_weight)
        loss.backward()
        norm = torch.nn.utils.clip_grad_norm_(self.head.parameters(), 1.0, error_if_nonfinite=True)
        self.optimizer.step()
        self.updates += 1
        self.examples += len(fb.previous)
        self.last_metrics = {"tv": float(tv), "confidence_bce": float(conf), "grad_norm": float(norm)}
        self.pending.clear()
        self.update_seconds += time.perf_counter() - t0


class RelayBranch(MaskedAttentionBranch):
    """The dual-view drafter with a relay head drawing its candidates sequentially."""

    def __init__(self, model, head: RelayHead, *, threshold: float = 0.0):
        super().__init__(model)
        if (head.config.vocab_size, head.config.hidden_size) != (model.config.vocab_size, model.config.hidden_size):
            raise ValueError("relay head and decoder dimensions differ")
        if not math.isfinite(threshold) or not 0 <= threshold <= 1:
            raise ValueError("the admission threshold must lie in [0, 1]")
        self.head, self.threshold = head, threshold

    def draft(self, anchor, cache, block_size, sampler: ProposalSampler, generator=None, feedback=None):
        inputs = anchor.new_full((1, block_size), self.model.config.mask_token_id)
        inputs[:, :1] = anchor
        out = self.model(inputs, view="draft", cache=cache)
        logits, hidden = out.logits[0, :-1], out.hidden[0, :-1]
        d = relay_candidates(self.head, logits, hidden, int(anchor[0, 0]), sampling=sampler.config,
                             threshold=self.threshold, generator=generator)
        n = d.tokens.numel()
        batch = DraftBatch(torch.cat((anchor, d.tokens[None].to(anchor.dtype)), 1), d.tokens.to(anchor.dtype), d.q,
                           cache, [], inputs)
        batch.relay = RelayFeedback(logits[:n], hidden[:n],
                                    torch.cat((anchor[0, :1], d.tokens[:-1].to(anchor.dtype))), logits[:0])
        return batch

    def feedback(self, learner: RelayLearner) -> "_RelayFeedbackHook":
        return _RelayFeedbackHook(learner)


class _RelayFeedbackHook:
    """The ``feedback`` protocol of ``generate``: hands each verified block's supervised
    depths (with the target logits as teacher) to the relay learner."""

    capture_layer = None

    def __init__(self, learner: RelayLearner):
        self.learner = learner

    def begin(self, prompt):
        self.learner.pending.clear()

    def commit(self, tokens):
        pass

    def observe(self, proposal, teacher_logits, target, *, used, fully_covered, done):
        fb = getattr(proposal, "relay", None)
        if fb is None or used <= 0:
            return
        self.learner.observe(RelayFeedback(fb.logits[:used], fb.hidden[:used], fb.previous[:used],
                                           teacher_logits[:used]), may_update=not done)

    def finish(self, result):
        self.learner.pending.clear()


__all__ = ["RelayBranch", "RelayConfig", "RelayDraft", "RelayFeedback", "RelayHead", "RelayLearner",
           "relay_candidates", "relay_loss"]
