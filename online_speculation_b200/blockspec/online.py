"""Online suffix learner of the dual-view draft attention (PyTorch module path).

Only the draft attention of the last ``last_layers`` layers learns; every other
tensor stays frozen (checked by version counters and a content fingerprint).
Each verified round can leave a feedback block: the frozen boundary hidden
state entering the suffix, the clean suffix KV, and the teacher (AR verify)
logits of the reached rows.  Every ``stride`` rounds the learner replays the
latest ``replay_blocks`` blocks with fp32 master weights, minimises full-
vocabulary TV or forward KL to the teacher, clips the gradient norm, takes an
AdamW step and publishes the masters into the execution weights.
Reference: online-speculation/src/blockspec/parallel/online.py:17-196 and
parallel/feedback.py.  The 1-layer draft head of the engine has its own
graph-captured learner (``engine/draft.py``).
"""

from __future__ import annotations

import copy
import hashlib
import math
import time
from collections import deque
from dataclasses import asdict, dataclass

import torch

from ..ops import kernels as K
from .model import DraftBoundary, DualViewDecoder


@dataclass(frozen=True)
class SuffixConfig:
    last_layers: int = 1
    stride: int = 16
    replay_blocks: int = 1
    learning_rate: float = 1e-5
    clip_norm: float = 1.0
    loss: str = "forward_kl"

    def __post_init__(self):
        if (any(type(v) is not int or v < 1 for v in (self.last_layers, self.stride, self.replay_blocks))
                or self.replay_blocks > self.stride
                or any(not math.isfinite(v) or v <= 0 for v in (self.learning_rate, self.clip_norm))
                or self.loss not in ("forward_kl", "tv")):
            raise ValueError("positive bounded windows, optimizer scales and a KL or TV loss required")


def divergence(student: torch.Tensor, teacher: torch.Tensor, kind: str = "forward_kl") -> torch.Tensor:
    """Per-row KL(teacher || student) or total variation at temperature one (fp32 or fp64)."""
    if student.shape != teacher.shape:
        raise ValueError("student / teacher shapes differ")
    dt = torch.float64 if student.dtype == torch.float64 else torch.float32
    lq = student.to(dt).log_softmax(-1)
    lp = teacher.detach().to(dt).log_softmax(-1)
    if kind == "forward_kl":
        return (lp.exp() * (lp - lq)).sum(-1)
    if kind == "tv":
        return 0.5 * (lq.exp() - lp.exp()).abs().sum(-1)
    raise ValueError(f"unknown loss {kind!r}")


@dataclass
class Feedback:
    inputs: torch.Tensor
    cache: tuple | None
    teacher_logits: torch.Tensor
    valid: int
    boundary: DraftBoundary
    fully_covered: bool = False

    def detached(self, cache_start: int = 0) -> "Feedback":
        cache = None if self.cache is None else tuple((k.detach(), v.detach()) for k, v in self.cache[cache_start:])
        return Feedback(self.inputs.detach().clone(), cache, self.teacher_logits.detach().clone(), self.valid,
                        self.boundary.detached(), self.fully_covered)


class SuffixLearner:
    def __init__(self, model: DualViewDecoder, config: SuffixConfig = SuffixConfig()):
        if config.last_layers > len(model.layers) or any(p.requires_grad for p in model.parameters()):
            raise ValueError("a frozen dual-view model and a suffix within its layers required")
        self.model, self.config = model, config
        self.capture_layer = len(model.layers) - config.last_layers
        self.execution = {n: p for n, p in model.named_parameters()
                          if n.startswith("layers.") and int(n.split(".")[1]) >= self.capture_layer
                          and ".attention.draft." in n}
        self.names = list(self.execution)
        flat = torch.cat([p.detach().float().flatten() for p in self.execution.values()])
        self.master = torch.nn.Parameter(flat)
        self.exp_avg = torch.zeros_like(flat)
        self.exp_avg_sq = torch.zeros_like(flat)
        self.step = 0
        self._frozen = [(p, p._version) for n, p in model.named_parameters() if n not in self.execution]
        h = hashlib.sha256()
        for n, p in model.named_parameters():
            if n not in self.execution:
                h.update(n.encode())
                h.update(p.detach().contiguous().cpu().float().numpy().tobytes())
        self.frozen_fingerprint = h.hexdigest()
        self.replay: deque[Feedback] = deque(maxlen=config.replay_blocks)
        self.rounds = self.updates = self.version = self.feedback_blocks = 0
        self.update_seconds, self.last_loss = 0.0, None

    def _views(self, flat):
        out, off = {}, 0
        for n, p in self.execution.items():
            out[n] = flat[off:off + p.numel()].view_as(p)
            off += p.numel()
        return out

    @property
    def trainable_parameters(self) -> int:
        return self.master.numel()

    @property
    def needs_decoder_feedback(self) -> bool:
        return self.config.stride - self.rounds % self.config.stride <= self.config.replay_blocks

    def _check(self):
        if any(p._version != v for p, v in self._frozen):
            raise RuntimeError("frozen representations changed; rebuild the learner")

    def clear_replay(self):
        self.replay.clear()

    def skip(self):
        self.rounds += 1

    def observe(self, fb: Feedback, *, may_update: bool = True):
        self._check()
        if fb.boundary.start_layer != self.capture_layer or not 0 < fb.valid < fb.inputs.shape[1]:
            raise ValueError("aligned boundary and reached teacher rows required")
        self.rounds += 1
        self.feedback_blocks += 1
        self.replay.append(fb.detached(cache_start=self.capture_layer))
        if may_update and self.rounds % self.config.stride == 0:
            return self.update()
        return None

    def _replay_items(self) -> list:
        """Replayed blocks that enter the next update."""
        return list(self.replay)

    def _replay_loss(self, fb: Feedback, logits: torch.Tensor, rows: int, blocks: int) -> torch.Tensor:
        """Loss of one replayed block; the update sums it over ``_replay_items``."""
        return divergence(logits, fb.teacher_logits, self.config.loss).sum() / rows

    def update(self):
        if not self.replay:
            return None
        self._check()
        start = time.perf_counter()
        items = self._replay_items()
        if not items:
            return None
        rows = sum(f.valid for f in items)
        total = 0.0
        grad = torch.zeros_like(self.master)
        with torch.enable_grad():
            for fb in items:
                weights = {n: v.to(self.execution[n].dtype) for n, v in self._views(self.master).items()}
                out = self.model.forward_suffix(fb.boundary, cache=fb.cache, logit_range=(0, fb.valid),
                                                draft_weights=weights)
                loss = self._replay_loss(fb, out.logits[0], rows, len(items))
                if not torch.isfinite(loss):
                    raise FloatingPointError("nonfinite online suffix loss")
                (g,) = torch.autograd.grad(loss, [self.master])
                grad += g
                total += float(loss.detach())
        self.step += 1
        norm_buf = torch.zeros(1, dtype=torch.float32, device=grad.device)
        sq = K.adamw_step(self.master.data, grad, self.exp_avg, self.exp_avg_sq, step=self.step,
                          lr=self.config.learning_rate, clip=self.config.clip_norm, norm_out=norm_buf)
        norm = float(torch.as_tensor(sq).sqrt()) if sq is not None else 0.0
        if not math.isfinite(norm):
            raise FloatingPointError("nonfinite gradient norm")
        self.publish()
        elapsed = time.perf_counter() - start
        self.updates += 1
        self.version += 1
        self.update_seconds += elapsed
        self.last_loss = total
        return {"loss": total, "gradient_norm": norm, "seconds": elapsed, "version": self.version}

    @torch.no_grad()
    def publish(self):
        for n, v in self._views(self.master.detach()).items():
            self.execution[n].copy_(v)

    def state_dict(self) -> dict:
        if self.replay:
            raise ValueError("save online state at a request boundary after clearing replay")
        return {"format": "blockspec-dual-suffix-v1", "config": asdict(self.config),
                "model_config": self.model.config.to_dict(), "frozen_fingerprint": self.frozen_fingerprint,
                "master": {n: v.detach().cpu().clone() for n, v in self._views(self.master).items()},
                "optimizer": {"exp_avg": self.exp_avg.cpu().clone(), "exp_avg_sq": self.exp_avg_sq.cpu().clone(),
                              "step": self.step},
                "rounds": self.rounds, "updates": self.updates, "version": self.version,
                "feedback_blocks": self.feedback_blocks, "update_seconds": self.update_seconds,
                "last_loss": self.last_loss}

    def load_state_dict(self, state: dict) -> None:
        self._check()
        if (state.get("format") != "blockspec-dual-suffix-v1" or state.get("config") != asdict(self.config)
                or state.get("model_config") != self.model.config.to_dict()
                or state.get("frozen_fingerprint") != self.frozen_fingerprint
                or set(state.get("master", {})) != set(self.names)):
            raise ValueError("online state must match its model, precision and update policy")
        with torch.no_grad():
            flat = torch.cat([state["master"][n].float().flatten() for n in self.names]).to(self.master.device)
            if not torch.isfinite(flat).all():
                raise ValueError("finite fp32 masters required")
            self.master.copy_(flat)
        self.exp_avg.copy_(state["optimizer"]["exp_avg"])
        self.exp_avg_sq.copy_(state["optimizer"]["exp_avg_sq"])
        self.step = int(state["optimizer"]["step"])
        for key in ("rounds", "updates", "version", "feedback_blocks", "update_seconds", "last_loss"):
            setattr(self, key, state[key])
        self.publish()
        self.clear_replay()


class OnlineFeedback:
    """Generation hooks that feed verified rounds into a :class:`SuffixLearner`."""

    def __init__(self, *, learner: SuffixLearner):
        self.learner = learner

    def begin(self, prompt):
        self._start = (self.learner.updates, self.learner.update_seconds, self.learner.feedback_blocks)
        self.learner.clear_replay()

    @property
    def capture_layer(self):
        return self.learner.capture_layer if self.learner.needs_decoder_feedback else None

    def commit(self, tokens):
        pass

    def observe(self, proposal, teacher_logits, target, *, used, fully_covered, done):
        if proposal.collect_feedback and proposal.boundary is not None and used > 0:
            fb = Feedback(proposal.draft_inputs, proposal.cache, teacher_logits[:used], used, proposal.boundary,
                          fully_covered)
            self.learner.observe(fb, may_update=not done)
        else:
            self.learner.skip()

    def finish(self, result):
        self.learner.clear_replay()
        u, s, f = self._start
        result.updates = self.learner.updates - u
        result.update_seconds = self.learner.update_seconds - s
        result.feedback_blocks = self.learner.feedback_blocks - f
