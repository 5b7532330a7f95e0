"""File-backed draft-view fitting with deterministic data order and bit-exact resume.

* ``TokenDataset``: indexed tokenized JSONL (``{"input_ids": [...]}`` per line);
  random windows stay inside one record.
* ``BatchStream``: seeded permutation + cursor, saved with its RNG state.
* ``FitConfig``: schedule (linear warm-up then cosine to ``minimum_lr_ratio``),
  AdamW hyper-parameters, precision.
* ``Trainer``: ``run`` / ``evaluate`` / ``save`` / ``resume``; a checkpoint
  is written only at optimizer-step boundaries and carries the data cursor,
  every RNG state and a fingerprint of the frozen base, so an interrupted run
  resumes to the same weights as an uninterrupted one.
Reference: online-speculation/src/blockspec/parallel/fitting.py:18-263
(training-state payload ``dual-fit-v1``).
"""

from __future__ import annotations

import hashlib
import json
import math
import time
from array import array
from contextlib import nullcontext
from dataclasses import asdict, dataclass
from pathlib import Path

import torch

from .training import distillation_loss, distillation_update, sample_anchors
from .weights import file_sha256, load_checkpoint, save_checkpoint


class TokenDataset:
    def __init__(self, path, vocab_size: int, sequence_length: int):
        if min(vocab_size, sequence_length) < 1:
            raise ValueError("positive vocabulary and window required")
        self.path = Path(path).resolve()
        self.vocab_size, self.sequence_length = vocab_size, sequence_length
        self.offsets, self.skipped = array("Q"), 0
        with self.path.open("rb") as f:
            while True:
                off = f.tell()
                line = f.readline()
                if not line:
                    break
                if not line.strip():
                    continue
                if len(self._decode(line)) >= sequence_length:
                    self.offsets.append(off)
                else:
                    self.skipped += 1
        if not self.offsets:
            raise ValueError("training data needs at least one complete window")
        self.fingerprint = file_sha256(self.path)

    def _decode(self, line: bytes) -> list[int]:
        ids = json.loads(line).get("input_ids")
        if not isinstance(ids, list) or not ids or any(type(x) is not int or not 0 <= x < self.vocab_size for x in ids):
            raise ValueError("each record needs valid input_ids")
        return ids

    def __len__(self) -> int:
        return len(self.offsets)

    def __getitem__(self, i: int) -> torch.Tensor:
        with self.path.open("rb") as f:
            f.seek(self.offsets[i])
            return torch.tensor(self._decode(f.readline()), dtype=torch.long)


class BatchStream:
    def __init__(self, dataset: TokenDataset, seed: int):
        self.dataset = dataset
        self.rng = torch.Generator().manual_seed(seed)
        self.order = torch.randperm(len(dataset), generator=self.rng)
        self.cursor = self.epoch = 0

    def batch(self, count: int) -> torch.Tensor:
        rows, L = [], self.dataset.sequence_length
        for _ in range(count):
            if self.cursor == len(self.order):
                self.order = torch.randperm(len(self.dataset), generator=self.rng)
                self.cursor = 0
                self.epoch += 1
            seq = self.dataset[int(self.order[self.cursor])]
            self.cursor += 1
            start = int(torch.randint(len(seq) - L + 1, (), generator=self.rng))
            rows.append(seq[start:start + L])
        return torch.stack(rows)

    def state_dict(self) -> dict:
        return {"rng": self.rng.get_state(), "order": self.order.clone(), "cursor": self.cursor, "epoch": self.epoch}

    def load_state_dict(self, state: dict) -> None:
        order = state["order"].cpu()
        if (order.shape != (len(self.dataset),) or not torch.equal(order.sort().values, torch.arange(len(self.dataset)))
                or not 0 <= state["cursor"] <= len(order) or state["epoch"] < 0):
            raise ValueError("invalid data permutation or cursor")
        self.rng.set_state(state["rng"].cpu())
        self.order, self.cursor, self.epoch = order, state["cursor"], state["epoch"]


@dataclass(frozen=True)
class FitConfig:
    steps: int = 1000
    batch_size: int = 1
    sequence_length: int = 256
    anchors_per_sequence: int = 4
    accumulate: int = 1
    chunk_rows: int = 32
    learning_rate: float = 1e-4
    warmup_steps: int = 50
    minimum_lr_ratio: float = 0.1
    weight_decay: float = 0.01
    clip_grad: float = 1.0
    precision: str = "fp32"
    seed: int = 731
    optimizer_impl: str = "single"

    def __post_init__(self):
        if min(self.steps, self.batch_size, self.sequence_length, self.anchors_per_sequence, self.accumulate,
               self.chunk_rows) < 1:
            raise ValueError("positive integer training dimensions required")
        if not 0 <= self.warmup_steps < self.steps:
            raise ValueError("warm-up must fit within the schedule")
        if (not all(math.isfinite(v) for v in (self.learning_rate, self.minimum_lr_ratio, self.weight_decay,
                                               self.clip_grad))
                or self.learning_rate <= 0 or self.clip_grad <= 0 or self.weight_decay < 0
                or not 0 <= self.minimum_lr_ratio <= 1):
            raise ValueError("finite positive learning rate / clip and a valid decay required")
        if self.precision not in ("fp32", "bf16") or self.optimizer_impl not in ("single", "fused"):
            raise ValueError("precision fp32/bf16 and optimizer single/fused")

    def make_optimizer(self, params):
        return torch.optim.AdamW(params, lr=self.learning_rate, weight_decay=self.weight_decay, foreach=False,
                                 fused=self.optimizer_impl == "fused")

    def rate(self, step: int) -> float:
        if step < self.warmup_steps:
            return self.learning_rate * (step + 1) / self.warmup_steps
        frac = (step - self.warmup_steps) / max(1, self.steps - self.warmup_steps - 1)
        return self.learning_rate * (self.minimum_lr_ratio
                                     + (1 - self.minimum_lr_ratio) * (1 + math.cos(math.pi * frac)) / 2)


def frozen_fingerprint(model) -> str:
    h = hashlib.sha256()
    for n, p in model.named_parameters():
        if ".attention.draft." in n:
            continue
        h.update((n + str(tuple(p.shape)) + str(p.dtype)).encode())
        h.update(p.detach().contiguous().cpu().float().numpy().tobytes())
    return h.hexdigest()


class Trainer:
    def __init__(self, model, data: TokenDataset, config: FitConfig = FitConfig()):
        if (data.sequence_length != config.sequence_length or data.vocab_size != model.config.vocab_size
                or config.sequence_length < model.config.block_size):
            raise ValueError("matching data windows and complete draft blocks required")
        if any(p.dtype != torch.float32 for p in model.parameters()):
            raise ValueError("training keeps fp32 parameters (optional bf16 autocast)")
        self.model = model.train_draft_only()
        self.config, self.data = config, data
        self.device = model.embedding.weight.device
        if config.precision == "bf16" and self.device.type != "cuda":
            raise ValueError("bf16 autocast needs CUDA")
        self.parameters = [p for p in model.parameters() if p.requires_grad]
        self.optimizer = config.make_optimizer(self.parameters)
        self.stream = BatchStream(data, config.seed)
        self.anchors_rng = torch.Generator().manual_seed(config.seed + 1)
        self.step = 0
        self.base_fingerprint = frozen_fingerprint(model)

    def _autocast(self):
        return torch.autocast("cuda", dtype=torch.bfloat16) if self.config.precision == "bf16" else nullcontext()

    def _runtime(self) -> dict:
        return {"torch": str(torch.__version__), "device_type": self.device.type,
                "device_name": torch.cuda.get_device_name(self.device) if self.device.type == "cuda" else "cpu",
                "threads": torch.get_num_threads(), "matmul_precision": torch.get_float32_matmul_precision()}

    def _batches(self, stream, rng):
        out = []
        for _ in range(self.config.accumulate):
            tokens = stream.batch(self.config.batch_size)
            anchors = sample_anchors(tokens, self.model.config.block_size, self.config.anchors_per_sequence,
                                     generator=rng)
            out.append((tokens.to(self.device), anchors.to(self.device)))
        return out

    def run(self, until: int | None = None, progress=None) -> list[dict]:
        end = self.config.steps if until is None else until
        if not self.step <= end <= self.config.steps:
            raise ValueError("stop boundary must lie within the schedule")
        records = []
        self.model.train()
        while self.step < end:
            t0 = time.perf_counter()
            metrics = distillation_update(self.model, self._batches(self.stream, self.anchors_rng), self.optimizer,
                                          learning_rate=self.config.rate(self.step), clip_grad=self.config.clip_grad,
                                          chunk_rows=self.config.chunk_rows, autocast=self._autocast)
            self.step += 1
            rec = {"step": self.step, **metrics, "seconds": time.perf_counter() - t0}
            records.append(rec)
            if progress is not None:
                progress(rec)
        return records

    @torch.no_grad()
    def evaluate(self, data: TokenDataset, batches: int = 4) -> float:
        stream = BatchStream(data, self.config.seed + 2)
        rng = torch.Generator().manual_seed(self.config.seed + 3)
        training = self.model.training
        self.model.eval()
        try:
            losses = []
            for _ in range(batches):
                tokens = stream.batch(self.config.batch_size)
                anchors = sample_anchors(tokens, self.model.config.block_size, self.config.anchors_per_sequence,
                                         generator=rng)
                with self._autocast():
                    losses.append(float(distillation_loss(self.model, tokens.to(self.device),
                                                          anchors.to(self.device), chunk_rows=self.config.chunk_rows)))
        finally:
            self.model.train(training)
        return sum(losses) / len(losses)

    def save(self, path) -> None:
        state = {"format": "dual-fit-v1", "config": asdict(self.config), "data_sha256": self.data.fingerprint,
                 "data_stream": self.stream.state_dict(), "anchors_rng": self.anchors_rng.get_state(),
                 "torch_rng": torch.get_rng_state(), "runtime": self._runtime(),
                 "cuda_rng": torch.cuda.get_rng_state(self.device) if self.device.type == "cuda" else None,
                 "base_fingerprint": self.base_fingerprint}
        save_checkpoint(path, self.model, optimizer=self.optimizer, step=self.step, training_state=state)

    @classmethod
    def resume(cls, path, data, *, device="cpu") -> "Trainer":
        model, saved = load_checkpoint(path, device=device)
        state = saved["training_state"]
        if not isinstance(state, dict) or state.get("format") != "dual-fit-v1" or saved["optimizer"] is None:
            raise ValueError("a complete training checkpoint is required")
        if not isinstance(data, TokenDataset):
            data = TokenDataset(data, model.config.vocab_size, state["config"]["sequence_length"])
        if state["data_sha256"] != data.fingerprint:
            raise ValueError("resume training data differs")
        trainer = cls(model, data, FitConfig(**state["config"]))
        if trainer.base_fingerprint != state["base_fingerprint"] or trainer._runtime() != state["runtime"]:
            raise ValueError("resume requires the same runtime and frozen base")
        trainer.optimizer.load_state_dict(saved["optimizer"])
        trainer.stream.load_state_dict(state["data_stream"])
        trainer.anchors_rng.set_state(state["anchors_rng"].cpu())
        torch.set_rng_state(state["torch_rng"].cpu())
        if trainer.device.type == "cuda" and state["cuda_rng"] is not None:
            torch.cuda.set_rng_state(state["cuda_rng"].cpu(), trainer.device)
        trainer.step = int(saved["step"])
        return trainer
