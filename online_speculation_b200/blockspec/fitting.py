"""File-backed draft-view fitting with a deterministic data order and bit-exact resume.

* ``TokenDataset``: tokenised JSONL (``{"input_ids": [...]}`` per line) indexed by byte
  offset; a training window never crosses records.
* ``BatchStream``: a seeded permutation walked by a cursor, reshuffled per epoch; its
  state (generator state, permutation, cursor, epoch) is saved with the checkpoint.
* ``FitConfig``: linear warm-up then cosine decay to ``minimum_lr_ratio``, AdamW
  settings and precision.
* ``Trainer``: ``run`` / ``evaluate`` / ``save`` / ``resume``.  Checkpoints are taken at
  optimizer-step boundaries and carry the data cursor, every RNG state, the runtime
  and a fingerprint of the frozen base, so an interrupted run resumes to the weights
  an uninterrupted run reaches.

The training-state payload (``format = "dual-fit-v1"`` and its keys) is the checkpoint
contract of online-speculation/src/blockspec/parallel/fitting.py.
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


def _token_ids(line: bytes, vocab_size: int) -> list[int]:
    ids = json.loads(line).get("input_ids")
    if not (isinstance(ids, list) and ids and all(type(t) is int and 0 <= t < vocab_size for t in ids)):
        raise ValueError("every record needs a non-empty input_ids list of vocabulary ids")
    return ids


class TokenDataset:
    def __init__(self, path, vocab_size: int, sequence_length: int):
        if vocab_size < 1 or sequence_length < 1:
            raise ValueError("vocab_size and sequence_length have to be positive")
        self.path = Path(path).resolve()
        self.vocab_size = vocab_size
        self.sequence_length = sequence_length
        self.offsets = array("Q")
        self.skipped = 0
        offset = 0
        with self.path.open("rb") as handle:
            for line in handle:
                if line.strip():
                    if len(_token_ids(line, vocab_size)) >= sequence_length:
                        self.offsets.append(offset)
                    else:
                        self.skipped += 1
                offset += len(line)
        if not self.offsets:
            raise ValueError(f"{self.path} has no record of at least {sequence_length} tokens")
        self.fingerprint = file_sha256(self.path)

    def __len__(self) -> int:
        return len(self.offsets)

    def __getitem__(self, i: int) -> torch.Tensor:
        with self.path.open("rb") as handle:
            handle.seek(self.offsets[i])
            return torch.tensor(_token_ids(handle.readline(), self.vocab_size), dtype=torch.long)


class BatchStream:
    def __init__(self, dataset: TokenDataset, seed: int):
        self.dataset = dataset
        self.rng = torch.Generator().manual_seed(seed)
        self.order = torch.randperm(len(dataset), generator=self.rng)
        self.cursor = 0
        self.epoch = 0

    def _next_record(self) -> torch.Tensor:
        if self.cursor >= len(self.order):
            self.order = torch.randperm(len(self.dataset), generator=self.rng)
            self.cursor = 0
            self.epoch += 1
        record = self.dataset[int(self.order[self.cursor])]
        self.cursor += 1
        return record

    def batch(self, count: int) -> torch.Tensor:
        width = self.dataset.sequence_length
        windows = []
        for _ in range(count):
            record = self._next_record()
            start = int(torch.randint(record.numel() - width + 1, (), generator=self.rng))
            windows.append(record[start:start + width])
        return torch.stack(windows)

    def state_dict(self) -> dict:
        return {"rng": self.rng.get_state(), "order": self.order.clone(), "cursor": self.cursor, "epoch": self.epoch}

    def load_state_dict(self, state: dict) -> None:
        order = state["order"].cpu()
        n = len(self.dataset)
        is_permutation = order.shape == (n,) and torch.equal(torch.sort(order).values, torch.arange(n))
        if not is_permutation or not 0 <= state["cursor"] <= n or state["epoch"] < 0:
            raise ValueError("the saved data stream does not fit this dataset")
        self.rng.set_state(state["rng"].cpu())
        self.order = order
        self.cursor = state["cursor"]
        self.epoch = state["epoch"]


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
        counts = (self.steps, self.batch_size, self.sequence_length, self.anchors_per_sequence, self.accumulate,
                  self.chunk_rows)
        scales = (self.learning_rate, self.minimum_lr_ratio, self.weight_decay, self.clip_grad)
        checks = (
            (min(counts) >= 1, "step, batch, window, anchor, accumulation and chunk counts must be positive"),
            (0 <= self.warmup_steps < self.steps, "the warm-up must end before the last step"),
            (all(math.isfinite(v) for v in scales), "optimizer scales must be finite"),
            (self.learning_rate > 0 and self.clip_grad > 0, "learning_rate and clip_grad must be positive"),
            (self.weight_decay >= 0 and 0 <= self.minimum_lr_ratio <= 1, "weight decay >= 0, min ratio in [0, 1]"),
            (self.precision in ("fp32", "bf16"), "precision is fp32 or bf16"),
            (self.optimizer_impl in ("single", "fused"), "optimizer_impl is single or fused"),
        )
        failed = [message for ok, message in checks if not ok]
        if failed:
            raise ValueError("invalid fit config: " + "; ".join(failed))

    def make_optimizer(self, params):
        return torch.optim.AdamW(params, lr=self.learning_rate, weight_decay=self.weight_decay, foreach=False,
                                 fused=self.optimizer_impl == "fused")

    def rate(self, step: int) -> float:
        if step < self.warmup_steps:
            return self.learning_rate * (step + 1) / self.warmup_steps
        progress = (step - self.warmup_steps) / max(1, self.steps - self.warmup_steps - 1)
        cosine = 0.5 * (1.0 + math.cos(math.pi * progress))
        return self.learning_rate * (self.minimum_lr_ratio + (1.0 - self.minimum_lr_ratio) * cosine)


def frozen_fingerprint(model) -> str:
    """SHA-256 over the names, shapes, dtypes and values of every non-draft parameter."""
    digest = hashlib.sha256()
    for name, p in model.named_parameters():
        if ".attention.draft." not in name:
            digest.update(f"{name}{tuple(p.shape)}{p.dtype}".encode())
            digest.update(p.detach().float().cpu().contiguous().numpy().tobytes())
    return digest.hexdigest()


class Trainer:
    def __init__(self, model, data: TokenDataset, config: FitConfig = FitConfig()):
        if data.sequence_length != config.sequence_length or data.vocab_size != model.config.vocab_size:
            raise ValueError("the dataset's window and vocabulary must match the config and model")
        if config.sequence_length < model.config.block_size:
            raise ValueError("a training window must hold at least one draft block")
        if any(p.dtype != torch.float32 for p in model.parameters()):
            raise ValueError("parameters stay fp32 during fitting (bf16 runs through autocast)")
        self.model = model.train_draft_only()
        self.config = config
        self.data = data
        self.device = model.embedding.weight.device
        if config.precision == "bf16" and self.device.type != "cuda":
            raise ValueError("bf16 autocast runs on CUDA only")
        self.parameters = [p for p in model.parameters() if p.requires_grad]
        self.optimizer = config.make_optimizer(self.parameters)
        self.stream = BatchStream(data, config.seed)
        self.anchors_rng = torch.Generator().manual_seed(config.seed + 1)
        self.step = 0
        self.base_fingerprint = frozen_fingerprint(model)

    def _autocast(self):
        return torch.autocast("cuda", dtype=torch.bfloat16) if self.config.precision == "bf16" else nullcontext()

    def _runtime(self) -> dict:
        on_cuda = self.device.type == "cuda"
        return {"torch": str(torch.__version__), "device_type": self.device.type,
                "device_name": torch.cuda.get_device_name(self.device) if on_cuda else "cpu",
                "threads": torch.get_num_threads(), "matmul_precision": torch.get_float32_matmul_precision()}

    def _micro_batch(self, stream: BatchStream, rng: torch.Generator):
        tokens = stream.batch(self.config.batch_size)
        anchors = sample_anchors(tokens, self.model.config.block_size, self.config.anchors_per_sequence,
                                 generator=rng)
        return tokens.to(self.device), anchors.to(self.device)

    def run(self, until: int | None = None, progress=None) -> list[dict]:
        end = self.config.steps if until is None else until
        if not self.step <= end <= self.config.steps:
            raise ValueError(f"cannot run from step {self.step} to {end} of {self.config.steps}")
        self.model.train()
        history = []
        while self.step < end:
            started = time.perf_counter()
            batches = [self._micro_batch(self.stream, self.anchors_rng) for _ in range(self.config.accumulate)]
            metrics = distillation_update(self.model, batches, self.optimizer, learning_rate=self.config.rate(self.step),
                                          clip_grad=self.config.clip_grad, chunk_rows=self.config.chunk_rows,
                                          autocast=self._autocast)
            self.step += 1
            record = {"step": self.step, **metrics, "seconds": time.perf_counter() - started}
            history.append(record)
            if progress is not None:
                progress(record)
        return history

    @torch.no_grad()
    def evaluate(self, data: TokenDataset, batches: int = 4) -> float:
        stream = BatchStream(data, self.config.seed + 2)
        rng = torch.Generator().manual_seed(self.config.seed + 3)
        was_training = self.model.training
        self.model.eval()
        total = 0.0
        try:
            for _ in range(batches):
                tokens, anchors = self._micro_batch(stream, rng)
                with self._autocast():
                    total += float(distillation_loss(self.model, tokens, anchors, chunk_rows=self.config.chunk_rows))
        finally:
            self.model.train(was_training)
        return total / batches

    def save(self, path) -> None:
        cuda_rng = torch.cuda.get_rng_state(self.device) if self.device.type == "cuda" else None
        state = {"format": "dual-fit-v1", "config": asdict(self.config), "data_sha256": self.data.fingerprint,
                 "data_stream": self.stream.state_dict(), "anchors_rng": self.anchors_rng.get_state(),
                 "torch_rng": torch.get_rng_state(), "runtime": self._runtime(), "cuda_rng": cuda_rng,
                 "base_fingerprint": self.base_fingerprint}
        save_checkpoint(path, self.model, optimizer=self.optimizer, step=self.step, training_state=state)

    @classmethod
    def resume(cls, path, data, *, device="cpu") -> "Trainer":
        model, saved = load_checkpoint(path, device=device)
        state = saved["training_state"]
        if not isinstance(state, dict) or state.get("format") != "dual-fit-v1" or saved["optimizer"] is None:
            raise ValueError(f"{path} is not a resumable dual-fit-v1 training checkpoint")
        if not isinstance(data, TokenDataset):
            data = TokenDataset(data, model.config.vocab_size, state["config"]["sequence_length"])
        if state["data_sha256"] != data.fingerprint:
            raise ValueError("the training data changed since the checkpoint was written")
        trainer = cls(model, data, FitConfig(**state["config"]))
        if trainer.base_fingerprint != state["base_fingerprint"]:
            raise ValueError("the frozen base weights changed since the checkpoint was written")
        if trainer._runtime() != state["runtime"]:
            raise ValueError("bit-exact resume needs the runtime the checkpoint was written with")
        trainer.optimizer.load_state_dict(saved["optimizer"])
        trainer.stream.load_state_dict(state["data_stream"])
        trainer.anchors_rng.set_state(state["anchors_rng"].cpu())
        torch.set_rng_state(state["torch_rng"].cpu())
        if trainer.device.type == "cuda" and state["cuda_rng"] is not None:
            torch.cuda.set_rng_state(state["cuda_rng"].cpu(), trainer.device)
        trainer.step = int(saved["step"])
        return trainer
