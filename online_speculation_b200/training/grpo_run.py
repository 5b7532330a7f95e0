"""A resumable GRPO run: output directory, run manifest, checkpoint-N directories.

Layout of ``output``:

* ``run_manifest.json`` -- status (initializing / training / interrupted /
  completed), the effective settings and their ``resume_fingerprint``: a SHA-256
  over the model shape, the GRPO hyper-parameters, the world size, the seed and
  the digest of the initial weights, without the step-count fields
  (``max_steps``, ``save_steps``, ``logging_steps``), so a run can be extended
  but not silently continued with different data or hyper-parameters;
* ``checkpoint-N/rank{r}.pt`` every ``save_steps`` steps (and at the end): each
  rank's fp32 master shard, AdamW moments, step and data RNG
  (:meth:`GRPOTrainer.state_dict`), plus ``trainer_state.json`` (step, log);
* ``log.jsonl`` -- one record per step.

``resume="auto"`` continues from the highest ``checkpoint-N``; a path resumes
from that directory; ``"none"`` starts fresh.  A manifest whose fingerprint
differs from the new run's is refused.  The directory rules follow
experiments/arllm/train_gsm8k_grpo.py:161-169 (latest checkpoint),
:201-206 (fingerprint without the step-count fields) and :311-318 (refusal).
"""

from __future__ import annotations

import argparse
import dataclasses
import hashlib
import json
import os
import time
from pathlib import Path

import torch

from ..models.decoder import DecoderConfig, random_state_dict
from .grpo import GRPOConfig, GRPOTrainer

STEP_COUNT_FIELDS = ("max_steps", "save_steps", "logging_steps")


def latest_checkpoint(output: Path) -> Path | None:
    best = None
    for path in Path(output).glob("checkpoint-*"):
        suffix = path.name.rsplit("-", 1)[-1]
        if path.is_dir() and suffix.isdigit() and (best is None or int(suffix) > best[0]):
            best = (int(suffix), path)
    return None if best is None else best[1]


def weights_digest(state_dict: dict) -> str:
    digest = hashlib.sha256()
    for name in sorted(state_dict):
        t = state_dict[name].detach().contiguous().cpu()
        digest.update(f"{name}{tuple(t.shape)}{t.dtype}".encode())
        digest.update(t.view(torch.uint8).numpy().tobytes() if t.dtype == torch.bfloat16 else t.numpy().tobytes())
    return digest.hexdigest()


def resume_fingerprint(effective: dict) -> str:
    stable = json.loads(json.dumps(effective, sort_keys=True))
    for key in STEP_COUNT_FIELDS:
        stable.get("training", {}).pop(key, None)
    return hashlib.sha256(json.dumps(stable, sort_keys=True).encode()).hexdigest()


def _write_json(path: Path, value) -> None:
    tmp = path.with_suffix(path.suffix + ".tmp")
    tmp.write_text(json.dumps(value, indent=2, sort_keys=True) + "\n", encoding="utf-8")
    os.replace(tmp, path)


class GRPORun:
    """Drive :class:`GRPOTrainer` for ``max_steps`` steps with checkpoints and auto-resume.

    ``data`` (optional) maps a step index to (ids, mask, rewards) for this rank and
    replaces the trainer's own rollouts (synthetic or offline data).
    """

    def __init__(self, output, model: DecoderConfig, config: GRPOConfig, *, max_steps: int, save_steps: int = 25,
                 logging_steps: int = 1, resume: str = "auto", group=None, device=None, seed: int = 0,
                 trainer_kwargs: dict | None = None, data=None, power_monitor: bool = False):
        if max_steps < 1 or save_steps < 1 or logging_steps < 1:
            raise ValueError("max_steps, save_steps and logging_steps are positive")
        self.output = Path(output)
        self.max_steps, self.save_steps, self.logging_steps = max_steps, save_steps, logging_steps
        self.group = group
        self.data = data
        self.power_monitor = power_monitor       # nvidia-smi power / utilisation summary in the manifest
        initial = random_state_dict(model, seed=seed, device="cpu")
        self.effective = {
            "model": dataclasses.asdict(model),
            "grpo": {k: list(v) if isinstance(v, tuple) else v for k, v in dataclasses.asdict(config).items()},
            "training": {"max_steps": max_steps, "save_steps": save_steps, "logging_steps": logging_steps,
                         "seed": seed, "data": "given" if data is not None else "rollouts"},
            "world_size": self._world(),
            "initial_weights_sha256": weights_digest(initial),
        }
        self.fingerprint = resume_fingerprint(self.effective)
        self.rank = self._rank()
        self.output.mkdir(parents=True, exist_ok=True)
        manifest_path = self.output / "run_manifest.json"
        if manifest_path.is_file():
            previous = json.loads(manifest_path.read_text(encoding="utf-8"))
            if previous.get("resume_fingerprint") != self.fingerprint:
                raise ValueError(f"{self.output} was created with different data or hyper-parameters; "
                                 "choose a new output directory")
        self.manifest_path = manifest_path
        self.manifest = {"schema_version": 1, "status": "initializing", "resume_fingerprint": self.fingerprint,
                         "effective": self.effective}
        self._barrier()
        if self.rank == 0:
            _write_json(manifest_path, self.manifest)
        kwargs = dict(trainer_kwargs or {})
        kwargs.setdefault("rollouts", data is None)
        self.trainer = GRPOTrainer(model, config, group=group, device=device, seed=seed,
                                   state_dict={k: v.to(device or "cpu") for k, v in initial.items()}, **kwargs)
        self.resumed_from = None
        checkpoint = (None if resume == "none" else latest_checkpoint(self.output) if resume == "auto"
                      else Path(resume))
        if checkpoint is not None:
            if not checkpoint.is_dir():
                raise FileNotFoundError(checkpoint)
            self._load(checkpoint)
        self.log: list[dict] = []

    # ---- process group helpers ----
    def _world(self) -> int:
        if self.group is None:
            return 1
        import torch.distributed as dist

        return dist.get_world_size(self.group)

    def _rank(self) -> int:
        if self.group is None:
            return 0
        import torch.distributed as dist

        return dist.get_rank(self.group)

    def _barrier(self) -> None:
        if self.group is not None:
            import torch.distributed as dist

            dist.barrier(group=self.group)

    # ---- checkpoints ----
    def _load(self, checkpoint: Path) -> None:
        state = torch.load(checkpoint / f"rank{self.rank}.pt", map_location="cpu", weights_only=False)
        if state.get("fingerprint") != self.fingerprint:
            raise ValueError(f"{checkpoint} belongs to a run with different data or hyper-parameters")
        self.trainer.load_state_dict(state["trainer"])
        self.resumed_from = str(checkpoint)

    def save(self) -> Path:
        step = self.trainer.step_count
        path = self.output / f"checkpoint-{step}"
        if self.rank == 0:
            path.mkdir(parents=True, exist_ok=True)
        self._barrier()
        path.mkdir(parents=True, exist_ok=True)
        tmp = path / f"rank{self.rank}.pt.tmp"
        torch.save({"fingerprint": self.fingerprint, "trainer": self.trainer.state_dict()}, tmp)
        os.replace(tmp, path / f"rank{self.rank}.pt")
        self._barrier()
        if self.rank == 0:
            _write_json(path / "trainer_state.json", {"step": step, "log": self.log[-self.save_steps:]})
        return path

    # ---- training ----
    def _set_status(self, status: str, **extra) -> None:
        if self.rank == 0:
            self.manifest.update(status=status, **extra)
            _write_json(self.manifest_path, self.manifest)

    def train(self) -> list[dict]:
        tr = self.trainer
        self._set_status("training", resume_from_checkpoint=self.resumed_from)
        started = time.perf_counter()
        monitor = None
        if self.power_monitor and tr.device.type == "cuda":
            from ..utils.power import PowerMonitor

            monitor = PowerMonitor(tr.device.index if tr.device.index is not None else 0).start()
        try:
            while tr.step_count < self.max_steps:
                if self.data is None:
                    record = tr.step()
                else:
                    ids, mask, rewards = self.data(tr.step_count)
                    record = tr.train_on(ids, mask, rewards)
                    record["step"] = tr.step_count
                self.log.append(record)
                if self.rank == 0 and tr.step_count % self.logging_steps == 0:
                    with (self.output / "log.jsonl").open("a", encoding="utf-8") as handle:
                        handle.write(json.dumps(record, sort_keys=True) + "\n")
                if tr.step_count % self.save_steps == 0:
                    self.save()
        except BaseException:
            extra = {"power": monitor.stop()} if monitor is not None else {}
            self._set_status("interrupted", elapsed_before_interruption_seconds=time.perf_counter() - started,
                             **extra)
            raise
        if latest_checkpoint(self.output) != self.output / f"checkpoint-{tr.step_count}":
            self.save()
        extra = {"power": monitor.stop()} if monitor is not None else {}
        if self.log and all("tokens" in r and "completions" in r for r in self.log):
            from ..shared.compute import estimate_grpo_compute_from_steps

            n = tr.params.trainable
            extra["compute"] = estimate_grpo_compute_from_steps(
                self.log, total_parameters=n, trainable_parameters=n, reference_scoring=tr.config.beta > 0,
                world=tr.world).as_dict()
        self._set_status("completed", train_seconds=time.perf_counter() - started, final_step=tr.step_count,
                         **extra)
        return self.log

    def close(self) -> None:
        self.trainer.close()


def main(argv=None) -> None:
    """GRPO on a named decoder shape with synthetic prompts and Bernoulli(0.5) rewards."""
    from ..models.decoder import PRESETS

    p = argparse.ArgumentParser(description=main.__doc__)
    p.add_argument("--output", required=True)
    p.add_argument("--model", default="qwen2.5-1.5b", choices=sorted(PRESETS))
    p.add_argument("--max-steps", type=int, default=100)
    p.add_argument("--save-steps", type=int, default=25)
    p.add_argument("--resume", default="auto", help="auto | none | a checkpoint directory")
    p.add_argument("--group-size", type=int, default=8)
    p.add_argument("--prompts-per-rank", type=int, default=1)
    p.add_argument("--prompt-length", type=int, default=256)
    p.add_argument("--completion-length", type=int, default=512)
    p.add_argument("--learning-rate", type=float, default=1e-6)
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--power-monitor", action="store_true", help="record nvidia-smi power / utilisation samples")
    args = p.parse_args(argv)
    group = None
    if int(os.environ.get("WORLD_SIZE", "1")) > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600))
        group = dist.group.WORLD
    config = GRPOConfig(group_size=args.group_size, prompts_per_rank=args.prompts_per_rank,
                        prompt_length=args.prompt_length, completion_length=args.completion_length,
                        learning_rate=args.learning_rate, seed=args.seed)
    run = GRPORun(args.output, PRESETS[args.model], config, max_steps=args.max_steps, save_steps=args.save_steps,
                  resume=args.resume, group=group, seed=args.seed, power_monitor=args.power_monitor)
    try:
        run.train()
    finally:
        run.close()
        if group is not None:
            import torch.distributed as dist

            dist.destroy_process_group()


if __name__ == "__main__":
    main()
