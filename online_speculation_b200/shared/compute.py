"""Token and dominant-matmul FLOP accounting (reference: src/inference_scaling/shared/compute.py:10-234).

``dense_forward_flops`` is the usual 2 x parameters x token-slots forward estimate.  The GRPO
estimate charges every model pass of a training run in forward-equivalent token slots:

* rollout generation feeds every prompt and completion token except each completion's last
  (that token is sampled, never fed);
* the frozen reference scores the whole sequence once when the KL coefficient is non-zero;
* the policy update is one forward pass, one activation-gradient pass and one weight-gradient
  pass over the trainable share of the weights (plus one recomputed forward with activation
  checkpointing);
* the optimizer is charged per trainable parameter and step: 14 flops for the fused AdamW
  update (clip scale, decoupled decay, two moment updates, bias corrections, square root,
  division, step) and 2 for the global gradient norm.

The report keys of :class:`GRPOComputeEstimate` are the reference's, so compute summaries of
both implementations line up.
"""

from __future__ import annotations

from collections.abc import Mapping, Sequence
from dataclasses import asdict, dataclass
from typing import Any

ADAMW_FLOPS_PER_PARAMETER = 16


def dense_forward_flops(parameter_count: int, forward_token_slots: int) -> int:
    """Conventional 2 * parameters * tokens forward estimate."""
    if parameter_count < 0 or forward_token_slots < 0:
        raise ValueError("parameter_count and forward_token_slots must be non-negative")
    return 2 * parameter_count * forward_token_slots


def training_step_flops(parameter_count: int, tokens: int, *, trainable_fraction: float = 1.0,
                        recompute: bool = False) -> int:
    """Forward (2N) + backward (2N for activations + 2N*trainable for weights) per token."""
    passes = 2.0 + 2.0 + 2.0 * trainable_fraction + (2.0 if recompute else 0.0)
    return int(passes * parameter_count * tokens)


@dataclass(frozen=True, slots=True)
class GRPOComputeEstimate:
    trainer_observed_prompt_plus_completion_tokens: int
    generated_completions: int
    rollout_generation_forward_token_slots: int
    reference_scoring_forward_token_slots: int
    policy_forward_backward_equivalent_token_slots: int
    total_forward_equivalent_token_slots: int
    total_parameters: int
    trainable_parameters: int
    optimizer_steps: int
    estimated_dense_model_flops: int
    estimated_optimizer_flops: int
    estimated_total_flops: int
    estimated_total_petaflops: float
    accounting_basis: str
    definition: str
    exclusions: str

    def as_dict(self) -> dict[str, Any]:
        return asdict(self)


def estimate_grpo_compute(*, model_sequence_tokens: int, generated_completions: int, total_parameters: int,
                          trainable_parameters: int, optimizer_steps: int, reference_scoring: bool,
                          recompute: bool = False) -> GRPOComputeEstimate:
    """Estimate a GRPO run from its prompt + completion token count and completion count."""
    counts = (model_sequence_tokens, generated_completions, total_parameters, trainable_parameters, optimizer_steps)
    if min(counts) < 0:
        raise ValueError("GRPO compute inputs must be non-negative")
    if generated_completions > model_sequence_tokens:
        raise ValueError("every completion holds at least one model token")
    if trainable_parameters > total_parameters:
        raise ValueError("trainable parameters are a part of all parameters")
    rollout = model_sequence_tokens - generated_completions
    reference = model_sequence_tokens if reference_scoring else 0
    share = trainable_parameters / total_parameters if total_parameters else 0.0
    # forward + activation gradients (+ recomputed forward), in whole passes; weight gradients by share
    whole = model_sequence_tokens * (3 if recompute else 2)
    policy = whole + int(round(share * model_sequence_tokens))
    total = rollout + reference + policy
    dense = dense_forward_flops(total_parameters, total)
    optimizer = ADAMW_FLOPS_PER_PARAMETER * trainable_parameters * optimizer_steps
    return GRPOComputeEstimate(
        model_sequence_tokens, generated_completions, rollout, reference, policy, total, total_parameters,
        trainable_parameters, optimizer_steps, dense, optimizer, dense + optimizer, (dense + optimizer) / 1e15,
        accounting_basis="prompt + completion tokens and completions counted by the trainer's step records",
        definition=("forward-equivalent token slots: rollout feeds all tokens but each completion's last; the "
                    "reference scores every token once when beta > 0; the policy update is a forward and an "
                    "activation-gradient pass plus a weight-gradient pass over the trainable share (and a "
                    "recomputed forward under checkpointing); dense FLOPs = 2 x parameters x slots; the "
                    f"optimizer is {ADAMW_FLOPS_PER_PARAMETER} flops per trainable parameter and step"),
        exclusions="attention score FLOPs, elementwise kernels, sampling, collectives, reward and host work")


def estimate_grpo_compute_from_steps(records: Sequence[Mapping[str, Any]], *, total_parameters: int,
                                     trainable_parameters: int, reference_scoring: bool, world: int = 1,
                                     recompute: bool = False) -> GRPOComputeEstimate:
    """The estimate over a run's per-step records (``tokens`` and ``completions`` per rank)."""
    if world < 1:
        raise ValueError("world must be positive")
    tokens = sum(int(r["tokens"]) for r in records) * world
    completions = sum(int(r["completions"]) for r in records) * world
    return estimate_grpo_compute(model_sequence_tokens=tokens, generated_completions=completions,
                                 total_parameters=total_parameters, trainable_parameters=trainable_parameters,
                                 optimizer_steps=len(records), reference_scoring=reference_scoring,
                                 recompute=recompute)
