"""Policy training on the sm_100a kernels: GRPO (autoregressive decoders)."""

from .grpo import GRPOConfig, GRPOTrainer, group_advantages, grpo_loss

__all__ = ["GRPOConfig", "GRPOTrainer", "group_advantages", "grpo_loss"]
