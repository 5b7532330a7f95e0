"""dLLM inference-scaling algorithms over the ``DiffusionBackend`` contract."""

from .is_sampling import (DiffusionConditionalISResult, DiffusionSIRResult, DiffusionStepwiseAdapter,
                          resample_diffusion_candidates, run_conditional_diffusion_is)
from .mh import DiffusionMHResult, run_diffusion_reward_mh
from .mh_acceleration import run_diffusion_replay_mixture_mh, run_diffusion_reward_mh_delayed
from .progressive_is import run_progressive_diffusion_is
from .search import run_diffusion_block_beam, run_diffusion_trajectory_power_mh
from .smc_forest import run_diffusion_smc_rollout_forest

__all__ = ["DiffusionConditionalISResult", "DiffusionMHResult", "DiffusionSIRResult", "DiffusionStepwiseAdapter",
           "resample_diffusion_candidates", "run_conditional_diffusion_is", "run_diffusion_block_beam",
           "run_diffusion_replay_mixture_mh", "run_diffusion_reward_mh", "run_diffusion_reward_mh_delayed",
           "run_diffusion_smc_rollout_forest", "run_diffusion_trajectory_power_mh", "run_progressive_diffusion_is"]
