"""Masked-diffusion LLM layer: configs, contracts, the block-diffusion backend, algorithms and VRPO."""

from .backend import DiffusionBackendSnapshot, DiffusionEngineBackend, ModuleLogits
from .config import (DiffusionBlockBeamConfig, DiffusionISConfig, DiffusionMHConfig, DiffusionPowerMHConfig,
                     DiffusionSamplingConfig, VRPOSamplingConfig, diffusion_decision_stage_lengths)
from .types import (DiffusionBackend, DiffusionGenerationRequest, DiffusionSample, DiffusionTraceStep,
                    DiffusionTrajectoryScoreRequest)

__all__ = ["DiffusionBackend", "DiffusionBackendSnapshot", "DiffusionBlockBeamConfig", "DiffusionEngineBackend",
           "DiffusionGenerationRequest", "DiffusionISConfig", "DiffusionMHConfig", "DiffusionPowerMHConfig",
           "DiffusionSample", "DiffusionSamplingConfig", "DiffusionTraceStep", "DiffusionTrajectoryScoreRequest",
           "ModuleLogits", "VRPOSamplingConfig", "diffusion_decision_stage_lengths"]
