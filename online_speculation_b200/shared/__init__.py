"""Model-agnostic algorithm layer: RNG streams, MH kernel, importance weights,
stepwise SIR, SMC resampling, budget allocation, verifiers and metrics."""

from .config import RuntimeConfig, SMCForestConfig, canonical_float
from .importance import (MonteCarloRolloutWeightProvider, ProbabilityObservation, RolloutObservation,
                         TruncatedReplayRolloutWeightProvider, corrected_replay_log_weight, logmeanexp)
from .metrics import (autocorrelation_ess, empirical_distribution, importance_effective_sample_size,
                      total_variation)
from .mh import (MetropolisHastingsDecision, MetropolisHastingsProposal, apply_metropolis_hastings,
                 decide_metropolis_hastings, metropolis_hastings_log_acceptance)
from .rng import SeedStream
from .smc import normalize_smc_log_weights, partition_resampled_reservoirs, systematic_resample
from .stepwise import (StepwiseCandidate, StepwiseGenerationBackend, categorical_index_from_uniform,
                       normalize_log_weights, run_stepwise_generation, select_stepwise_candidate)
from .types import TokenSequence
