"""Model-independent Metropolis--Hastings transition kernel.

Backends build the current/proposed target log densities and the forward /
reverse proposal log-probabilities; this module does the accept/reject with an
explicit uniform so the decision is reproducible
(reference: src/inference_scaling/shared/mh.py:20-137).
"""

from __future__ import annotations

from dataclasses import dataclass
from math import exp, isfinite, log
from sys import float_info
from typing import Generic, TypeVar

StateT = TypeVar("StateT")


@dataclass(frozen=True, slots=True)
class MetropolisHastingsProposal(Generic[StateT]):
    state: StateT
    current_target_log_density: float
    proposed_target_log_density: float
    forward_proposal_log_probability: float = 0.0
    reverse_proposal_log_probability: float = 0.0

    @property
    def log_hastings_ratio(self) -> float:
        return (self.proposed_target_log_density - self.current_target_log_density
                + self.reverse_proposal_log_probability - self.forward_proposal_log_probability)


@dataclass(frozen=True, slots=True)
class MetropolisHastingsDecision:
    log_acceptance: float
    acceptance_probability: float
    accepted: bool


@dataclass(frozen=True, slots=True)
class MetropolisHastingsTransition(Generic[StateT]):
    previous_state: StateT
    proposal: MetropolisHastingsProposal[StateT]
    state: StateT
    decision: MetropolisHastingsDecision


def metropolis_hastings_log_acceptance(*, current_target_log_density: float, proposed_target_log_density: float,
                                       forward_proposal_log_probability: float = 0.0,
                                       reverse_proposal_log_probability: float = 0.0) -> float:
    terms = (current_target_log_density, proposed_target_log_density, forward_proposal_log_probability,
             reverse_proposal_log_probability)
    if not all(isfinite(float(t)) for t in terms):
        raise ValueError("MH target and proposal log terms must be finite")
    ratio = (float(proposed_target_log_density) - float(current_target_log_density)
             + float(reverse_proposal_log_probability) - float(forward_proposal_log_probability))
    return min(0.0, ratio)


def decide_metropolis_hastings(*, current_target_log_density: float, proposed_target_log_density: float,
                               uniform: float, forward_proposal_log_probability: float = 0.0,
                               reverse_proposal_log_probability: float = 0.0) -> MetropolisHastingsDecision:
    u = float(uniform)
    if not isfinite(u) or not 0.0 <= u < 1.0:
        raise ValueError("MH uniform variate must lie in [0, 1)")
    log_a = metropolis_hastings_log_acceptance(
        current_target_log_density=current_target_log_density,
        proposed_target_log_density=proposed_target_log_density,
        forward_proposal_log_probability=forward_proposal_log_probability,
        reverse_proposal_log_probability=reverse_proposal_log_probability,
    )
    return MetropolisHastingsDecision(log_a, exp(log_a), log(max(u, float_info.min)) <= log_a)


def apply_metropolis_hastings(current_state: StateT, proposal: MetropolisHastingsProposal[StateT], *,
                              uniform: float) -> MetropolisHastingsTransition[StateT]:
    decision = decide_metropolis_hastings(
        current_target_log_density=proposal.current_target_log_density,
        proposed_target_log_density=proposal.proposed_target_log_density,
        forward_proposal_log_probability=proposal.forward_proposal_log_probability,
        reverse_proposal_log_probability=proposal.reverse_proposal_log_probability,
        uniform=uniform,
    )
    return MetropolisHastingsTransition(current_state, proposal,
                                        proposal.state if decision.accepted else current_state, decision)
