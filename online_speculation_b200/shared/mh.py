"""Metropolis--Hastings accept/reject, scalar and batched.

The suffix-MH engines decide many chains at once, so the primitive here is
:func:`mh_log_acceptance_batch`, which evaluates ``min(0, log pi(y) - log pi(x) +
log q(x|y) - log q(y|x))`` over arrays; the scalar helpers used by the
sequential algorithms are thin views of it.  A decision compares ``log u`` with
the log acceptance for an explicit uniform ``u``, so it is reproducible from the
uniform's random stream alone.  The public types and keyword names follow
src/inference_scaling/shared/mh.py (the algorithm contract).
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Generic, TypeVar

import numpy as np

StateT = TypeVar("StateT")

_TINY = np.finfo(np.float64).tiny


def mh_log_acceptance_batch(current, proposed, forward=0.0, reverse=0.0) -> np.ndarray:
    """Elementwise log acceptance probabilities (float64 arrays broadcast together)."""
    terms = np.broadcast_arrays(*(np.asarray(t, dtype=np.float64) for t in (current, proposed, forward, reverse)))
    if not all(np.isfinite(t).all() for t in terms):
        raise ValueError("every target and proposal log term of an MH step has to be finite")
    cur, prop, fwd, rev = terms
    return np.minimum(0.0, (prop - cur) + (rev - fwd))


def mh_accept_batch(log_acceptance, uniforms) -> np.ndarray:
    """Boolean decisions ``log(u) <= log_acceptance`` for uniforms in [0, 1)."""
    u = np.asarray(uniforms, dtype=np.float64)
    if not (np.isfinite(u).all() and (u >= 0.0).all() and (u < 1.0).all()):
        raise ValueError("MH decisions need uniforms in [0, 1)")
    return np.log(np.maximum(u, _TINY)) <= np.asarray(log_acceptance, dtype=np.float64)


@dataclass(frozen=True, slots=True)
class MetropolisHastingsProposal(Generic[StateT]):
    state: StateT
    current_target_log_density: float
    proposed_target_log_density: float
    forward_proposal_log_probability: float = 0.0
    reverse_proposal_log_probability: float = 0.0

    @property
    def log_hastings_ratio(self) -> float:
        return float((self.proposed_target_log_density - self.current_target_log_density)
                     + (self.reverse_proposal_log_probability - self.forward_proposal_log_probability))


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
    return float(mh_log_acceptance_batch(current_target_log_density, proposed_target_log_density,
                                         forward_proposal_log_probability, reverse_proposal_log_probability))


def decide_metropolis_hastings(*, current_target_log_density: float, proposed_target_log_density: float,
                               uniform: float, forward_proposal_log_probability: float = 0.0,
                               reverse_proposal_log_probability: float = 0.0) -> MetropolisHastingsDecision:
    log_a = mh_log_acceptance_batch(current_target_log_density, proposed_target_log_density,
                                    forward_proposal_log_probability, reverse_proposal_log_probability)
    accepted = bool(mh_accept_batch(log_a, uniform))
    return MetropolisHastingsDecision(float(log_a), float(np.exp(log_a)), accepted)


def apply_metropolis_hastings(current_state: StateT, proposal: MetropolisHastingsProposal[StateT], *,
                              uniform: float) -> MetropolisHastingsTransition[StateT]:
    decision = decide_metropolis_hastings(
        current_target_log_density=proposal.current_target_log_density,
        proposed_target_log_density=proposal.proposed_target_log_density,
        forward_proposal_log_probability=proposal.forward_proposal_log_probability,
        reverse_proposal_log_probability=proposal.reverse_proposal_log_probability,
        uniform=uniform)
    kept = proposal.state if decision.accepted else current_state
    return MetropolisHastingsTransition(current_state, proposal, kept, decision)
