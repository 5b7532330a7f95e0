"""CPU tests of the engine backend's draft-acceptance rule and the speculation config table
(reference: transformers_backend.py:468-642, loader.py:81-116)."""

import pytest

from online_speculation_b200.arllm.acceleration import ActiveBatchSpeculationConfig, SpeculationTier
from online_speculation_b200.arllm.backends.loader import speculation_from_config
from online_speculation_b200.engine.backend import draft_acceptance


def test_draft_acceptance_rule():
    # whole draft matches: the draw after it is kept too
    assert draft_acceptance((5, 6, 7), (5, 6, 7, 9), room=10, eos=None) == (4, 3, False)
    # first mismatch is kept and ends the run
    assert draft_acceptance((5, 6, 7), (5, 8, 7, 9), room=10, eos=None) == (2, 1, False)
    assert draft_acceptance((5, 6, 7), (4, 6, 7, 9), room=10, eos=None) == (1, 0, False)
    # EOS ends the run, matched or not
    assert draft_acceptance((5, 0, 7), (5, 0, 7, 9), room=10, eos=0) == (2, 2, True)
    assert draft_acceptance((5, 6, 7), (5, 0, 7, 9), room=10, eos=0) == (2, 1, True)
    assert draft_acceptance((5, 6), (5, 6, 0), room=10, eos=0) == (3, 2, True)
    # budget: no draw past the request's remaining tokens
    assert draft_acceptance((5, 6, 7), (5, 6, 7, 9), room=3, eos=None) == (3, 3, False)
    assert draft_acceptance((5, 6, 7), (5, 6, 7, 9), room=2, eos=None) == (2, 2, False)
    assert draft_acceptance((5, 6, 7), (5, 6, 7, 9), room=1, eos=None) == (1, 1, False)


def test_speculation_from_config():
    assert speculation_from_config({}) is None
    assert speculation_from_config({"acceleration": {"speculation": {"enabled": False}}}) is None
    cfg = speculation_from_config({"acceleration": {"speculation": {
        "enabled": True, "tiers": [[2, 6], [64, 0]], "stochastic_tree": True, "min_token_probability": 0.2}}})
    assert isinstance(cfg, ActiveBatchSpeculationConfig)
    assert cfg.tiers == (SpeculationTier(2, 6), SpeculationTier(64, 0))
    assert cfg.stochastic_tree and cfg.min_token_probability == 0.2
    assert cfg.draft_tokens(1) == 6 and cfg.draft_tokens(3) == 0
    with pytest.raises(ValueError):
        speculation_from_config({"acceleration": {"speculation": {"enabled": True, "bogus": 1}}})
    with pytest.raises(ValueError):
        speculation_from_config({"acceleration": {"speculation": {"enabled": True, "tiers": [[1]]}}})
