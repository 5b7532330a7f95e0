"""The adaptive speculation policy of the MH engine (decision rule only, no GPU)."""

from types import SimpleNamespace

from online_speculation_b200.engine.mh_engine import MHEngine


def _state(**kw):
    base = dict(spec_policy="adaptive", probe_every=8, plain_steps=1, _t_spec=None, _t_plain=None, _accept_ema=None,
                _since_spec=0)
    base.update(kw)
    return SimpleNamespace(**base)


def test_fixed_policies():
    assert MHEngine._speculate_next(_state(spec_policy="always", _t_spec=9.0, _t_plain=1.0, _accept_ema=1.0))
    assert not MHEngine._speculate_next(_state(spec_policy="never", _t_spec=1.0, _t_plain=9.0, _accept_ema=4.0))


def test_adaptive_measures_both_then_compares_tokens_per_second():
    assert MHEngine._speculate_next(_state())                                  # nothing measured: draft
    assert not MHEngine._speculate_next(_state(_t_spec=9.0, _accept_ema=1.0))  # plain not measured yet
    # 1.01 tokens per 9.3 ms against 1 token per 4.3 ms: plain decoding wins
    assert not MHEngine._speculate_next(_state(_t_spec=9.3, _t_plain=4.3, _accept_ema=1.01, _since_spec=2))
    # 3 tokens per 9.3 ms beats 1 per 4.3 ms
    assert MHEngine._speculate_next(_state(_t_spec=9.3, _t_plain=4.3, _accept_ema=3.0, _since_spec=2))
    # a probe round is due after probe_every - 1 plain rounds
    assert MHEngine._speculate_next(_state(_t_spec=9.3, _t_plain=4.3, _accept_ema=1.01, _since_spec=7))
    # a plain round of 4 chained steps yields 4 tokens per job: 3 tokens per 9.3 ms lose to 4 per 12 ms
    assert not MHEngine._speculate_next(_state(_t_spec=9.3, _t_plain=12.0, _accept_ema=3.0, _since_spec=2,
                                               plain_steps=4))
