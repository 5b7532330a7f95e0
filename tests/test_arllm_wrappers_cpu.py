"""arllm backend wrappers and rewards on the tabular CPU backend."""

import math
import threading

import numpy as np
import pytest

from online_speculation_b200.arllm.backends.absorbing import AbsorbingEOSBackend
from online_speculation_b200.arllm.backends.batching import ContinuousBatchingBackend
from online_speculation_b200.arllm.backends.cache import ScoreCachingBackend
from online_speculation_b200.arllm.backends.candidate_cache import CachedCandidateBackend
from online_speculation_b200.arllm.backends.reference import ReferencePolicyBackend
from online_speculation_b200.arllm.backends.stopping import StoppedSequenceBackend
from online_speculation_b200.arllm.backends.tabular import TabularBackend
from online_speculation_b200.arllm.config import SamplingConfig
from online_speculation_b200.arllm.rewards import ConsilienceReward, SequenceLogProbabilityReward
from online_speculation_b200.arllm.types import GenerationRequest, ScoreRequest
from online_speculation_b200.shared.output import ThinkingFormat

V = 8
EOS = 7


def _tab(seed=0):
    rng = np.random.default_rng(seed)
    table = {}

    def row(prefix):
        key = tuple(prefix[-2:])
        if key not in table:
            table[key] = rng.dirichlet(np.ones(V) * 0.7)
        return table[key]
    return TabularBackend(row, V, model_id="tab")


def test_stopped_sequence_keeps_marker_and_pads_with_eos():
    b = _tab()
    st = StoppedSequenceBackend(b, stop_token_sequences=((3, 4),), eos_token_id=EOS, protected_prefix_length=1,
                                generation_chunk_size=2)
    reqs = [GenerationRequest((1,), 12, SamplingConfig(), seed=s, request_id=str(s)) for s in range(20)]
    for r, s in zip(reqs, st.sample_batch(reqs)):
        toks = s.token_ids
        assert len(toks) == 12
        ends = [i + 2 for i in range(len(toks) - 1) if toks[i:i + 2] == (3, 4)] + [i + 1 for i, t in enumerate(toks)
                                                                                  if t == EOS]
        if ends:
            e = min(ends)
            assert all(t == EOS for t in toks[e:]) and all(v == 0.0 for v in s.token_logprobs[e:])
        sc = st.score_batch([ScoreRequest(r.prefix, (toks,), None)])[0]
        assert sc == pytest.approx(s.token_logprobs)
    bad = st.score_batch([ScoreRequest((1,), ((3, 4, 2),), None)])[0]
    assert bad[2] == -math.inf


def test_absorbing_eos_requires_unset_outer_eos():
    a = AbsorbingEOSBackend(_tab(), EOS)
    with pytest.raises(ValueError):
        a.sample_batch([GenerationRequest((1,), 4, SamplingConfig(eos_token_id=EOS), 0, "x")])
    out = a.sample_batch([GenerationRequest((1,), 6, SamplingConfig(), 0, "x")])[0]
    assert len(out.token_ids) == 6


def test_reference_policy_translates_temperature():
    b = _tab()
    ref = ReferencePolicyBackend(b, temperature=0.5)
    s = ref.sample_batch([GenerationRequest((1,), 4, SamplingConfig(), 3, "r")])[0]
    direct = b.sample_batch([GenerationRequest((1,), 4, SamplingConfig(temperature=0.5), 3, "r")])[0]
    assert s.token_ids == direct.token_ids and s.policy_id == SamplingConfig().policy_id
    assert s.reference_token_logprobs == pytest.approx(direct.token_logprobs)


def test_score_cache_hits_and_candidate_replay():
    b = _tab()
    c = ScoreCachingBackend(b, maximum_entries=2)
    r = ScoreRequest((1,), ((2, 3), (4,)), None)
    first = c.score_batch([r])
    assert c.score_batch([r]) == first and c.snapshot().hits == 2
    c.score_batch([ScoreRequest((1,), ((5,),), None)])
    assert c.snapshot().evictions == 1
    samples = b.sample_batch([GenerationRequest((1,), 3, SamplingConfig(), 0, "cand-0")])
    cc = CachedCandidateBackend(b, samples)
    assert cc.sample_batch([GenerationRequest((1,), 3, SamplingConfig(), 9, "cand-0")]) == samples
    with pytest.raises(KeyError):
        cc.sample_batch([GenerationRequest((1,), 3, SamplingConfig(), 9, "other")])


def test_continuous_batching_merges_threads_without_changing_samples():
    b = _tab()
    cb = ContinuousBatchingBackend(b, max_batch_size=64, batch_wait_seconds=0.05)
    reqs = [[GenerationRequest((1, i), 5, SamplingConfig(), seed=10 * i + j, request_id=f"{i}:{j}") for j in range(3)]
            for i in range(6)]
    got = [None] * 6

    def work(i):
        got[i] = cb.sample_batch(reqs[i])

    ts = [threading.Thread(target=work, args=(i,)) for i in range(6)]
    for t in ts:
        t.start()
    for t in ts:
        t.join()
    for i in range(6):
        assert [s.token_ids for s in got[i]] == [s.token_ids for s in b.sample_batch(reqs[i])]
    snap = cb.snapshot()
    assert snap.sample_requests == 18 and snap.sample_batches < 6
    cb.close()
    with pytest.raises(RuntimeError):
        cb.sample_batch(reqs[0])


def test_consilience_and_logprob_rewards():
    b = _tab(1)
    lp = SequenceLogProbabilityReward(b, scale=0.5)
    assert lp((1,), (2, 3)) == pytest.approx(0.5 * sum(b.score_batch([ScoreRequest((1,), ((2, 3),), None)])[0]))
    r = ConsilienceReward(b, top_k=3, scope="full", window_fraction=0.5, skip_fraction=0.0, initial_penalty=1.0)
    comp = (2, 3, 4, 5)
    stats = b.score_statistics_batch([ScoreRequest((1,), (comp,), None)], confidence_top_k=3)[0]
    c = stats.token_topk_confidences
    assert r((1,), comp) == pytest.approx((c[2] + c[3]) / 2 - (c[0] + c[1]) / 2)
    th = ConsilienceReward(b, top_k=2, thinking_format=ThinkingFormat(end_token_ids=(6,), start_token_ids=(5,)))
    th.batch((1,), [(5, 2, 3, 6, 4), (2, 2)])
    st = th.scope_statistics()
    assert st["thinking_sequences"] == 1 and st["full_sequences"] == 1
