"""Host-side race tests (the sanitizer substitute for the threaded wrappers): many threads drive
the continuous-batching wrapper, the score cache and the rollout token tree at once, mixing
sample, score and observe calls; every result must equal the serial result on the exact tabular
backend, every call must finish within a deadline, and the counters must add up."""

import random
import threading

from online_speculation_b200.arllm.acceleration import RolloutTokenTree
from online_speculation_b200.arllm.backends.batching import ContinuousBatchingBackend
from online_speculation_b200.arllm.backends.cache import ScoreCachingBackend
from online_speculation_b200.arllm.backends.tabular import TabularBackend
from online_speculation_b200.arllm.config import SamplingConfig
from online_speculation_b200.arllm.types import GenerationRequest, ScoreRequest

THREADS, CALLS = 12, 25


def _work(seed):
    rng = random.Random(seed)
    out = []
    for c in range(CALLS):
        prefix = tuple(rng.randrange(16) for _ in range(rng.randint(1, 4)))
        pol = SamplingConfig(temperature=rng.choice((0.7, 1.0, 1.3)))
        if rng.random() < 0.6:
            reqs = [GenerationRequest(prefix, rng.randint(1, 6), pol, seed=rng.randrange(1 << 30),
                                      request_id=f"t{seed}:{c}:{k}") for k in range(rng.randint(1, 4))]
            out.append(("sample", reqs))
        else:
            conts = tuple(tuple(rng.randrange(16) for _ in range(rng.randint(1, 5))) for _ in range(rng.randint(1, 3)))
            out.append(("score", [ScoreRequest(prefix, conts, pol)]))
    return out


def _run(backend, call):
    kind, reqs = call
    if kind == "sample":
        return [tuple(s.token_ids) for s in backend.sample_batch(reqs)], [tuple(s.token_logprobs)
                                                                         for s in backend.sample_batch(reqs)]
    return backend.score_batch(reqs)


def test_wrappers_under_concurrent_mixed_calls():
    base = TabularBackend.per_position_logits(16, 12, seed=9, prompt_length=4)
    batching = ContinuousBatchingBackend(base, max_batch_size=16, max_batch_tokens=512, batch_wait_seconds=0.001)
    cached = ScoreCachingBackend(batching, maximum_entries=64)       # small: forces evictions under contention
    tree = RolloutTokenTree(max_context_tokens=4, max_contexts=200, min_context_tokens=2)
    plans = {t: _work(t) for t in range(THREADS)}
    got: dict[int, list] = {}
    errors: list[BaseException] = []

    def worker(t):
        try:
            res = []
            for call in plans[t]:
                r = _run(cached, call)
                res.append(r)
                if call[0] == "sample":
                    for toks in r[0]:
                        tree.observe((1, 2) + toks)
                    tree.draft((1, 2), 3)
            got[t] = res
        except BaseException as err:          # noqa: BLE001 - reported below
            errors.append(err)

    threads = [threading.Thread(target=worker, args=(t,), daemon=True) for t in range(THREADS)]
    for th in threads:
        th.start()
    for th in threads:
        th.join(timeout=120)
    try:
        assert not any(th.is_alive() for th in threads), "a wrapper call did not finish (deadlock)"
        assert not errors, errors[0]
        for t in range(THREADS):
            for call, r in zip(plans[t], got[t]):
                assert r == _run(base, call), (t, call[0])
        snap = batching.snapshot()
        want = sum(len(reqs) for plan in plans.values() for kind, reqs in plan if kind == "sample")
        assert snap.sample_requests == 2 * want          # every sample call issued twice per plan entry
        tsnap = tree.snapshot()
        assert tsnap.queries == sum(1 for plan in plans.values() for kind, _ in plan if kind == "sample")
        assert tsnap.contexts <= 200
    finally:
        batching.close()
