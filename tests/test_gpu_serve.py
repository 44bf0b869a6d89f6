"""Continuous batching on the device (nexus_cuda_serve_step) against the oracle.

Requests of different prompt lengths and token budgets arrive over time; the
scheduler admits them FIFO up to max_batch_size running requests and a KV
page budget smaller than the model's pool (so some wait for pages), binds
each request's page ids to a free device sequence, prefills it and decodes
every running request in one batched step per tick.  Every request's tokens
must equal the oracle's greedy generate(prompt, max_tokens) run on its own
(the reference's InferenceEngine::generate_with_config at temperature 0,
src/engine/mod.rs:1196-1238).  A request the model cannot hold ends with an
error event, a cancelled request gives its sequence and pages back, and
requests with max_tokens 0 end without a step.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

VOCAB = 4096
MAX_SEQ = 96


def _engine(nb, path, max_batch=4):
    be = nb.CudaBackend(device=0, max_batch=max_batch, max_seq_len=MAX_SEQ)
    eng = nb.InferenceEngine(be)
    eng.load_model(path)
    return be, eng


def _requests(seed, n):
    rng = np.random.default_rng(seed)
    out = []
    for i in range(n):
        plen = int(rng.integers(1, 40))
        out.append((f"req{i}", rng.integers(0, VOCAB, plen).tolist(), int(rng.integers(0, 18))))
    return out


def test_serve_matches_oracle_generate(nb, oracle, tiny_path):
    be, eng = _engine(nb, tiny_path)
    ref = oracle.Model(tiny_path, max_seq_len=MAX_SEQ)
    assert eng.info.page_tokens == 16 and eng.info.max_batch == 4
    reqs = _requests(5, 9)
    reqs[3] = (reqs[3][0], reqs[3][1], 0)                       # nothing to generate
    batcher = nb.ContinuousBatcher(eng, max_batch_size=3, max_kv_pages=9)
    # first wave now, the rest while the first ones run
    for r in reqs[:5]:
        batcher.add_request(*r)
    got, running_max, ticks = {}, 0, 0
    while True:
        if ticks == 3:
            for r in reqs[5:]:
                batcher.add_request(*r)
        p, r_, _ = batcher.scheduler.stats()
        if ticks > 3 and p == 0 and r_ == 0:
            break
        events = batcher.tick()
        ticks += 1
        running_max = max(running_max, len([e for e in events if e.status == 0]))
        assert len(events) <= 3
        for e in events:
            assert e.status == 0
            if e.done:
                got[e.request_id] = batcher.scheduler.tokens(e.request_id)
        used, budget = batcher.scheduler.kv_page_stats()
        assert used <= budget == 9
        assert ticks < 400
    assert running_max == 3
    for rid, prompt, mt in reqs:
        want = ref.generate(prompt, mt)
        assert got[rid] == want, rid
    eng.close()
    be.close()


def test_serve_rejects_and_cancels(nb, oracle, tiny_path):
    be, eng = _engine(nb, tiny_path)
    ref = oracle.Model(tiny_path, max_seq_len=MAX_SEQ)
    batcher = nb.ContinuousBatcher(eng, max_batch_size=2, max_kv_pages=16)
    rng = np.random.default_rng(9)
    long_prompt = rng.integers(0, VOCAB, 90).tolist()
    a = rng.integers(0, VOCAB, 12).tolist()
    b = rng.integers(0, VOCAB, 7).tolist()
    batcher.add_request("too_long", long_prompt, 10)    # 90 + 10 - 1 > 96
    batcher.add_request("a", a, 12)
    batcher.add_request("b", b, 12)
    ev = batcher.tick()
    rej = [e for e in ev if e.request_id == "too_long"]
    assert len(rej) == 1 and rej[0].done and rej[0].status != 0
    assert {e.request_id for e in ev if e.status == 0} == {"a"}
    batcher.tick()
    assert batcher.scheduler.complete_request("a")       # cancelled while running
    got = {}
    for _ in range(40):
        for e in batcher.tick():
            if e.done:
                got[e.request_id] = batcher.scheduler.tokens(e.request_id)
        if batcher.scheduler.stats()[:2] == (0, 0):
            break
    assert got["b"] == ref.generate(b, 12)
    assert batcher.scheduler.kv_page_stats()[0] == 0
    # the cancelled request's sequence and pages are free again: a new
    # request runs to the oracle's tokens
    batcher.add_request("c", a, 5)
    assert batcher.run()["c"] == ref.generate(a, 5)
    eng.close()
    be.close()
