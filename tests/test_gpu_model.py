"""Decode-step parity on the GPU through the C ABI, against the CPU oracle.

Bars (north star): logits within 2e-3 max-abs, greedy token sequences
identical, KV cache lengths equal.  The tiny configuration (4 layers,
hidden 256, all Q4_K) runs in full: 128-token prompt (seed 1) + 64 greedy
tokens.  The 8B shape is checked on a short prompt.
"""
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

LOGIT_TOL = 2e-3


@pytest.fixture(scope="module")
def tiny_engine(nb, tiny_path):
    b = nb.CudaBackend(device=0, max_batch=4)
    e = nb.InferenceEngine(b)
    e.load_model(tiny_path)
    yield e
    e.close()
    b.close()


def prompt(seed, n, vocab):
    return np.random.default_rng(seed).integers(0, vocab, n).tolist()


def test_tiny_info(tiny_engine):
    i = tiny_engine.info
    assert (i.num_layers, i.hidden_size, i.num_heads, i.num_kv_heads, i.head_dim) == (4, 256, 8, 4, 32)
    assert i.vocab_rows == 4096 and i.rope_freq_base == 10000.0


def test_tiny_prefill_and_decode_logits(tiny_engine, oracle, tiny_path):
    m = oracle.Model(tiny_path)
    p = prompt(1, 128, 4096)
    ref = m.prefill(p)
    got, tok = tiny_engine.prefill(p)
    assert np.max(np.abs(got - ref)) < LOGIT_TOL
    assert tok == oracle.greedy(ref)
    assert tiny_engine.seq_len() == 128
    for i in range(5):
        t = oracle.greedy(ref)
        ref = m.decode(t, 128 + i)
        got, tok = tiny_engine.decode_with_cache(t, 128 + i)
        assert np.max(np.abs(got - ref)) < LOGIT_TOL
        assert tok == oracle.greedy(ref)


def test_tiny_generate_token_identical(tiny_engine, oracle, tiny_path):
    """Config 1 in full: 128-token random prompt (seed 1), 64 greedy tokens."""
    m = oracle.Model(tiny_path)
    p = prompt(1, 128, 4096)
    ref = m.generate(p, 64)
    got = tiny_engine.generate(p, 64)
    assert got == ref
    assert tiny_engine.seq_len() == m.seq_len(0) == 192


def test_tiny_single_token_steps_match_chunked_prefill(tiny_engine):
    p = prompt(7, 11, 4096)
    a, ta = tiny_engine.prefill(p)
    tiny_engine.prefill(p[:1])
    for i, t in enumerate(p[1:], start=1):
        b, tb = tiny_engine.decode_with_cache(t, i)
    assert np.max(np.abs(a - b)) < 1e-4 and ta == tb


def test_tiny_decode_batch_matches_single(tiny_engine, oracle, tiny_path):
    seqs = [prompt(100 + s, 9 + s, 4096) for s in range(3)]
    refs = []
    for s, p in enumerate(seqs):
        m = oracle.Model(tiny_path)
        l0 = m.prefill(p)
        t = oracle.greedy(l0)
        refs.append((t, m.decode(t, len(p))))
        tiny_engine.prefill(p, seq_id=s)
    items = [(s, refs[s][0], len(seqs[s])) for s in range(3)]
    toks, logits = tiny_engine.decode_batch(items, want_logits=True)
    for s in range(3):
        assert np.max(np.abs(logits[s] - refs[s][1])) < LOGIT_TOL
        assert toks[s] == oracle.greedy(refs[s][1])
        assert tiny_engine.seq_len(s) == len(seqs[s]) + 1


def test_tiny_decode_batch_tensor_core_path(nb, oracle, tiny_path):
    """12 sequences in one decode batch run on the tcgen05 GEMM (batches of 8+);
    every sequence's logits and greedy token match the oracle's single-stream decode."""
    b = nb.CudaBackend(device=0, max_batch=16)
    e = nb.InferenceEngine(b)
    e.load_model(tiny_path)
    seqs = [prompt(200 + s, 3 + s, 4096) for s in range(12)]
    refs = []
    for s, p in enumerate(seqs):
        m = oracle.Model(tiny_path)
        t = oracle.greedy(m.prefill(p))
        refs.append((t, m.decode(t, len(p))))
        e.prefill(p, seq_id=s)
    items = [(s, refs[s][0], len(seqs[s])) for s in range(12)]
    toks, logits = e.decode_batch(items, want_logits=True)
    for s in range(12):
        assert np.max(np.abs(logits[s] - refs[s][1])) < LOGIT_TOL, s
        assert toks[s] == oracle.greedy(refs[s][1])
    e.close()
    b.close()


@pytest.mark.parametrize("bits", [(4, 4), (3, 2)])
def test_tiny_packed_kv(nb, oracle, tiny_path, bits):
    """Packed low-bit KV.  Packing itself is bit-exact (test_kv_quantize_bit_exact);
    here K/V come from the GEMV, whose ~1e-5 relative rounding difference can
    move a value across a quantization boundary (one step = range/(2^bits-1)),
    so the logit bound is the float-KV bound plus the effect of such flips."""
    b = nb.CudaBackend(device=0, kv_bits=bits)
    e = nb.InferenceEngine(b)
    e.load_model(tiny_path)
    m = oracle.Model(tiny_path, kv_bits=bits)
    p = prompt(2, 40, 4096)
    ref = m.prefill(p)
    got, tok = e.prefill(p)
    err = float(np.max(np.abs(got - ref)))
    print(f"packed kv {bits}: max |logit diff| = {err:.3e}")
    assert err < 2e-2, err
    assert tok == oracle.greedy(ref)
    gen, refgen = e.generate(p, 16), m.generate(p, 16)
    e.close()
    b.close()
    assert gen == refgen


@pytest.mark.parametrize("bits", [(4, 4), (3, 2)])
def test_head_dim_128_packed_kv(nb, oracle, bits):
    """Packed KV on a head_dim-128 model (the tensor-core attention kernel):
    a 140-token prefill in one step, then three decode steps."""
    path = nb.model_path("tp_small")
    b = nb.CudaBackend(device=0, kv_bits=bits)
    e = nb.InferenceEngine(b)
    e.load_model(path)
    m = oracle.Model(path, kv_bits=bits, threads=os.cpu_count() or 1)
    p = prompt(5, 140, 8192)
    ref = m.prefill(p)
    got, tok = e.prefill(p)
    errs = [float(np.max(np.abs(got - ref)))]
    assert tok == oracle.greedy(ref)
    for i in range(3):
        ref = m.decode(tok, len(p) + i)
        got, tok2 = e.decode_with_cache(tok, len(p) + i)
        errs.append(float(np.max(np.abs(got - ref))))
        assert tok2 == oracle.greedy(ref)
        tok = tok2
    e.close()
    b.close()
    print(f"head_dim 128, packed kv {bits}: max |logit diff| = {max(errs):.3e}")
    assert max(errs) < 2e-2, errs


RING = 24  # max_seq_len of the full-cache tests


@pytest.mark.parametrize("flags,kv_bits", [(0, (0, 0)), (0, (4, 4)), (0x4, (0, 0))],
                         ids=["graph", "packed", "persistent"])
def test_full_cache_drops_oldest_token(nb, oracle, tiny_path, flags, kv_bits):
    """KvCache::add on a full cache drops its oldest token and appends the new
    one (src/engine/mod.rs:410-426), so decoding continues past max_seq_len
    with attention over the last max_seq_len tokens.  Device-chained generate,
    single decodes with logits, a prompt longer than the cache and the draft
    verify path all match the oracle's shifting cache."""
    b = nb.CudaBackend(device=0, max_seq_len=RING, kv_bits=kv_bits, flags=flags)
    e = nb.InferenceEngine(b)
    e.load_model(tiny_path)
    ref = oracle.Model(tiny_path, kv_bits=kv_bits, max_seq_len=RING)
    tol = LOGIT_TOL if kv_bits == (0, 0) else 2e-2
    p = prompt(3, 20, 4096)
    want = ref.generate(p, 30)
    assert e.generate(p, 30) == want
    assert e.seq_len() == RING
    # single-token decodes past the boundary, logits each step
    ref2 = oracle.Model(tiny_path, kv_bits=kv_bits, max_seq_len=RING)
    q = prompt(4, 22, 4096)
    got, tok = e.prefill(q)
    assert np.max(np.abs(got - ref2.prefill(q))) < tol
    for i in range(8):
        got, tok2 = e.decode_with_cache(tok, len(q) + i)
        want_l = ref2.decode(tok, len(q) + i)
        assert np.max(np.abs(got - want_l)) < tol, i
        tok = tok2
    assert e.seq_len() == RING
    # a prompt longer than the cache: the chunks stop at the wrap
    ref3 = oracle.Model(tiny_path, kv_bits=kv_bits, max_seq_len=RING)
    r = prompt(5, 61, 4096)
    got, _ = e.prefill(r)
    assert np.max(np.abs(got - ref3.prefill(r))) < tol
    # draft verify across the boundary: the greedy tokens as the draft
    cont = ref.generate(p, 12)
    out, (acc, rej) = e.generate_with_draft_tokens(p, 12, cont[len(p):], window=8)
    assert out == cont and (acc, rej) == (12, 0)
    e.close()
    b.close()


def test_full_cache_decode_batch(nb, oracle, tiny_path):
    """Two sequences decoded together past max_seq_len (one wraps first)."""
    b = nb.CudaBackend(device=0, max_seq_len=RING, max_batch=2)
    e = nb.InferenceEngine(b)
    e.load_model(tiny_path)
    ps = [prompt(6, 18, 4096), prompt(7, 23, 4096)]
    want = [oracle.Model(tiny_path, max_seq_len=RING).generate(p, 14) for p in ps]
    toks = []
    for s, p in enumerate(ps):
        toks.append(e.prefill(p, seq_id=s, want_logits=False)[1])
    got = [[t] for t in toks]
    for i in range(13):
        toks, _ = e.decode_batch([(s, toks[s], len(ps[s]) + i) for s in range(2)])
        for s in range(2):
            got[s].append(toks[s])
    for s in range(2):
        assert ps[s] + got[s] == want[s], s
        assert e.seq_len(s) == RING
    e.close()
    b.close()


def test_missing_tensor_is_an_error(nb, tmp_path):
    from tests.gguf_writer import write_gguf
    path = tmp_path / "empty.gguf"
    write_gguf(path, {"general.architecture": "llama", "llama.embedding_length": 256, "llama.block_count": 1,
                      "llama.attention.head_count": 8}, [])
    b = nb.CudaBackend(device=0)
    e = nb.InferenceEngine(b)
    with pytest.raises(nb.NexusError) as err:
        e.load_model(path)
    assert err.value.code == nb._lib.NEXUS_E_MISSING_TENSOR
    b.close()


@pytest.mark.slow
def test_llama8b_shape_short_prompt(nb, oracle):
    """8B shape (Q4_K body, Q8_0 embedding/head): 6-token prompt + 3 greedy tokens."""
    path = nb.model_path("llama8b_q4k")
    b = nb.CudaBackend(device=0, max_seq_len=64)
    e = nb.InferenceEngine(b)
    e.load_model(path)
    m = oracle.Model(path, threads=32, max_seq_len=64)
    p = prompt(1, 6, 128256)
    ref = m.prefill(p)
    got, tok = e.prefill(p)
    err = float(np.max(np.abs(got - ref)))
    print(f"8B shape, 6-token prompt: max |logit diff| = {err:.3e}")
    assert err < LOGIT_TOL, err
    assert tok == oracle.greedy(ref)
    assert e.generate(p, 3) == m.generate(p, 3)
    e.close()
    b.close()


@pytest.mark.parametrize("persistent", [True, False])
def test_head_dim_128_single_token_paths(nb, oracle, persistent):
    """A head_dim-128, G=2 model with the float cache: single-token steps run
    on the persistent whole-step kernel (NEXUS_CFG_PERSISTENT: one launch per
    token, weights streamed across phase boundaries) or on the kernel-per-op
    graph.  Both match the oracle: logits at every step within
    2e-3 and 12 greedy tokens identical; the KV length advances."""
    path = nb.model_path("tp_small")
    b = nb.CudaBackend(device=0, max_seq_len=256, flags=nb._lib.CFG_PERSISTENT if persistent else 0)
    e = nb.InferenceEngine(b)
    e.load_model(path)
    m = oracle.Model(path, threads=os.cpu_count() or 1, max_seq_len=256)
    p = prompt(6, 37, 8192)
    ref = m.prefill(p)
    got, tok = e.prefill(p)
    assert np.max(np.abs(got - ref)) < LOGIT_TOL
    errs = []
    for i in range(6):
        t = oracle.greedy(ref)
        assert tok == t
        ref = m.decode(t, len(p) + i)
        got, tok = e.decode_with_cache(t, len(p) + i)
        errs.append(float(np.max(np.abs(got - ref))))
    assert max(errs) < LOGIT_TOL, errs
    assert e.seq_len() == len(p) + 6
    # device-chained greedy generation (the bench's `value` path)
    assert e.generate(p, 12) == m.generate(p, 12)
    e.close()
    b.close()


@pytest.mark.parametrize("window", [1, 4, 8, 32])
def test_generate_with_draft_tokens(nb, oracle, tiny_path, window):
    """generate_with_draft_tokens at temperature 0 (src/engine/mod.rs:1244-1291):
    the output is the greedy continuation whatever the draft; accepted counts the
    draft positions equal to it.  Windows of draft tokens are verified in one
    multi-token step each (8+ tokens on the tensor-core GEMM)."""
    b = nb.CudaBackend(device=0, max_seq_len=256)
    e = nb.InferenceEngine(b)
    e.load_model(tiny_path)
    m = oracle.Model(tiny_path)
    p = prompt(8, 30, 4096)
    ref = m.generate(p, 24)
    good = ref[30:]
    bad = list(good[:20])
    for q in (2, 9, 15):
        bad[q] = (bad[q] + 1) % 4096
    for draft, want in [(good, (24, 0)), (bad, (17, 3)), ([], (0, 0)), (good + [5] * 10, (24, 0))]:
        out, stats = e.generate_with_draft_tokens(p, 24, draft, window=window)
        assert out == ref
        assert stats == want
        assert e.seq_len() == 30 + 24
    e.close()
    b.close()


def test_generate_with_draft_tokens_head_dim_128(nb, oracle):
    path = nb.model_path("tp_small")
    b = nb.CudaBackend(device=0, max_seq_len=128)
    e = nb.InferenceEngine(b)
    e.load_model(path)
    m = oracle.Model(path, threads=os.cpu_count() or 1, max_seq_len=128)
    p = prompt(9, 17, 8192)
    ref = m.generate(p, 20)
    draft = list(ref[17:])
    draft[11] = (draft[11] + 7) % 8192
    out, stats = e.generate_with_draft_tokens(p, 20, draft, window=8)
    assert out == ref and stats == (19, 1)
    e.close()
    b.close()


def test_chunked_prefill_attention_matches_single_steps(nb, oracle):
    """A 300-token prompt as chunks of 256 and 44 tokens runs its attention as
    one causal kernel per chunk on the tensor cores (f16 hi/lo products, f32
    accumulate); the logits equal those of 300 single-token decode steps within
    1e-4, and the oracle's within 2e-3."""
    path = nb.model_path("tp_small")
    b = nb.CudaBackend(device=0, max_seq_len=320)
    e = nb.InferenceEngine(b)
    e.load_model(path)
    p = prompt(12, 300, 8192)
    a, ta = e.prefill(p)
    e.prefill(p[:1])
    for i, t in enumerate(p[1:], start=1):
        c, tc = e.decode_with_cache(t, i, want_logits=i == len(p) - 1)
    assert np.max(np.abs(a - c)) < 1e-4 and ta == tc
    m = oracle.Model(path, threads=os.cpu_count() or 1, max_seq_len=320)
    ref = m.prefill_batched(p)
    assert np.max(np.abs(a - ref)) < LOGIT_TOL
    e.close()
    b.close()
