"""Device-resident paged KV driven by scheduler page lists, through the C ABI.

The reference's scheduler gives every request ceil((prompt + max_tokens)/16)
KV page ids (Scheduler::allocate_kv_pages, src/scheduler.rs:333-361) and
ships them with each decode item (ScheduledDecode.kv_pages, :108-115).  The
backend stores token t of a sequence in page page_ids[t / page_tokens] of a
per-layer page pool.  Where the pages sit must not change a single bit of
the results: a sequence on shuffled, non-contiguous pages gives the same
logits as on the library's contiguous pages, for the float cache and the
packed cache (per-element and tensor-core kernels), on the single-token GEMV
path and the batched tensor-core GEMM path, and for several page sizes.
Lists that cannot hold the step, ids outside the pool, repeated ids, pages
of another sequence and lists that would move cached tokens are refused.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

PT = 16


def _prompt(seed, n, vocab):
    return np.random.default_rng(seed).integers(0, vocab, n).tolist()


def _run(nb, path, kv_bits, pages_for, prompt_len=40, steps=6, batch=1, page_tokens=0, max_pages=0, vocab=4096):
    """Prefill `batch` sequences (seed 11 + s), then `steps` decode_batch steps
    over all of them; pages_for(s) gives sequence s's page list or None (the
    library's pages).  Returns the logits of every step, [steps+1][batch][V]."""
    be = nb.CudaBackend(device=0, kv_bits=kv_bits, max_batch=batch, max_seq_len=prompt_len + steps + 8,
                        page_tokens=page_tokens, max_pages=max_pages)
    eng = nb.InferenceEngine(be)
    eng.load_model(path)
    pages = [pages_for(s) for s in range(batch)]
    out = [[]]
    toks = []
    for s in range(batch):
        if pages[s] is not None:
            eng.seq_set_pages(s, pages[s])
        lg, t = eng.prefill(_prompt(11 + s, prompt_len, vocab), seq_id=s)
        out[0].append(lg)
        toks.append(t)
    for i in range(steps):
        items = [(s, toks[s], prompt_len + i) for s in range(batch)]
        toks, lg = eng.decode_batch(items, want_logits=True,
                                    page_ids=None if all(p is None for p in pages) else
                                    [p if p is not None else [] for p in pages])
        out.append(list(lg))
        for s in range(batch):
            assert eng.seq_len(s) == prompt_len + i + 1
    eng.close()
    be.close()
    return np.asarray(out)


def _shuffled(seed, n_pages, pool):
    return np.random.default_rng(seed).permutation(pool)[:n_pages].tolist()


def _bits(a):
    return np.asarray(a, np.float32).view(np.uint32)


@pytest.mark.parametrize("kv_bits", [(0, 0), (4, 4), (3, 2)])
def test_shuffled_pages_bit_identical_tiny(nb, tiny_path, kv_bits):
    """Tiny model (head_dim 32): float cache and the per-element packed kernel;
    one sequence (GEMV steps) and a prefill of 40 tokens (GEMM chunks)."""
    need = (40 + 6 + 8 + PT - 1) // PT
    ref = _run(nb, tiny_path, kv_bits, lambda s: None)
    got = _run(nb, tiny_path, kv_bits, lambda s: _shuffled(3, need, 64), max_pages=64)
    assert np.array_equal(_bits(ref), _bits(got))


@pytest.mark.parametrize("kv_bits", [(0, 0), (4, 4)])
def test_shuffled_pages_bit_identical_batched_head_dim_128(nb, kv_bits):
    """head_dim 128 (the tensor-core packed kernel), 8 sequences per step (the
    tcgen05 GEMM path), every sequence on its own shuffled pages drawn from
    one pool, against the library's contiguous pages."""
    path = nb.model_path("tp_small")
    need = (40 + 6 + 8 + PT - 1) // PT
    perm = np.random.default_rng(5).permutation(8 * need + 5).tolist()
    ref = _run(nb, path, kv_bits, lambda s: None, batch=8, vocab=8192)
    got = _run(nb, path, kv_bits, lambda s: perm[s * need:(s + 1) * need], batch=8, vocab=8192,
               max_pages=8 * need + 5)
    assert np.array_equal(_bits(ref), _bits(got))


@pytest.mark.parametrize("page_tokens", [1, 8, 64])
def test_page_sizes_bit_identical(nb, tiny_path, page_tokens):
    ref = _run(nb, tiny_path, (0, 0), lambda s: None)
    need = (40 + 6 + 8 + page_tokens - 1) // page_tokens
    got = _run(nb, tiny_path, (0, 0), lambda s: _shuffled(4, need, 2 * need + 3), page_tokens=page_tokens,
               max_pages=2 * need + 3)
    assert np.array_equal(_bits(ref), _bits(got))


def test_page_list_rejections(nb, tiny_path):
    from nexus_b200 import NexusError
    be = nb.CudaBackend(device=0, max_batch=2, max_seq_len=128, max_pages=32)
    eng = nb.InferenceEngine(be)
    eng.load_model(tiny_path)
    p = _prompt(1, 40, 4096)
    with pytest.raises(NexusError):
        eng.seq_set_pages(0, [0, 1, 32])          # beyond the pool of 32 pages
    with pytest.raises(NexusError):
        eng.seq_set_pages(0, [3, 4, 3])           # a page listed twice
    eng.seq_set_pages(0, [9, 2, 30])              # 48 tokens
    _, t = eng.prefill(p, seq_id=0)
    with pytest.raises(NexusError):
        eng.seq_set_pages(1, [30, 5])             # page 30 belongs to sequence 0
    with pytest.raises(NexusError):
        eng.seq_set_pages(0, [9, 3, 30])          # would move cached tokens 16..31
    with pytest.raises(NexusError):
        eng.seq_set_pages(0, [9, 2])              # shorter than the 40 cached tokens
    # decode up to the end of the three pages, then a step that needs a fourth
    pos = 40
    for _ in range(8):
        toks, _ = eng.decode_batch([(0, t, pos)], page_ids=[[9, 2, 30]])
        t, pos = toks[0], pos + 1
    assert eng.seq_len(0) == 48
    with pytest.raises(NexusError):
        eng.decode_batch([(0, t, pos)], page_ids=[[9, 2, 30]])
    assert eng.seq_len(0) == 48
    # extending the list keeps the cached pages in place and the step goes on
    toks, _ = eng.decode_batch([(0, t, pos)], page_ids=[[9, 2, 30, 17]])
    assert eng.seq_len(0) == 49
    # releasing the pages clears the sequence and frees them for another one
    eng.seq_set_pages(0, [])
    assert eng.seq_len(0) == 0
    eng.seq_set_pages(1, [30, 5])
    eng.close()
    be.close()


def test_pool_smaller_than_library_pages(nb, tiny_path):
    """With max_pages below max_batch x pages(max_seq_len), a sequence whose
    library pages fall outside the pool needs a page list."""
    from nexus_b200 import NexusError
    be = nb.CudaBackend(device=0, max_batch=4, max_seq_len=64, max_pages=6)  # 4 pages per sequence
    eng = nb.InferenceEngine(be)
    eng.load_model(tiny_path)
    eng.prefill(_prompt(2, 20, 4096), seq_id=0)        # library pages 0..3
    eng.prefill(_prompt(2, 20, 4096), seq_id=1)        # library pages 4..5 (32 tokens) hold 20
    with pytest.raises(NexusError):
        eng.prefill(_prompt(3, 40, 4096), seq_id=1)    # ... but not 40
    with pytest.raises(NexusError):
        eng.prefill(_prompt(2, 20, 4096), seq_id=2)    # no library pages left in the pool
    eng.seq_set_pages(0, [])                           # sequence 0 done: pages 0..3 free
    eng.seq_set_pages(2, [3, 0])
    eng.prefill(_prompt(2, 20, 4096), seq_id=2)
    assert eng.seq_len(2) == 20
    eng.close()
    be.close()
