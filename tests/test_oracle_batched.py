"""The oracle's layer-major prefill and synthetic writer against their references.

orc_model_prefill_batched (used to make the long-context parity fixtures)
must give the same bits as the reference-ordered token-by-token prefill, for
logits and for every later decode step (which reads the KV cache it wrote).
orc_synth_write must write the same bytes as the CUDA library's synthetic
writer, so fixtures and the bench's CPU legs see the model the GPU sees.
"""
import numpy as np
import pytest

from nexus_b200 import Q2_K, Q4_0, Q4_K, Q8_0

SMALL = dict(num_layers=2, hidden_size=512, num_heads=4, num_kv_heads=2, ff_dim=768, vocab_size=1024,
             context_length=256, rope_theta=500000.0, attn_format=Q8_0, ffn_format=Q2_K, embd_format=Q4_0,
             head_format=Q8_0, norm_format=Q4_K)


def _same_bits(a, b):
    return np.array_equal(np.asarray(a, np.float32).view(np.uint32), np.asarray(b, np.float32).view(np.uint32))


@pytest.mark.parametrize("kv", [(0, 0), (4, 4), (3, 2)])
def test_batched_prefill_equals_token_by_token(oracle, tiny_path, kv):
    seq = oracle.Model(tiny_path, kv_bits=kv, threads=2, max_seq_len=160)
    bat = oracle.Model(tiny_path, kv_bits=kv, threads=3, max_seq_len=160)
    prompt = np.random.default_rng(5).integers(0, 4096, 77).tolist()  # two full 32-token tiles + a ragged one
    a, b = seq.prefill(prompt), bat.prefill_batched(prompt)
    assert _same_bits(a, b)
    tok = oracle.greedy(a)
    for i in range(3):
        la, lb = seq.decode(tok, 77 + i), bat.decode(tok, 77 + i)
        assert _same_bits(la, lb)
        tok = oracle.greedy(la)
    assert seq.seq_len(0) == bat.seq_len(0) == 80


def test_batched_prefill_other_formats_and_gqa(oracle, tmp_path):
    path = tmp_path / "small.gguf"
    oracle.write_synthetic_model(str(path), seed=3, threads=2, **SMALL)
    seq = oracle.Model(path, threads=1, max_seq_len=64)
    bat = oracle.Model(path, threads=4, max_seq_len=64)
    prompt = np.random.default_rng(9).integers(0, 1024, 40).tolist()
    assert _same_bits(seq.prefill(prompt), bat.prefill_batched(prompt))


def test_batched_prefill_rejects_prompts_longer_than_the_cache(oracle, tiny_path):
    m = oracle.Model(tiny_path, threads=1, max_seq_len=16)
    with pytest.raises(RuntimeError):
        m.prefill_batched(list(range(17)))


@pytest.mark.parametrize("variant", ["tiny", "small", "tied_repeat"])
def test_oracle_writer_matches_library_writer(nb, oracle, tmp_path, variant):
    cfg = dict(nb.CONFIGS["tiny"]) if variant == "tiny" else dict(SMALL)
    if variant == "tied_repeat":
        cfg.update(head_format=-1, repeat_chunks=1)
    a, b = tmp_path / "lib.gguf", tmp_path / "orc.gguf"
    nb.write_synthetic_model(str(a), seed=7, threads=2, **cfg)
    oracle.write_synthetic_model(str(b), seed=7, threads=3, **cfg)
    assert a.read_bytes() == b.read_bytes()
