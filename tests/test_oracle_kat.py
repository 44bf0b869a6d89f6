"""The CPU oracle against the reference's own known-answer tests.

The oracle (oracle/nexus_oracle.c) restates the reference's Rust CPU path;
these cases pin it to the assertions of the reference's inline tests,
transcribed in tests/golden/reference_kats.json (see make_kats.py).
"""
import json
import math
from pathlib import Path

import numpy as np
import pytest

from tests.gguf_writer import f32_bytes, write_gguf

KATS = json.loads((Path(__file__).parent / "golden" / "reference_kats.json").read_text())


def test_q8_0_known_answer(oracle):
    k = KATS["q8_0_dequant"]
    h = oracle.f32_to_f16(k["scale"])
    blk = np.zeros(34, np.uint8)
    blk[0], blk[1] = h & 0xFF, h >> 8
    blk[2:] = np.array(k["q"], np.int8).view(np.uint8)
    v = oracle.dequantize(oracle.Q8_0, blk, 32)
    for idx, want in k["expect"].items():
        assert v[int(idx)] == want


def test_k_quant_sizes(oracle):
    k = KATS["k_quant_sizes"]
    data = (np.arange(k["n"], dtype=np.float32) / np.float32(31.0) - np.float32(4.0)).astype(np.float32)
    for name, want in k["bytes"].items():
        fmt = getattr(oracle, name)
        q = oracle.quantize(fmt, data)
        assert q.size == want
        assert oracle.dequantize(fmt, q, data.size).size == data.size


def _ramp(spec, n):
    i = np.arange(n, dtype=np.float32)
    if spec == "i/16-2":
        return (i / np.float32(16.0) - np.float32(2.0)).astype(np.float32)
    return (i / np.float32(31.0) - np.float32(4.0)).astype(np.float32)


@pytest.mark.parametrize("case", KATS["roundtrip_bounds"]["cases"], ids=lambda c: c["format"])
def test_roundtrip_bounds(oracle, case):
    fmt = getattr(oracle, case["format"])
    data = _ramp(case["ramp"], case["n"])
    back = oracle.dequantize(fmt, oracle.quantize(fmt, data), data.size)
    assert np.max(np.abs(back - data)) < case["max_abs_err"]


def test_truncated_payload_rejected(oracle):
    q = oracle.quantize(oracle.Q4_K, np.ones(256, np.float32))
    with pytest.raises(ValueError):
        oracle.dequantize(oracle.Q4_K, q[:-1], 256)


def test_rms_norm_known_answer(oracle):
    k = KATS["rms_norm"]
    out = oracle.rms_norm(np.array(k["input"], np.float32), np.array(k["weight"], np.float32), k["eps"])
    scale = np.float32(1.0) / np.sqrt(np.float32(30.0) / np.float32(4.0))
    assert np.all(np.abs(out - np.array(k["input"], np.float32) * scale) < k["tol"])


def test_rope_position_zero_is_identity(oracle):
    k = KATS["rope_pos0_identity"]
    x = np.array(k["input"], np.float32)
    out = oracle.rope_single(x, k["position"], k["head_dim"], k["base"])
    assert np.all(np.abs(out - x) < k["tol"])


def test_rope_matches_formula(oracle):
    # NeoX half-split rotation with angle pos / base^(2d/D) (src/kernel/mod.rs:258-271)
    rng = np.random.default_rng(5)
    x = rng.standard_normal(64).astype(np.float32)
    out = oracle.rope_single(x, 37, 64, 500000.0)
    d = np.arange(32, dtype=np.float64)
    ang = 37.0 / np.power(500000.0, 2 * d / 64)
    x0, x1 = x[:32].astype(np.float64), x[32:].astype(np.float64)
    ref = np.concatenate([x0 * np.cos(ang) - x1 * np.sin(ang), x0 * np.sin(ang) + x1 * np.cos(ang)])
    assert np.max(np.abs(out - ref)) < 1e-5


def test_packed_kv_roundtrip(oracle):
    k = KATS["packed_kv_roundtrip"]
    kk = oracle.PackedKv(k["bits"], k["head_dim"], k["max_seq_len"])
    vv = oracle.PackedKv(k["bits"], k["head_dim"], k["max_seq_len"])
    kk.add(0, np.array(k["key"], np.float32))
    vv.add(0, np.array(k["value"], np.float32))
    assert np.all(np.abs(kk.get_all(1) - np.array(k["key"], np.float32)) <= k["tol"])
    assert np.all(np.abs(vv.get_all(1) - np.array(k["value"], np.float32)) <= k["tol"])


def test_packed_kv_attention_is_finite(oracle):
    k = KATS["packed_kv_attention_finite"]
    kk = oracle.PackedKv(k["bits"], k["head_dim"], 4)
    vv = oracle.PackedKv(k["bits"], k["head_dim"], 4)
    for i, (key, val) in enumerate(zip(k["keys"], k["values"])):
        kk.add(i, np.array(key, np.float32))
        vv.add(i, np.array(val, np.float32))
    keys = kk.get_all(2).reshape(2, 2)
    vals = vv.get_all(2).reshape(2, 2)
    s = keys @ np.array(k["q"], np.float32) / np.sqrt(np.float32(2.0))
    p = np.exp(s - s.max())
    out = (p / p.sum()) @ vals
    assert np.all(np.isfinite(out)) and out.size == 2


def test_packed_kv_bit_layout(oracle):
    # values are written LSB-first at bit offset i*bits (write_bits, src/engine/mod.rs:288-299)
    kv = oracle.PackedKv(3, 8, 2)
    vals = np.array([0, 1, 2, 3, 4, 5, 6, 7], np.float32)  # min 0, scale 1 -> q = i
    kv.add(0, vals)
    data, mins, scales = kv.raw(1)
    bits = "".join(format(b, "08b")[::-1] for b in data[:3])
    assert [int(bits[3 * i:3 * i + 3][::-1], 2) for i in range(8)] == list(range(8))
    assert mins[0] == 0.0 and scales[0] == 1.0


def test_packed_kv_constant_vector_uses_unit_scale(oracle):
    kv = oracle.PackedKv(4, 4, 1)
    kv.add(0, np.full(4, 0.25, np.float32))
    _, mins, scales = kv.raw(1)
    assert scales[0] == 1.0 and mins[0] == np.float32(0.25)
    assert np.all(kv.get_all(1) == np.float32(0.25))


def test_greedy_known_answer_and_ties(oracle):
    k = KATS["greedy"]
    assert oracle.greedy(np.array(k["logits"], np.float32)) == k["expect"]
    # Iterator::max_by keeps the last maximum; non-finite values are skipped
    assert oracle.greedy(np.array([1.0, 3.0, 3.0, 0.5], np.float32)) == 2
    assert oracle.greedy(np.array([np.nan, np.inf, 2.0, -np.inf], np.float32)) == 2
    assert oracle.greedy(np.array([np.nan, np.inf], np.float32)) == 0
    # total_cmp orders -0.0 below +0.0
    assert oracle.greedy(np.array([0.0, -0.0], np.float32)) == 0


def _zero_layer_model(tmp_path, k):
    path = tmp_path / "zero_layer.gguf"
    write_gguf(path, {"general.architecture": "llama", "llama.embedding_length": 2, "llama.block_count": 0,
                      "llama.attention.head_count": 1, "llama.attention.head_count_kv": 1,
                      "llama.feed_forward_length": 2},
               [("token_embd.weight", [2, 2], 0, f32_bytes(k["token_embd"])),
                ("output_norm.weight", [2], 0, f32_bytes(k["output_norm"])),
                ("output.weight", [2, 2], 0, f32_bytes(k["output"]))])
    return path


def test_prefill_zero_layer_known_answer(oracle, tmp_path):
    k = KATS["prefill_zero_layer"]
    m = oracle.Model(_zero_layer_model(tmp_path, k))
    m.set_eps(k["eps"])
    logits = m.prefill(k["tokens"])
    assert logits.size == len(k["expect"])
    assert np.all(np.abs(logits - np.array(k["expect"], np.float32)) < k["tol"])


def test_tiny_decode_shapes(oracle, tiny_path):
    k = KATS["decode_one_layer_shapes"]
    m = oracle.Model(tiny_path)
    logits = m.decode(0, 0)
    assert logits.size == m.info.vocab_rows == 4096
    assert m.seq_len(0) == k["expect_seq_len"]
    assert np.all(np.isfinite(logits))


def test_kv_cache_shift_keeps_capacity(oracle, tiny_path):
    k = KATS["kv_cache_shift"]
    m = oracle.Model(tiny_path, max_seq_len=k["max_seq_len"])
    for pos in range(k["adds"]):
        m.decode(pos, pos)
    assert m.seq_len(0) == k["expect_seq_len"]


def test_prefill_resets_cache_and_generate_is_greedy(oracle, tiny_path):
    m = oracle.Model(tiny_path)
    rng = np.random.default_rng(1)
    prompt = rng.integers(0, 4096, 6).tolist()
    logits = m.prefill(prompt)
    assert m.seq_len(0) == 6
    out = m.generate(prompt, 3)
    assert out[:6] == prompt
    assert out[6] == oracle.greedy(logits)
    assert m.seq_len(0) == 9


def test_threads_do_not_change_results(oracle, tiny_path):
    a = oracle.Model(tiny_path, threads=1)
    b = oracle.Model(tiny_path, threads=4)
    for pos, tok in enumerate([3, 1000, 77]):
        la, lb = a.decode(tok, pos), b.decode(tok, pos)
        assert np.array_equal(la.view(np.uint32), lb.view(np.uint32))
