"""Kernel-level parity on the GPU through the C ABI, against the CPU oracle.

Bars: block-format conversions are bit-exact; the fused GEMV (and every other
floating-point op) is within 1e-3 relative error, measured as
max|y - y_ref| / max|y_ref| over the output (per-op tolerance of the north
star), with f32 accumulation.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

FORMATS = ["Q8_0", "Q4_0", "Q4_K", "Q2_K"]
REL_TOL = 1e-3


def rel_err(y, ref):
    return float(np.max(np.abs(y - ref)) / max(np.max(np.abs(ref)), 1e-30))


def weights(rng, n):
    return (rng.standard_normal(n) * 0.02).astype(np.float32)


@pytest.mark.parametrize("fmt", FORMATS)
def test_dequantize_bit_exact(backend, oracle, nb, fmt):
    rng = np.random.default_rng(21)
    for n in (32, 256, 300, 4096 * 3 + 64):
        if fmt in ("Q4_K", "Q2_K") and n % 256 and n < 256:
            continue
        x = (rng.standard_normal(n) * 0.3).astype(np.float32)
        q = oracle.quantize(getattr(oracle, fmt), x)
        ref = oracle.dequantize(getattr(oracle, fmt), q, n)
        got = backend.dequantize(getattr(nb, fmt), q, n)
        assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))


@pytest.mark.parametrize("fmt", FORMATS)
def test_quantize_bit_exact(backend, oracle, nb, fmt):
    rng = np.random.default_rng(22)
    for n in (1, 33, 256, 300, 256 * 40 + 7):
        x = (rng.standard_normal(n) * 0.05).astype(np.float32)
        assert np.array_equal(backend.quantize(getattr(nb, fmt), x), oracle.quantize(getattr(oracle, fmt), x))
    x = np.zeros(512, np.float32)
    x[256:] = 1.0
    assert np.array_equal(backend.quantize(getattr(nb, fmt), x), oracle.quantize(getattr(oracle, fmt), x))


@pytest.mark.parametrize("fmt", FORMATS)
def test_tile_layout_roundtrip_bit_exact(backend, oracle, nb, fmt):
    rng = np.random.default_rng(23)
    rows, cols = 72, 768  # partial last row group
    q = oracle.quantize(getattr(oracle, fmt), weights(rng, rows * cols))
    w = nb.QWeight(backend, getattr(nb, fmt), rows, cols, q)
    ref = oracle.dequantize(getattr(oracle, fmt), q, rows * cols)
    assert np.array_equal(w.dequantize().view(np.uint32), ref.view(np.uint32))
    w.close()


SWEEP = [(4096, 4096), (1024, 4096), (14336, 4096), (4096, 14336), (128256, 4096)]


@pytest.mark.parametrize("fmt", FORMATS)
@pytest.mark.parametrize("shape", SWEEP, ids=lambda s: f"{s[0]}x{s[1]}")
def test_qmatvec_sweep_shapes(backend, oracle, nb, fmt, shape):
    """Config-2 sweep shapes, batch 1 and 4, against the oracle's sequential f32 matvec."""
    n, k = shape
    rng = np.random.default_rng(31 + n + k)
    q = oracle.quantize(getattr(oracle, fmt), weights(rng, n * k))
    w = nb.QWeight(backend, getattr(nb, fmt), n, k, q)
    x = rng.standard_normal((4, k)).astype(np.float32)
    y = w.matvec(x)
    for t in (0, 3):
        ref = oracle.qmatvec(getattr(oracle, fmt), q, n, k, x[t], threads=16)
        assert rel_err(y[t], ref) < REL_TOL, (t, rel_err(y[t], ref))
    y1 = w.matvec(x[:1])
    assert np.array_equal(y1[0], y[0])  # batch composition does not change a row's result
    w.close()


@pytest.mark.parametrize("m", [1, 2, 3, 5, 16])
def test_qmatvec_batches(backend, oracle, nb, m):
    rng = np.random.default_rng(40 + m)
    n, k = 512, 1024
    q = oracle.quantize(oracle.Q4_K, weights(rng, n * k))
    x = rng.standard_normal((m, k)).astype(np.float32)
    y = backend.qmatvec(nb.Q4_K, q, n, k, x)
    for t in range(m):
        assert rel_err(y[t], oracle.qmatvec(oracle.Q4_K, q, n, k, x[t])) < REL_TOL


def test_qmatvec_input_edge_cases(backend, oracle, nb):
    rng = np.random.default_rng(44)
    n, k = 64, 512
    q = oracle.quantize(oracle.Q4_K, weights(rng, n * k))
    x = np.zeros((3, k), np.float32)
    x[1, :256] = rng.standard_normal(256) * 1e4  # large and zero super-blocks
    x[2] = rng.standard_normal(k) * 1e-6
    y = backend.qmatvec(nb.Q4_K, q, n, k, x)
    assert np.all(y[0] == 0.0)
    for t in (1, 2):
        assert rel_err(y[t], oracle.qmatvec(oracle.Q4_K, q, n, k, x[t])) < REL_TOL


@pytest.mark.parametrize("fmt", FORMATS)
@pytest.mark.parametrize("m", [8, 16, 17, 64, 100])
@pytest.mark.parametrize("shape", [(4096, 4096), (1024, 4096), (4096, 14336)], ids=lambda s: f"{s[0]}x{s[1]}")
def test_qgemm_batched(backend, oracle, nb, shape, m, fmt):
    """Batches of 8+ tokens run on the tcgen05 GEMM; tokens 0, m/2 and m-1
    are checked against the oracle's sequential f32 matvec."""
    n, k = shape
    rng = np.random.default_rng(60 + m + n + k)
    q = oracle.quantize(getattr(oracle, fmt), weights(rng, n * k))
    w = nb.QWeight(backend, getattr(nb, fmt), n, k, q)
    x = rng.standard_normal((m, k)).astype(np.float32)
    y = w.matvec(x)
    for t in sorted({0, m // 2, m - 1}):
        ref = oracle.qmatvec(getattr(oracle, fmt), q, n, k, x[t], threads=16)
        assert rel_err(y[t], ref) < REL_TOL, (t, rel_err(y[t], ref))
    w.close()


@pytest.mark.parametrize("fmt", FORMATS)
@pytest.mark.parametrize("shape", SWEEP, ids=lambda s: f"{s[0]}x{s[1]}")
def test_qgemm_sweep_shapes_all_batches(backend, oracle, nb, shape, fmt):
    """Config S in full on the tensor-core path: all five weight shapes, all
    four formats, M in {16, 64, 512} (and the GEMV's 1 and 4 above); tokens 0,
    M/2 and M-1 against the oracle's sequential f32 matvec.  The 128256-row
    head repeats 4096 drawn rows (quantizing 525M values would dominate the
    test); every other shape is drawn in full."""
    n, k = shape
    rng = np.random.default_rng(90 + n + k)
    if n > 16384:
        base = oracle.quantize(getattr(oracle, fmt), weights(rng, 4096 * k))
        q = np.tile(base.reshape(4096, -1), (n // 4096 + 1, 1))[:n].reshape(-1)
    else:
        q = oracle.quantize(getattr(oracle, fmt), weights(rng, n * k))
    w = nb.QWeight(backend, getattr(nb, fmt), n, k, q)
    for m in (16, 64, 512):
        x = rng.standard_normal((m, k)).astype(np.float32)
        y = w.matvec(x)
        for t in sorted({0, m // 2, m - 1}):
            ref = oracle.qmatvec(getattr(oracle, fmt), q, n, k, x[t], threads=16)
            assert rel_err(y[t], ref) < REL_TOL, (m, t, rel_err(y[t], ref))
    w.close()


@pytest.mark.parametrize("fmt", ["Q8_0", "Q4_0"])
@pytest.mark.parametrize("m", [33, 64, 130])
def test_qgemm_wide_matrix_token_tile(backend, oracle, nb, m, fmt):
    """Matrices whose 128-row tiles cover every SM run the block formats with
    64-token tiles (m > 32); padded tokens in the last tile stay unused."""
    n, k = 149 * 128 + 32, 512
    rng = np.random.default_rng(63 + m)
    q = oracle.quantize(getattr(oracle, fmt), weights(rng, n * k))
    w = nb.QWeight(backend, getattr(nb, fmt), n, k, q)
    x = rng.standard_normal((m, k)).astype(np.float32)
    y = w.matvec(x)
    for t in sorted({0, 31, 32, m // 2, m - 1}):
        ref = oracle.qmatvec(getattr(oracle, fmt), q, n, k, x[t], threads=16)
        assert rel_err(y[t], ref) < REL_TOL, (t, rel_err(y[t], ref))
    w.close()


@pytest.mark.parametrize("fmt", FORMATS)
def test_qgemm_edge_cases(backend, oracle, nb, fmt):
    """Zero, huge, tiny and mixed-scale tokens; a partial 128-row tile."""
    rng = np.random.default_rng(61)
    n, k = 72, 768
    F = getattr(oracle, fmt)
    q = oracle.quantize(F, weights(rng, n * k))
    x = rng.standard_normal((9, k)).astype(np.float32)
    x[0] = 0.0
    x[1] *= 3e4
    x[2] *= 1e-6
    x[3, :256] *= 1e4
    x[4, 256:] = 0.0
    y = backend.qmatvec(getattr(nb, fmt), q, n, k, x)
    assert np.all(y[0] == 0.0)
    for t in range(1, 9):
        assert rel_err(y[t], oracle.qmatvec(F, q, n, k, x[t])) < REL_TOL, t


def test_qgemm_matches_gemv_path(backend, nb, oracle):
    """The same tokens through the GEMV (batch of 4) and the GEMM (batch of 8)."""
    rng = np.random.default_rng(62)
    n, k = 2048, 2048
    q = oracle.quantize(oracle.Q4_K, weights(rng, n * k))
    w = nb.QWeight(backend, nb.Q4_K, n, k, q)
    x = rng.standard_normal((8, k)).astype(np.float32)
    y8 = w.matvec(x)
    y4 = np.concatenate([w.matvec(x[:4]), w.matvec(x[4:])])
    assert rel_err(y8, y4) < 1e-4
    w.close()


def test_rms_norm_op(backend, oracle):
    rng = np.random.default_rng(50)
    x = rng.standard_normal((3, 4096)).astype(np.float32)
    w = rng.standard_normal(4096).astype(np.float32)
    y = backend.rms_norm(x, w, 1e-5)
    for r in range(3):
        assert rel_err(y[r], oracle.rms_norm(x[r], w, 1e-5)) < 1e-5
    kat = backend.rms_norm(np.array([1, 2, 3, 4], np.float32), np.ones(4, np.float32), 1e-5)
    assert np.all(np.abs(kat - np.array([1, 2, 3, 4], np.float32) / np.sqrt(np.float32(7.5))) < 1e-5)


def test_softmax_layer_norm_add_mul(backend, oracle):
    rng = np.random.default_rng(51)
    x = rng.standard_normal((2, 1000)).astype(np.float32)
    s = backend.softmax(x)
    for r in range(2):
        assert rel_err(s[r], oracle.softmax(x[r])) < 1e-5
    w = rng.standard_normal(1000).astype(np.float32)
    b = rng.standard_normal(1000).astype(np.float32)
    ln = backend.layer_norm(x, w, b, 1e-5)
    xd = x.astype(np.float64)
    ref = (xd - xd.mean(1, keepdims=True)) / np.sqrt(xd.var(1, keepdims=True) + 1e-5) * w + b
    assert np.max(np.abs(ln - ref)) < 1e-4
    a = rng.standard_normal(777).astype(np.float32)
    c = rng.standard_normal(777).astype(np.float32)
    from nexus_b200 import _lib as L
    assert np.array_equal(backend.binary(L.OP_ADD, a, c), a + c)
    assert np.array_equal(backend.binary(L.OP_MUL, a, c), a * c)


@pytest.mark.parametrize("transpose_b", [True, False])
def test_matmul_op(backend, transpose_b):
    import torch
    rng = np.random.default_rng(52)
    a = rng.standard_normal((37, 70)).astype(np.float32)
    b = rng.standard_normal((45, 70) if transpose_b else (70, 45)).astype(np.float32)
    c = backend.matmul(a, b, transpose_b)
    ref = torch.from_numpy(a).double() @ (torch.from_numpy(b).double().T if transpose_b else torch.from_numpy(b).double())
    assert np.max(np.abs(c - ref.numpy())) < 1e-3
    kat = backend.matmul(np.array([[1, 2], [3, 4]], np.float32), np.array([[5, 6], [7, 8]], np.float32), False)
    assert np.array_equal(kat, np.array([[19, 22], [43, 50]], np.float32))  # src/backend/cpu.rs:232-237


def test_rope_and_argmax_ops(backend, oracle):
    rng = np.random.default_rng(53)
    x = rng.standard_normal(8 * 128).astype(np.float32)
    # the generic op evaluates powf/cosf/sinf on the device (the decode path uses
    # a host table with glibc's values); at position 511 the angles reach 511 rad
    # and the two libms differ by a few ulp
    for pos in (0, 1, 511):
        got = backend.rope(x, pos, 128, 500000.0)
        assert np.max(np.abs(got - oracle.rope_single(x, pos, 128, 500000.0))) < 1e-4
    logits = rng.standard_normal(128256).astype(np.float32)
    assert backend.argmax(logits) == oracle.greedy(logits)
    tie = np.array([1.0, 3.0, 3.0, np.nan, np.inf], np.float32)
    assert backend.argmax(tie) == oracle.greedy(tie) == 2
    assert backend.argmax(np.array([np.nan, -np.inf], np.float32)) == 0


@pytest.mark.parametrize("hq,hkv,d,seq", [(8, 4, 32, 1), (8, 4, 32, 130), (32, 8, 128, 577), (4, 4, 64, 33)])
def test_attention_op(backend, hq, hkv, d, seq):
    rng = np.random.default_rng(54 + seq)
    q = rng.standard_normal(hq * d).astype(np.float32)
    k = rng.standard_normal((seq, hkv * d)).astype(np.float32)
    v = rng.standard_normal((seq, hkv * d)).astype(np.float32)
    out = backend.attention(q, k, v, hq, hkv, d)
    g = hq // hkv
    ref = np.zeros(hq * d)
    for h in range(hq):
        kh = k[:, (h // g) * d:(h // g + 1) * d].astype(np.float64)
        vh = v[:, (h // g) * d:(h // g + 1) * d].astype(np.float64)
        s = kh @ q[h * d:(h + 1) * d] / np.sqrt(d)
        p = np.exp(s - s.max())
        ref[h * d:(h + 1) * d] = (p / p.sum()) @ vh
    assert np.max(np.abs(out - ref)) < 1e-4


def _packed_stream(oracle, bits, x):
    """PackedKvBuffer of rows x [seq][kv_dim] (src/engine/mod.rs:209-232):
    (codes, mins, scales) and the values the cache reads back (value_at)."""
    seq, kv_dim = x.shape
    pk = oracle.PackedKv(bits, kv_dim, seq)
    for t in range(seq):
        pk.add(t, x[t])
    return pk.raw(seq), pk.get_all(seq).reshape(seq, kv_dim)


def _attention_ref(q, kval, vval, hq, hkv, d):
    g = hq // hkv
    ref = np.zeros(hq * d)
    for h in range(hq):
        kh = kval[:, (h // g) * d:(h // g + 1) * d].astype(np.float64)
        vh = vval[:, (h // g) * d:(h // g + 1) * d].astype(np.float64)
        s = kh @ q[h * d:(h + 1) * d].astype(np.float64) / np.sqrt(d)
        p = np.exp(s - s.max())
        ref[h * d:(h + 1) * d] = (p / p.sum()) @ vh
    return ref


@pytest.mark.parametrize("hq,hkv,d,seq,bits", [
    (32, 8, 128, 1, (4, 4)), (32, 8, 128, 577, (4, 4)), (32, 8, 128, 4133, (4, 4)),
    (64, 8, 128, 300, (4, 4)), (8, 8, 128, 130, (4, 4)), (16, 8, 128, 70, (4, 4)),
    (32, 8, 128, 515, (3, 2)), (32, 8, 128, 515, (3, 4)), (32, 8, 128, 515, (6, 6)),
    (32, 8, 128, 515, (8, 8)), (32, 8, 128, 515, (2, 2)), (64, 8, 128, 260, (8, 4)),
    (8, 4, 64, 200, (4, 4)), (8, 4, 32, 65, (3, 2)), (32, 8, 128, 100, (5, 7))])
def test_attention_packed_op(backend, oracle, hq, hkv, d, seq, bits):
    """Decode attention over packed K/V (head_dim 128 with bits 2/3/4/6/8 runs on
    the tensor-core kernel, the rest on the per-element one) against float64
    attention over the values the packed cache reads back."""
    rng = np.random.default_rng(90 + seq + 7 * bits[0] + bits[1])
    q = (rng.standard_normal(hq * d) * 2.0).astype(np.float32)
    k = (rng.standard_normal((seq, hkv * d)) + 0.3).astype(np.float32)
    v = rng.standard_normal((seq, hkv * d)).astype(np.float32)
    kraw, kval = _packed_stream(oracle, bits[0], k)
    vraw, vval = _packed_stream(oracle, bits[1], v)
    out = backend.attention_packed(q, kraw, vraw, hq, hkv, d, bits[0], bits[1])
    ref = _attention_ref(q, kval, vval, hq, hkv, d)
    err = np.max(np.abs(out - ref))
    assert err < 2e-4 * max(1.0, np.max(np.abs(ref))), err


def test_attention_packed_extreme_scales(backend, oracle):
    """Per-token scales spanning 2^-20 .. 2^10 and a constant token (range 0 ->
    scale 1.0): the value weights stay in f16 range relative to their maximum."""
    rng = np.random.default_rng(97)
    hq, hkv, d, seq = 32, 8, 128, 300
    q = rng.standard_normal(hq * d).astype(np.float32)
    mag = np.exp2(rng.uniform(-20, 10, seq)).astype(np.float32)[:, None]
    k = (rng.standard_normal((seq, hkv * d)) * 0.05).astype(np.float32)
    v = (rng.standard_normal((seq, hkv * d)) * mag).astype(np.float32)
    v[7] = 0.25
    kraw, kval = _packed_stream(oracle, 4, k)
    vraw, vval = _packed_stream(oracle, 4, v)
    out = backend.attention_packed(q, kraw, vraw, hq, hkv, d, 4, 4)
    ref = _attention_ref(q, kval, vval, hq, hkv, d)
    assert np.max(np.abs(out - ref)) < 2e-4 * np.max(np.abs(ref))


def test_dequantize_truncated_payload_is_an_error(backend, oracle, nb):
    q = oracle.quantize(oracle.Q4_K, np.ones(512, np.float32))
    with pytest.raises(nb.NexusError) as e:
        backend.dequantize(nb.Q4_K, q[:-1], 512)
    assert e.value.code == nb._lib.NEXUS_E_TRUNCATED


@pytest.mark.parametrize("bits", [2, 3, 4, 6, 8])
def test_kv_quantize_bit_exact(backend, oracle, bits):
    """Device packing of one KV vector equals PackedKvBuffer::add bit for bit."""
    rng = np.random.default_rng(60 + bits)
    for n, scale in ((1024, 1.0), (128, 0.05), (8, 3.0)):
        v = (rng.standard_normal(n) * scale).astype(np.float32)
        data, mn, sc = backend.kv_quantize(v, bits)
        ref = oracle.PackedKv(bits, n, 1)
        ref.add(0, v)
        rdata, rmin, rscale = ref.raw(1)
        assert np.array_equal(data, rdata)
        assert np.float32(mn) == rmin[0] and np.float32(sc) == rscale[0]
    const = np.full(64, 0.75, np.float32)  # range <= 1e-8 -> scale 1.0
    data, mn, sc = backend.kv_quantize(const, bits)
    assert sc == 1.0 and np.float32(mn) == np.float32(0.75) and not data.any()
