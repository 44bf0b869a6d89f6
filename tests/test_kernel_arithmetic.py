"""Host restatements of the integer arithmetic the CUDA kernels rely on,
checked on the CPU (no GPU, no CUDA library):

* packed-cache attention (nexus_b200/csrc/kernels_attn_pk.cu): the query as a
  20-bit integer split into three signed 7-bit digits, and the affine split
  q.k_t = min_t*sum(q) + scale_t*sum_d q_d*code_{t,d} over the codes that
  PackedKvBuffer stores (src/engine/mod.rs:209-256);
* the GEMV input planes (nexus_b200/csrc/kernels_gemv.cuh): x ~= u*z with z a
  24-bit integer held as a signed high byte and unsigned middle and low
  bytes (or a 16-bit one as a signed high and an unsigned low byte), the
  clamp that keeps the top byte in range, the error of the 24-bit form
  against the 16-bit one on heavy-tailed inputs, and the 16-bit form's error
  on normalized inputs.
"""
import numpy as np
import pytest


def q_digits(qi):
    """kernels_attn_pk.cu qdigit: qi = d2*2^14 + d1*2^7 + d0, signed digits."""
    qi = np.asarray(qi, np.int64)
    d0 = ((qi + 64) & 127) - 64
    r1 = (qi - d0) >> 7
    d1 = ((r1 + 64) & 127) - 64
    d2 = (r1 - d1) >> 7
    return d2, d1, d0


def q_scale_exponent(amax):
    """Power-of-two exponent e with amax * 2^e < 2^20 (kernels_attn_pk.cu)."""
    bits = np.float32(amax).view(np.uint32)
    eb = int((bits >> 23) & 255)
    return 60 if eb == 0 else max(-60, min(60, 20 - (eb - 126)))


@pytest.mark.parametrize("seed", range(5))
def test_query_digits_recombine_exactly(seed):
    rng = np.random.default_rng(seed)
    q = (rng.standard_normal(128) * 10.0 ** rng.uniform(-4, 4)).astype(np.float32)
    e = q_scale_exponent(np.max(np.abs(q)))
    qi = np.rint(q.astype(np.float64) * 2.0 ** e).astype(np.int64)
    assert np.max(np.abs(qi)) < 2 ** 20
    d2, d1, d0 = q_digits(qi)
    for d in (d2, d1, d0):
        assert d.min() >= -128 and d.max() <= 127  # each fits an s8 operand
    assert np.array_equal(d2 * 16384 + d1 * 128 + d0, qi)
    # the rounding of q to 2^-e steps is far below f32 attention noise
    assert np.max(np.abs(qi * 2.0 ** -e - q)) <= 2.0 ** -e * 0.5 + 1e-30


@pytest.mark.parametrize("bits", [2, 3, 4, 6, 8])
def test_affine_split_of_packed_scores(oracle, bits):
    """Scores from the packed codes via min*sum(q) + scale*sum(q*code) equal the
    dot products with the values the packed cache reads back (value_at)."""
    rng = np.random.default_rng(70 + bits)
    d, seq = 128, 40
    pk = oracle.PackedKv(bits, d, seq)
    k = (rng.standard_normal((seq, d)) * 0.7 + 0.2).astype(np.float32)
    for t in range(seq):
        pk.add(t, k[t])
    data, mins, scales = pk.raw(seq)
    vals = pk.get_all(seq).reshape(seq, d).astype(np.float64)
    # unpack the codes LSB-first at bit offset i*bits (PackedKvBuffer::add)
    bpt = (d * bits + 7) // 8
    rows = data.reshape(seq, bpt)
    allbits = np.unpackbits(rows, axis=1, bitorder="little")[:, :d * bits].reshape(seq, d, bits)
    codes = (allbits * (1 << np.arange(bits))).sum(axis=2)
    q = rng.standard_normal(d).astype(np.float32)
    e = q_scale_exponent(np.max(np.abs(q)))
    qi = np.rint(q.astype(np.float64) * 2.0 ** e).astype(np.int64)
    exact_int = codes.astype(np.int64) @ qi                      # the mma's integer sums
    scores = mins.astype(np.float64) * q.astype(np.float64).sum() + scales * exact_int * 2.0 ** -e
    ref = vals @ q.astype(np.float64)
    assert np.max(np.abs(scores - ref)) < 1e-4 * max(1.0, np.max(np.abs(ref)))


def planes24(z):
    """kernels_gemv.cuh prep_sb_vals: signed high byte, unsigned middle and low."""
    z = np.asarray(z, np.int64)
    h = ((z >> 16) & 0xFF).astype(np.uint8).view(np.int8).astype(np.int64)
    m = (z >> 8) & 0xFF
    lo = z & 0xFF
    return h, m, lo


def quantize24(v):
    amax = np.float32(np.max(np.abs(v)))
    inv = np.float32(8388607.0) / amax
    z = np.rint((v.astype(np.float32) * inv).astype(np.float32)).astype(np.int64)
    return np.clip(z, -8388607, 8388607), amax / np.float32(8388607.0)


def test_24bit_planes_recombine_and_clamp():
    z = np.concatenate([np.arange(-300, 300), [-8388607, -8388606, -65536, -1, 0, 1, 65535, 8388606, 8388607]])
    h, m, lo = planes24(z)
    assert np.array_equal(h * 65536 + m * 256 + lo, z)
    # without the clamp the largest element can round to 2^23, whose high
    # byte reads back as -128: the clamp keeps every super-block in range
    rng = np.random.default_rng(3)
    overflow = 0
    for _ in range(2000):
        v = rng.standard_normal(256).astype(np.float32) * np.float32(10.0 ** rng.uniform(-3, 3))
        amax = np.float32(np.max(np.abs(v)))
        raw = np.rint((v * (np.float32(8388607.0) / amax)).astype(np.float32))
        overflow += int(np.any(raw > 8388607))
        zc, _ = quantize24(v)
        h, m, lo = planes24(zc)
        assert np.array_equal(h * 65536 + m * 256 + lo, zc)
    assert overflow > 0


def test_24bit_error_on_heavy_tailed_inputs():
    """SwiGLU-like inputs (products of Gaussians): the 16-bit form's dot-product
    error is ~2^8 times the 24-bit form's."""
    rng = np.random.default_rng(11)
    k = 4096
    g, u = rng.standard_normal(k), rng.standard_normal(k)
    x = (g / (1 + np.exp(-g)) * u).astype(np.float32)
    w = rng.standard_normal(k)
    exact = w @ x.astype(np.float64)
    errs = {}
    for levels in (32767, 8388607):
        approx = 0.0
        for s in range(k // 256):
            v = x[256 * s:256 * (s + 1)]
            amax = np.max(np.abs(v))
            z = np.clip(np.rint(v.astype(np.float64) * levels / amax), -levels, levels)
            approx += (amax / levels) * (w[256 * s:256 * (s + 1)] @ z)
        errs[levels] = abs(approx - exact) / (np.abs(w) @ np.abs(x))
    assert errs[8388607] < errs[32767] / 50
    assert errs[8388607] < 1e-7


def planes16(z):
    """kernels_gemv.cuh prep_sb_vals<2>: signed high byte, unsigned low byte."""
    z = np.asarray(z, np.int64)
    h = ((z >> 8) & 0xFF).astype(np.uint8).view(np.int8).astype(np.int64)
    return h, z & 0xFF


def test_16bit_planes_recombine_and_clamp():
    z = np.concatenate([np.arange(-600, 600), [-32767, -32766, -256, -1, 0, 1, 255, 32766, 32767]])
    h, lo = planes16(z)
    assert np.array_equal(h * 256 + lo, z)
    rng = np.random.default_rng(4)
    for _ in range(2000):
        v = rng.standard_normal(256).astype(np.float32) * np.float32(10.0 ** rng.uniform(-3, 3))
        amax = np.float32(np.max(np.abs(v)))
        zc = np.clip(np.rint((v * (np.float32(32767.0) / amax)).astype(np.float32)).astype(np.int64), -32767, 32767)
        h, lo = planes16(zc)
        assert np.array_equal(h * 256 + lo, zc)


def test_16bit_error_on_normalized_inputs():
    """RMSNorm outputs (Gaussian-like, the inputs of q/k/v, o_proj, gate/up and
    the head): the 16-bit form keeps the dot-product error near 1e-5 of the
    absolute sum, the range the per-op 1e-3 bound leaves far behind."""
    rng = np.random.default_rng(12)
    k = 4096
    x = rng.standard_normal(k)
    x = (x / np.sqrt(np.mean(x * x))).astype(np.float32)
    w = rng.standard_normal(k)
    exact = w @ x.astype(np.float64)
    approx = 0.0
    for s in range(k // 256):
        v = x[256 * s:256 * (s + 1)].astype(np.float64)
        amax = np.max(np.abs(v))
        z = np.clip(np.rint(v * 32767 / amax), -32767, 32767)
        approx += (amax / 32767) * (w[256 * s:256 * (s + 1)] @ z)
    assert abs(approx - exact) / (np.abs(w) @ np.abs(x)) < 2e-5
