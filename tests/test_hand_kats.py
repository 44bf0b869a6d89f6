"""Byte-level known answers for the K-quant formats and the GGUF container,
written down by hand from the reference's definitions (not computed by the
oracle), and a transcription of the reference's GGUF byte-stream test.

Q4_K (`dequantize_q4_k`, src/gguf/mod.rs:1032-1054; scale unpacking
`unpack_q4_k_scales`, :1547-1554): a 144-byte block is d (f16) | dmin (f16) |
12 packed scale bytes | 128 code bytes.  scales[i] = p[i] & 63,
mins[i] = p[i+4] & 63, scales[i+4] = (p[i+8] & 15) | (p[i] >> 6) << 4,
mins[i+4] = (p[i+8] >> 4) | (p[i+4] >> 6) << 4 (i < 4); element i uses the low
nibble of qs[i] for i < 128 and the high nibble of qs[i-128] above, sub-block
i / 32, value d*scale*q - dmin*min.

Q2_K (`dequantize_q2_k`, :1057-1088): 84 bytes = 16 scale bytes | 64 code
bytes | d | dmin; q = (qs[i/4] >> 2*(i%4)) & 3, scale byte i/16: low nibble
scale, high nibble min.

The products d*scale*q and dmin*min are exact in f32 for these formats (an
f16 mantissa of 11 bits times at most 10 bits), so only the final subtraction
rounds; the second d/dmin pair below is not a power of two, so those expected
values are that one rounding, stated as f32 bit patterns.

The CPU tests pin the oracle; the GPU test runs the same blocks through the
device dequantization (tile layout, then tile to f32).
"""
import struct

import numpy as np
import pytest

# Q4_K block: scale bytes p[0..11]; qs[j] = (7j + 3) mod 256
Q4K_SCALES = [0x41, 0x02, 0xC3, 0x04, 0x05, 0x46, 0x07, 0x88, 0x21, 0x43, 0x65, 0x87]
# unpacked by hand: scales = [1, 2, 3, 4, 17, 3, 53, 7], mins = [5, 6, 7, 8, 2, 20, 6, 40]
Q4K_QS = [(7 * j + 3) & 0xFF for j in range(128)]
# element: (q, sub-block) derivation, value at d = 0.5, dmin = 0.25
Q4K_EXACT = {
    0: 0.25,     # qs[0] = 3 -> low 3; sub 0 (1, 5): 0.5*1*3 - 0.25*5
    33: 8.5,     # qs[33] = 234 = 0xEA -> low 10; sub 1 (2, 6): 10 - 1.5
    100: 28.0,   # qs[100] = 191 = 0xBF -> low 15; sub 3 (4, 8): 30 - 2
    130: 8.0,    # qs[2] = 17 = 0x11 -> high 1; sub 4 (17, 2): 8.5 - 0.5
    200: 396.0,  # qs[72] = 251 = 0xFB -> high 15; sub 6 (53, 6): 397.5 - 1.5
    255: 14.5,   # qs[127] = 124 = 0x7C -> high 7; sub 7 (7, 40): 24.5 - 10
}
# d = f16 0x2E66 = 0.0999755859375, dmin = f16 0x2A3D = 0.048736572265625
Q4K_ROUNDED = {0: 0x3D666000, 33: 0x3FDA8200, 100: 0x40B37A00, 130: 0x3FCD1200, 200: 0x429E6058,
               255: 0x403CC200}

# Q2_K block: scale byte j = (j + 1) & 15 | (15 - j) << 4; qs[k] = (37k + 11) mod 256
Q2K_SCALES = [((j + 1) & 0xF) | ((15 - j) << 4) for j in range(16)]
Q2K_QS = [(37 * k + 11) & 0xFF for k in range(64)]
Q2K_EXACT = {
    0: -2.25,    # qs[0] = 0b00001011, bits 0-1 = 3; scale byte 0 (1, 15): 1.5 - 3.75
    5: -3.75,    # qs[1] = 0b00110000, bits 2-3 = 0: 0 - 3.75
    6: -2.25,    # qs[1], bits 4-5 = 3: 1.5 - 3.75
    100: -2.25,  # qs[25] = 0b10101000, bits 0-1 = 0; scale byte 6 (7, 9): 0 - 2.25
    103: 4.75,   # qs[25], bits 6-7 = 2: 7 - 2.25
    230: -0.25,  # qs[57] = 0b01001000, bits 4-5 = 0; scale byte 14 (15, 1): 0 - 0.25
    231: 7.25,   # qs[57], bits 6-7 = 1: 7.5 - 0.25
    255: 0.0,    # scale byte 15 = 0x00 (16 & 15 = 0, min 0)
}
Q2K_ROUNDED = {0: 0xBEDCBC00, 5: 0xBF3B2600, 6: 0xBEDCBC00, 100: 0xBEE09400, 103: 0x3F760600,
               230: 0xBD47A000, 231: 0x3FB9B700, 255: 0x00000000}

HALF, QUARTER, D_ODD, DMIN_ODD = 0x3800, 0x3400, 0x2E66, 0x2A3D


def q4k_block(d_bits, dmin_bits):
    return np.frombuffer(struct.pack("<HH", d_bits, dmin_bits) + bytes(Q4K_SCALES) + bytes(Q4K_QS), np.uint8)


def q2k_block(d_bits, dmin_bits):
    return np.frombuffer(bytes(Q2K_SCALES) + bytes(Q2K_QS) + struct.pack("<HH", d_bits, dmin_bits), np.uint8)


CASES = [
    ("Q4_K", q4k_block, 144, Q4K_EXACT, Q4K_ROUNDED),
    ("Q2_K", q2k_block, 84, Q2K_EXACT, Q2K_ROUNDED),
]


def _check(values, exact, rounded_bits, which):
    if which == "exact":
        for i, v in exact.items():
            assert values[i] == np.float32(v), (i, values[i], v)
    else:
        bits = values.view(np.uint32)
        for i, b in rounded_bits.items():
            assert int(bits[i]) == b, (i, hex(int(bits[i])), hex(b))


@pytest.mark.parametrize("fmt,make,nbytes,exact,rounded", CASES, ids=[c[0] for c in CASES])
def test_oracle_kquant_byte_known_answers(oracle, fmt, make, nbytes, exact, rounded):
    code = getattr(oracle, fmt)
    blk = make(HALF, QUARTER)
    assert blk.size == nbytes == oracle.type_size(code, 256)
    _check(oracle.dequantize(code, blk, 256), exact, rounded, "exact")
    _check(oracle.dequantize(code, make(D_ODD, DMIN_ODD), 256), exact, rounded, "rounded")
    # a second block after the first: element 256 + i equals element i of the second block
    two = np.concatenate([make(D_ODD, DMIN_ODD), blk])
    out = oracle.dequantize(code, two, 512)
    _check(out[256:], exact, rounded, "exact")
    _check(out[:256], exact, rounded, "rounded")


@pytest.mark.gpu
@pytest.mark.parametrize("fmt,make,nbytes,exact,rounded", CASES, ids=[c[0] for c in CASES])
def test_device_kquant_byte_known_answers(backend, nb, fmt, make, nbytes, exact, rounded):
    code = getattr(nb, fmt)
    _check(backend.dequantize(code, make(HALF, QUARTER), 256), exact, rounded, "exact")
    _check(backend.dequantize(code, make(D_ODD, DMIN_ODD), 256), exact, rounded, "rounded")
    # as a resident matrix: 32 rows (one row group) of 2 super-blocks, the
    # tile layout's chunk reordering undone by the tile-to-f32 kernel
    rows = [np.concatenate([make(D_ODD, DMIN_ODD), make(HALF, QUARTER)]) if r % 2 else
            np.concatenate([make(HALF, QUARTER), make(D_ODD, DMIN_ODD)]) for r in range(32)]
    w = nb.QWeight(backend, code, 32, 512, np.concatenate(rows))
    got = w.dequantize().reshape(32, 512)
    w.close()
    for r in range(32):
        first, second = ("rounded", "exact") if r % 2 else ("exact", "rounded")
        _check(got[r, :256], exact, rounded, first)
        _check(got[r, 256:], exact, rounded, second)


# -- GGUF byte stream: src/gguf/mod.rs:1636-1679 (test_parse_file_reads_real_tensor_data) --

def _u32(v):
    return struct.pack("<I", v)


def _u64(v):
    return struct.pack("<Q", v)


def _str(s):
    return _u64(len(s)) + s.encode()


def _kv_u32(key, v):
    return _str(key) + _u32(4) + _u32(v)      # GgufValueType::U32 = 4


def _kv_str(key, v):
    return _str(key) + _u32(8) + _str(v)      # GgufValueType::String = 8


def gguf_bytes():
    b = b"GGUF" + _u32(3) + _u64(1) + _u64(4)
    b += _kv_u32("general.alignment", 32) + _kv_str("general.architecture", "llama")
    b += _kv_u32("llama.embedding_length", 4) + _kv_u32("llama.block_count", 1)
    b += _str("token_embd.weight") + _u32(1) + _u64(4) + _u32(0) + _u64(0)   # 1 dim of 4, F32, offset 0
    b += bytes(-len(b) % 32)
    return b + np.array([1.0, -2.0, 3.5, 4.25], "<f4").tobytes()


def test_oracle_gguf_byte_stream(oracle, tmp_path):
    import ctypes as C
    data = gguf_bytes()
    path = tmp_path / "stream.gguf"
    path.write_bytes(data)
    lib = oracle.load()

    class TensorInfo(C.Structure):
        _fields_ = [("name", C.c_char * 256), ("n_dims", C.c_uint32), ("shape", C.c_uint64 * 4),
                    ("type", C.c_int), ("offset", C.c_uint64)]

    lib.orc_gguf_open.argtypes = [C.c_char_p, C.POINTER(C.c_void_p)]
    lib.orc_gguf_close.argtypes = [C.c_void_p]
    lib.orc_gguf_tensor_count.argtypes = [C.c_void_p]
    lib.orc_gguf_tensor_count.restype = C.c_size_t
    lib.orc_gguf_tensor.argtypes = [C.c_void_p, C.c_size_t]
    lib.orc_gguf_tensor.restype = C.POINTER(TensorInfo)
    lib.orc_gguf_tensor_data.argtypes = [C.c_void_p, C.POINTER(TensorInfo)]
    lib.orc_gguf_tensor_data.restype = C.POINTER(C.c_float)
    lib.orc_gguf_data_offset.argtypes = [C.c_void_p]
    lib.orc_gguf_data_offset.restype = C.c_uint64
    lib.orc_gguf_get_usize.argtypes = [C.c_void_p, C.c_char_p, C.POINTER(C.c_uint64)]
    g = C.c_void_p()
    assert lib.orc_gguf_open(str(path).encode(), C.byref(g)) == 0
    try:
        assert lib.orc_gguf_data_offset(g) == len(data) - 16
        v = C.c_uint64()
        for key, want in [(b"general.alignment", 32), (b"llama.embedding_length", 4), (b"llama.block_count", 1)]:
            assert lib.orc_gguf_get_usize(g, key, C.byref(v)) == 1 and v.value == want, key
        assert lib.orc_gguf_tensor_count(g) == 1
        t = lib.orc_gguf_tensor(g, 0)
        assert t.contents.name == b"token_embd.weight" and t.contents.n_dims == 1
        assert t.contents.shape[0] == 4 and t.contents.type == 0 and t.contents.offset == 0
        p = lib.orc_gguf_tensor_data(g, t)
        assert [p[i] for i in range(4)] == [1.0, -2.0, 3.5, 4.25]
    finally:
        lib.orc_gguf_close(g)
    # the same stream cut inside the tensor data is rejected
    path.write_bytes(data[:-1])
    g2 = C.c_void_p()
    rc = lib.orc_gguf_open(str(path).encode(), C.byref(g2))
    if rc == 0:
        t = lib.orc_gguf_tensor(g2, 0)
        assert not lib.orc_gguf_tensor_data(g2, t), "truncated tensor data must not be readable"
        lib.orc_gguf_close(g2)
