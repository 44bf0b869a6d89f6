"""ctypes wrapper of the CPU parity oracle (oracle/liboracle.so).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the
CPU-baseline legs of bench.py, never by the shipped package.  The oracle is a
C restatement of the reference's (luen-eth/Nexus) CPU decode path; see
oracle/nexus_oracle.c for the file:line citations.
"""
from __future__ import annotations

import ctypes as C
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / "liboracle.so"

F32, F16, Q4_0, Q8_0, Q2_K, Q4_K, BF16 = 0, 1, 2, 8, 10, 12, 28
ORC_OK = 0


class SynthConfig(C.Structure):
    _fields_ = [("num_layers", C.c_uint32), ("hidden_size", C.c_uint32), ("num_heads", C.c_uint32),
                ("num_kv_heads", C.c_uint32), ("ff_dim", C.c_uint32), ("vocab_size", C.c_uint32),
                ("context_length", C.c_uint32), ("rope_theta", C.c_float), ("weight_std", C.c_float),
                ("seed", C.c_uint64), ("attn_format", C.c_int), ("ffn_format", C.c_int), ("embd_format", C.c_int),
                ("head_format", C.c_int), ("norm_format", C.c_int), ("threads", C.c_int),
                ("repeat_chunks", C.c_uint32)]


class ModelInfo(C.Structure):
    _fields_ = [("num_layers", C.c_uint32), ("hidden_size", C.c_uint32), ("ff_dim", C.c_uint32),
                ("num_heads", C.c_uint32), ("num_kv_heads", C.c_uint32), ("head_dim", C.c_uint32),
                ("vocab_rows", C.c_uint32), ("max_seq_len", C.c_uint32), ("rope_freq_base", C.c_float),
                ("rms_norm_eps", C.c_float), ("kv_bits_k", C.c_uint32), ("kv_bits_v", C.c_uint32)]


_lib = None


def build() -> Path:
    srcs = [HERE / "nexus_oracle.c", HERE / "nexus_oracle.h", HERE / "Makefile"]
    if not LIB.exists() or any(s.stat().st_mtime > LIB.stat().st_mtime for s in srcs):
        subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB


def load() -> C.CDLL:
    global _lib
    if _lib is None:
        build()
        lib = C.CDLL(str(LIB))
        P = C.c_void_p
        sig = {
            "orc_f32_to_f16": (C.c_uint16, [C.c_float]),
            "orc_f16_to_f32": (C.c_float, [C.c_uint16]),
            "orc_type_size": (C.c_size_t, [C.c_int, C.c_size_t]),
            "orc_quantize": (C.c_size_t, [C.c_int, P, C.c_size_t, P]),
            "orc_dequantize": (C.c_int, [C.c_int, P, C.c_size_t, C.c_size_t, P]),
            "orc_rms_norm": (None, [P, P, C.c_size_t, C.c_float, P]),
            "orc_rope_single": (None, [P, C.c_size_t, C.c_size_t, C.c_float]),
            "orc_matvec": (None, [P, C.c_size_t, C.c_size_t, P, P]),
            "orc_qmatvec": (C.c_int, [C.c_int, P, C.c_size_t, C.c_size_t, P, P, C.c_int]),
            "orc_greedy": (C.c_uint32, [P, C.c_size_t]),
            "orc_softmax": (None, [P, C.c_size_t, P]),
            "orc_packed_kv_new": (P, [C.c_uint32, C.c_size_t, C.c_size_t]),
            "orc_packed_kv_free": (None, [P]),
            "orc_packed_kv_add": (None, [P, C.c_size_t, P]),
            "orc_packed_kv_value_at": (C.c_float, [P, C.c_size_t, C.c_size_t]),
            "orc_packed_kv_get_all": (None, [P, C.c_size_t, P]),
            "orc_packed_kv_shift_left": (None, [P, C.c_size_t]),
            "orc_packed_kv_bytes_per_token": (C.c_size_t, [P]),
            "orc_packed_kv_data": (P, [P]),
            "orc_packed_kv_mins": (P, [P]),
            "orc_packed_kv_scales": (P, [P]),
            "orc_model_load": (C.c_int, [C.c_char_p, C.c_uint32, C.c_uint32, C.c_int, C.c_uint32, C.POINTER(P)]),
            "orc_model_free": (None, [P]),
            "orc_model_get_info": (None, [P, C.POINTER(ModelInfo)]),
            "orc_model_set_threads": (None, [P, C.c_int]),
            "orc_model_set_eps": (None, [P, C.c_float]),
            "orc_model_decode": (C.c_int, [P, C.c_uint32, C.c_size_t, P]),
            "orc_model_prefill": (C.c_int, [P, P, C.c_size_t, P]),
            "orc_model_generate": (C.c_int, [P, P, C.c_size_t, C.c_size_t, P]),
            "orc_model_seq_len": (C.c_size_t, [P, C.c_uint32]),
            "orc_model_last_hidden": (P, [P]),
            "orc_model_prefill_batched": (C.c_int, [P, P, C.c_size_t, P]),
            "orc_synth_write": (C.c_int, [C.c_char_p, P]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


def write_synthetic_model(path: str, *, num_layers: int, hidden_size: int, num_heads: int, num_kv_heads: int,
                          ff_dim: int, vocab_size: int, context_length: int, rope_theta: float,
                          attn_format: int, ffn_format: int, embd_format: int, head_format: int,
                          norm_format: int, weight_std: float = 0.02, seed: int = 0, threads: int = 0,
                          repeat_chunks: int = 0) -> None:
    """The seeded synthetic GGUF, byte-identical to the CUDA library's writer
    (so CPU-only runs need not load that library)."""
    cfg = SynthConfig(num_layers=num_layers, hidden_size=hidden_size, num_heads=num_heads,
                      num_kv_heads=num_kv_heads, ff_dim=ff_dim, vocab_size=vocab_size,
                      context_length=context_length, rope_theta=rope_theta, weight_std=weight_std, seed=seed,
                      attn_format=attn_format, ffn_format=ffn_format, embd_format=embd_format,
                      head_format=head_format, norm_format=norm_format, threads=threads,
                      repeat_chunks=repeat_chunks)
    rc = load().orc_synth_write(str(path).encode(), C.byref(cfg))
    if rc != ORC_OK:
        raise RuntimeError(f"oracle synthetic writer failed: {rc}")


def _p(a: np.ndarray) -> int:
    return a.ctypes.data


def f32_to_f16(x: float) -> int:
    return int(load().orc_f32_to_f16(x))


def f16_to_f32(h: int) -> float:
    return float(load().orc_f16_to_f32(h))


def type_size(fmt: int, n: int) -> int:
    return int(load().orc_type_size(fmt, n))


def quantize(fmt: int, x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    out = np.zeros(type_size(fmt, x.size), np.uint8)
    n = load().orc_quantize(fmt, _p(x), x.size, _p(out))
    assert n == out.size, (n, out.size)
    return out


def dequantize(fmt: int, data: np.ndarray, n: int) -> np.ndarray:
    data = np.ascontiguousarray(data, np.uint8)
    out = np.zeros(n, np.float32)
    rc = load().orc_dequantize(fmt, _p(data), data.size, n, _p(out))
    if rc != ORC_OK:
        raise ValueError(f"oracle dequantize failed: {rc}")
    return out


def rms_norm(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    w = np.ascontiguousarray(w, np.float32)
    out = np.zeros_like(x)
    load().orc_rms_norm(_p(x), _p(w), x.size, eps, _p(out))
    return out


def rope_single(x: np.ndarray, position: int, head_dim: int, base: float) -> np.ndarray:
    x = np.array(x, np.float32, copy=True)
    for h in range(0, x.size, head_dim):
        seg = np.ascontiguousarray(x[h:h + head_dim])
        load().orc_rope_single(_p(seg), position, head_dim, base)
        x[h:h + head_dim] = seg
    return x


def matvec(w: np.ndarray, rows: int, cols: int, x: np.ndarray) -> np.ndarray:
    w = np.ascontiguousarray(w, np.float32)
    x = np.ascontiguousarray(x, np.float32)
    y = np.zeros(rows, np.float32)
    load().orc_matvec(_p(w), rows, cols, _p(x), _p(y))
    return y


def qmatvec(fmt: int, w: np.ndarray, rows: int, cols: int, x: np.ndarray, threads: int = 1) -> np.ndarray:
    w = np.ascontiguousarray(w, np.uint8)
    x = np.ascontiguousarray(x, np.float32)
    y = np.zeros(rows, np.float32)
    rc = load().orc_qmatvec(fmt, _p(w), rows, cols, _p(x), _p(y), threads)
    assert rc == ORC_OK
    return y


def greedy(logits: np.ndarray) -> int:
    logits = np.ascontiguousarray(logits, np.float32)
    return int(load().orc_greedy(_p(logits), logits.size))


def softmax(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    out = np.zeros_like(x)
    load().orc_softmax(_p(x), x.size, _p(out))
    return out


class PackedKv:
    """PackedKvBuffer (src/engine/mod.rs:187-313)."""

    def __init__(self, bits: int, head_dim: int, max_seq_len: int):
        self.lib = load()
        self.h = self.lib.orc_packed_kv_new(bits, head_dim, max_seq_len)
        self.head_dim = head_dim

    def add(self, position: int, values: np.ndarray) -> None:
        v = np.ascontiguousarray(values, np.float32)
        self.lib.orc_packed_kv_add(self.h, position, _p(v))

    def value_at(self, position: int, dim: int) -> float:
        return float(self.lib.orc_packed_kv_value_at(self.h, position, dim))

    def get_all(self, seq_len: int) -> np.ndarray:
        out = np.zeros(seq_len * self.head_dim, np.float32)
        self.lib.orc_packed_kv_get_all(self.h, seq_len, _p(out))
        return out

    def shift_left(self, seq_len: int) -> None:
        self.lib.orc_packed_kv_shift_left(self.h, seq_len)

    def raw(self, seq_len: int):
        bpt = int(self.lib.orc_packed_kv_bytes_per_token(self.h))
        data = np.ctypeslib.as_array(C.cast(self.lib.orc_packed_kv_data(self.h), C.POINTER(C.c_uint8)),
                                     (seq_len * bpt,)).copy()
        mins = np.ctypeslib.as_array(C.cast(self.lib.orc_packed_kv_mins(self.h), C.POINTER(C.c_float)),
                                     (seq_len,)).copy()
        scales = np.ctypeslib.as_array(C.cast(self.lib.orc_packed_kv_scales(self.h), C.POINTER(C.c_float)),
                                       (seq_len,)).copy()
        return data, mins, scales

    def __del__(self):
        try:
            self.lib.orc_packed_kv_free(self.h)
        except Exception:
            pass


class Model:
    """InferenceEngine on the CPU (decode_with_cache / prefill / greedy generate)."""

    def __init__(self, path, kv_bits=(0, 0), threads: int = 1, max_seq_len: int = 0):
        self.lib = load()
        h = C.c_void_p()
        rc = self.lib.orc_model_load(str(path).encode(), kv_bits[0], kv_bits[1], threads, max_seq_len,
                                     C.byref(h))
        if rc != ORC_OK:
            raise RuntimeError(f"oracle model load failed: {rc}")
        self.h = h
        info = ModelInfo()
        self.lib.orc_model_get_info(h, C.byref(info))
        self.info = info

    def set_eps(self, eps: float) -> None:
        self.lib.orc_model_set_eps(self.h, eps)

    def set_threads(self, threads: int) -> None:
        self.lib.orc_model_set_threads(self.h, threads)

    def decode(self, token: int, position: int) -> np.ndarray:
        out = np.zeros(self.info.vocab_rows, np.float32)
        rc = self.lib.orc_model_decode(self.h, token, position, _p(out))
        if rc != ORC_OK:
            raise RuntimeError(f"oracle decode failed: {rc}")
        return out

    def prefill(self, tokens) -> np.ndarray:
        t = np.ascontiguousarray(np.asarray(tokens, np.uint32))
        out = np.zeros(self.info.vocab_rows, np.float32)
        rc = self.lib.orc_model_prefill(self.h, _p(t) if t.size else None, t.size, _p(out))
        if rc != ORC_OK:
            raise RuntimeError(f"oracle prefill failed: {rc}")
        return out

    def prefill_batched(self, tokens) -> np.ndarray:
        """prefill with the layer-major schedule: same bits as prefill()."""
        t = np.ascontiguousarray(np.asarray(tokens, np.uint32))
        out = np.zeros(self.info.vocab_rows, np.float32)
        rc = self.lib.orc_model_prefill_batched(self.h, _p(t) if t.size else None, t.size, _p(out))
        if rc != ORC_OK:
            raise RuntimeError(f"oracle batched prefill failed: {rc}")
        return out

    def generate(self, prompt, max_tokens: int) -> list:
        p = np.ascontiguousarray(np.asarray(prompt, np.uint32))
        out = np.zeros(p.size + max_tokens, np.uint32)
        rc = self.lib.orc_model_generate(self.h, _p(p) if p.size else None, p.size, max_tokens, _p(out))
        if rc != ORC_OK:
            raise RuntimeError(f"oracle generate failed: {rc}")
        return out.tolist()

    def seq_len(self, layer: int = 0) -> int:
        return int(self.lib.orc_model_seq_len(self.h, layer))

    def last_hidden(self) -> np.ndarray:
        p = self.lib.orc_model_last_hidden(self.h)
        return np.ctypeslib.as_array(C.cast(p, C.POINTER(C.c_float)), (self.info.hidden_size,)).copy()

    def __del__(self):
        try:
            self.lib.orc_model_free(self.h)
        except Exception:
            pass
