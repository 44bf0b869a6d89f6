"""Python mirror of the reference's backend and engine surface over the C ABI.

Names follow the reference (luen-eth/Nexus, Rust):
  - ``BackendFactory`` / ``CudaBackend``: ``trait Backend`` and
    ``BackendFactory`` (src/backend/mod.rs:75-240).  The CUDA backend is
    available when an sm_100 device is present; selecting it never falls
    back to the CPU.
  - ``InferenceEngine``: ``load_model`` / ``decode_with_cache`` / ``prefill`` /
    ``generate`` (src/engine/mod.rs:539-1238), with greedy sampling.
  - ``decode_batch``: one step for several sequences, the items of
    ``Scheduler::decode_batch`` (src/scheduler.rs:207-229).
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass
from typing import Optional, Sequence

import numpy as np

from . import _lib as L


def _ptr(a: np.ndarray) -> int:
    return a.ctypes.data


@dataclass
class BackendCapabilities:
    backend: str
    available: bool
    features: list
    supported_ops: list
    device_count: int = 0


@dataclass
class MemoryInfo:
    total_memory: int
    free_memory: int
    used_memory: int

    def utilization(self) -> float:
        return 0.0 if self.total_memory == 0 else self.used_memory / self.total_memory


def cuda_capabilities() -> BackendCapabilities:
    lib = L.load()
    caps = L.Caps()
    L.check(lib.nexus_cuda_capabilities(C.byref(caps)))
    return BackendCapabilities(
        backend=caps.backend.decode(), available=bool(caps.available),
        features=[caps.features[i].decode() for i in range(caps.n_features)],
        supported_ops=[caps.supported_ops[i].decode() for i in range(caps.n_supported_ops)],
        device_count=caps.device_count)


class CudaBackend:
    """``Backend`` trait implementation for BackendType::Cuda."""

    def __init__(self, device: int = 0, kv_bits: tuple[int, int] = (0, 0), max_batch: int = 1,
                 max_seq_len: int = 0, flags: int = 0, page_tokens: int = 0, max_pages: int = 0,
                 tp_timeout_ms: int = 0):
        lib = L.load()
        cfg = L.Config()
        lib.nexus_cuda_config_default(C.byref(cfg))
        cfg.device = device
        cfg.kv_bits_k, cfg.kv_bits_v = kv_bits
        cfg.max_batch = max_batch
        cfg.max_seq_len = max_seq_len
        cfg.flags = flags
        if page_tokens:
            cfg.page_tokens = page_tokens
        cfg.max_pages = max_pages
        cfg.tp_timeout_ms = tp_timeout_ms
        h = C.c_void_p()
        L.check(lib.nexus_cuda_backend_create(C.byref(cfg), C.byref(h)))
        self._lib = lib
        self.handle = h

    # -- tensor parallelism (one process per GPU) --
    def tp_init(self, rank: int, world: int, uid: bytes) -> None:
        """Join the tensor-parallel group `uid` (from tp_unique_id on rank 0)."""
        buf = C.create_string_buffer(bytes(uid), L.TP_ID_BYTES)
        L.check(self._lib.nexus_cuda_tp_init(self.handle, rank, world, buf, L.TP_ID_BYTES), self.handle)

    def tp_allreduce_kind(self) -> str:
        """"none", "nccl" or "peer": how the hidden-state all-reduces run."""
        return {L.TP_NONE: "none", L.TP_NCCL: "nccl", L.TP_PEER: "peer"}[
            self._lib.nexus_cuda_tp_allreduce_kind(self.handle)]

    # -- trait methods --
    def name(self) -> str:
        return self._lib.nexus_cuda_backend_name(self.handle).decode()

    def backend_type(self) -> str:
        return "cuda"

    def is_available(self) -> bool:
        return True

    def memory_info(self) -> MemoryInfo:
        t, f, u = C.c_size_t(), C.c_size_t(), C.c_size_t()
        L.check(self._lib.nexus_cuda_memory_info(self.handle, C.byref(t), C.byref(f), C.byref(u)), self.handle)
        return MemoryInfo(t.value, f.value, u.value)

    def capabilities(self) -> BackendCapabilities:
        return cuda_capabilities()

    def synchronize(self) -> None:
        L.check(self._lib.nexus_cuda_synchronize(self.handle), self.handle)

    def execute(self, op: L.Op) -> None:
        L.check(self._lib.nexus_cuda_execute(self.handle, C.byref(op)), self.handle)

    def close(self) -> None:
        if self.handle:
            self._lib.nexus_cuda_backend_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # -- KernelOp helpers (host arrays) --
    def dequantize(self, fmt: int, blocks: np.ndarray, n: int) -> np.ndarray:
        out = np.empty(n, np.float32)
        blocks = np.ascontiguousarray(blocks, np.uint8)
        op = L.Op(kind=L.OP_DEQUANTIZE, a=_ptr(blocks), out=_ptr(out), len=n, m=blocks.nbytes, format=fmt)
        self.execute(op)
        return out

    def quantize(self, fmt: int, x: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, np.float32)
        out = np.empty(self._lib.nexus_format_bytes(fmt, x.size), np.uint8)
        self.execute(L.Op(kind=L.OP_QUANTIZE, a=_ptr(x), out=_ptr(out), len=x.size, format=fmt))
        return out

    def qmatvec(self, fmt: int, w_blocks: np.ndarray, rows: int, cols: int, x: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, np.float32).reshape(-1, cols)
        w_blocks = np.ascontiguousarray(w_blocks, np.uint8)
        out = np.empty((x.shape[0], rows), np.float32)
        self.execute(L.Op(kind=L.OP_QMATVEC, a=_ptr(x), b=_ptr(w_blocks), out=_ptr(out), m=x.shape[0], n=rows,
                          k=cols, format=fmt))
        return out

    def rms_norm(self, x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
        x = np.ascontiguousarray(x, np.float32)
        x2 = x.reshape(-1, x.shape[-1])
        w = np.ascontiguousarray(w, np.float32)
        out = np.empty_like(x2)
        self.execute(L.Op(kind=L.OP_RMS_NORM, a=_ptr(x2), b=_ptr(w), out=_ptr(out), m=x2.shape[0], n=x2.shape[1],
                          eps=eps))
        return out.reshape(x.shape)

    def layer_norm(self, x: np.ndarray, w: np.ndarray, b: Optional[np.ndarray], eps: float) -> np.ndarray:
        x = np.ascontiguousarray(x, np.float32)
        x2 = x.reshape(-1, x.shape[-1])
        w = np.ascontiguousarray(w, np.float32)
        bb = None if b is None else np.ascontiguousarray(b, np.float32)
        out = np.empty_like(x2)
        self.execute(L.Op(kind=L.OP_LAYER_NORM, a=_ptr(x2), b=_ptr(w), c=None if bb is None else _ptr(bb),
                          out=_ptr(out), m=x2.shape[0], n=x2.shape[1], eps=eps))
        return out.reshape(x.shape)

    def softmax(self, x: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, np.float32)
        x2 = x.reshape(-1, x.shape[-1])
        out = np.empty_like(x2)
        self.execute(L.Op(kind=L.OP_SOFTMAX, a=_ptr(x2), out=_ptr(out), m=x2.shape[0], n=x2.shape[1]))
        return out.reshape(x.shape)

    def matmul(self, a: np.ndarray, b: np.ndarray, transpose_b: bool) -> np.ndarray:
        a = np.ascontiguousarray(a, np.float32)
        b = np.ascontiguousarray(b, np.float32)
        m, k = a.shape
        n = b.shape[0] if transpose_b else b.shape[1]
        out = np.empty((m, n), np.float32)
        self.execute(L.Op(kind=L.OP_MATMUL, a=_ptr(a), b=_ptr(b), out=_ptr(out), m=m, n=n, k=k,
                          transpose_b=int(transpose_b)))
        return out

    def binary(self, kind: int, a: np.ndarray, b: np.ndarray) -> np.ndarray:
        a = np.ascontiguousarray(a, np.float32)
        b = np.ascontiguousarray(b, np.float32)
        out = np.empty_like(a)
        self.execute(L.Op(kind=kind, a=_ptr(a), b=_ptr(b), out=_ptr(out), len=a.size))
        return out

    def rope(self, x: np.ndarray, position: int, head_dim: int, base: float) -> np.ndarray:
        x = np.array(x, np.float32, copy=True)
        self.execute(L.Op(kind=L.OP_ROPE, a=_ptr(x), out=_ptr(x), m=x.size // head_dim, k=head_dim,
                          position=position, scale=base))
        return x

    def argmax(self, x: np.ndarray) -> int:
        x = np.ascontiguousarray(x, np.float32)
        out = np.zeros(1, np.uint32)
        self.execute(L.Op(kind=L.OP_ARGMAX, a=_ptr(x), out=_ptr(out), len=x.size))
        return int(out[0])

    def kv_quantize(self, values: np.ndarray, bits: int):
        """PackedKvBuffer::add of one vector: (packed bytes, min, scale)."""
        v = np.ascontiguousarray(values, np.float32)
        bpt = (v.size * bits + 7) // 8
        out = np.zeros(bpt + 8, np.uint8)
        self.execute(L.Op(kind=L.OP_KV_QUANTIZE, a=_ptr(v), out=_ptr(out), len=v.size, k=bits))
        return out[:bpt], float(out[bpt:bpt + 4].view(np.float32)[0]), float(out[bpt + 4:].view(np.float32)[0])

    def attention(self, q: np.ndarray, keys: np.ndarray, values: np.ndarray, num_q_heads: int,
                  num_kv_heads: int, head_dim: int, scale: float = 0.0) -> np.ndarray:
        q = np.ascontiguousarray(q, np.float32)
        keys = np.ascontiguousarray(keys, np.float32)
        values = np.ascontiguousarray(values, np.float32)
        seq = keys.size // (num_kv_heads * head_dim)
        out = np.empty(num_q_heads * head_dim, np.float32)
        self.execute(L.Op(kind=L.OP_ATTENTION, a=_ptr(q), b=_ptr(keys), c=_ptr(values), out=_ptr(out),
                          m=num_q_heads, n=seq, k=head_dim, kv_heads=num_kv_heads, scale=scale))
        return out

    def attention_packed(self, q: np.ndarray, keys: tuple, values: tuple, num_q_heads: int, num_kv_heads: int,
                         head_dim: int, bits_k: int, bits_v: int, scale: float = 0.0) -> np.ndarray:
        """Decode attention over packed caches; keys/values = (codes [seq][bpt] u8,
        mins [seq] f32, scales [seq] f32) as PackedKvBuffer holds them."""
        q = np.ascontiguousarray(q, np.float32)

        def blob(kv):
            data, mins, scales = kv
            return np.concatenate([np.ascontiguousarray(data, np.uint8).ravel(),
                                   np.ascontiguousarray(mins, np.float32).view(np.uint8),
                                   np.ascontiguousarray(scales, np.float32).view(np.uint8)])
        kb, vb = blob(keys), blob(values)
        seq = np.asarray(keys[1]).size
        out = np.empty(num_q_heads * head_dim, np.float32)
        self.execute(L.Op(kind=L.OP_ATTENTION_PACKED, a=_ptr(q), b=_ptr(kb), c=_ptr(vb), out=_ptr(out),
                          m=num_q_heads, n=seq, k=head_dim, kv_heads=num_kv_heads, scale=scale,
                          format=bits_k | (bits_v << 8)))
        return out


class QWeight:
    """A quantized matrix resident on the device in the GEMV tile layout."""

    def __init__(self, backend: CudaBackend, fmt: int, rows: int, cols: int, blocks: np.ndarray):
        self.backend = backend
        blocks = np.ascontiguousarray(blocks, np.uint8)
        h = C.c_void_p()
        L.check(backend._lib.nexus_cuda_qweight_create(backend.handle, fmt, rows, cols, _ptr(blocks), blocks.nbytes,
                                                       C.byref(h)), backend.handle)
        self.handle, self.rows, self.cols, self.fmt = h, rows, cols, fmt

    def matvec(self, x: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, np.float32).reshape(-1, self.cols)
        y = np.empty((x.shape[0], self.rows), np.float32)
        L.check(self.backend._lib.nexus_cuda_qmatvec_host(self.handle, _ptr(x), x.shape[0], _ptr(y)),
                self.backend.handle)
        return y

    def matvec_device(self, x_ptr: int, m: int, y_ptr: int) -> None:
        L.check(self.backend._lib.nexus_cuda_qmatvec_device(self.handle, x_ptr, m, y_ptr), self.backend.handle)

    def bench(self, x_ptr: int, m: int, y_ptr: int, iters: int = 20, flush_bytes: int = 256 << 20) -> float:
        """Mean device time (ms) of one GEMV launch, cold L2 before each."""
        ms = C.c_float()
        L.check(self.backend._lib.nexus_cuda_qmatvec_bench(self.handle, x_ptr, m, y_ptr, iters, flush_bytes,
                                                           C.byref(ms)), self.backend.handle)
        return ms.value

    def dequantize(self) -> np.ndarray:
        out = np.empty(self.rows * self.cols, np.float32)
        L.check(self.backend._lib.nexus_cuda_qweight_dequantize(self.handle, _ptr(out)), self.backend.handle)
        return out

    def nbytes(self) -> int:
        return int(self.backend._lib.nexus_cuda_qweight_bytes(self.handle))

    def close(self):
        if self.handle:
            self.backend._lib.nexus_cuda_qweight_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class InferenceEngine:
    """``InferenceEngine`` on the CUDA backend (src/engine/mod.rs:503-1238)."""

    def __init__(self, backend: CudaBackend):
        self.backend = backend
        self._lib = backend._lib
        self.model = None
        self.info: Optional[L.ModelInfo] = None

    def load_model(self, path: str) -> None:
        h = C.c_void_p()
        L.check(self._lib.nexus_cuda_model_load(self.backend.handle, str(path).encode(), C.byref(h)),
                self.backend.handle)
        self.model = h
        info = L.ModelInfo()
        L.check(self._lib.nexus_cuda_model_get_info(h, C.byref(info)))
        self.info = info
        self.vocab_size = info.vocab_rows
        self.num_layers = info.num_layers
        self.hidden_size = info.hidden_size

    def decode_with_cache(self, token: int, position: int, seq_id: int = 0,
                          want_logits: bool = True) -> tuple[Optional[np.ndarray], int]:
        logits = np.empty(self.info.vocab_rows, np.float32) if want_logits else None
        tok = C.c_uint32()
        L.check(self._lib.nexus_cuda_decode(self.model, seq_id, token, position,
                                            None if logits is None else _ptr(logits), C.byref(tok)),
                self.backend.handle)
        return logits, tok.value

    def prefill(self, tokens: Sequence[int], seq_id: int = 0,
                want_logits: bool = True) -> tuple[Optional[np.ndarray], int]:
        toks = np.ascontiguousarray(np.asarray(tokens, np.uint32))
        logits = np.empty(self.info.vocab_rows, np.float32) if (want_logits and toks.size) else None
        tok = C.c_uint32()
        L.check(self._lib.nexus_cuda_prefill(self.model, seq_id, _ptr(toks) if toks.size else None, toks.size,
                                             None if logits is None else _ptr(logits), C.byref(tok)),
                self.backend.handle)
        return logits, tok.value

    def generate(self, prompt: Sequence[int], max_tokens: int, seq_id: int = 0) -> list[int]:
        p = np.ascontiguousarray(np.asarray(prompt, np.uint32))
        out = np.zeros(p.size + max_tokens, np.uint32)
        L.check(self._lib.nexus_cuda_generate(self.model, seq_id, _ptr(p) if p.size else None, p.size, max_tokens,
                                              _ptr(out)), self.backend.handle)
        return out.tolist()

    def generate_with_draft_tokens(self, prompt: Sequence[int], max_tokens: int, draft: Sequence[int],
                                   window: int = 8, seq_id: int = 0) -> tuple[list[int], tuple[int, int]]:
        """generate_with_draft_tokens at temperature 0 (src/engine/mod.rs:1244-1291):
        returns (prompt + greedy continuation, (accepted, rejected)); draft
        windows are verified in one multi-token step each."""
        p = np.ascontiguousarray(np.asarray(prompt, np.uint32))
        d = np.ascontiguousarray(np.asarray(draft, np.uint32))
        out = np.zeros(p.size + max_tokens, np.uint32)
        acc, rej = C.c_uint32(), C.c_uint32()
        L.check(self._lib.nexus_cuda_generate_with_draft(self.model, seq_id, _ptr(p) if p.size else None, p.size,
                                                         _ptr(d) if d.size else None, d.size, max_tokens, window,
                                                         _ptr(out), C.byref(acc), C.byref(rej)), self.backend.handle)
        return out.tolist(), (acc.value, rej.value)

    def decode_batch(self, items: Sequence[tuple[int, int, int]], want_logits: bool = False,
                     page_ids: Optional[Sequence[Sequence[int]]] = None):
        """items: (seq_id, token, position) per sequence; page_ids: optional
        scheduler page list per item (Scheduler::allocate_kv_pages,
        src/scheduler.rs:333-361; an empty list keeps the sequence's current
        pages); returns (tokens, logits)."""
        n = len(items)
        arr = (L.DecodeItem * max(n, 1))()
        keep = []
        for i, (sid, tok, pos) in enumerate(items):
            arr[i].seq_id, arr[i].token, arr[i].position = sid, tok, pos
            arr[i].n_pages, arr[i].page_ids = 0, None
            if page_ids is not None and len(page_ids[i]):
                pg = np.ascontiguousarray(np.asarray(page_ids[i], np.uint32))
                keep.append(pg)
                arr[i].n_pages = pg.size
                arr[i].page_ids = pg.ctypes.data_as(C.POINTER(C.c_uint32))
        toks = np.zeros(max(n, 1), np.uint32)
        logits = np.empty((n, self.info.vocab_rows), np.float32) if want_logits else None
        L.check(self._lib.nexus_cuda_decode_batch(self.model, arr, n, _ptr(toks),
                                                  None if logits is None else _ptr(logits)),
                self.backend.handle)
        return toks[:n].tolist(), logits

    def seq_set_pages(self, seq_id: int, page_ids: Optional[Sequence[int]]) -> None:
        """Bind a request's KV page list (Scheduler::allocate_kv_pages,
        src/scheduler.rs:333-361) before its prefill; None or [] releases the
        pages and clears the sequence."""
        pg = np.ascontiguousarray(np.asarray(page_ids if page_ids is not None else [], np.uint32))
        L.check(self._lib.nexus_cuda_seq_set_pages(self.model, seq_id, _ptr(pg) if pg.size else None, pg.size),
                self.backend.handle)

    def seq_len(self, seq_id: int = 0) -> int:
        v = C.c_uint32()
        L.check(self._lib.nexus_cuda_seq_len(self.model, seq_id, C.byref(v)), self.backend.handle)
        return v.value

    def last_step_ms(self) -> float:
        v = C.c_float()
        L.check(self._lib.nexus_cuda_last_step_ms(self.model, C.byref(v)))
        return v.value

    def profile_decode(self, token: int, steps: int, seq_id: int = 0) -> list[dict]:
        """Per-kernel CUDA-event timings of `steps` decode steps (no graph)."""
        recs = (L.KernelProfile * 32)()
        n = C.c_int()
        L.check(self._lib.nexus_cuda_profile_decode(self.model, seq_id, token, steps, recs, 32, C.byref(n)),
                self.backend.handle)
        return [dict(name=recs[i].name.decode(), launches=recs[i].launches, total_ms=recs[i].total_ms,
                     bytes_per_launch=recs[i].bytes_per_launch) for i in range(n.value)]

    def close(self):
        if self.model:
            self._lib.nexus_cuda_model_free(self.model)
            self.model = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def tp_unique_id() -> bytes:
    """A fresh tensor-parallel group id (rank 0 creates it, every rank passes it to tp_init)."""
    lib = L.load()
    buf = C.create_string_buffer(L.TP_ID_BYTES)
    L.check(lib.nexus_cuda_tp_unique_id(buf, L.TP_ID_BYTES))
    return buf.raw


def tp_plan(num_heads: int, num_kv_heads: int, head_dim: int, ff_dim: int, vocab_rows: int, rank: int,
            world: int) -> dict:
    """The slice of the model one rank holds (nexus_tp_plan)."""
    lib = L.load()
    out = L.TpSlice()
    L.check(lib.nexus_tp_plan(num_heads, num_kv_heads, head_dim, ff_dim, vocab_rows, rank, world, C.byref(out)))
    return {k: getattr(out, k) for k, _ in L.TpSlice._fields_}


def write_synthetic_model(path: str, *, num_layers: int, hidden_size: int, num_heads: int, num_kv_heads: int,
                          ff_dim: int, vocab_size: int, context_length: int, rope_theta: float,
                          attn_format: int, ffn_format: int, embd_format: int, head_format: int,
                          norm_format: int, weight_std: float = 0.02, seed: int = 0, threads: int = 0,
                          repeat_chunks: int = 0) -> None:
    """Seeded LLaMA-style GGUF v3 in nexus-convert's file conventions
    (repeat_chunks > 0: each tensor repeats its first repeat_chunks * 65536
    drawn elements, for quick generation of very large models)."""
    lib = L.load()
    cfg = L.SynthConfig(num_layers=num_layers, hidden_size=hidden_size, num_heads=num_heads,
                        num_kv_heads=num_kv_heads, ff_dim=ff_dim, vocab_size=vocab_size,
                        context_length=context_length, rope_theta=rope_theta, weight_std=weight_std, seed=seed,
                        attn_format=attn_format, ffn_format=ffn_format, embd_format=embd_format,
                        head_format=head_format, norm_format=norm_format, threads=threads,
                        repeat_chunks=repeat_chunks)
    L.check(lib.nexus_synth_model_write(str(path).encode(), C.byref(cfg)))


def quantize_host(fmt: int, x: np.ndarray) -> np.ndarray:
    lib = L.load()
    x = np.ascontiguousarray(x, np.float32)
    out = np.empty(lib.nexus_format_bytes(fmt, x.size), np.uint8)
    n = lib.nexus_quantize_host(fmt, _ptr(x), x.size, _ptr(out))
    if n != out.size:
        raise L.NexusError(L.NEXUS_E_UNSUPPORTED_FORMAT, "host quantize failed")
    return out
