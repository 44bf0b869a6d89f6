"""ctypes binding of ``include/nexus_cuda.h`` (the C ABI of libnexus_cuda.so).

This is the same stub a Rust ``extern "C"`` crate, cgo or N-API binding would
be: plain pointers, sizes and int status codes.  The library is loaded from
this package directory; when it is missing the import fails loudly (there is
no CPU fallback for the CUDA backend).
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

HERE = Path(__file__).resolve().parent
# NEXUS_CUDA_LIB selects another build of the library (e.g. one built with
# different kernel parameters by nexus_b200/build.py --out ...)
LIB_PATH = Path(os.environ.get("NEXUS_CUDA_LIB", str(HERE / "libnexus_cuda.so")))

# status codes
NEXUS_OK = 0
NEXUS_E_INVALID = 1
NEXUS_E_UNSUPPORTED_FORMAT = 2
NEXUS_E_OOM = 3
NEXUS_E_CUDA = 4
NEXUS_E_COMM = 5
NEXUS_E_TIMEOUT = 6
NEXUS_E_IO = 7
NEXUS_E_MISSING_TENSOR = 8
NEXUS_E_TRUNCATED = 9
NEXUS_E_UNAVAILABLE = 10

# formats (GGUF type ids)
F32, F16, Q4_0, Q8_0, Q2_K, Q4_K, BF16 = 0, 1, 2, 8, 10, 12, 28
FORMAT_NAMES = {F32: "F32", F16: "F16", Q4_0: "Q4_0", Q8_0: "Q8_0", Q2_K: "Q2_K", Q4_K: "Q4_K", BF16: "BF16"}
FORMAT_IDS = {v: k for k, v in FORMAT_NAMES.items()}

# op kinds
OP_MATMUL, OP_ATTENTION, OP_LAYER_NORM, OP_RMS_NORM, OP_ADD, OP_MUL, OP_SOFTMAX = range(7)
OP_QUANTIZE, OP_DEQUANTIZE, OP_QMATVEC, OP_ROPE, OP_ARGMAX, OP_KV_QUANTIZE = 7, 8, 9, 10, 11, 12
OP_ATTENTION_PACKED = 13

CFG_NO_GRAPH = 0x1
CFG_NO_PDL = 0x2
CFG_PERSISTENT = 0x4
CFG_NCCL_ALLREDUCE = 0x8
TP_NONE, TP_NCCL, TP_PEER = 0, 1, 2
CFG_FAULT_STALL_BARRIER = 0x100


class Caps(C.Structure):
    _fields_ = [("available", C.c_int), ("device_count", C.c_int), ("backend", C.c_char_p),
                ("features", C.c_char_p * 16), ("n_features", C.c_int),
                ("supported_ops", C.c_char_p * 16), ("n_supported_ops", C.c_int)]


class Config(C.Structure):
    _fields_ = [("device", C.c_int), ("tp", C.c_int), ("kv_bits_k", C.c_uint32), ("kv_bits_v", C.c_uint32),
                ("max_batch", C.c_uint32), ("max_seq_len", C.c_uint32), ("page_tokens", C.c_uint32),
                ("max_pages", C.c_uint32), ("flags", C.c_uint32), ("tp_timeout_ms", C.c_uint32)]


class Op(C.Structure):
    _fields_ = [("kind", C.c_int), ("device_ptrs", C.c_int), ("a", C.c_void_p), ("b", C.c_void_p),
                ("c", C.c_void_p), ("out", C.c_void_p), ("m", C.c_size_t), ("n", C.c_size_t),
                ("k", C.c_size_t), ("len", C.c_size_t), ("kv_heads", C.c_size_t), ("position", C.c_size_t),
                ("scale", C.c_float), ("eps", C.c_float), ("format", C.c_int), ("transpose_b", C.c_int)]


class ModelInfo(C.Structure):
    _fields_ = [("num_layers", C.c_uint32), ("hidden_size", C.c_uint32), ("ff_dim", C.c_uint32),
                ("num_heads", C.c_uint32), ("num_kv_heads", C.c_uint32), ("head_dim", C.c_uint32),
                ("vocab_rows", C.c_uint32), ("max_seq_len", C.c_uint32), ("rope_freq_base", C.c_float),
                ("rms_norm_eps", C.c_float), ("weight_bytes", C.c_uint64), ("body_format", C.c_int),
                ("max_batch", C.c_uint32), ("page_tokens", C.c_uint32), ("max_pages", C.c_uint32)]


class DecodeItem(C.Structure):
    _fields_ = [("seq_id", C.c_uint32), ("token", C.c_uint32), ("position", C.c_uint32),
                ("n_pages", C.c_uint32), ("page_ids", C.POINTER(C.c_uint32))]


class ScheduledDecode(C.Structure):
    _fields_ = [("id", C.c_uint64), ("token", C.c_uint32), ("position", C.c_uint32), ("generated", C.c_uint32),
                ("prompt_len", C.c_uint32), ("n_pages", C.c_uint32), ("kv_pages", C.POINTER(C.c_uint32))]


class ServeEvent(C.Structure):
    _fields_ = [("request_id", C.c_uint64), ("token", C.c_uint32), ("index", C.c_uint32), ("done", C.c_uint32),
                ("status", C.c_int32)]


class KernelProfile(C.Structure):
    _fields_ = [("name", C.c_char * 24), ("launches", C.c_uint32), ("total_ms", C.c_float),
                ("bytes_per_launch", C.c_double)]


class SynthConfig(C.Structure):
    _fields_ = [("num_layers", C.c_uint32), ("hidden_size", C.c_uint32), ("num_heads", C.c_uint32),
                ("num_kv_heads", C.c_uint32), ("ff_dim", C.c_uint32), ("vocab_size", C.c_uint32),
                ("context_length", C.c_uint32), ("rope_theta", C.c_float), ("weight_std", C.c_float),
                ("seed", C.c_uint64), ("attn_format", C.c_int), ("ffn_format", C.c_int),
                ("embd_format", C.c_int), ("head_format", C.c_int), ("norm_format", C.c_int),
                ("threads", C.c_int), ("repeat_chunks", C.c_uint32)]


P = C.c_void_p
# (name, restype, argtypes) of every symbol declared in include/nexus_cuda.h
class TpSlice(C.Structure):
    _fields_ = [("q_head_begin", C.c_uint32), ("q_heads", C.c_uint32), ("kv_head_begin", C.c_uint32),
                ("kv_heads", C.c_uint32), ("ffn_begin", C.c_uint32), ("ffn_rows", C.c_uint32),
                ("vocab_begin", C.c_uint32), ("vocab_rows", C.c_uint32)]


TP_ID_BYTES = 128

SIGNATURES = [
    ("nexus_cuda_is_available", C.c_int, []),
    ("nexus_cuda_capabilities", C.c_int, [C.POINTER(Caps)]),
    ("nexus_cuda_config_default", None, [C.POINTER(Config)]),
    ("nexus_cuda_backend_create", C.c_int, [C.POINTER(Config), C.POINTER(P)]),
    ("nexus_cuda_backend_destroy", C.c_int, [P]),
    ("nexus_cuda_backend_name", C.c_char_p, [P]),
    ("nexus_cuda_memory_info", C.c_int, [P, C.POINTER(C.c_size_t), C.POINTER(C.c_size_t), C.POINTER(C.c_size_t)]),
    ("nexus_cuda_synchronize", C.c_int, [P]),
    ("nexus_cuda_last_error", C.c_char_p, [P]),
    ("nexus_cuda_tp_unique_id", C.c_int, [P, C.c_size_t]),
    ("nexus_cuda_tp_init", C.c_int, [P, C.c_int, C.c_int, P, C.c_size_t]),
    ("nexus_cuda_tp_allreduce_kind", C.c_int, [P]),
    ("nexus_tp_plan", C.c_int, [C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32, C.c_int, C.c_int,
                                C.POINTER(TpSlice)]),
    ("nexus_cuda_execute", C.c_int, [P, C.POINTER(Op)]),
    ("nexus_cuda_qweight_create", C.c_int, [P, C.c_int, C.c_size_t, C.c_size_t, P, C.c_size_t, C.POINTER(P)]),
    ("nexus_cuda_qweight_destroy", C.c_int, [P]),
    ("nexus_cuda_qmatvec_device", C.c_int, [P, P, C.c_size_t, P]),
    ("nexus_cuda_qmatvec_host", C.c_int, [P, P, C.c_size_t, P]),
    ("nexus_cuda_qweight_dequantize", C.c_int, [P, P]),
    ("nexus_cuda_qweight_bytes", C.c_size_t, [P]),
    ("nexus_cuda_qmatvec_bench", C.c_int, [P, P, C.c_size_t, P, C.c_int, C.c_size_t, C.POINTER(C.c_float)]),
    ("nexus_cuda_model_load", C.c_int, [P, C.c_char_p, C.POINTER(P)]),
    ("nexus_cuda_model_free", C.c_int, [P]),
    ("nexus_cuda_model_get_info", C.c_int, [P, C.POINTER(ModelInfo)]),
    ("nexus_cuda_seq_reset", C.c_int, [P, C.c_uint32]),
    ("nexus_cuda_seq_len", C.c_int, [P, C.c_uint32, C.POINTER(C.c_uint32)]),
    ("nexus_cuda_seq_set_pages", C.c_int, [P, C.c_uint32, P, C.c_uint32]),
    ("nexus_cuda_decode", C.c_int, [P, C.c_uint32, C.c_uint32, C.c_uint32, P, C.POINTER(C.c_uint32)]),
    ("nexus_cuda_prefill", C.c_int, [P, C.c_uint32, P, C.c_size_t, P, C.POINTER(C.c_uint32)]),
    ("nexus_cuda_generate", C.c_int, [P, C.c_uint32, P, C.c_size_t, C.c_size_t, P]),
    ("nexus_cuda_decode_batch", C.c_int, [P, C.POINTER(DecodeItem), C.c_size_t, P, P]),
    ("nexus_cuda_generate_with_draft", C.c_int, [P, C.c_uint32, P, C.c_size_t, P, C.c_size_t, C.c_size_t,
                                                 C.c_uint32, P, C.POINTER(C.c_uint32), C.POINTER(C.c_uint32)]),
    ("nexus_scheduler_last_error", C.c_char_p, []),
    ("nexus_scheduler_create", C.c_int, [C.c_uint32, C.c_uint32, C.c_uint32, C.POINTER(P)]),
    ("nexus_scheduler_destroy", C.c_int, [P]),
    ("nexus_scheduler_add_request", C.c_int, [P, C.c_uint64, P, C.c_size_t, C.c_uint32]),
    ("nexus_scheduler_get_next_batch", C.c_int, [P, P, C.c_size_t, C.POINTER(C.c_size_t)]),
    ("nexus_scheduler_decode_batch", C.c_int, [P, C.POINTER(ScheduledDecode), C.c_size_t, C.POINTER(C.c_size_t)]),
    ("nexus_scheduler_append_generated", C.c_int, [P, C.c_uint64, C.c_uint32, C.POINTER(C.c_int)]),
    ("nexus_scheduler_step", C.c_int, [P, P, C.c_size_t, C.POINTER(C.c_size_t)]),
    ("nexus_scheduler_get_completed", C.c_int, [P, P, C.c_size_t, C.POINTER(C.c_size_t)]),
    ("nexus_scheduler_complete_request", C.c_int, [P, C.c_uint64, C.POINTER(C.c_int)]),
    ("nexus_scheduler_stats", C.c_int, [P, C.POINTER(C.c_size_t), C.POINTER(C.c_size_t), C.POINTER(C.c_size_t)]),
    ("nexus_scheduler_kv_page_stats", C.c_int, [P, C.POINTER(C.c_size_t), C.POINTER(C.c_size_t)]),
    ("nexus_scheduler_kv_allocation", C.c_int, [P, C.c_uint64, P, C.c_size_t, C.POINTER(C.c_size_t), C.POINTER(C.c_size_t)]),
    ("nexus_scheduler_tokens", C.c_int, [P, C.c_uint64, P, C.c_size_t, C.POINTER(C.c_size_t)]),
    ("nexus_cuda_serve_step", C.c_int, [P, P, C.POINTER(ServeEvent), C.c_size_t, C.POINTER(C.c_size_t)]),
    ("nexus_cuda_last_step_ms", C.c_int, [P, C.POINTER(C.c_float)]),
    ("nexus_cuda_profile_decode", C.c_int, [P, C.c_uint32, C.c_uint32, C.c_uint32, C.POINTER(KernelProfile),
                                            C.c_int, C.POINTER(C.c_int)]),
    ("nexus_cuda_attention_noalloc", C.c_int, [P, P, P, P, P, C.c_size_t, C.c_size_t, C.c_size_t, C.c_size_t,
                                               C.c_float]),
    ("nexus_quantize_host", C.c_size_t, [C.c_int, P, C.c_size_t, P]),
    ("nexus_format_bytes", C.c_size_t, [C.c_int, C.c_size_t]),
    ("nexus_synth_model_write", C.c_int, [C.c_char_p, C.POINTER(SynthConfig)]),
]

_lib = None


def load() -> C.CDLL:
    """Load libnexus_cuda.so (building it first if the sources are newer)."""
    global _lib
    if _lib is not None:
        return _lib
    if os.environ.get("NEXUS_NO_BUILD") != "1" and "NEXUS_CUDA_LIB" not in os.environ:
        from . import build as _build
        _build.build()
    if not LIB_PATH.exists():
        raise ImportError(f"{LIB_PATH} is missing: the CUDA backend has no CPU fallback; run nexus_b200/build.py")
    lib = C.CDLL(str(LIB_PATH))
    for name, res, args in SIGNATURES:
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


class NexusError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"nexus status {code}: {msg}")
        self.code = code


def check(rc: int, backend=None) -> None:
    if rc != NEXUS_OK:
        lib = load()
        msg = lib.nexus_cuda_last_error(backend)
        raise NexusError(rc, msg.decode() if msg else "")


def check_scheduler(rc: int) -> None:
    """Status of a nexus_scheduler_* call, with the scheduler's message."""
    if rc != NEXUS_OK:
        msg = load().nexus_scheduler_last_error()
        raise NexusError(rc, msg.decode() if msg else "")
