"""Synthetic model configurations of the benchmark workloads.

Random-init LLaMA-style models with the shapes of the reference's headline
configurations (weights N(0, 0.02^2), seed 0, norms 1.0 quantized with the
body format as nexus-convert does, tools/nexus-convert/main.rs:151).  No
public dataset or checkpoint is involved: every input is seeded and synthetic.
"""
from __future__ import annotations

import hashlib
import json
import os
from pathlib import Path

from ._lib import Q2_K, Q4_K, Q8_0

GENERATOR_VERSION = 1

CONFIGS = {
    # tiny: 4 layers, hidden 256, 8/4 heads, head_dim 32, FFN 768, vocab 4096, all Q4_K
    "tiny": dict(num_layers=4, hidden_size=256, num_heads=8, num_kv_heads=4, ff_dim=768, vocab_size=4096,
                 context_length=512, rope_theta=10000.0, attn_format=Q4_K, ffn_format=Q4_K, embd_format=Q4_K,
                 head_format=Q4_K, norm_format=Q4_K),
    # small model whose heads, FFN rows and vocab split over 2/4/8 tensor-parallel
    # ranks (per-rank column slices of whole super-blocks): 2 layers, hidden 2048,
    # 16/8 heads, head_dim 128, FFN 4096, vocab 8192, all Q4_K
    "tp_small": dict(num_layers=2, hidden_size=2048, num_heads=16, num_kv_heads=8, ff_dim=4096, vocab_size=8192,
                     context_length=512, rope_theta=10000.0, attn_format=Q4_K, ffn_format=Q4_K, embd_format=Q4_K,
                     head_format=Q4_K, norm_format=Q4_K),
    # Llama-3-8B shape, Q4_K body, Q8_0 embedding and LM head
    "llama8b_q4k": dict(num_layers=32, hidden_size=4096, num_heads=32, num_kv_heads=8, ff_dim=14336,
                        vocab_size=128256, context_length=8448, rope_theta=500000.0, attn_format=Q4_K,
                        ffn_format=Q4_K, embd_format=Q8_0, head_format=Q8_0, norm_format=Q4_K),
    # Llama-3-8B shape, Q8_0 everywhere (packed-KV serving workload)
    "llama8b_q8": dict(num_layers=32, hidden_size=4096, num_heads=32, num_kv_heads=8, ff_dim=14336,
                       vocab_size=128256, context_length=8448, rope_theta=500000.0, attn_format=Q8_0,
                       ffn_format=Q8_0, embd_format=Q8_0, head_format=Q8_0, norm_format=Q8_0),
    # Llama-3-70B shape, Q4_K attention, Q2_K FFN, Q8_0 embedding/head (assumed).
    # Each tensor repeats its first 64 x 65536 drawn elements (4 Mi values, a
    # few MB of quantized bytes) so the 27 GB file is written in seconds; the
    # kernels stream every byte from its own address all the same.
    "llama70b": dict(num_layers=80, hidden_size=8192, num_heads=64, num_kv_heads=8, ff_dim=28672,
                     vocab_size=128256, context_length=4352, rope_theta=500000.0, attn_format=Q4_K,
                     ffn_format=Q2_K, embd_format=Q8_0, head_format=Q8_0, norm_format=Q4_K, repeat_chunks=64),
    # parity subsamples of the long-context workloads (every element drawn):
    # the config-P model's widths and formats with 2 layers (8k-token contexts
    # on the packed cache) and the config-X model's with 2 layers (Q4_K
    # attention, Q2_K FFN at the 70B widths)
    "llama8b_q8_l2": dict(num_layers=2, hidden_size=4096, num_heads=32, num_kv_heads=8, ff_dim=14336,
                          vocab_size=128256, context_length=8448, rope_theta=500000.0, attn_format=Q8_0,
                          ffn_format=Q8_0, embd_format=Q8_0, head_format=Q8_0, norm_format=Q8_0),
    # the config-E model's widths and formats with 2 layers (a small case of
    # the same kernels for ncu captures)
    "llama8b_q4k_l2": dict(num_layers=2, hidden_size=4096, num_heads=32, num_kv_heads=8, ff_dim=14336,
                           vocab_size=128256, context_length=8448, rope_theta=500000.0, attn_format=Q4_K,
                           ffn_format=Q4_K, embd_format=Q8_0, head_format=Q8_0, norm_format=Q4_K),
    "llama70b_l2": dict(num_layers=2, hidden_size=8192, num_heads=64, num_kv_heads=8, ff_dim=28672,
                        vocab_size=128256, context_length=4352, rope_theta=500000.0, attn_format=Q4_K,
                        ffn_format=Q2_K, embd_format=Q8_0, head_format=Q8_0, norm_format=Q4_K),
}


def config_key(cfg: dict) -> str:
    blob = json.dumps({"v": GENERATOR_VERSION, **cfg}, sort_keys=True).encode()
    return hashlib.sha1(blob).hexdigest()[:12]


def model_dir() -> Path:
    d = Path(os.environ.get("NEXUS_MODEL_DIR", "/tmp/nexus_models"))
    d.mkdir(parents=True, exist_ok=True)
    return d


def model_path(name_or_cfg, seed: int = 0, threads: int = 0, writer=None) -> Path:
    """Path of the synthetic GGUF for a configuration, writing it on first use.

    writer: the function that writes the file (default: the CUDA library's
    nexus_synth_model_write).  CPU-only callers pass the oracle's writer, which
    produces the same bytes without loading the CUDA library."""
    if writer is None:
        from .engine import write_synthetic_model as writer

    cfg = dict(CONFIGS[name_or_cfg]) if isinstance(name_or_cfg, str) else dict(name_or_cfg)
    cfg["seed"] = seed
    tag = name_or_cfg if isinstance(name_or_cfg, str) else "custom"
    path = model_dir() / f"{tag}-{config_key(cfg)}.gguf"
    done = path.with_suffix(".ok")
    if not (path.exists() and done.exists()):
        # a private temporary name: several processes (one per GPU) may write
        # the same model at once; the last rename wins with identical bytes
        tmp = path.with_suffix(f".{os.getpid()}.tmp")
        writer(str(tmp), threads=threads, **cfg)
        os.replace(tmp, path)
        done.write_text("ok")
    return path
