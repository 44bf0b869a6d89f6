#!/usr/bin/env python
"""Decode benchmark of the B200 backend (one JSON line on rank 0).

Workload (the metric's configuration): the
Llama-3-8B-shaped model, random init, Q4_K body with Q8_0 embedding and LM
head, a 512-token random prompt (seed 1), greedy decode at batch 1.  A step is
one decode step (one token through all 32 layers, LM head and argmax).

  value  tokens/s of K device-chained decode steps, inputs resident in HBM,
         CUDA events on the backend stream (max over ranks for N > 1).
  e2e    the same steps through the public C ABI call nexus_cuda_decode with
         host buffers: the step's token goes host->device, the argmax comes
         back device->host, every step.
  roofline  the dominant kernel (the fused gate/up dequant-GEMV) from a live
         per-kernel CUDA-event profile of real decode steps; achieved =
         algorithmic bytes per launch / mean launch time; peak = measured HBM
         copy bandwidth (MEASURED_PEAKS.json).
  cpu_baseline  the CPU restatement of the reference decode path (oracle/) on
         the host cores, bounded sample.

--impl reference times the reference's CPU decode path (the oracle port, a C
restatement of the Rust reference, which cannot be built here) on the same
config and metric: the same 512-token prompt (prefilled with the oracle's
layer-major schedule, bit-identical to the reference's token-by-token
prefill), then decode steps at contexts 512+ on all host threads, plus one
single-threaded step (the reference's decode path is single-threaded).  That
arm writes its model with the oracle's synthetic writer and never loads the
CUDA library.

Multi-GPU: tensor parallelism over the torchrun ranks (heads, FFN rows and
vocabulary rows per rank; one all-reduce per sublayer, by the one-shot
peer-memory kernel over NVLink, NCCL as fallback).  One decode
stream is served by all ranks, so the scaling is strong: `value` is the
stream's tokens per second, timed on the device as the max over ranks.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

PROMPT_LEN = 512
GEN_TOKENS = 128
SEED_PROMPT = 1


# DRAM bytes per launch (dram__bytes_read.sum + dram__bytes_write.sum) of the
# dominant kernel, from one ncu capture of the same kernel and shape (the
# command and the full table are in the profiles/ summary named here).
DOMINANT_TRAFFIC = {
    "gate_up": (66329088, "ncu --set full capture of k_gemv<Q4_K> 28672x4096, 1 token "
                          "(profiles/k_gemv_q4k_gateup_28672x4096_m1.md)"),
}


def measured_peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "source": "measured"}
    return {"hbm_gbs": 6650.0, "source": "fallback"}


class ClockSampler:
    """nvidia-smi clocks/throttle reasons sampled during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device = device
        self.rows = []
        self._stop = threading.Event()
        self._thr = None

    def _run(self):
        while not self._stop.is_set():
            try:
                out = subprocess.run(["nvidia-smi", "-i", str(self.device), f"--query-gpu={self.FIELDS}",
                                      "--format=csv,noheader,nounits"], capture_output=True, text=True,
                                     timeout=5).stdout.strip()
                if out:
                    self.rows.append([c.strip() for c in out.split(",")])
            except Exception:
                pass
            self._stop.wait(0.2)

    def __enter__(self):
        self._thr = threading.Thread(target=self._run, daemon=True)
        self._thr.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        self._thr.join(timeout=10)

    def summary(self) -> dict:
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in self.rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in self.rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in self.rows for i in range(4) if len(r) > 5 + i and r[5 + i] == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.rows)}


def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def init_dist(world: int, backend: str):
    if world <= 1:
        return None
    import datetime

    import torch.distributed as dist
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    dist.init_process_group(backend=backend, timeout=datetime.timedelta(seconds=600))
    return dist


def reduce_max(dist, value: float, device) -> float:
    if dist is None:
        return value
    import torch
    t = torch.tensor([value], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(dist, device):
    if dist is not None:
        import torch
        dist.barrier(device_ids=[device.index] if device.type == "cuda" else None)


def cpu_threads() -> int:
    try:
        return max(1, min(64, len(os.sched_getaffinity(0))))
    except Exception:
        return max(1, min(64, os.cpu_count() or 1))


METRIC = "decode tok/s, Llama-3-8B-shape Q4_K, b=1"


def time_oracle(model_path: Path, steps: int, warmup: int, budget_s: float, threads: int,
                prompt_len: int = PROMPT_LEN, single_core_steps: int = 0) -> dict:
    """The CPU restatement of the reference's decode (oracle port) on a bounded
    sample: a `prompt_len`-token prompt of the bench's seed (prefilled with the
    oracle's layer-major schedule, the same bits as token-by-token), then up to
    `steps` decode steps timed one by one (stopping once `budget_s` of timed
    work is spent), on `threads` threads; then `single_core_steps` more steps on
    one thread."""
    from oracle import oracle as O

    m = O.Model(model_path, threads=threads, max_seq_len=prompt_len + steps + warmup + single_core_steps + 8)
    prompt = np.random.default_rng(SEED_PROMPT).integers(0, m.info.vocab_rows, prompt_len).tolist()
    logits = m.prefill_batched(prompt)
    tok = O.greedy(logits)
    pos = len(prompt)
    for _ in range(warmup):
        logits = m.decode(tok, pos)
        tok = O.greedy(logits)
        pos += 1
    times = []
    ctx0 = pos
    t_start = time.perf_counter()
    for _ in range(steps):
        t0 = time.perf_counter()
        logits = m.decode(tok, pos)
        tok = O.greedy(logits)
        pos += 1
        times.append(time.perf_counter() - t0)
        if time.perf_counter() - t_start > budget_s:
            break
    total = sum(times)
    r = {"tok_s": len(times) / total, "steps": len(times), "s_per_token": total / len(times),
         "threads": threads, "ctx": (ctx0, pos - 1)}
    if single_core_steps:
        m.set_threads(1)
        t0 = time.perf_counter()
        for _ in range(single_core_steps):
            logits = m.decode(tok, pos)
            tok = O.greedy(logits)
            pos += 1
        dt = time.perf_counter() - t0
        r["single_core"] = {"value": single_core_steps / dt, "unit": "tok/s", "cores": 1, "steps": single_core_steps,
                            "s_per_token": dt / single_core_steps}
    return r


def oracle_model_path(config: str) -> Path:
    """The bench model written by the oracle's synthetic writer (the same bytes
    as the CUDA library's writer), so CPU-only legs never load that library."""
    from nexus_b200.configs import model_path
    from oracle import oracle as O
    return model_path(config, threads=cpu_threads(), writer=O.write_synthetic_model)


def run_reference(args):
    world, rank, local = dist_env()
    if rank != 0:
        return 0
    path = oracle_model_path(args.config)
    threads = cpu_threads()
    r = time_oracle(path, args.steps, args.warmup, budget_s=args.ref_budget, threads=threads,
                    single_core_steps=1)
    sample = (f"{r['steps']} decode steps at contexts {r['ctx'][0]}-{r['ctx'][1]} after the bench's {PROMPT_LEN}-token "
              f"prompt (seed {SEED_PROMPT}), {threads} threads splitting matvec rows (bit-identical per row)")
    line = {
        "impl": "reference", "metric": METRIC, "value": r["tok_s"],
        "unit": "tok/s", "n_gpus": 0, "steps": r["steps"], "warmup": args.warmup,
        "ms_per_step": 1000 * r["s_per_token"],
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded random-init weights and prompt)",
        "config": {"workload": f"{args.config}: prompt {PROMPT_LEN} (seed {SEED_PROMPT}), greedy decode b=1, "
                               f"context {r['ctx'][0]}-{r['ctx'][1]}",
                   "model": args.config, "global_batch": 1, "seq_len": PROMPT_LEN + GEN_TOKENS, "parallelism": "cpu"},
        "cpu_baseline": {"value": r["tok_s"], "unit": "tok/s", "cores": threads, "kind": "port", "sample": sample,
                         "single_core": r["single_core"]},
        "e2e": {"value": r["tok_s"], "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def run_ncu_case(args):
    """Small, fixed launch sequence for `ncu` captures: prefill 8 tokens as one
    8-token step on the tensor-core GEMM path, then ncu_steps single-token
    decode steps from the captured graph (5 kernels per layer + 3 per step)."""
    import nexus_b200 as nb
    path = nb.model_path(args.config, threads=cpu_threads())
    b = max(1, args.ncu_batch)
    backend = nb.CudaBackend(device=0, max_seq_len=64, max_batch=b)
    eng = nb.InferenceEngine(backend)
    eng.load_model(path)
    if b == 1:
        prompt = np.random.default_rng(SEED_PROMPT).integers(0, eng.info.vocab_rows, 8).tolist()
        out = eng.generate(prompt, args.ncu_steps)
        print(json.dumps({"ncu_case": args.config, "prefill": 8, "decode_steps": args.ncu_steps,
                          "tokens": out[8:], "kernels_per_step": 5 * eng.info.num_layers + 3}), flush=True)
    else:
        # b sequences of 8 prompt tokens (seed 1 + i), then ncu_steps batched
        # decode steps over all of them (the tensor-core GEMM path)
        toks = []
        for i in range(b):
            prompt = np.random.default_rng(SEED_PROMPT + i).integers(0, eng.info.vocab_rows, 8).tolist()
            toks.append(eng.prefill(prompt, seq_id=i, want_logits=False)[1])
        import torch
        torch.cuda.synchronize()
        torch.cuda.profiler.start()  # ncu --profile-from-start off captures the decode steps only
        for s in range(args.ncu_steps):
            toks, _ = eng.decode_batch([(i, toks[i], 8 + s) for i in range(b)])
        torch.cuda.synchronize()
        torch.cuda.profiler.stop()
        print(json.dumps({"ncu_case": args.config, "batch": b, "prefill": 8, "decode_steps": args.ncu_steps}),
              flush=True)
    eng.close()
    backend.close()
    return 0


def tp_join(dist, nb, backend, rank: int, world: int) -> None:
    """Tensor parallelism over the torchrun ranks: rank 0's NCCL group id is
    broadcast and every rank joins before loading its slice of the model."""
    if world <= 1:
        return
    uid = [nb.tp_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(uid, src=0)
    backend.tp_init(rank, world, uid[0])


def run_batched(nb, L, path, batch: int, prompt_len: int, steps: int, warmup: int, device: int, dist=None,
                rank: int = 0, world: int = 1) -> dict:
    """Config E at batch `batch`: every sequence gets its own random prompt of
    `prompt_len` tokens (seed 1 + index), then `steps` decode steps each
    advance all sequences by one token through nexus_cuda_decode_batch.  The
    device time is the CUDA-event time of each batched step; the end-to-end
    time is the host wall clock around the calls (token ids in, argmax ids out)."""
    import torch
    be = nb.CudaBackend(device=device, max_batch=batch, max_seq_len=prompt_len + steps + warmup + 8)
    tp_join(dist, nb, be, rank, world)
    eng = nb.InferenceEngine(be)
    eng.load_model(path)
    V = eng.info.vocab_rows
    toks, pos = [], []
    t0 = time.perf_counter()
    for s in range(batch):
        p = np.random.default_rng(SEED_PROMPT + s).integers(0, V, prompt_len).tolist()
        _, t = eng.prefill(p, seq_id=s, want_logits=False)
        toks.append(t)
        pos.append(prompt_len)
    torch.cuda.synchronize()
    prefill_s = time.perf_counter() - t0
    prefill_ms_last = eng.last_step_ms()

    def step():
        nonlocal toks
        items = [(s, toks[s], pos[s]) for s in range(batch)]
        out, _ = eng.decode_batch(items, want_logits=False)
        toks = [int(v) for v in out]
        for s in range(batch):
            pos[s] += 1

    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    dev_ms = 0.0
    t0 = time.perf_counter()
    for _ in range(steps):
        step()
        dev_ms += eng.last_step_ms()
    wall = time.perf_counter() - t0
    eng.close()
    be.close()
    dev_ms = reduce_max(dist, dev_ms, torch.device("cuda", device))
    wall = reduce_max(dist, wall, torch.device("cuda", device))
    return {"value": batch * steps / (dev_ms / 1000.0), "unit": "tok/s", "batch": batch, "steps": steps,
            "ms_per_step": dev_ms / steps,
            "e2e": {"value": batch * steps / wall, "unit": "tok/s", "h2d_bytes_per_step": 28 * batch,
                    "d2h_bytes_per_step": 4 * batch},
            "prefill": {"tokens": batch * prompt_len, "seconds": prefill_s,
                        "tok_s": batch * prompt_len / prefill_s, "last_prompt_ms": prefill_ms_last}}


SWEEP_SHAPES = [(4096, 4096), (1024, 4096), (14336, 4096), (4096, 14336), (128256, 4096)]
SWEEP_FORMATS = ["Q8_0", "Q4_0", "Q4_K", "Q2_K"]
SWEEP_M = [1, 4, 16, 64, 512]


def sweep_weight(nb, fmt: int, n: int, k: int, seed: int = 0):
    """A seeded N(0, 0.02^2) weight quantized on the host: 256 distinct rows
    repeated down the matrix (the timing does not depend on the values)."""
    rng = np.random.default_rng(seed)
    base = (rng.standard_normal((256, k), dtype=np.float32) * 0.02).reshape(-1)
    blk = nb.quantize_host(fmt, base)
    return np.tile(blk.reshape(256, -1), (n // 256, 1))


def run_matvec(args):
    """Config S (quantized matvec/matmul sweep): device time per launch with a
    cold L2 (256 MB written between launches), HBM GB/s of the algorithmic
    bytes (weights + x + y) and, for 64+ tokens, useful TFLOP/s (2*M*N*K).
    --matvec FMT N K M runs one case three times (the ncu target)."""
    import torch
    import nexus_b200 as nb
    be = nb.CudaBackend(device=0)
    peaks = measured_peaks()
    cases = []
    if args.matvec:
        f, n, k, m = args.matvec
        cases = [(f, int(n), int(k), [int(m)])]
    else:
        cases = [(f, n, k, SWEEP_M) for (n, k) in SWEEP_SHAPES for f in SWEEP_FORMATS]
    rows = []
    for fname, n, k, ms in cases:
        fmt = getattr(nb, fname)
        qw = nb.QWeight(be, fmt, n, k, sweep_weight(nb, fmt, n, k))
        for m in ms:
            x = torch.randn(m, k, device="cuda", generator=torch.Generator("cuda").manual_seed(3))
            y = torch.empty(m, n, device="cuda")
            torch.cuda.synchronize()
            if args.matvec:
                for _ in range(3):
                    qw.matvec_device(x.data_ptr(), m, y.data_ptr())
                be.synchronize()
                ms_ = qw.bench(x.data_ptr(), m, y.data_ptr(), iters=3)
            else:
                qw.bench(x.data_ptr(), m, y.data_ptr(), iters=2)
                ms_ = qw.bench(x.data_ptr(), m, y.data_ptr(), iters=10 if m < 512 else 4)
            byts = qw.nbytes() + 4.0 * m * k + 4.0 * m * n
            row = {"format": fname, "n": n, "k": k, "m": m, "us": ms_ * 1e3, "gbs": byts / (ms_ * 1e-3) / 1e9,
                   "hbm_frac": byts / (ms_ * 1e-3) / 1e9 / peaks["hbm_gbs"],
                   "path": "tcgen05 GEMM" if m >= 8 else "dp4a GEMV"}
            if m >= 64:
                row["tflops"] = 2.0 * m * n * k / (ms_ * 1e-3) / 1e12
            rows.append(row)
            print(json.dumps(row), flush=True)
        qw.close()
    be.close()
    return 0


def run_workload_p(args):
    """Config P: the 8B shape with Q8_0 weights and the 4-bit packed KV cache;
    64 requests with context lengths uniform in [1024, 8192] (seed 2) of random
    token ids (seed 1 + request), then `steps` continuous decode steps that
    advance all 64 requests by one token each through nexus_cuda_decode_batch,
    with scheduler-style 16-token page lists (src/scheduler.rs:333-361): every
    request's KV lives in the pages its list names."""
    import torch
    import nexus_b200 as nb
    n_req, gen = 64, args.steps
    path = nb.model_path("llama8b_q8", threads=cpu_threads())
    ctx = np.random.default_rng(2).integers(args.p_ctx[0], args.p_ctx[1] + 1, n_req)
    be = nb.CudaBackend(device=0, kv_bits=(4, 4), max_batch=n_req, max_seq_len=int(ctx.max()) + gen + args.warmup + 8)
    eng = nb.InferenceEngine(be)
    eng.load_model(path)
    V = eng.info.vocab_rows
    toks, pos, pages, next_page = [], [], [], 0
    t0 = time.perf_counter()
    for r in range(n_req):
        # the scheduler's allocation: ceil((prompt + max_tokens) / 16) ids from a
        # running counter, bound before the prefill writes the request's KV
        npg = (int(ctx[r]) + gen + args.warmup + 15) // 16
        pages.append(list(range(next_page, next_page + npg)))
        next_page += npg
        eng.seq_set_pages(r, pages[r])
        prompt = np.random.default_rng(SEED_PROMPT + r).integers(0, V, int(ctx[r])).tolist()
        _, t = eng.prefill(prompt, seq_id=r, want_logits=False)
        toks.append(t)
        pos.append(int(ctx[r]))
    torch.cuda.synchronize()
    prefill_s = time.perf_counter() - t0

    def step():
        nonlocal toks
        out, _ = eng.decode_batch([(r, toks[r], pos[r]) for r in range(n_req)], want_logits=False,
                                  page_ids=pages)
        toks = [int(v) for v in out]
        for r in range(n_req):
            pos[r] += 1

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    dev_ms = 0.0
    t0 = time.perf_counter()
    if args.profile_range:
        torch.cuda.profiler.start()
    with ClockSampler(0) as clk:
        for _ in range(gen):
            step()
            dev_ms += eng.last_step_ms()
    wall = time.perf_counter() - t0
    if args.profile_range:
        torch.cuda.synchronize()
        torch.cuda.profiler.stop()
    mean_ctx = float(ctx.mean()) + args.warmup + gen / 2
    kv_bytes = 2 * eng.info.num_layers * mean_ctx * (eng.info.num_kv_heads * eng.info.head_dim * 4 // 8 + 8) * n_req
    step_bytes = eng.info.weight_bytes + kv_bytes
    line = {"metric": "continuous decode tok/s, 8B-shape Q8_0, 4-bit packed KV, 64 requests (config P)",
            "value": n_req * gen / (dev_ms / 1000.0), "unit": "tok/s", "n_gpus": 1, "steps": gen,
            "warmup": args.warmup, "ms_per_step": dev_ms / gen, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f16 tensor-core (exact Q8_0 hi/lo) + f32", "data": "synthetic",
            "config": {"workload": f"llama8b_q8, 64 requests, ctx U[{args.p_ctx[0]},{args.p_ctx[1]}] seed 2, KV 4/4-bit packed, "
                                   "16-token pages", "model": "llama8b_q8", "global_batch": n_req,
                       "mean_ctx": mean_ctx, "l2": "inputs larger than L2 (weights + KV per step)"},
            "e2e": {"value": n_req * gen / wall, "unit": "tok/s", "h2d_bytes_per_step": 28 * n_req,
                    "d2h_bytes_per_step": 4 * n_req},
            "roofline": {"bound": "hbm", "kernel": "whole step", "achieved": step_bytes / (dev_ms / gen / 1000) / 1e9,
                         "peak": measured_peaks()["hbm_gbs"], "unit": "GB/s",
                         "frac": step_bytes / (dev_ms / gen / 1000) / 1e9 / measured_peaks()["hbm_gbs"],
                         "traffic": None, "bytes_per_step": step_bytes},
            "prefill": {"tokens": int(ctx.sum()), "seconds": prefill_s, "tok_s": float(ctx.sum()) / prefill_s},
            "clocks": clk.summary()}
    eng.close()
    be.close()
    print(json.dumps(line), flush=True)
    return 0


def run_workload_x(args, dist, rank: int, world: int, local: int):
    """Config X: the 70B shape (Q4_K attention, Q2_K FFN, Q8_0 embedding and
    head), tensor parallel over the ranks: a 4096-token random prompt, then
    `steps` greedy decode steps at batch 1 (device-chained), and the same at
    batch 16 through nexus_cuda_decode_batch."""
    import torch
    import nexus_b200 as nb
    device = torch.device("cuda", local)
    prompt_len = 4096
    if rank == 0:
        path = nb.model_path("llama70b", threads=cpu_threads())
    barrier(dist, device)
    if rank != 0:
        path = nb.model_path("llama70b")
    be = nb.CudaBackend(device=local, max_seq_len=prompt_len + args.steps + args.warmup + 8)
    tp_join(dist, nb, be, rank, world)
    eng = nb.InferenceEngine(be)
    eng.load_model(path)
    info = eng.info
    prompt = np.random.default_rng(SEED_PROMPT).integers(0, info.vocab_rows, prompt_len).tolist()
    t0 = time.perf_counter()
    eng.prefill(prompt, want_logits=False)
    torch.cuda.synchronize()
    prefill_s = reduce_max(dist, time.perf_counter() - t0, device)
    eng.generate(prompt, args.warmup)
    barrier(dist, device)
    with ClockSampler(local) as clk:
        eng.generate(prompt, args.steps)
        torch.cuda.synchronize()
    ms = reduce_max(dist, eng.last_step_ms(), device)
    eng.close()
    be.close()
    b16 = run_batched(nb, None, path, 16, prompt_len=prompt_len, steps=min(args.steps, 16), warmup=args.warmup,
                      device=local, dist=dist, rank=rank, world=world)
    line = {"metric": "decode tok/s, Llama-3-70B-shape (Q4_K attn, Q2_K FFN), b=1 (b=16 in b16)",
            "value": args.steps / (ms / 1000.0), "unit": "tok/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "int8x4 dp4a + f32 (b=1); f16 tensor-core (b=16)", "data": "synthetic",
            "config": {"workload": f"llama70b: prompt {prompt_len} (seed {SEED_PROMPT}), greedy decode",
                       "model": "llama70b", "global_batch": 1,
                       "parallelism": f"tp{world}" if world > 1 else "single GPU",
                       "weight_bytes_per_token_per_rank": info.weight_bytes,
                       "l2": "inputs larger than L2"},
            "roofline": {"bound": "hbm", "kernel": "whole step",
                         "achieved": info.weight_bytes / (ms / args.steps / 1000) / 1e9,
                         "peak": measured_peaks()["hbm_gbs"], "unit": "GB/s",
                         "frac": info.weight_bytes / (ms / args.steps / 1000) / 1e9 / measured_peaks()["hbm_gbs"],
                         "traffic": None},
            "prefill": {"tokens": prompt_len, "seconds": prefill_s, "tok_s": prompt_len / prefill_s},
            "b16": b16, "clocks": clk.summary()}
    if rank == 0:
        print(json.dumps(line), flush=True)
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", default="llama8b_q4k")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--ref-budget", type=float, default=60.0)
    ap.add_argument("--profile-steps", type=int, default=4)
    ap.add_argument("--batch", type=int, default=32, help="batched-decode measurement (config E at b=32); 1 = off")
    ap.add_argument("--ncu-batch", type=int, default=1,
                    help="with --ncu-steps: batched decode steps over this many sequences (8-token prompts each)")
    ap.add_argument("--ncu-steps", type=int, default=0,
                    help="profiling run for ncu: 8-token prefill (2 fused 4-token steps), then this many "
                         "device-chained decode steps; prints a short JSON line")
    ap.add_argument("--workload", default="E", choices=["E", "P", "X"],
                    help="E: 8B Q4_K b=1 (+b=32) [default]; P: 8B Q8_0, packed KV, 64 requests; X: 70B shape, TP")
    ap.add_argument("--p-ctx", nargs=2, type=int, default=[1024, 8192], metavar=("LO", "HI"),
                    help="workload P context lengths, uniform in [LO, HI] (a smaller range gives a smaller ncu case)")
    ap.add_argument("--profile-range", action="store_true",
                    help="workload P: bracket the timed steps with cudaProfilerStart/Stop "
                         "(for ncu --profile-from-start off)")
    ap.add_argument("--sweep", action="store_true", help="config S: quantized matvec/matmul sweep, one JSON line per case")
    ap.add_argument("--matvec", nargs=4, metavar=("FMT", "N", "K", "M"), help="one config-S case, three launches")
    args = ap.parse_args()
    if args.sweep or args.matvec:
        return run_matvec(args)
    if args.warmup < 3:
        args.warmup = 3
    if args.steps + args.warmup > GEN_TOKENS:
        args.steps = GEN_TOKENS - args.warmup
    if args.impl == "reference":
        return run_reference(args)
    if args.ncu_steps:
        return run_ncu_case(args)

    if args.workload == "P":
        return run_workload_p(args)
    world, rank, local = dist_env()
    import torch
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    dist = init_dist(world, "nccl")
    if args.workload == "X":
        rc = run_workload_x(args, dist, rank, world, local)
        if dist is not None:
            barrier(dist, device)
            dist.destroy_process_group()
        return rc

    import nexus_b200 as nb
    from nexus_b200 import _lib as L
    # rank 0 writes the synthetic model; the others wait for it
    if rank == 0:
        path = nb.model_path(args.config, threads=cpu_threads())
    barrier(dist, device)
    if rank != 0:
        path = nb.model_path(args.config)

    backend = nb.CudaBackend(device=local, max_seq_len=PROMPT_LEN + GEN_TOKENS + 8)
    tp_join(dist, nb, backend, rank, world)
    eng = nb.InferenceEngine(backend)
    eng.load_model(path)
    info = eng.info
    prompt = np.random.default_rng(SEED_PROMPT).integers(0, info.vocab_rows, PROMPT_LEN).tolist()

    # ---- value: device-chained decode steps (generate), inputs resident ----
    eng.prefill(prompt)
    lib, model = eng._lib, eng.model
    import ctypes as C
    out = np.zeros(PROMPT_LEN + args.warmup, np.uint32)
    p = np.asarray(prompt, np.uint32)
    # warm-up (captures the graph), untimed
    L.check(lib.nexus_cuda_generate(model, 0, p.ctypes.data, p.size, args.warmup, out.ctypes.data), backend.handle)
    out = np.zeros(PROMPT_LEN + args.steps, np.uint32)
    barrier(dist, device)
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        L.check(lib.nexus_cuda_generate(model, 0, p.ctypes.data, p.size, args.steps, out.ctypes.data),
                backend.handle)
        torch.cuda.synchronize()
    gen_ms = eng.last_step_ms()  # CUDA events around the K chained steps (excludes the prefill)
    ms_max = reduce_max(dist, gen_ms, device)
    # one decode stream served by all ranks (tensor parallel): tokens per second of the job
    value = args.steps / (ms_max / 1000.0)

    # ---- e2e: nexus_cuda_decode with host token in / argmax out per step ----
    _, tok = eng.prefill(prompt, want_logits=False)
    pos = PROMPT_LEN
    for _ in range(args.warmup):
        _, tok = eng.decode_with_cache(tok, pos, want_logits=False)
        pos += 1
    eng.prefill(prompt, want_logits=False)
    pos = PROMPT_LEN
    barrier(dist, device)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    tok_c = C.c_uint32(tok)
    for _ in range(args.steps):
        L.check(lib.nexus_cuda_decode(model, 0, tok_c.value, pos, None, C.byref(tok_c)), backend.handle)
        pos += 1
    torch.cuda.synchronize()
    e2e_s = reduce_max(dist, time.perf_counter() - t0, device)
    e2e_value = args.steps / e2e_s

    # ---- live per-kernel profile (CUDA events per launch, no graph) ----
    eng.prefill(prompt, want_logits=False)
    prof = eng.profile_decode(int(out[PROMPT_LEN]), args.profile_steps)
    peaks = measured_peaks()
    kern = {r["name"]: r for r in prof}
    dom = max(prof, key=lambda r: r["total_ms"])
    dom_ms = dom["total_ms"] / dom["launches"]
    achieved = dom["bytes_per_launch"] / (dom_ms / 1000.0) / 1e9
    step_ms_prof = sum(r["total_ms"] for r in prof) / args.profile_steps
    barrier(dist, device)

    line = {
        "metric": METRIC,
        "value": value, "unit": "tok/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms_max / args.steps, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "int8x4 dp4a + f32 (Q4_K/Q8_0 weights)", "data": "synthetic (seeded random-init weights, random prompt)",
        "config": {"workload": f"{args.config}: prompt {PROMPT_LEN} (seed {SEED_PROMPT}), greedy decode b=1, "
                               f"context {PROMPT_LEN}-{PROMPT_LEN + args.warmup + args.steps}",
                   "model": args.config, "global_batch": 1, "seq_len": PROMPT_LEN + GEN_TOKENS,
                   "parallelism": f"tp{world} (heads, FFN and vocab rows per rank; one all-reduce per sublayer, "
                                  f"{backend.tp_allreduce_kind()})" if world > 1 else "single GPU",
                   "l2": "inputs larger than L2: every step streams all weights "
                         f"({info.weight_bytes / 1e9:.3f} GB) from HBM",
                   "weight_bytes_per_token": info.weight_bytes},
        "e2e": {"value": e2e_value, "unit": "tok/s", "h2d_bytes_per_step": 28, "d2h_bytes_per_step": 4},
        "gpu_launches": None,
        "roofline": {"bound": "hbm", "kernel": dom["name"], "achieved": achieved, "peak": peaks["hbm_gbs"],
                     "unit": "GB/s", "frac": achieved / peaks["hbm_gbs"],
                     "traffic": DOMINANT_TRAFFIC.get(dom["name"], (None, None))[0],
                     "traffic_source": DOMINANT_TRAFFIC.get(dom["name"], (None, "no capture of this kernel"))[1],
                     "peak_source": peaks["source"],
                     "step_achieved_gbs": info.weight_bytes / (ms_max / args.steps / 1000.0) / 1e9},
        "kernels": {r["name"]: {"launches_per_step": r["launches"] / args.profile_steps,
                                "ms_per_step": r["total_ms"] / args.profile_steps,
                                "gbs": r["bytes_per_launch"] * r["launches"] / (r["total_ms"] / 1000.0) / 1e9}
                    for r in prof},
        "profile_step_ms": step_ms_prof,
        "clocks": clk.summary(),
    }
    launches_per_step = sum(r["launches"] for r in prof) / args.profile_steps
    line["gpu_launches"] = int(round(launches_per_step * args.steps))

    eng.close()
    backend.close()
    # ---- b=32: one decode step advances 32 sequences (tensor-core GEMM path) ----
    if args.batch > 1:
        line["b32"] = run_batched(nb, L, path, args.batch, prompt_len=PROMPT_LEN, steps=min(args.steps, 32),
                                  warmup=args.warmup, device=local, dist=dist, rank=rank, world=world)

    if rank == 0 and not args.no_cpu_baseline:
        # bounded (~20 s): a short prompt, so no long CPU prefill holds the GPU;
        # the reference arm times the same steps at the bench's contexts 512+
        r = time_oracle(path, 64, 1, budget_s=20.0, threads=cpu_threads(), prompt_len=4, single_core_steps=1)
        line["cpu_baseline"] = {"value": r["tok_s"], "unit": "tok/s", "cores": r["threads"], "kind": "port",
                                "sample": f"{r['steps']} decode steps of the same model at contexts "
                                          f"{r['ctx'][0]}-{r['ctx'][1]} after a 4-token prompt (oracle restatement "
                                          "of the reference CPU path; the reference arm times contexts 512+)",
                                # the reference's decode path is single-threaded (src/engine/mod.rs:775-801)
                                "single_core": r["single_core"]}
    if dist is not None:
        barrier(dist, device)
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
