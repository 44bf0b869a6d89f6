"""Model-level parity fixtures of the benchmarked configurations, from the oracle.

Runs the CPU oracle (oracle/, the C restatement of the reference's decode
path) on the seeded synthetic models of BASELINE.json's configurations and
writes, per case, the prompt, the greedy continuation and sampled logits to
tests/golden/model_<case>.npz, with the case list in model_cases.json.  The
GPU tests (tests/test_gpu_parity_configs.py) replay the same prompts through
the CUDA backend and compare.

Prompts are prefilled with the oracle's layer-major schedule
(orc_model_prefill_batched), which gives the same bits as the reference's
token-by-token prefill (checked on the CPU by tests/test_oracle_batched.py);
the decode steps then run token by token.  Each step feeds back the oracle's
own greedy token.  Models are written with the oracle's synthetic writer
(byte-identical to the CUDA library's), so this script never loads the CUDA
library.

Cases (config letters as in BASELINE.json's list):
  e_s1..e_s4   config E (Llama-3-8B shape, Q4_K body, Q8_0 embedding/head,
               float KV): 512-token prompts of seeds 1..4, 8 greedy steps;
               e_s1 is the b=1 bench workload, e_s1..e_s4 the b=32 subsample.
  p_1k         config P's model (Q8_0, 4/4-bit packed KV): a 1031-token prompt.
  p_8k_l2      config P's widths and formats with 2 layers: an 8191-token prompt
               on the packed cache.
  x_l2         config X's widths and formats (Q4_K attention, Q2_K FFN, Q8_0
               embedding/head) with 2 layers: a 4096-token prompt.

Usage: python tests/golden/make_model_fixtures.py [case ...] [--threads N]
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import time
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT))

CASES = {
    "e_s1": dict(config="llama8b_q4k", kv_bits=[0, 0], seed=1, prompt_len=512, steps=8, max_seq_len=640),
    "e_s2": dict(config="llama8b_q4k", kv_bits=[0, 0], seed=2, prompt_len=512, steps=8, max_seq_len=640),
    "e_s3": dict(config="llama8b_q4k", kv_bits=[0, 0], seed=3, prompt_len=512, steps=8, max_seq_len=640),
    "e_s4": dict(config="llama8b_q4k", kv_bits=[0, 0], seed=4, prompt_len=512, steps=8, max_seq_len=640),
    "p_1k": dict(config="llama8b_q8", kv_bits=[4, 4], seed=1, prompt_len=1031, steps=4, max_seq_len=1088),
    "p_8k_l2": dict(config="llama8b_q8_l2", kv_bits=[4, 4], seed=2, prompt_len=8191, steps=4, max_seq_len=8256),
    "x_l2": dict(config="llama70b_l2", kv_bits=[0, 0], seed=1, prompt_len=4096, steps=4, max_seq_len=4160),
}
VOCAB = 128256


def logit_indices(logits: np.ndarray) -> np.ndarray:
    """Every 64th vocabulary row plus the 64 largest logits."""
    top = np.argsort(logits)[-64:]
    return np.unique(np.concatenate([np.arange(0, logits.size, 64), top])).astype(np.int32)


def top2_gap(logits: np.ndarray) -> float:
    s = np.sort(logits[np.isfinite(logits)])
    return float(s[-1] - s[-2])


def make_case(name: str, spec: dict, threads: int) -> dict:
    from nexus_b200.configs import model_path
    from oracle import oracle as O

    path = model_path(spec["config"], threads=threads, writer=O.write_synthetic_model)
    m = O.Model(path, kv_bits=tuple(spec["kv_bits"]), threads=threads, max_seq_len=spec["max_seq_len"])
    prompt = np.random.default_rng(spec["seed"]).integers(0, VOCAB, spec["prompt_len"]).astype(np.uint32)
    t0 = time.time()
    first = m.prefill_batched(prompt.tolist())
    t_pre = time.time() - t0
    idx = logit_indices(first)
    tokens, gaps = [O.greedy(first)], [top2_gap(first)]
    last = first
    for i in range(spec["steps"]):
        last = m.decode(tokens[-1], spec["prompt_len"] + i)
        tokens.append(O.greedy(last))
        gaps.append(top2_gap(last))
    idx_last = logit_indices(last)
    np.savez_compressed(HERE / f"model_{name}.npz", prompt=prompt, tokens=np.asarray(tokens, np.uint32),
                        gaps=np.asarray(gaps, np.float32), idx_first=idx, logits_first=first[idx],
                        idx_last=idx_last, logits_last=last[idx_last])
    print(f"{name}: prefill {spec['prompt_len']} in {t_pre:.0f} s, total {time.time() - t0:.0f} s, "
          f"tokens {tokens}", flush=True)
    return dict(spec, file=f"model_{name}.npz")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("cases", nargs="*", default=list(CASES))
    ap.add_argument("--threads", type=int, default=os.cpu_count() or 1)
    a = ap.parse_args()
    meta_path = HERE / "model_cases.json"
    meta = json.loads(meta_path.read_text()) if meta_path.exists() else {}
    for name in a.cases:
        meta[name] = make_case(name, CASES[name], a.threads)
        meta_path.write_text(json.dumps(meta, indent=1, sort_keys=True) + "\n")


if __name__ == "__main__":
    main()
