"""One rank of a tensor-parallel parity run (launched by torch.distributed.run
from tests/test_tp_gpu.py): the tp_small model split over the world, run
twice -- with the one-shot peer-memory all-reduce and with NCCL
(NEXUS_CFG_NCCL_ALLREDUCE) -- on the same calls: a 24-token prefill and 16
greedy tokens, a 300-token prefill (one 256-token chunk, then the rest), and
4 batched steps of 8 sequences.  Rank 0 compares both against the CPU oracle
and against each other and writes the verdict as JSON.  Every rank loads
(and validates) before the first collective, so a failing rank stops the run
on the host side."""
import json
import os
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))

BATCH, BATCH_STEPS = 8, 4


def _run(nb, L, local, rank, world, uid, model, flags, dist):
    be = nb.CudaBackend(device=local, max_seq_len=512, max_batch=BATCH, flags=flags)
    be.tp_init(rank, world, uid)
    kind = be.tp_allreduce_kind()
    eng = nb.InferenceEngine(be)
    eng.load_model(model)
    dist.barrier()  # every rank loaded before the first collective
    vocab = eng.info.vocab_rows
    rng = np.random.default_rng(5)
    prompt = rng.integers(0, vocab, 24).tolist()
    long_prompt = rng.integers(0, vocab, 300).tolist()
    out = {"kind": kind}
    logits, tok = eng.prefill(prompt)
    out["logits"], out["tok"] = logits, int(tok)
    out["gen"] = eng.generate(prompt, 16)
    out["long_logits"], out["long_tok"] = eng.prefill(long_prompt)
    prompts = [rng.integers(0, vocab, 10 + 3 * s).tolist() for s in range(BATCH)]
    toks = [eng.prefill(p, seq_id=s, want_logits=False)[1] for s, p in enumerate(prompts)]
    steps = [list(toks)]
    for i in range(BATCH_STEPS):
        items = [(s, toks[s], len(prompts[s]) + i) for s in range(BATCH)]
        toks, lg = eng.decode_batch(items, want_logits=i == BATCH_STEPS - 1)
        toks = list(toks)
        steps.append(toks)
    out["batch_tokens"], out["batch_logits"] = steps, lg
    out["prompts"], out["prompt"], out["long_prompt"] = prompts, prompt, long_prompt
    eng.close()
    be.close()
    dist.barrier()
    return out


def main():
    import datetime

    import torch
    import torch.distributed as dist

    out_path, model = sys.argv[1], sys.argv[2]
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=120))
    import nexus_b200 as nb
    from nexus_b200 import _lib as L

    torch.cuda.set_device(local)
    runs = {}
    for mode, flags in [("peer", 0), ("nccl", L.CFG_NCCL_ALLREDUCE)]:
        uid = [nb.tp_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        runs[mode] = _run(nb, L, local, rank, world, uid[0], model, flags, dist)
    if rank == 0:
        from oracle import oracle as O
        O.load()
        p, n = runs["peer"], runs["nccl"]
        m = O.Model(model, max_seq_len=512)
        ref = m.prefill(p["prompt"])
        refgen = O.Model(model, max_seq_len=512).generate(p["prompt"], 16)
        ref_long = O.Model(model, max_seq_len=512).prefill(p["long_prompt"])
        # per batch sequence: the prefill's token, then one per batched step
        ref_batch = [O.Model(model, max_seq_len=512).generate(q, BATCH_STEPS + 1)[len(q):] for q in p["prompts"]]
        ref_batch = [list(t) for t in zip(*ref_batch)]
        res = {"world": world, "kinds": [p["kind"], n["kind"]], "ref_tok": int(O.greedy(ref)), "ref_gen": refgen,
               "ref_long_tok": int(O.greedy(ref_long)), "ref_batch_tokens": ref_batch}
        for mode, r in runs.items():
            res[mode] = {"max_abs": float(np.max(np.abs(r["logits"] - ref))), "tok": r["tok"], "gen": r["gen"],
                         "long_max_abs": float(np.max(np.abs(r["long_logits"] - ref_long))),
                         "long_tok": int(r["long_tok"]), "batch_tokens": r["batch_tokens"]}
        res["peer_vs_nccl"] = {
            "logits": float(np.max(np.abs(p["logits"] - n["logits"]))),
            "long_logits": float(np.max(np.abs(p["long_logits"] - n["long_logits"]))),
            "batch_logits": float(np.max(np.abs(np.asarray(p["batch_logits"]) - np.asarray(n["batch_logits"])))),
        }
        Path(out_path).write_text(json.dumps(res))
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
