"""One rank of a tensor-parallel parity run (launched by torch.distributed.run
from tests/test_tp_gpu.py): the tp_small model split over the world, a prompt
prefilled and greedy tokens generated; rank 0 compares against the CPU oracle
and writes the verdict as JSON.  Every rank loads (and validates) before the
first collective, so a failing rank stops the run on the host side."""
import json
import os
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))


def main():
    import datetime

    import torch
    import torch.distributed as dist

    out_path, model = sys.argv[1], sys.argv[2]
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=120))
    import nexus_b200 as nb

    torch.cuda.set_device(local)
    uid = [nb.tp_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(uid, src=0)
    be = nb.CudaBackend(device=local, max_seq_len=128)
    be.tp_init(rank, world, uid[0])
    eng = nb.InferenceEngine(be)
    eng.load_model(model)
    dist.barrier()  # every rank loaded before the first NCCL collective
    info = eng.info
    prompt = np.random.default_rng(5).integers(0, info.vocab_rows, 24).tolist()
    logits, tok = eng.prefill(prompt)
    gen = eng.generate(prompt, 16)
    single = None
    eng.close()
    be.close()
    dist.barrier()
    if rank == 0:
        from oracle import oracle as O
        O.load()
        m = O.Model(model)
        ref = m.prefill(prompt)
        m2 = O.Model(model)
        refgen = m2.generate(prompt, 16)
        res = {"world": world, "max_abs": float(np.max(np.abs(logits - ref))), "tok": int(tok),
               "ref_tok": int(O.greedy(ref)), "gen": gen, "ref_gen": refgen}
        Path(out_path).write_text(json.dumps(res))
    dist.barrier()
    dist.destroy_process_group()
    del single


if __name__ == "__main__":
    main()
