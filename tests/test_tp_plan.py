"""Tensor-parallel shard plan (host arithmetic, no GPU): every rank's slice of
heads, FFN rows and vocab rows partitions the model exactly, and shapes that
cannot split into whole super-blocks are rejected.  The gloo test runs the
plan on two CPU ranks and checks the gathered slices, as the launcher would."""
import os
import socket

import pytest

from nexus_b200 import configs


def plans(cfg, world):
    import nexus_b200 as nb
    D = cfg["hidden_size"] // cfg["num_heads"]
    return [nb.tp_plan(cfg["num_heads"], cfg["num_kv_heads"], D, cfg["ff_dim"], cfg["vocab_size"], r, world)
            for r in range(world)]


def check_partition(ps, cfg):
    for key_b, key_n, total in (("q_head_begin", "q_heads", cfg["num_heads"]),
                                ("kv_head_begin", "kv_heads", cfg["num_kv_heads"]),
                                ("ffn_begin", "ffn_rows", cfg["ff_dim"]),
                                ("vocab_begin", "vocab_rows", cfg["vocab_size"])):
        covered = []
        for p in ps:
            covered.extend(range(p[key_b], p[key_b] + p[key_n]))
        assert covered == list(range(total)), key_b
    # each rank's query heads map onto its own KV heads (GQA groups stay whole)
    G = cfg["num_heads"] // cfg["num_kv_heads"]
    for p in ps:
        assert p["q_head_begin"] // G == p["kv_head_begin"] and p["q_heads"] == G * p["kv_heads"]


@pytest.mark.parametrize("name", ["llama8b_q4k", "llama70b", "tp_small"])
@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_plan_partitions_model(nb, name, world):
    cfg = configs.CONFIGS[name]
    check_partition(plans(cfg, world), cfg)


def test_plan_rejects_unaligned_split(nb):
    # tiny: 8 heads of 32 -> 128 columns per rank at world 2, not a whole super-block
    with pytest.raises(nb.NexusError):
        plans(configs.CONFIGS["tiny"], 2)
    with pytest.raises(nb.NexusError):
        nb.tp_plan(16, 8, 128, 4096, 8192, 2, 2)  # rank outside the world


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _gloo_worker(rank, world, port, name, out):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    import nexus_b200 as nb
    cfg = configs.CONFIGS[name]
    D = cfg["hidden_size"] // cfg["num_heads"]
    mine = nb.tp_plan(cfg["num_heads"], cfg["num_kv_heads"], D, cfg["ff_dim"], cfg["vocab_size"], rank, world)
    got = [None] * world
    dist.all_gather_object(got, mine)
    if rank == 0:
        check_partition(got, cfg)
        out.put("ok")
    dist.destroy_process_group()


@pytest.mark.parametrize("name", ["llama8b_q4k", "tp_small"])
def test_plan_two_gloo_ranks(nb, name):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gloo_worker, args=(r, 2, port, name, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs)
    assert q.get(timeout=5) == "ok"
