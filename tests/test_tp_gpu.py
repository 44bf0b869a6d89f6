"""Tensor-parallel decode on 2 GPUs (one process per GPU, one all-reduce per
sublayer) against the CPU oracle: logits within 2e-3, greedy tokens identical,
for both all-reduces -- the one-shot kernel over NVLink peer memory (the
default) and NCCL -- which must also agree with each other.  Single-token
steps, a chunked prefill and batched steps.  NVLS stays off (the peer kernel
uses plain peer loads and stores).  Skipped when fewer than two GPUs are
visible."""
import json
import os
import socket
import subprocess
import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parents[1]


def _gpus():
    import torch
    return torch.cuda.device_count() if torch.cuda.is_available() else 0


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


@pytest.mark.skipif(_gpus() < 2, reason="needs 2 GPUs")
def test_tp2_matches_oracle(nb, tmp_path):
    model = nb.model_path("tp_small")
    out = tmp_path / "tp.json"
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr=127.0.0.1", f"--master-port={_port()}", str(ROOT / "tests" / "tp_worker.py"), str(out),
           str(model)]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]
    res = json.loads(out.read_text())
    print(json.dumps({k: v for k, v in res.items() if k in ("kinds", "peer_vs_nccl")}))
    assert res["kinds"] == ["peer", "nccl"], res["kinds"]
    for mode in ("peer", "nccl"):
        r = res[mode]
        assert r["max_abs"] < 2e-3 and r["long_max_abs"] < 2e-3, (mode, r)
        assert r["tok"] == res["ref_tok"] and r["long_tok"] == res["ref_long_tok"], mode
        assert r["gen"] == res["ref_gen"], mode
        assert r["batch_tokens"] == res["ref_batch_tokens"], mode
    # both all-reduces add the two ranks' partials once: the same float sums
    for k, v in res["peer_vs_nccl"].items():
        assert v < 1e-5, (k, v)
