"""Failure paths of the CUDA backend, made without faulting the GPU.

* A device wait that runs out: the persistent step kernel's grid barrier is
  told (NEXUS_CFG_FAULT_STALL_BARRIER) to wait for a CTA that does not exist.
  Every CTA gives up after its bounded wait, sets the device error flag, waits
  for its weight copies in flight and leaves; the call returns
  NEXUS_E_TIMEOUT, the barrier and arrival counters are reset, the next call
  times out the same way instead of hanging, and a fresh model on the same
  device decodes correctly afterwards.
* A failed device allocation: a KV page pool far larger than the GPU makes
  cudaMalloc fail during the model load, which returns NEXUS_E_OOM (not a
  generic CUDA error), frees what it had allocated, and leaves the context
  usable.
* Bad tensor-parallel arguments are refused on the host before NCCL is
  touched.
* A tensor-parallel rank that never joins: rank 0 of a world of 2 calls
  nexus_cuda_tp_init and nobody else does.  The join waits on the host (a
  nonblocking NCCL communicator polled against tp_timeout_ms), gives up with
  NEXUS_E_COMM, tears its half of the group down, and the same process then
  runs a single-GPU model.  The rank runs as a child process with its own
  time limit, so a join that did not give up could not stall the test run;
  no kernel is in flight at any point.

The reference has no device path; its decode errors are Result<_, String>
and it falls back silently to a stateless decode when a tensor is missing
(src/engine/mod.rs:1160-1166).  Here errors are status codes.
"""
import os
import subprocess
import sys
import time
from pathlib import Path

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _prompt(seed, n, vocab):
    return np.random.default_rng(seed).integers(0, vocab, n).tolist()


def test_device_wait_timeout_reports_and_recovers(nb, oracle):
    from nexus_b200 import NexusError
    from nexus_b200 import _lib as L
    path = nb.model_path("tp_small")
    p = _prompt(3, 20, 8192)
    be = nb.CudaBackend(device=0, max_seq_len=64, flags=L.CFG_PERSISTENT | L.CFG_FAULT_STALL_BARRIER)
    e = nb.InferenceEngine(be)
    e.load_model(path)
    _, tok = e.prefill(p)            # prefill runs on the batched path, not the step kernel
    for _ in range(2):
        with pytest.raises(NexusError) as err:
            e.decode_with_cache(tok, len(p))
        assert err.value.code == L.NEXUS_E_TIMEOUT
        assert e.seq_len() == len(p)  # the failed step did not advance the sequence
    e.close()
    be.close()
    # the device and the library still work
    be = nb.CudaBackend(device=0, max_seq_len=64, flags=L.CFG_PERSISTENT)
    e = nb.InferenceEngine(be)
    e.load_model(path)
    m = oracle.Model(path, max_seq_len=64)
    ref = m.prefill(p)
    got, t0 = e.prefill(p)
    assert t0 == oracle.greedy(ref)
    ref = m.decode(t0, len(p))
    got, t1 = e.decode_with_cache(t0, len(p))
    assert np.max(np.abs(got - ref)) < 2e-3 and t1 == oracle.greedy(ref)
    e.close()
    be.close()


def test_device_allocation_failure_is_oom(nb, tiny_path):
    from nexus_b200 import NexusError
    from nexus_b200 import _lib as L
    # 2^20 sequences x 512 tokens of float K and V for 4 layers: ~550 GB
    be = nb.CudaBackend(device=0, max_batch=1 << 20, max_seq_len=512)
    e = nb.InferenceEngine(be)
    with pytest.raises(NexusError) as err:
        e.load_model(tiny_path)
    assert err.value.code == L.NEXUS_E_OOM
    be.close()
    be = nb.CudaBackend(device=0)
    e = nb.InferenceEngine(be)
    e.load_model(tiny_path)
    assert len(e.generate(_prompt(1, 8, 4096), 4)) == 12
    e.close()
    be.close()


def test_tensor_parallel_bad_arguments_refused(nb):
    from nexus_b200 import NexusError
    from nexus_b200 import _lib as L
    be = nb.CudaBackend(device=0)
    uid = nb.tp_unique_id()
    for rank, world in [(2, 2), (-1, 2), (0, 0)]:
        with pytest.raises(NexusError) as err:
            be.tp_init(rank, world, uid)
        assert err.value.code == L.NEXUS_E_INVALID
    be.close()


_NEVER_JOINS = r"""
import sys, time
sys.path.insert(0, sys.argv[1])
import numpy as np
import nexus_b200 as nb
from nexus_b200 import NexusError
from nexus_b200 import _lib as L
be = nb.CudaBackend(device=0, tp_timeout_ms=3000)
t0 = time.time()
try:
    be.tp_init(0, 2, nb.tp_unique_id())
    code = 0
except NexusError as e:
    code, msg = e.code, str(e)
took = time.time() - t0
assert code == L.NEXUS_E_COMM, code
assert be.tp_allreduce_kind() == "none"
be.close()
be = nb.CudaBackend(device=0)
e = nb.InferenceEngine(be)
e.load_model(sys.argv[2])
assert len(e.generate(list(range(1, 9)), 4)) == 12
e.close()
be.close()
print("OK", round(took, 2), msg)
"""


def test_tensor_parallel_rank_never_joins(nb, tiny_path):
    root = Path(__file__).resolve().parents[1]
    t0 = time.time()
    r = subprocess.run([sys.executable, "-c", _NEVER_JOINS, str(root), str(tiny_path)], capture_output=True,
                       text=True, timeout=180, env={**os.environ, "NCCL_NVLS_ENABLE": "0"})
    print(r.stdout[-500:], r.stderr[-1500:])
    assert r.returncode == 0, r.stderr[-3000:]
    took = float(r.stdout.split("OK", 1)[1].split()[0])
    assert 2.5 < took < 60, took
    assert time.time() - t0 < 170
