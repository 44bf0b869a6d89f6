"""The allocation-free attention entry point against the regular one.

nexus_cuda_attention_noalloc serves callers that must not allocate device
memory while they run (inside a stream capture, in loops that cannot take
cudaMalloc/cudaFree's device-wide synchronization, or with memory owned by
their own pool).  It keeps its scratch in one fixed device array.  Here it
is called through the C ABI on device buffers the test owns, twice in a row
(the second call reuses the array left by the first), and each result is
compared with nexus_cuda_execute(NEXUS_OP_ATTENTION) on the same inputs,
within the attention tolerance of tests/test_gpu_ops.py (1e-4 absolute).
This file is collected last so a failure here comes after every other test.
"""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ATTN_TOL = 1e-4


def _regular(backend, nb, q, k, v, hq, hkv, d, seq):
    from nexus_b200 import _lib as L
    out = __import__("torch").empty(hq * d, dtype=__import__("torch").float32, device="cuda")
    op = L.Op(kind=L.OP_ATTENTION, device_ptrs=1, a=q.data_ptr(), b=k.data_ptr(), c=v.data_ptr(),
              out=out.data_ptr(), m=hq, n=seq, k=d, kv_heads=hkv)
    backend.execute(op)
    return out


@pytest.mark.parametrize("hq,hkv,d,seq", [(32, 8, 128, 577), (8, 4, 32, 130)])
def test_noalloc_attention_matches_regular_twice(nb, hq, hkv, d, seq):
    import torch
    from nexus_b200 import _lib as L

    lib = L.load()
    if not lib.nexus_cuda_is_available():
        pytest.fail("no sm_100 CUDA device")
    backend = nb.CudaBackend(device=0)
    torch.cuda.set_device(0)
    for call in range(2):
        g = torch.Generator(device="cpu").manual_seed(70 + call + seq)
        q = torch.randn(hq * d, generator=g).cuda()
        k = torch.randn(seq * hkv * d, generator=g).cuda()
        v = torch.randn(seq * hkv * d, generator=g).cuda()
        out = torch.full((hq * d,), float("nan"), device="cuda")
        torch.cuda.synchronize()
        rc = lib.nexus_cuda_attention_noalloc(backend.handle, q.data_ptr(), k.data_ptr(), v.data_ptr(),
                                              out.data_ptr(), hq, hkv, d, seq, C.c_float(0.0))
        L.check(rc, backend.handle)
        ref = _regular(backend, nb, q, k, v, hq, hkv, d, seq)
        torch.cuda.synchronize()
        diff = (out - ref).abs().max().item()
        assert diff < ATTN_TOL, (call, diff)
    backend.close()


def test_noalloc_attention_rejects_oversized_scratch(nb):
    import torch
    from nexus_b200 import _lib as L

    lib = L.load()
    backend = nb.CudaBackend(device=0)
    x = torch.zeros(16, device="cuda")
    # 64 KV heads x 64 slices x 8 x 130 floats is far beyond the fixed 1 MiB
    rc = lib.nexus_cuda_attention_noalloc(backend.handle, x.data_ptr(), x.data_ptr(), x.data_ptr(), x.data_ptr(),
                                          512, 64, 128, 8192, C.c_float(0.0))
    assert rc == L.NEXUS_E_INVALID
    assert b"1 MiB" in lib.nexus_cuda_last_error(backend.handle)
    backend.close()
