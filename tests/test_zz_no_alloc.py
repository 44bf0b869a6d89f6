"""The allocation-free attention entry point against the regular one.

nexus_cuda_attention_noalloc serves callers that cannot allocate device
memory while they run: serving loops that cannot take cudaMalloc/cudaFree's
device-wide synchronization, and engines whose device memory is all in
their own pool.  It keeps its scratch in one fixed device array.  Here it is
called through the C ABI on device buffers the test owns, twice in a row (the
second call reuses the array the first one left), and each result is
compared with nexus_cuda_execute(NEXUS_OP_ATTENTION) on the same inputs and
with a float64 softmax attention computed on the host, within the attention
tolerance of tests/test_gpu_ops.py (1e-4 absolute).  This file is collected
last so a failure here comes after every other test.
"""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ATTN_TOL = 1e-4
MIB = 1 << 20


def _regular(backend, q, k, v, hq, hkv, d, seq):
    import torch
    from nexus_b200 import _lib as L
    out = torch.empty(hq * d, dtype=torch.float32, device="cuda")
    op = L.Op(kind=L.OP_ATTENTION, device_ptrs=1, a=q.data_ptr(), b=k.data_ptr(), c=v.data_ptr(),
              out=out.data_ptr(), m=hq, n=seq, k=d, kv_heads=hkv)
    backend.execute(op)
    return out


def _float64_attention(q, k, v, hq, hkv, d, seq):
    """softmax(q.k / sqrt(d)) . v per query head, GQA head h -> KV head h / (hq/hkv)."""
    q = q.reshape(hq, d).astype(np.float64)
    k = k.reshape(seq, hkv, d).astype(np.float64)
    v = v.reshape(seq, hkv, d).astype(np.float64)
    g = hq // hkv
    out = np.empty((hq, d))
    for h in range(hq):
        s = k[:, h // g, :] @ q[h] / np.sqrt(d)
        p = np.exp(s - s.max())
        out[h] = (p / p.sum()) @ v[:, h // g, :]
    return out.reshape(-1)


def _scratch_bytes(hq, hkv, d, seq):
    """The kernel's slice partials: min(64, ceil(seq/64)) slices per KV head."""
    nsplit = min(64, -(-seq // 64))
    return hkv * nsplit * (hq // hkv) * (d + 2) * 4


# (hq, hkv, d, seq): the 8B shape, a small shape, one past 4096 tokens (the
# 64-slice cap), G = 1, and G = 4 just under the 1 MiB scratch bound
SHAPES = [(32, 8, 128, 577), (8, 4, 32, 130), (8, 8, 64, 5000), (32, 8, 128, 3969)]


@pytest.mark.parametrize("hq,hkv,d,seq", SHAPES)
def test_noalloc_attention_matches_regular_twice(nb, hq, hkv, d, seq):
    import torch
    from nexus_b200 import _lib as L

    lib = L.load()
    if not lib.nexus_cuda_is_available():
        pytest.fail("no sm_100 CUDA device")
    assert _scratch_bytes(hq, hkv, d, seq) <= MIB
    backend = nb.CudaBackend(device=0)
    torch.cuda.set_device(0)
    for call in range(2):
        g = torch.Generator(device="cpu").manual_seed(70 + call + seq)
        qh = torch.randn(hq * d, generator=g)
        kh = torch.randn(seq * hkv * d, generator=g)
        vh = torch.randn(seq * hkv * d, generator=g)
        q, k, v = qh.cuda(), kh.cuda(), vh.cuda()
        out = torch.full((hq * d,), float("nan"), device="cuda")
        torch.cuda.synchronize()
        rc = lib.nexus_cuda_attention_noalloc(backend.handle, q.data_ptr(), k.data_ptr(), v.data_ptr(),
                                              out.data_ptr(), hq, hkv, d, seq, C.c_float(0.0))
        L.check(rc, backend.handle)
        assert torch.cuda.current_device() == 0
        ref = _regular(backend, q, k, v, hq, hkv, d, seq)
        torch.cuda.synchronize()
        diff = (out - ref).abs().max().item()
        assert diff < ATTN_TOL, (call, diff)
        want = _float64_attention(qh.numpy(), kh.numpy(), vh.numpy(), hq, hkv, d, seq)
        diff64 = float(np.max(np.abs(out.cpu().numpy().astype(np.float64) - want)))
        assert diff64 < ATTN_TOL, (call, diff64)
    backend.close()


def test_noalloc_attention_rejects_bad_shapes(nb):
    import torch
    from nexus_b200 import _lib as L

    lib = L.load()
    backend = nb.CudaBackend(device=0)
    x = torch.zeros(16, device="cuda")

    def call(hq, hkv, d, seq):
        return lib.nexus_cuda_attention_noalloc(backend.handle, x.data_ptr(), x.data_ptr(), x.data_ptr(),
                                                x.data_ptr(), hq, hkv, d, seq, C.c_float(0.0))

    # 64 KV heads x 64 slices x 8 x 130 floats is far beyond the fixed 1 MiB
    assert call(512, 64, 128, 8192) == L.NEXUS_E_INVALID
    assert b"1 MiB" in lib.nexus_cuda_last_error(backend.handle)
    # the neighbour of the accepted (32, 8, 128, 3969): one more slice crosses the bound
    assert _scratch_bytes(32, 8, 128, 4033) > MIB
    assert call(32, 8, 128, 4033) == L.NEXUS_E_INVALID
    # no query heads, a ratio that is not a power of two, an unsupported head_dim
    assert call(0, 8, 128, 64) == L.NEXUS_E_INVALID
    assert call(24, 8, 128, 64) == L.NEXUS_E_INVALID
    assert call(8, 8, 96, 64) == L.NEXUS_E_INVALID
    assert call(8, 8, 128, 0) == L.NEXUS_E_INVALID
    backend.close()
