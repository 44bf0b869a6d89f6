// noalloc.cu -- GQA decode attention for callers that cannot allocate memory.
//
// Some callers of this library cannot allocate device memory while they run:
// serving loops that cannot take the device-wide synchronization that
// cudaFree (and often cudaMalloc) imposes between steps, embedders whose whole
// device memory is handed to their own pool or arena up front (a cudaMalloc
// would fail, or steal memory the pool has accounted for), and latency-bound
// paths that must not meet an out-of-memory error in the middle of serving.
// The regular
// attention entry point (nexus_cuda_execute with NEXUS_OP_ATTENTION) obtains
// its scratch -- the per-slice softmax partials, the per-head arrival counters
// and the step descriptor -- with cudaMalloc on every call.  The entry point in
// this file runs the same kernel with that scratch placed in a fixed
// file-scope device array instead, so it allocates nothing.  Inputs and the
// output stay in the caller's device buffers.
//
// Limits and sharing:
//   - The array holds kNoAllocScratchBytes (1 MiB) of slice partials; calls
//     whose num_kv_heads * slices * (num_q_heads/num_kv_heads) * (head_dim+2)
//     floats exceed it are rejected with NEXUS_E_INVALID.  (slices =
//     min(64, ceil(seq_len / 64)).)
//   - Every GPU that loads the library holds the array until the process exits.
//   - All calls share the one array and it keeps the last call's contents;
//     the counters that must start at zero are cleared at the start of every
//     call.  Calls that overlap on the GPU (different streams, or different
//     host threads on one stream without ordering) race on the array; order
//     them on one stream.
//   - The first call on a device looks up the array's device address with
//     cudaGetSymbolAddress (the host-side name of a __device__ array is only a
//     stand-in, not a device address).  Make that first call before any stream
//     capture begins.
#include <cuda_runtime.h>

#include <mutex>
#include <string>

#include "../../include/nexus_cuda.h"
#include "kernels.h"

namespace nx {

constexpr size_t kNoAllocScratchBytes = 1u << 20;            // slice partials
constexpr size_t kNoAllocCounterSlots = 256;                  // KV heads
constexpr size_t kNoAllocTotal = kNoAllocScratchBytes + kNoAllocCounterSlots * 4 + 256;

// The scratch array: [partials | counters | DevSeq | seq_id]
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocTotal];

namespace {
std::mutex g_addr_mu;
void *g_addr[64] = {};  // device address of g_noalloc_scratch per device ordinal

__global__ void k_noalloc_step(DevSeq *seq, uint32_t *sid, unsigned seq_len) {
    DevSeq s = {};
    s.seq_len = seq_len;
    s.slot = seq_len - 1;
    *seq = s;
    *sid = 0u;
}
}  // namespace

}  // namespace nx

using namespace nx;

// Backend accessors implemented in engine.cu.
extern int nexus_backend_stream_device(nexus_cuda_backend *b, cudaStream_t *stream, int *device);
extern int nexus_backend_fail(nexus_cuda_backend *b, int code, const char *msg);

extern "C" int nexus_cuda_attention_noalloc(nexus_cuda_backend *b, const float *q_dev, const float *k_dev,
                                            const float *v_dev, float *out_dev, size_t num_q_heads,
                                            size_t num_kv_heads, size_t head_dim, size_t seq_len, float scale) {
    cudaStream_t st = nullptr;
    int dev = 0;
    if (!b || nexus_backend_stream_device(b, &st, &dev) != NEXUS_OK)
        return nexus_backend_fail(b, NEXUS_E_INVALID, "attention_noalloc: NULL backend");
    if (!q_dev || !k_dev || !v_dev || !out_dev)
        return nexus_backend_fail(b, NEXUS_E_INVALID, "attention_noalloc: NULL device pointer");
    if (seq_len == 0 || num_kv_heads == 0 || num_q_heads == 0 || num_q_heads % num_kv_heads ||
        seq_len > 0x7fffffffu)
        return nexus_backend_fail(b, NEXUS_E_INVALID, "attention_noalloc: bad shape");
    if (head_dim != 32 && head_dim != 64 && head_dim != 128)
        return nexus_backend_fail(b, NEXUS_E_INVALID, "attention_noalloc: head_dim must be 32, 64 or 128");
    const size_t G = num_q_heads / num_kv_heads;
    if (G > 8 || (G & (G - 1))) return nexus_backend_fail(b, NEXUS_E_INVALID, "attention_noalloc: q/kv head ratio must be 1, 2, 4 or 8");
    if (num_kv_heads > kNoAllocCounterSlots)
        return nexus_backend_fail(b, NEXUS_E_INVALID, "attention_noalloc: more than 256 KV heads");
    const size_t nsplit = seq_len / 64 + (seq_len % 64 ? 1 : 0) > 64 ? 64 : seq_len / 64 + (seq_len % 64 ? 1 : 0);
    const size_t need = num_kv_heads * nsplit * G * (head_dim + 2) * sizeof(float);
    if (need > kNoAllocScratchBytes)
        return nexus_backend_fail(b, NEXUS_E_INVALID,
                                  ("attention_noalloc: needs " + std::to_string(need) +
                                   " scratch bytes, more than the fixed 1 MiB")
                                      .c_str());
    if (dev < 0 || dev >= 64) return nexus_backend_fail(b, NEXUS_E_INVALID, "attention_noalloc: device ordinal >= 64");
    // the backend's device is made current for the call; the caller's is restored on return
    int caller_dev = -1;
    if (cudaGetDevice(&caller_dev) != cudaSuccess) caller_dev = -1;
    struct RestoreDevice {
        int d;
        ~RestoreDevice() {
            if (d >= 0) cudaSetDevice(d);
        }
    } restore{caller_dev};
    cudaError_t e = cudaSetDevice(dev);
    void *base = nullptr;
    if (e == cudaSuccess) {
        std::lock_guard<std::mutex> lk(g_addr_mu);
        if (!g_addr[dev]) {
            e = cudaGetSymbolAddress(&g_addr[dev], g_noalloc_scratch);
            if (e != cudaSuccess) g_addr[dev] = nullptr;
        }
        base = g_addr[dev];
    }
    if (e != cudaSuccess || !base)
        return nexus_backend_fail(b, NEXUS_E_CUDA,
                                  (std::string("attention_noalloc: scratch address: ") + cudaGetErrorString(e)).c_str());
    unsigned char *p = static_cast<unsigned char *>(base);
    float *part = reinterpret_cast<float *>(p);
    unsigned *counters = reinterpret_cast<unsigned *>(p + kNoAllocScratchBytes);
    DevSeq *seq = reinterpret_cast<DevSeq *>(p + kNoAllocScratchBytes + kNoAllocCounterSlots * 4);
    uint32_t *sid = reinterpret_cast<uint32_t *>(p + kNoAllocScratchBytes + kNoAllocCounterSlots * 4 + 64);
    // the counters must start at zero; the previous call may have left anything
    e = cudaMemsetAsync(counters, 0, num_kv_heads * sizeof(unsigned), st);
    if (e == cudaSuccess) {
        k_noalloc_step<<<1, 1, 0, st>>>(seq, sid, (unsigned)seq_len);
        e = cudaGetLastError();
    }
    if (e == cudaSuccess) {
        AttnParams a = {};
        a.hq = (int)num_q_heads;
        a.hkv = (int)num_kv_heads;
        a.head_dim = (int)head_dim;
        a.m = 1;
        a.q = q_dev;
        a.out = out_dev;
        a.scale = scale != 0.0f ? scale : 1.0f / sqrtf((float)head_dim);
        a.k_cache = k_dev;
        a.v_cache = v_dev;
        a.seqs = seq;
        a.seq_ids = sid;
        a.kv_dim = (int)(num_kv_heads * head_dim);
        a.nsplit = (int)nsplit;
        a.part = part;
        a.counters = counters;
        e = launch_attention(a, st);
    }
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e != cudaSuccess)
        return nexus_backend_fail(b, NEXUS_E_CUDA, (std::string("attention_noalloc: ") + cudaGetErrorString(e)).c_str());
    return NEXUS_OK;
}
