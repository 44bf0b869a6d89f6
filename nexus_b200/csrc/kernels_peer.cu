// kernels_peer.cu -- one-shot all-reduce of the hidden state over NVLink peer
// memory, for tensor-parallel decode.
//
// Under tensor parallelism every o_proj and down GEMV leaves a partial sum of
// the hidden state on each rank, and the sublayer needs their sum on every
// rank (64 all-reduces per token for the Llama-3-8B shape; the reference has
// no multi-GPU path).  At batch 1 the vector is 16 KB: the cost is latency,
// not bandwidth.  This kernel does it in one launch and one NVLink round trip:
// each CTA stages its slice of this rank's partial in a buffer the other ranks
// map (CUDA IPC), publishes an epoch flag with release semantics, waits
// (bounded) for every peer's flag of the same epoch, then reads the peers'
// slices directly over NVLink and adds all partials in rank order -- the same
// order on every rank, so every rank holds bit-identical sums.
//
// Buffers are double-buffered by epoch parity: a rank can only reuse a buffer
// two epochs later, after every peer has finished reading it (a peer starts
// epoch e + 1, and sets that flag, only after its epoch-e kernel completed).
// Every launch has kPeerCtas CTAs, whatever n, so that every CTA's epoch
// advances on every call and a CTA's parity never lags another CTA's slice
// of the same buffer.  A wait that gives up sets the error flag and leaves x
// as this rank's partial; the host reports NEXUS_E_TIMEOUT and refuses
// further tensor-parallel steps.
#include <cuda_runtime.h>

#include "kernels.h"

namespace nx {

namespace {

constexpr unsigned kPeerSpin = 1u << 22;

__device__ __forceinline__ void st_release_sys(unsigned *p, unsigned v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned *p) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__global__ void __launch_bounds__(512) k_peer_allreduce(PeerReduce pr, float *x, size_t n) {
    const int b = blockIdx.x, nb = gridDim.x;
    const size_t s0 = n * b / nb, s1 = n * (b + 1) / nb;
    __shared__ unsigned e_s;
    __shared__ int ok_s;
    if (threadIdx.x == 0) e_s = pr.epoch[b] + 1u;
    __syncthreads();
    const unsigned e = e_s;
    const int par = (int)(e & 1u);
    float *mine = pr.bufs[pr.rank][par];
    for (size_t i = s0 + threadIdx.x; i < s1; i += blockDim.x) mine[i] = x[i];
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence_system();
        st_release_sys(&pr.flags[pr.rank][2 * b + par], e);
        int ok = 1;
        for (int r = 0; r < pr.world && ok; r++) {
            if (r == pr.rank) continue;
            unsigned k = 0;
            while ((int)(ld_acquire_sys(&pr.flags[r][2 * b + par]) - e) < 0) {
                if (++k > kPeerSpin) {
                    ok = 0;
                    if (pr.err) atomicExch(pr.err, 3);
                    break;
                }
                __nanosleep(32);
            }
        }
        pr.epoch[b] = e;
        ok_s = ok;
    }
    __syncthreads();
    if (!ok_s) return;
    for (size_t i = s0 + threadIdx.x; i < s1; i += blockDim.x) {
        const float own = x[i];
        float tot = 0.0f;
        for (int r = 0; r < pr.world; r++) tot += r == pr.rank ? own : __ldcv(pr.bufs[r][par] + i);
        x[i] = tot;
    }
}

}  // namespace

cudaError_t launch_peer_allreduce(const PeerReduce &pr, float *x, size_t n, cudaStream_t st) {
    if (n == 0 || n > pr.max_floats || pr.world < 2 || pr.world > kPeerMaxRanks) return cudaErrorInvalidValue;
    k_peer_allreduce<<<kPeerCtas, 512, 0, st>>>(pr, x, n);
    return cudaGetLastError();
}

}  // namespace nx
