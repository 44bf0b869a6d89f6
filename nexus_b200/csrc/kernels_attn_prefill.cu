// kernels_attn_prefill.cu -- causal GQA attention for a chunk of one sequence
// (prefill, speculative-verify windows) on the tensor cores.
//
// The reference prefills token by token (InferenceEngine::prefill,
// src/engine/mod.rs:1149-1170), each token running KvCache::attention_decode
// (:452-499) over the tokens before it.  A chunk of m prompt tokens processed
// in one step needs the same m attentions; run as m decode attentions each
// token re-reads its whole prefix.  Here one CTA owns one KV head and a tile of
// the chunk's tokens (its 64 rows are (token, query head) pairs of that KV
// head), loads each 32-key tile of K and V once into shared memory for all of
// its rows, and computes S = Q K^T and O += P V with mma.sync (m16n8k16, f32
// accumulate) under an online softmax, masking every key past the row's own
// position (causal).
//
// Precision: Q, K, P and V are split into f16 halves x = hi + lo (22
// significant bits) and every product is hi*hi + hi*lo + lo*hi, so scores and
// outputs keep ~2^-21 relative error (the reference computes in f32).
//
// Applies to the float cache, head_dim 128 (paged keys through KvPages).
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <math.h>

#include "common.cuh"
#include "kernels.h"

namespace nx {
namespace pf {

constexpr int D = 128;
constexpr int NW = 4;            // warps per CTA; 16 rows each
constexpr int ROWS = NW * 16;
constexpr int TK = 32;           // keys per tile
constexpr int KS = D + 8;        // K row stride in halves (padded against bank conflicts)
constexpr int VS = TK + 8;       // V^T row stride in halves

__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t h2u(__half2 h) { return *reinterpret_cast<uint32_t *>(&h); }

// (x0, x1) -> packed f16 hi pair and lo pair with x = hi + lo
__device__ __forceinline__ void split2(float x0, float x1, uint32_t &hi, uint32_t &lo) {
    const __half2 h = __floats2half2_rn(x0, x1);
    const float2 hf = __half22float2(h);
    hi = h2u(h);
    lo = h2u(__floats2half2_rn(x0 - hf.x, x1 - hf.y));
}

struct Smem {
    __half kh[TK][KS], kl[TK][KS];     // K tile, [key][dim]
    __half vh[D][VS], vl[D][VS];       // V tile transposed, [dim][key]
};

// grid (hkv, ceil(m / (ROWS / G))), block NW * 32.  The step's m tokens are
// consecutive positions of the sequence in cache row seq_ids[0]: token t sits
// at slot seqs[0].slot + t and attends to slots 0 .. seqs[0].slot + t.
template <int G>
__global__ void __launch_bounds__(NW * 32, 2) k_attn_prefill(AttnParams p) {
    __shared__ __align__(16) Smem sm;
    constexpr int TQ = ROWS / G;  // tokens per CTA
    const int h = blockIdx.x;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int gid = lane >> 2, tig = lane & 3;
    if (p.pdl) {
        pdl_launch_dependents();
        pdl_wait();
    }
    const uint32_t base = p.seqs[0].slot;
    const uint32_t sid = p.seq_ids[0];
    const int t_first = blockIdx.y * TQ;
    const int t_last = min(p.m, t_first + TQ) - 1;  // last token of this CTA
    const int kmax = (int)base + t_last + 1;          // keys the CTA's rows can see
    const float scale = p.scale;

    // this thread's two rows: r = warp*16 + gid (+8) -> token r / G, head r % G
    int tok[2], slot[2];
    bool valid[2];
#pragma unroll
    for (int i = 0; i < 2; i++) {
        const int r = warp * 16 + gid + 8 * i;
        tok[i] = t_first + r / G;
        valid[i] = tok[i] <= t_last;
        slot[i] = (int)base + tok[i];
    }
    // Q fragments (A operand), 8 k-steps of 16 dims, hi and lo
    uint32_t qh[8][4], ql[8][4];
#pragma unroll
    for (int ks = 0; ks < 8; ks++) {
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const int i = j & 1;                   // row gid (0) or gid + 8 (1)
            const int col = ks * 16 + tig * 2 + (j >> 1) * 8;
            const int r = warp * 16 + gid + 8 * i;
            float x0 = 0.0f, x1 = 0.0f;
            if (valid[i]) {
                const float *q = p.q + (size_t)tok[i] * p.hq * D + (size_t)(h * G + r % G) * D + col;
                const float2 v = __ldcg(reinterpret_cast<const float2 *>(q));
                x0 = v.x;
                x1 = v.y;
            }
            split2(x0, x1, qh[ks][j], ql[ks][j]);
        }
    }
    float o[16][4];
#pragma unroll
    for (int nd = 0; nd < 16; nd++)
#pragma unroll
        for (int c = 0; c < 4; c++) o[nd][c] = 0.0f;
    float mrow[2] = {-INFINITY, -INFINITY}, lrow[2] = {0.0f, 0.0f};

    for (int k0 = 0; k0 < kmax; k0 += TK) {
        // ---- K and V tile: thread i loads key i / 4, dims (i % 4) * 32 .. + 31 ----
        {
            const int kk = threadIdx.x >> 2, d0 = (threadIdx.x & 3) * 32;
            const int key = k0 + kk;
            const bool in = key < kmax;
            const size_t ph = kv_phys(p.pages, sid, (uint32_t)(in ? key : 0));
            const float *kr = p.k_cache + ph * p.kv_dim + h * D + d0;
            const float *vr = p.v_cache + ph * p.kv_dim + h * D + d0;
#pragma unroll
            for (int c = 0; c < 8; c++) {
                float4 kv = in ? __ldcg(reinterpret_cast<const float4 *>(kr) + c) : make_float4(0.f, 0.f, 0.f, 0.f);
                float4 vv = in ? __ldcg(reinterpret_cast<const float4 *>(vr) + c) : make_float4(0.f, 0.f, 0.f, 0.f);
                uint32_t a, b;
                split2(kv.x, kv.y, a, b);
                *reinterpret_cast<uint32_t *>(&sm.kh[kk][d0 + 4 * c]) = a;
                *reinterpret_cast<uint32_t *>(&sm.kl[kk][d0 + 4 * c]) = b;
                split2(kv.z, kv.w, a, b);
                *reinterpret_cast<uint32_t *>(&sm.kh[kk][d0 + 4 * c + 2]) = a;
                *reinterpret_cast<uint32_t *>(&sm.kl[kk][d0 + 4 * c + 2]) = b;
                const float vx[4] = {vv.x, vv.y, vv.z, vv.w};
#pragma unroll
                for (int e = 0; e < 4; e++) {
                    const __half hv = __float2half_rn(vx[e]);
                    sm.vh[d0 + 4 * c + e][kk] = hv;
                    sm.vl[d0 + 4 * c + e][kk] = __float2half_rn(vx[e] - __half2float(hv));
                }
            }
        }
        __syncthreads();
        // ---- S = Q K^T for this warp's 16 rows x 32 keys ----
        float s[4][4];
#pragma unroll
        for (int nf = 0; nf < 4; nf++) {
#pragma unroll
            for (int c = 0; c < 4; c++) s[nf][c] = 0.0f;
            const int key = nf * 8 + gid;
#pragma unroll
            for (int ks = 0; ks < 8; ks++) {
                const int col = ks * 16 + tig * 2;
                const uint32_t bh0 = *reinterpret_cast<const uint32_t *>(&sm.kh[key][col]);
                const uint32_t bh1 = *reinterpret_cast<const uint32_t *>(&sm.kh[key][col + 8]);
                const uint32_t bl0 = *reinterpret_cast<const uint32_t *>(&sm.kl[key][col]);
                const uint32_t bl1 = *reinterpret_cast<const uint32_t *>(&sm.kl[key][col + 8]);
                mma16816(s[nf], qh[ks][0], qh[ks][1], qh[ks][2], qh[ks][3], bh0, bh1);
                mma16816(s[nf], qh[ks][0], qh[ks][1], qh[ks][2], qh[ks][3], bl0, bl1);
                mma16816(s[nf], ql[ks][0], ql[ks][1], ql[ks][2], ql[ks][3], bh0, bh1);
            }
        }
        // ---- scale, causal mask, online softmax per row ----
        float corr[2];
#pragma unroll
        for (int i = 0; i < 2; i++) {
            float mx = -INFINITY;
#pragma unroll
            for (int nf = 0; nf < 4; nf++)
#pragma unroll
                for (int c = 0; c < 2; c++) {
                    const int key = k0 + nf * 8 + tig * 2 + c;
                    float v = s[nf][2 * i + c] * scale;
                    if (!valid[i] || key > slot[i]) v = -INFINITY;
                    s[nf][2 * i + c] = v;
                    mx = fmaxf(mx, v);
                }
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
            const float mn = fmaxf(mrow[i], mx);
            corr[i] = mn == -INFINITY ? 1.0f : expf(mrow[i] - mn);
            float sum = 0.0f;
#pragma unroll
            for (int nf = 0; nf < 4; nf++)
#pragma unroll
                for (int c = 0; c < 2; c++) {
                    const float v = s[nf][2 * i + c];
                    const float e = v == -INFINITY ? 0.0f : expf(v - mn);
                    s[nf][2 * i + c] = e;
                    sum += e;
                }
            sum += __shfl_xor_sync(0xffffffffu, sum, 1);
            sum += __shfl_xor_sync(0xffffffffu, sum, 2);
            lrow[i] = lrow[i] * corr[i] + sum;
            mrow[i] = mn;
        }
#pragma unroll
        for (int nd = 0; nd < 16; nd++) {
            o[nd][0] *= corr[0];
            o[nd][1] *= corr[0];
            o[nd][2] *= corr[1];
            o[nd][3] *= corr[1];
        }
        // ---- O += P V: P from the score fragments (two 8-key groups per k-step) ----
#pragma unroll
        for (int ks = 0; ks < 2; ks++) {
            uint32_t ah[4], al[4];
            split2(s[2 * ks][0], s[2 * ks][1], ah[0], al[0]);
            split2(s[2 * ks][2], s[2 * ks][3], ah[1], al[1]);
            split2(s[2 * ks + 1][0], s[2 * ks + 1][1], ah[2], al[2]);
            split2(s[2 * ks + 1][2], s[2 * ks + 1][3], ah[3], al[3]);
            const int kc = ks * 16 + tig * 2;
#pragma unroll
            for (int nd = 0; nd < 16; nd++) {
                const int dim = nd * 8 + gid;
                const uint32_t bh0 = *reinterpret_cast<const uint32_t *>(&sm.vh[dim][kc]);
                const uint32_t bh1 = *reinterpret_cast<const uint32_t *>(&sm.vh[dim][kc + 8]);
                const uint32_t bl0 = *reinterpret_cast<const uint32_t *>(&sm.vl[dim][kc]);
                const uint32_t bl1 = *reinterpret_cast<const uint32_t *>(&sm.vl[dim][kc + 8]);
                mma16816(o[nd], ah[0], ah[1], ah[2], ah[3], bh0, bh1);
                mma16816(o[nd], ah[0], ah[1], ah[2], ah[3], bl0, bl1);
                mma16816(o[nd], al[0], al[1], al[2], al[3], bh0, bh1);
            }
        }
        __syncthreads();
    }
    // ---- normalize and store: rows gid (c0, c1) and gid + 8 (c2, c3) ----
#pragma unroll
    for (int i = 0; i < 2; i++) {
        if (!valid[i]) continue;
        const int r = warp * 16 + gid + 8 * i;
        // a head whose softmax sum is not positive stays zero (src/engine/mod.rs:483-485)
        const float inv = lrow[i] > 0.0f ? 1.0f / lrow[i] : 0.0f;
        float *out = p.out + (size_t)tok[i] * p.hq * D + (size_t)(h * G + r % G) * D;
#pragma unroll
        for (int nd = 0; nd < 16; nd++) {
            float2 v = make_float2(o[nd][2 * i] * inv, o[nd][2 * i + 1] * inv);
            if (lrow[i] <= 0.0f) v = make_float2(0.0f, 0.0f);
            *reinterpret_cast<float2 *>(out + nd * 8 + tig * 2) = v;
        }
    }
}

template <int G>
cudaError_t launch_g(const AttnParams &p, cudaStream_t st) {
    constexpr int TQ = ROWS / G;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(p.hkv, (p.m + TQ - 1) / TQ);
    cfg.blockDim = dim3(NW * 32);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = p.pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, k_attn_prefill<G>, p);
}

}  // namespace pf

bool attention_prefill_supported(const AttnParams &p) {
    const int G = p.hkv > 0 ? p.hq / p.hkv : 0;
    return p.bits_k == 0 && p.head_dim == 128 && p.hkv > 0 && p.hq % p.hkv == 0 &&
           (G == 1 || G == 2 || G == 4 || G == 8);
}

cudaError_t launch_attention_prefill(const AttnParams &p, cudaStream_t st) {
    if (!attention_prefill_supported(p) || p.m < 1) return cudaErrorInvalidValue;
    switch (p.hq / p.hkv) {
    case 1: return pf::launch_g<1>(p, st);
    case 2: return pf::launch_g<2>(p, st);
    case 4: return pf::launch_g<4>(p, st);
    default: return pf::launch_g<8>(p, st);
    }
}

}  // namespace nx
