// kernels_attn.cu -- GQA decode attention over the KV cache (float or packed).
//
// Replaces KvCache::attention_decode (src/engine/mod.rs:452-499): for query
// head qh, kv head kvh = qh / (Hq/Hkv); s_t = (q . k_t) * (1/sqrt(D));
// o = sum_t softmax(s)_t * v_t.  Packed caches are read directly in their
// low-bit form: value = min_t + q * scale_t (PackedKvBuffer::value_at,
// src/engine/mod.rs:252-256), one (min, scale) per token across all KV heads.
//
// Split-context ("flash decoding") layout: grid (Hkv, nsplit, batch).  Each
// CTA owns one KV head, a contiguous slice of the context and all G query
// heads that share that KV head, so every K/V element is read from HBM once.
// Four warps stride over the slice's tokens; lane i holds head_dim/32 dims.
// Each warp keeps an online softmax per query head; warps are merged in
// shared memory, splits through a scratch buffer by the last CTA to finish
// (an atomic counter per (sequence, KV head) that it resets for the next use).
#include <cuda_runtime.h>
#include <math.h>

#include "common.cuh"
#include "kernels.h"

namespace nx {

template <int VEC>
__device__ __forceinline__ void load_f32(const float *p, float (&v)[VEC]) {
    if constexpr (VEC == 4) {
        float4 t = *reinterpret_cast<const float4 *>(p);
        v[0] = t.x; v[1] = t.y; v[2] = t.z; v[3] = t.w;
    } else if constexpr (VEC == 2) {
        float2 t = *reinterpret_cast<const float2 *>(p);
        v[0] = t.x; v[1] = t.y;
    } else {
#pragma unroll
        for (int i = 0; i < VEC; i++) v[i] = p[i];
    }
}

// VEC values of `bits` bits starting at element e0 of a packed token row.
template <int VEC>
__device__ __forceinline__ void load_packed(const uint8_t *row, int e0, int bits, float mn, float sc,
                                            float (&v)[VEC]) {
    const unsigned mask = (1u << bits) - 1u;
#pragma unroll
    for (int i = 0; i < VEC; i++) {
        const int bit = (e0 + i) * bits;
        const unsigned lo = row[bit >> 3], hi = row[(bit >> 3) + 1];
        const unsigned q = ((lo | (hi << 8)) >> (bit & 7)) & mask;
        // min + q * scale, each rounded once (value_at, src/engine/mod.rs:255)
        v[i] = __fadd_rn(mn, __fmul_rn((float)q, sc));
    }
}

template <int VEC, int G>
__global__ void __launch_bounds__(128) k_attn(AttnParams p) {
    constexpr int D = VEC * 32;
    constexpr int NW = 4;
    const int h = blockIdx.x, split = blockIdx.y, t = blockIdx.z;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __shared__ float sm_m[NW][G], sm_l[NW][G];
    __shared__ float sm_o[NW][G][D];
    __shared__ bool is_last;

    if (p.pdl) {
        pdl_launch_dependents();
        pdl_wait();
    }
    const DevSeq sq = p.seqs[t];
    const uint32_t sid = p.seq_ids[t];
    const int seq_len = (int)sq.seq_len;
    const int per = (seq_len + p.nsplit - 1) / p.nsplit;
    const int t0 = split * per, t1 = min(seq_len, t0 + per);

    float qv[G][VEC];
#pragma unroll
    for (int g = 0; g < G; g++)
        load_f32<VEC>(p.q + (size_t)t * p.hq * D + (size_t)(h * G + g) * D + lane * VEC, qv[g]);
    float m[G], l[G], o[G][VEC];
#pragma unroll
    for (int g = 0; g < G; g++) {
        m[g] = -INFINITY;
        l[g] = 0.0f;
#pragma unroll
        for (int i = 0; i < VEC; i++) o[g][i] = 0.0f;
    }

    const bool packed = p.bits_k > 0;
    for (int tok = t0 + warp; tok < t1; tok += NW) {
        float kv[VEC], vv[VEC];
        const int e0 = h * D + lane * VEC;
        if (!packed) {
            const size_t off = (size_t)sid * p.seq_stride + (size_t)tok * p.kv_dim + e0;
            load_f32<VEC>(p.k_cache + off, kv);
            load_f32<VEC>(p.v_cache + off, vv);
        } else {
            const size_t mi = (size_t)sid * p.pk_seq_tokens + tok;
            load_packed<VEC>(p.kp_data + (size_t)sid * p.pk_seq_stride_k + (size_t)tok * p.pk_bpt_k, e0,
                             p.bits_k, p.kp_min[mi], p.kp_scale[mi], kv);
            load_packed<VEC>(p.vp_data + (size_t)sid * p.pk_seq_stride_v + (size_t)tok * p.pk_bpt_v, e0,
                             p.bits_v, p.vp_min[mi], p.vp_scale[mi], vv);
        }
        float dot[G];
#pragma unroll
        for (int g = 0; g < G; g++) {
            float s = 0.0f;
#pragma unroll
            for (int i = 0; i < VEC; i++) s += qv[g][i] * kv[i];
            dot[g] = s;
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1)
#pragma unroll
            for (int g = 0; g < G; g++) dot[g] += __shfl_xor_sync(0xffffffffu, dot[g], off);
#pragma unroll
        for (int g = 0; g < G; g++) {
            const float s = dot[g] * p.scale;
            const float mn = fmaxf(m[g], s);
            const float corr = expf(m[g] - mn);
            const float pe = expf(s - mn);
            l[g] = l[g] * corr + pe;
#pragma unroll
            for (int i = 0; i < VEC; i++) o[g][i] = o[g][i] * corr + pe * vv[i];
            m[g] = mn;
        }
    }

    // merge the warps of this CTA
#pragma unroll
    for (int g = 0; g < G; g++) {
        if (lane == 0) {
            sm_m[warp][g] = m[g];
            sm_l[warp][g] = l[g];
        }
#pragma unroll
        for (int i = 0; i < VEC; i++) sm_o[warp][g][lane * VEC + i] = o[g][i];
    }
    __syncthreads();
    const int stride = D + 2;
    float *part = p.part + (((size_t)t * p.hkv + h) * p.nsplit) * G * stride;
    for (int idx = threadIdx.x; idx < G * D; idx += blockDim.x) {
        const int g = idx / D, d = idx % D;
        float M = -INFINITY;
        for (int w = 0; w < NW; w++) M = fmaxf(M, sm_m[w][g]);
        float L = 0.0f, O = 0.0f;
        for (int w = 0; w < NW; w++) {
            const float wt = sm_m[w][g] == -INFINITY ? 0.0f : expf(sm_m[w][g] - M);
            L += wt * sm_l[w][g];
            O += wt * sm_o[w][g][d];
        }
        float *ps = part + ((size_t)split * G + g) * stride;
        ps[d] = O;
        if (d == 0) {
            ps[D] = M;
            ps[D + 1] = L;
        }
    }
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
        unsigned *ctr = p.counters + (size_t)t * p.hkv + h;
        const unsigned prev = atomicAdd(ctr, 1u);
        is_last = prev == (unsigned)(p.nsplit - 1);
        if (is_last) *ctr = 0u;
    }
    __syncthreads();
    if (!is_last) return;
    __threadfence();
    for (int idx = threadIdx.x; idx < G * D; idx += blockDim.x) {
        const int g = idx / D, d = idx % D;
        float M = -INFINITY;
        for (int s = 0; s < p.nsplit; s++) M = fmaxf(M, __ldcg(part + ((size_t)s * G + g) * stride + D));
        float L = 0.0f, O = 0.0f;
        for (int s = 0; s < p.nsplit; s++) {
            const float *ps = part + ((size_t)s * G + g) * stride;
            const float ms = __ldcg(ps + D);
            const float wt = ms == -INFINITY ? 0.0f : expf(ms - M);
            L += wt * __ldcg(ps + D + 1);
            O += wt * __ldcg(ps + d);
        }
        // a head whose softmax sum is not positive stays zero (src/engine/mod.rs:483-485)
        p.out[(size_t)t * p.hq * D + (size_t)(h * G + g) * D + d] = L > 0.0f ? O / L : 0.0f;
    }
}

template <int VEC, int G>
static cudaError_t launch_attn_t(const AttnParams &p, cudaStream_t st) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(p.hkv, p.nsplit, p.m);
    cfg.blockDim = dim3(128);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = p.pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, k_attn<VEC, G>, p);
}

template <int VEC>
static cudaError_t launch_attn_g(const AttnParams &p, cudaStream_t st) {
    switch (p.hq / p.hkv) {
    case 1: return launch_attn_t<VEC, 1>(p, st);
    case 2: return launch_attn_t<VEC, 2>(p, st);
    case 4: return launch_attn_t<VEC, 4>(p, st);
    case 8: return launch_attn_t<VEC, 8>(p, st);
    default: return cudaErrorInvalidValue;
    }
}

cudaError_t launch_attention(const AttnParams &p, cudaStream_t st) {
    if (p.hkv <= 0 || p.hq % p.hkv != 0) return cudaErrorInvalidValue;
    switch (p.head_dim) {
    case 32: return launch_attn_g<1>(p, st);
    case 64: return launch_attn_g<2>(p, st);
    case 128: return launch_attn_g<4>(p, st);
    default: return cudaErrorInvalidValue;
    }
}

}  // namespace nx
