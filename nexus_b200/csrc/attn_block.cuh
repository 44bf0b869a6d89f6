#pragma once
// attn_block.cuh -- one (KV head, context slice, token) block of GQA decode
// attention, shared by the standalone attention kernel (kernels_attn.cu) and
// the persistent decode-step kernel (kernels_step.cu).
//
// Replaces KvCache::attention_decode (src/engine/mod.rs:452-499): for query
// head qh, kv head kvh = qh / (Hq/Hkv); s_t = (q . k_t) * (1/sqrt(D));
// o = sum_t softmax(s)_t * v_t.  Packed caches are read directly in their
// low-bit form: value = min_t + q * scale_t (PackedKvBuffer::value_at,
// src/engine/mod.rs:252-256), one (min, scale) per token across all KV heads.
//
// A block owns one KV head, a contiguous slice of at least TPS tokens of the
// context, and all G query heads sharing that KV head, so every K/V element
// is read from HBM once.  NW warps stride over the slice; each warp issues the
// loads of kBatch tokens before using any of them (one memory round trip per
// batch); lane i holds head_dim/32 dims of each row.  Warps keep an online
// softmax per query head and are merged in shared memory; slices are merged
// by the last block to finish (an atomic counter per (sequence, KV head),
// reset by that block).  All shared memory comes from the caller (AttnSmem).
#include <cuda_runtime.h>
#include <math.h>

#include "common.cuh"
#include "kernels.h"

namespace nx {

constexpr int kBatch = 8;

template <int VEC, int G, int NW>
struct AttnSmem {
    float m[NW][G], l[NW][G];
    float o[NW][G][VEC * 32];
    float w[64][G];
    float p[NW][kBatch][G], c[NW][G];
    float M[G], L[G];
    float ls[64][G];
    int is_last;
};

template <int VEC>
__device__ __forceinline__ void load_f32(const float *p, float (&v)[VEC]) {
    if constexpr (VEC == 4) {
        float4 t = __ldcg(reinterpret_cast<const float4 *>(p));
        v[0] = t.x; v[1] = t.y; v[2] = t.z; v[3] = t.w;
    } else if constexpr (VEC == 2) {
        float2 t = __ldcg(reinterpret_cast<const float2 *>(p));
        v[0] = t.x; v[1] = t.y;
    } else {
#pragma unroll
        for (int i = 0; i < VEC; i++) v[i] = __ldcg(p + i);
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

template <int TPS>
__device__ __forceinline__ int active_splits(int seq_len, int nsplit_grid) {
    int s = (seq_len + TPS - 1) / TPS;
    return max(1, min(s, nsplit_grid));
}

// Completes NV partial sums spread over the warp with one transpose-reduce:
// at each xor step a lane keeps the half of its values that its lane bit
// selects and adds the partner's copy of that half (31 shuffles for 32
// values instead of 160).  Afterwards value i is complete in lane i >> 1 as
// element i & 1 (NV = 64), in lane i (NV = 32), or in lanes
// i << s .. (i << s) + 2^s - 1 (NV = 32 >> s, all holding the same sum).
template <int NV>
__device__ __forceinline__ void transpose_reduce(float (&v)[NV], int lane) {
#pragma unroll
    for (int step = 0; step < 5; step++) {
        const int o = 16 >> step;
        const int n = NV >> step;  // values per lane before this step
        if (n >= 2) {
            const bool up = (lane & o) != 0;
#pragma unroll
            for (int i = 0; i < n / 2; i++) {
                const float keep = up ? v[n / 2 + i] : v[i];
                const float send = up ? v[i] : v[n / 2 + i];
                v[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
            }
        } else {
            v[0] += __shfl_xor_sync(0xffffffffu, v[0], o);
        }
    }
}

template <int VEC, int G, int NW, int TPS>
__device__ __forceinline__ void attn_block(const AttnParams &p, int h, int split, int t,
                                           AttnSmem<VEC, G, NW> &sm) {
    constexpr int D = VEC * 32;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    auto &sm_m = sm.m;
    auto &sm_l = sm.l;
    auto &sm_o = sm.o;
    auto &sm_w = sm.w;
    auto &sm_p = sm.p;
    auto &sm_c = sm.c;
    auto &sm_M = sm.M;
    auto &sm_L = sm.L;
    auto &sm_ls = sm.ls;
    // q and the step descriptor are independent loads: issue both first
    float qv[G][VEC];
#pragma unroll
    for (int g = 0; g < G; g++)
        load_f32<VEC>(p.q + (size_t)t * p.hq * D + (size_t)(h * G + g) * D + lane * VEC, qv[g]);
    const DevSeq sq = p.seqs[t];
    const uint32_t sid = p.seq_ids[t];
    const int seq_len = (int)sq.seq_len;
    const int nsplit = active_splits<TPS>(seq_len, p.nsplit);
    if (split >= nsplit) return;
    const int per = (seq_len + nsplit - 1) / nsplit;
    const int t0 = split * per, t1 = min(seq_len, t0 + per);
    // After the batch's dot products are reduced, lane `lane` holds R of its
    // kBatch x G scores (token j, head g): index lane * R + r when there are
    // 32 or more, else lane >> SH, repeated in 2^SH lanes of which the first
    // ("lead") carries it.  Every lane keeps the running maximum of the
    // head(s) it holds and its lead share of that head's softmax sum; the
    // batch's weights and rescale factors meet in shared memory.
    constexpr int NV = kBatch * G;
    constexpr int R = NV >= 32 ? NV / 32 : 1;
    constexpr int SH = NV >= 32 ? 0 : (NV == 16 ? 1 : NV == 8 ? 2 : NV == 4 ? 3 : 4);
    const bool lead = (lane & ((1 << SH) - 1)) == 0;
    float ml[R], ll[R], o[G][VEC];
#pragma unroll
    for (int r = 0; r < R; r++) {
        ml[r] = -INFINITY;
        ll[r] = 0.0f;
    }
#pragma unroll
    for (int g = 0; g < G; g++)
#pragma unroll
        for (int i = 0; i < VEC; i++) o[g][i] = 0.0f;

    const bool packed = p.bits_k > 0;
    const int e0 = h * D + lane * VEC;
    for (int base = t0 + warp * kBatch; base < t1; base += NW * kBatch) {
        float kv[kBatch][VEC], vv[kBatch][VEC];
        // issue every load of the batch first
#pragma unroll
        for (int j = 0; j < kBatch; j++) {
            const int tok = min(base + j, t1 - 1);
            const size_t ph = kv_phys(p.pages, sid, (uint32_t)tok);
            if (!packed) {
                const size_t off = ph * p.kv_dim + e0;
                load_f32<VEC>(p.k_cache + off, kv[j]);
                load_f32<VEC>(p.v_cache + off, vv[j]);
            } else {
                load_packed<VEC>(p.kp_data + ph * p.pk_bpt_k, e0, p.bits_k, p.kp_min[ph], p.kp_scale[ph], kv[j]);
                load_packed<VEC>(p.vp_data + ph * p.pk_bpt_v, e0, p.bits_v, p.vp_min[ph], p.vp_scale[ph], vv[j]);
            }
        }
        float pd[NV];
#pragma unroll
        for (int j = 0; j < kBatch; j++)
#pragma unroll
            for (int g = 0; g < G; g++) {
                float s = 0.0f;
#pragma unroll
                for (int i = 0; i < VEC; i++) s += qv[g][i] * kv[j][i];
                pd[j * G + g] = s;
            }
        transpose_reduce<NV>(pd, lane);
#pragma unroll
        for (int r = 0; r < R; r++) {
            const int idx = NV >= 32 ? lane * R + r : lane >> SH;
            const int j = idx / G, g = idx % G;
            const float s = base + j < t1 ? pd[r] * p.scale : -INFINITY;
            // the lanes of one head differ in lane bits 2..4 (token j)
            float mx = s;
#pragma unroll
            for (int off = 4; off < 32; off <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
            const float mn = fmaxf(ml[r], mx);  // finite: token base is valid
            const float corr = expf(ml[r] - mn);
            const float pe = expf(s - mn);
            ml[r] = mn;
            ll[r] = ll[r] * corr + (lead ? pe : 0.0f);
            if (lead) {
                sm_p[warp][j][g] = pe;
                if (j == 0) sm_c[warp][g] = corr;
            }
        }
        __syncwarp();
#pragma unroll
        for (int g = 0; g < G; g++) {
            const float c = sm_c[warp][g];
#pragma unroll
            for (int i = 0; i < VEC; i++) o[g][i] *= c;
        }
#pragma unroll
        for (int j = 0; j < kBatch; j++)
#pragma unroll
            for (int g = 0; g < G; g++) {
                const float pe = sm_p[warp][j][g];
#pragma unroll
                for (int i = 0; i < VEC; i++) o[g][i] = fmaf(pe, vv[j][i], o[g][i]);
            }
        __syncwarp();
    }

    // merge the warps of this CTA
#pragma unroll
    for (int r = 0; r < R; r++) {
        float l = ll[r];
#pragma unroll
        for (int off = 4; off < 32; off <<= 1) l += __shfl_xor_sync(0xffffffffu, l, off);
        const int idx = NV >= 32 ? lane * R + r : lane >> SH;
        if (lead && idx < G) {
            sm_m[warp][idx] = ml[r];
            sm_l[warp][idx] = l;
        }
    }
#pragma unroll
    for (int g = 0; g < G; g++)
#pragma unroll
        for (int i = 0; i < VEC; i++) sm_o[warp][g][lane * VEC + i] = o[g][i];
    __syncthreads();
    if (nsplit == 1) {
        // the whole context is this CTA's slice: normalize and write directly
        for (int idx = threadIdx.x; idx < G * D; idx += blockDim.x) {
            const int g = idx / D, d = idx % D;
            float M = -INFINITY;
#pragma unroll
            for (int w = 0; w < NW; w++) M = fmaxf(M, sm_m[w][g]);
            float L = 0.0f, O = 0.0f;
#pragma unroll
            for (int w = 0; w < NW; w++) {
                const float wt = sm_m[w][g] == -INFINITY ? 0.0f : expf(sm_m[w][g] - M);
                L += wt * sm_l[w][g];
                O += wt * sm_o[w][g][d];
            }
            p.out[(size_t)t * p.hq * D + (size_t)(h * G + g) * D + d] = L > 0.0f ? O / L : 0.0f;
        }
        return;
    }
    const int stride = D + 2;
    float *part = p.part + (((size_t)t * p.hkv + h) * p.nsplit) * G * stride;
    for (int idx = threadIdx.x; idx < G * D; idx += blockDim.x) {
        const int g = idx / D, d = idx % D;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < NW; w++) M = fmaxf(M, sm_m[w][g]);
        float L = 0.0f, O = 0.0f;
#pragma unroll
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
        sm.is_last = prev == (unsigned)(nsplit - 1);
        if (sm.is_last) *ctr = 0u;
    }
    __syncthreads();
    if (!sm.is_last) return;
    __threadfence();
    // slice merge: maxima and sums of every (slice, head) in parallel ...
    for (int idx = threadIdx.x; idx < nsplit * G; idx += blockDim.x) {
        const int s = idx / G, g = idx % G;
        sm_w[s][g] = __ldcg(part + ((size_t)s * G + g) * stride + D);
        sm_ls[s][g] = __ldcg(part + ((size_t)s * G + g) * stride + D + 1);
    }
    __syncthreads();
    if (threadIdx.x < G) {
        const int g = threadIdx.x;
        float M = -INFINITY;
        for (int s = 0; s < nsplit; s++) M = fmaxf(M, sm_w[s][g]);
        float L = 0.0f;
        for (int s = 0; s < nsplit; s++) {
            const float ms = sm_w[s][g];
            const float wt = ms == -INFINITY ? 0.0f : expf(ms - M);
            L += wt * sm_ls[s][g];
            sm_w[s][g] = wt;
        }
        sm_M[g] = M;
        sm_L[g] = L;
    }
    __syncthreads();
    // ... then every output element from independent loads
    for (int idx = threadIdx.x; idx < G * D; idx += blockDim.x) {
        const int g = idx / D, d = idx % D;
        float O = 0.0f;
#pragma unroll 8
        for (int s = 0; s < nsplit; s++) O += sm_w[s][g] * __ldcg(part + ((size_t)s * G + g) * stride + d);
        const float L = sm_L[g];
        // a head whose softmax sum is not positive stays zero (src/engine/mod.rs:483-485)
        p.out[(size_t)t * p.hq * D + (size_t)(h * G + g) * D + d] = L > 0.0f ? O / L : 0.0f;
    }
}


}  // namespace nx
