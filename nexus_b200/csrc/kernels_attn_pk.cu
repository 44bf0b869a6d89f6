// kernels_attn_pk.cu -- GQA decode attention over the packed KV cache on the
// tensor cores (head_dim 128).
//
// Same result as KvCache::attention_decode over KvCacheBuffer::Quantized
// (src/engine/mod.rs:452-499): value = min_t + q * scale_t per element
// (PackedKvBuffer::value_at, src/engine/mod.rs:252-256), s_t = (q . k_t) *
// score_scale, o = sum_t softmax(s)_t * v_t.  The packed codes are never
// expanded to floats one element at a time; the affine form is split off:
//
//   q . k_t = min_t * sum(q) + scale_t * sum_d q_d * code_{t,d}
//   o_d     = sum_t p_t * min_t + sum_t (p_t * scale_t) * code_{t,d}
//
// Scores.  sum_d q_d * code_{t,d} is an exact integer product: q (per head)
// is rounded to a 20-bit integer at a power-of-two scale and split into three
// signed 7-bit digits; the codes are the unsigned bytes mask-extracted from
// the packed words.  One mma.m16n8k32 (u8 x s8 -> s32) covers 16 tokens x 32
// dims x 8 columns (4 heads x the two high digits, then the low digit), so
// the integer sums are exact and only the final recombination rounds.
//
// Values.  mma.m16n8k16 (f16 x f16 -> f32) with A = the codes of a 16-dim x
// 16-token block as exact f16 integers (f * code: byte permutes and masks
// place the code in the mantissa of 1024, one f16x2 subtract removes the
// 1024) and B = the per-token weights p_t * scale_t split into f16 hi + lo
// (22 significant bits).  The weights are kept relative to their own running
// maximum (of log2 p_t + log2 scale_t), so they stay in f16 range whatever the
// scales.
//
// Layout: grid (Hkv, slices, batch), 4 warps.  A warp owns a tile of 32
// tokens of one KV head at a time and all G query
// heads sharing it; lane (g, c) = (lane / 4, lane % 4) holds, per 16-token
// block, tokens g and g + 8 of head c's scores and dims 16g .. 16g+15 of head
// c's output.  Tiles reach shared memory by cp.async into two stages per warp,
// the next tile's copies issued before the current tile's math.  Warps and
// slices merge as in the float kernel (partials + the last slice to finish,
// deterministic order).
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <math.h>

#include "common.cuh"
#include "kernels.h"

namespace nx {
namespace {

constexpr int kPkWarps = 4;
constexpr int kPkD = 128;
constexpr float kLog2e = 1.4426950408889634f;

__device__ __forceinline__ void mma_u8s8(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void mma_f16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                        uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// four 8x8 b16 matrices, transposed: lane l gives the row address of matrix
// l / 8, row l % 8
__device__ __forceinline__ void ldsm_x4_trans(uint32_t (&r)[4], const void *row) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(smem_u32(row))
                 : "memory");
}

// bits of the little-endian word array w starting at bit `pos`, moved to bit 0
// (upper bits not masked); pos is a compile-time constant after unrolling
template <int NW>
__device__ __forceinline__ uint32_t bits_at(const uint32_t (&w)[NW], int pos) {
    const int i = pos >> 5, s = pos & 31;
    if (s == 0) return w[i];
    if (i + 1 < NW) return __funnelshift_r(w[i], w[i + 1], s);
    return w[i] >> s;
}

// ---- K codes: the lane's 32 dims (c*32 .. c*32+31 of the head) of one token
// are 4*BK bytes = BK words.  kfrag(j, half) is the A register of k32-chunk j
// for k = 4c..4c+3 (half 0) or 4c+16..4c+19 (half 1): four code bytes whose
// dims (within the lane's 32) are kdim(j, half, 0..3).
template <int BK>
__device__ __forceinline__ uint32_t kfrag(const uint32_t (&w)[BK], int j, int half) {
    if constexpr (BK == 4) {
        return half ? (w[j] >> 4) & 0x0F0F0F0Fu : w[j] & 0x0F0F0F0Fu;
    } else if constexpr (BK == 8) {
        return w[2 * j + half];
    } else if constexpr (BK == 2) {
        return (w[j >> 1] >> (2 * (2 * (j & 1) + half))) & 0x03030303u;
    } else {
        constexpr uint32_t mask = (1u << BK) - 1u;
        uint32_t r = 0;
#pragma unroll
        for (int i = 0; i < 4; i++) r |= (bits_at<BK>(w, (8 * j + 4 * half + i) * BK) & mask) << (8 * i);
        return r;
    }
}
template <int BK>
__device__ __forceinline__ constexpr int kdim(int j, int half, int i) {
    return BK == 4 ? 8 * j + 2 * i + half : BK == 2 ? 16 * (j >> 1) + 4 * i + 2 * (j & 1) + half : 8 * j + 4 * half + i;
}

// ---- V codes: the lane's 16 dims (g*16 .. g*16+15 of the head) of one token
// are 2*BV bytes, held in (BV+1)/2 words.  vfrag(a, b, d) is an f16x2
// register with token a's code of dim d in the low half and token b's in the
// high half, as vfactor(d) * code (exact in f16).
template <int BV>
__device__ __forceinline__ constexpr int vwords() { return (BV + 1) / 2; }

__device__ __forceinline__ uint32_t pair_bytes(uint32_t a, uint32_t b, int byte) {
    // [a.byte, a.byte, b.byte, b.byte]
    const uint32_t sel = (uint32_t)byte | ((uint32_t)byte << 4) | ((uint32_t)(byte + 4) << 8) | ((uint32_t)(byte + 4) << 12);
    return __byte_perm(a, b, sel);
}

// (1024 + x) - 1024 in both halves, exact for the integers x < 1024 here
__device__ __forceinline__ uint32_t unbias(uint32_t r) {
    uint32_t out;
    asm("sub.f16x2 %0, %1, %2;" : "=r"(out) : "r"(r), "r"(0x64006400u));
    return out;
}

template <int BV>
__device__ __forceinline__ uint32_t vfrag(const uint32_t (&a)[vwords<BV>()], const uint32_t (&b)[vwords<BV>()], int d) {
    constexpr uint32_t magic = 0x64006400u;  // f16 1024 in both halves
    if constexpr (BV == 4) {
        const uint32_t z = pair_bytes(a[d >> 3], b[d >> 3], (d & 7) >> 1);
        return unbias((d & 1) ? ((z & 0x00F000F0u) | magic) : ((z & 0x000F000Fu) | magic));
    } else if constexpr (BV == 8) {
        const uint32_t z = pair_bytes(a[d >> 2], b[d >> 2], d & 3);
        return unbias((z & 0x00FF00FFu) | magic);
    } else if constexpr (BV == 2) {
        const uint32_t z = pair_bytes(a[0], b[0], d >> 2);
        const uint32_t m = 0x00030003u << (2 * (d & 3));
        return unbias((z & m) | magic);
    } else {
        constexpr uint32_t mask = (1u << BV) - 1u;
        const uint32_t lo = bits_at<vwords<BV>()>(a, d * BV) & mask;
        const uint32_t hi = bits_at<vwords<BV>()>(b, d * BV) & mask;
        return unbias(lo | (hi << 16) | magic);
    }
}
template <int BV>
__device__ __forceinline__ constexpr float vfactor(int d) {
    return BV == 4 ? ((d & 1) ? 16.0f : 1.0f) : BV == 2 ? (float)(1 << (2 * (d & 3))) : 1.0f;
}

__device__ __forceinline__ float pow2f(int e) { return __int_as_float((127 + e) << 23); }

// asynchronous global -> shared copies (no registers held while in flight)
__device__ __forceinline__ void cp_async16(void *dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async4(void *dst, const void *src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait1() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }

// Shared-memory row of tile token tt in the V buffer.  4-bit rows (64 B) are
// permuted so that the four tokens 2c+r (c = 0..3) one fragment load reads
// fall in both halves of the banks; 8-bit rows (128 B) XOR their 16-byte
// units with the token instead.
template <int BV>
__device__ __forceinline__ int vrow(int tt) { return BV == 4 ? tt ^ ((tt >> 1) & 1) : tt; }
template <int BV>
__device__ __forceinline__ int vunit(int tt, int u) { return BV == 8 ? u ^ (tt & 7) : u; }

// Per-warp tile buffers: K rows, V rows (16*bits bytes each), and the four
// per-token floats (kmin, kscale, vmin, vscale); two stages.
template <int BK, int BV, int TT>
struct PkTile {
    static constexpr int K = 0;
    static constexpr int V = K + TT * 16 * BK;
    static constexpr int MS = V + TT * 16 * BV;
    static constexpr int BYTES = MS + TT * 16;
};

// signed 7-bit digit k (0 = lowest) of qi = d2*2^14 + d1*2^7 + d0
__device__ __forceinline__ int qdigit(int qi, int k) {
    const int d0 = ((qi + 64) & 127) - 64;
    const int r1 = (qi - d0) >> 7;
    if (k == 0) return d0;
    const int d1 = ((r1 + 64) & 127) - 64;
    if (k == 1) return d1;
    return (r1 - d1) >> 7;
}

template <int BK, int BV, int NG>
__global__ void __launch_bounds__(kPkWarps * 32, NG == 1 ? 4 : 2) k_attn_pk(AttnParams p) {
    constexpr int D = kPkD, NW = kPkWarps, G = 4 * NG;  // G: heads per KV head, padded
    constexpr int MT = 2;                                // 16-token blocks per tile
    constexpr int TT = 16 * MT;
    constexpr int NVW = vwords<BV>();
    const int h = blockIdx.x, split = blockIdx.y, t = blockIdx.z;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int gq = lane >> 2, c = lane & 3;
    const int hq_real = p.hq / p.hkv;  // query heads of this KV head (1, 2, 4 or 8)

    __shared__ float sQ[G][D];
    __shared__ float sQa[G], sQb[G];
    __shared__ int sE[G];
    __shared__ __align__(16) uint32_t sP[NW][NG][TT][4];  // per token: 8 f16 columns (head hi, lo)
    __shared__ float sO[NW][G][D];
    __shared__ float sM[NW][G], sL[NW][G];
    __shared__ float sw[64][G], sls[64][G], sMg[G], sLg[G];
    __shared__ bool is_last;

    if (p.pdl) {
        pdl_launch_dependents();
        pdl_wait();
    }
    const DevSeq sq = p.seqs[t];
    const uint32_t sid = p.seq_ids[t];
    const int seq_len = (int)sq.seq_len;
    const int tiles = (seq_len + TT - 1) / TT;
    const int nsp0 = max(1, min(p.nsplit, (tiles + NW - 1) / NW));
    const int tps = (tiles + nsp0 - 1) / nsp0;
    const int nsp = (tiles + tps - 1) / tps;
    if (split >= nsp) return;
    const int t0 = split * tps * TT, t1 = min(seq_len, t0 + tps * TT);

    // ---- q: per head a power-of-two scale 2^e with max|q| * 2^e < 2^20, and sum(q)
    for (int i = threadIdx.x; i < G * D; i += blockDim.x) {
        const int g = i / D;
        sQ[g][i % D] = g < hq_real ? __ldcg(p.q + (size_t)t * p.hq * D + (size_t)(h * hq_real + g) * D + (i % D)) : 0.0f;
    }
    __syncthreads();
    const float sl2 = p.scale * kLog2e;
    for (int g = warp; g < G; g += NW) {
        float amax = 0.0f, sum = 0.0f;
#pragma unroll
        for (int i = 0; i < D / 32; i++) {
            const float v = sQ[g][lane + 32 * i];
            amax = fmaxf(amax, fabsf(v));
            sum += v;
        }
        for (int o = 16; o > 0; o >>= 1) {
            amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
            sum += __shfl_xor_sync(0xffffffffu, sum, o);
        }
        if (lane == 0) {
            const int eb = (__float_as_int(amax) >> 23) & 255;  // amax in [2^(eb-127), 2^(eb-126))
            const int e = eb == 0 ? 60 : max(-60, min(60, 20 - (eb - 126)));
            sE[g] = e;
            sQa[g] = sum * sl2;
            sQb[g] = pow2f(-e) * sl2;
        }
    }
    __syncthreads();

    // B registers of the score mma: column gq = head (gq >> 1) of group hg;
    // ntl 0 holds digits 2 (even gq) and 1 (odd gq), ntl 1 digit 0 (even gq)
    uint32_t qB[NG][2][4][2];
#pragma unroll
    for (int hg = 0; hg < NG; hg++) {
        const int g = 4 * hg + (gq >> 1);
        const float sc = pow2f(sE[g]);
#pragma unroll
        for (int ntl = 0; ntl < 2; ntl++) {
            const int dig = ntl == 0 ? ((gq & 1) ? 1 : 2) : ((gq & 1) ? -1 : 0);
#pragma unroll
            for (int j = 0; j < 4; j++)
#pragma unroll
                for (int half = 0; half < 2; half++) {
                    uint32_t r = 0;
                    if (dig >= 0) {
#pragma unroll
                        for (int i = 0; i < 4; i++) {
                            const int qi = __float2int_rn(sQ[g][32 * c + kdim<BK>(j, half, i)] * sc);
                            r |= ((uint32_t)qdigit(qi, dig) & 0xFFu) << (8 * i);
                        }
                    }
                    qB[hg][ntl][j][half] = r;
                }
        }
    }
    float qa[NG], qb[NG];
#pragma unroll
    for (int hg = 0; hg < NG; hg++) {
        qa[hg] = sQa[4 * hg + c];
        qb[hg] = sQb[4 * hg + c];
    }

    // ---- the warp's tiles
    float acc[NG][8][4];
    float m[NG], mp[NG], L[NG], MN[NG];
#pragma unroll
    for (int hg = 0; hg < NG; hg++) {
        m[hg] = mp[hg] = -INFINITY;
        L[hg] = MN[hg] = 0.0f;
#pragma unroll
        for (int i = 0; i < 8; i++)
#pragma unroll
            for (int r = 0; r < 4; r++) acc[hg][i][r] = 0.0f;
    }
    // the KV head's segment of every physical slot; tokens map to slots through the page table
    const uint8_t *kseq = p.kp_data + (size_t)h * (16 * BK);
    const uint8_t *vseq = p.vp_data + (size_t)h * (16 * BV);
    using TL = PkTile<BK, BV, TT>;
    extern __shared__ __align__(16) uint8_t pk_dyn[];
    uint8_t *wbuf = pk_dyn + (size_t)warp * 2 * TL::BYTES;
    // copies of the tile at `base` into stage st: the KV head's row segment of
    // every token (tokens past the slice repeat its last one) and min/scale
    auto issue = [&](int base, int st) {
        uint8_t *b = wbuf + st * TL::BYTES;
#pragma unroll
        for (int i = 0; i < TT * BK / 32; i++) {
            const int ch = lane + 32 * i, tt = ch / BK, part = ch % BK;
            const size_t ph = kv_phys(p.pages, sid, (uint32_t)min(base + tt, t1 - 1));
            cp_async16(b + TL::K + tt * 16 * BK + part * 16, kseq + ph * p.pk_bpt_k + part * 16);
        }
#pragma unroll
        for (int i = 0; i < TT * BV / 32; i++) {
            const int ch = lane + 32 * i, tt = ch / BV, part = ch % BV;
            const size_t ph = kv_phys(p.pages, sid, (uint32_t)min(base + tt, t1 - 1));
            cp_async16(b + TL::V + vrow<BV>(tt) * 16 * BV + vunit<BV>(tt, part) * 16,
                       vseq + ph * p.pk_bpt_v + part * 16);
        }
#pragma unroll
        for (int i = 0; i < TT / 32; i++) {
            const int tt = lane + 32 * i;
            const size_t ph = kv_phys(p.pages, sid, (uint32_t)min(base + tt, t1 - 1));
            float *ms = reinterpret_cast<float *>(b + TL::MS) + 4 * tt;
            cp_async4(ms + 0, p.kp_min + ph);
            cp_async4(ms + 1, p.kp_scale + ph);
            cp_async4(ms + 2, p.vp_min + ph);
            cp_async4(ms + 3, p.vp_scale + ph);
        }
    };
    int base = t0 + warp * TT, st = 0;
    if (base < t1) issue(base, 0);
    cp_async_commit();
    for (; base < t1; base += NW * TT, st ^= 1) {
        // the next tile's copies go out before this tile's math
        if (base + NW * TT < t1) issue(base + NW * TT, st ^ 1);
        cp_async_commit();
        cp_async_wait1();
        __syncwarp();
        const uint8_t *tb = wbuf + st * TL::BYTES;
        const float4 *sMS = reinterpret_cast<const float4 *>(tb + TL::MS);
        uint32_t wk[MT][2][BK];
        uint32_t wv[MT][4][NVW];
#pragma unroll
        for (int mt = 0; mt < MT; mt++)
#pragma unroll
            for (int r = 0; r < 2; r++) {
                const uint32_t *src = reinterpret_cast<const uint32_t *>(tb + TL::K + (16 * mt + gq + 8 * r) * 16 * BK +
                                                                         c * 4 * BK);
#pragma unroll
                for (int i = 0; i < BK; i++) wk[mt][r][i] = src[i];
            }
#pragma unroll
        for (int kc = 0; kc < MT; kc++)
#pragma unroll
            for (int r = 0; r < 4; r++) {
                const int tt = 16 * kc + 2 * c + (r & 1) + 8 * (r >> 1);
                const int byte = gq * 2 * BV;  // the lane's 2*BV bytes inside the row
                const uint8_t *row = tb + TL::V + vrow<BV>(tt) * 16 * BV;
                if constexpr (BV == 8) {
                    const uint4 v = *reinterpret_cast<const uint4 *>(row + vunit<BV>(tt, gq) * 16);
                    wv[kc][r][0] = v.x; wv[kc][r][1] = v.y; wv[kc][r][2] = v.z; wv[kc][r][3] = v.w;
                } else if constexpr (BV == 4) {
                    const uint2 v = *reinterpret_cast<const uint2 *>(row + byte);
                    wv[kc][r][0] = v.x; wv[kc][r][1] = v.y;
                } else if constexpr (BV % 2 == 0) {
#pragma unroll
                    for (int i = 0; i < NVW; i++) wv[kc][r][i] = reinterpret_cast<const uint32_t *>(row + byte)[i];
                } else {
                    const uint16_t *hp = reinterpret_cast<const uint16_t *>(row + byte);
#pragma unroll
                    for (int i = 0; i < NVW; i++)
                        wv[kc][r][i] = (uint32_t)hp[2 * i] | (2 * i + 1 < BV ? (uint32_t)hp[2 * i + 1] << 16 : 0u);
                }
            }

        // scores: exact integer q . codes per (token, head)
        float s2[NG][MT][2], u2[NG][MT][2];
#pragma unroll
        for (int mt = 0; mt < MT; mt++) {
            const float4 ms0 = sMS[16 * mt + gq], ms1 = sMS[16 * mt + gq + 8];
#pragma unroll
            for (int hg = 0; hg < NG; hg++) {
                int ck[2][4] = {{0, 0, 0, 0}, {0, 0, 0, 0}};
#pragma unroll
                for (int ntl = 0; ntl < 2; ntl++)
#pragma unroll
                    for (int j = 0; j < 4; j++)
                        mma_u8s8(ck[ntl], kfrag<BK>(wk[mt][0], j, 0), kfrag<BK>(wk[mt][1], j, 0),
                                 kfrag<BK>(wk[mt][0], j, 1), kfrag<BK>(wk[mt][1], j, 1), qB[hg][ntl][j][0],
                                 qB[hg][ntl][j][1]);
                const bool valid = 4 * hg + c < hq_real;
#pragma unroll
                for (int r = 0; r < 2; r++) {
                    const float4 ms = r ? ms1 : ms0;
                    const float R = (float)ck[0][2 * r] * 16384.0f + (float)ck[0][2 * r + 1] * 128.0f + (float)ck[1][2 * r];
                    const bool ok = valid && base + 16 * mt + gq + 8 * r < t1;
                    const float s = fmaf(ms.x, qa[hg], ms.y * R * qb[hg]);
                    s2[hg][mt][r] = ok ? s : -INFINITY;
                    u2[hg][mt][r] = ok ? s + __log2f(ms.w) : -INFINITY;
                }
            }
        }

        // online softmax; the value weights P = 2^(u2 - mp) go to smem as f16 hi/lo
#pragma unroll
        for (int hg = 0; hg < NG; hg++) {
            float mx = -INFINITY, mu = -INFINITY;
#pragma unroll
            for (int mt = 0; mt < MT; mt++)
#pragma unroll
                for (int r = 0; r < 2; r++) {
                    mx = fmaxf(mx, s2[hg][mt][r]);
                    mu = fmaxf(mu, u2[hg][mt][r]);
                }
#pragma unroll
            for (int o = 4; o < 32; o <<= 1) {
                mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
                mu = fmaxf(mu, __shfl_xor_sync(0xffffffffu, mu, o));
            }
            const float mn_new = fmaxf(m[hg], mx), mp_new = fmaxf(mp[hg], mu);
            const float ms_ = mn_new == -INFINITY ? 0.0f : mn_new;
            const float mps = mp_new == -INFINITY ? 0.0f : mp_new;
            const float corr = exp2f(m[hg] - ms_), corrp = exp2f(mp[hg] - mps);
            m[hg] = mn_new;
            mp[hg] = mp_new;
            L[hg] *= corr;
            MN[hg] *= corr;
#pragma unroll
            for (int i = 0; i < 8; i++)
#pragma unroll
                for (int r = 0; r < 4; r++) acc[hg][i][r] *= corrp;
#pragma unroll
            for (int mt = 0; mt < MT; mt++)
#pragma unroll
                for (int r = 0; r < 2; r++) {
                    const int tt = 16 * mt + gq + 8 * r;
                    const float pe = exp2f(s2[hg][mt][r] - ms_);
                    L[hg] += pe;
                    MN[hg] = fmaf(pe, sMS[tt].z, MN[hg]);
                    const float P = exp2f(u2[hg][mt][r] - mps);
                    const __half hi = __float2half_rn(P);
                    const __half lo = __float2half_rn(P - __half2float(hi));
                    const __half2 pr = __halves2half2(hi, lo);
                    sP[warp][hg][tt][c] = *reinterpret_cast<const uint32_t *>(&pr);
                }
        }
        __syncwarp();

        // values: O^T[dim][column] += codes^T . P over the tile's tokens
#pragma unroll
        for (int kc2 = 0; kc2 < MT; kc2 += 2) {
            uint32_t bp[NG][4];
            const int q = lane >> 3, rr = lane & 7;
#pragma unroll
            for (int hg = 0; hg < NG; hg++)
                ldsm_x4_trans(bp[hg], &sP[warp][hg][16 * (kc2 + (q >> 1)) + 8 * (q & 1) + rr][0]);
#pragma unroll
            for (int kk = 0; kk < 2; kk++) {
                const int kc = kc2 + kk;
#pragma unroll
                for (int i = 0; i < 8; i++) {
                    const uint32_t a0 = vfrag<BV>(wv[kc][0], wv[kc][1], 2 * i);
                    const uint32_t a1 = vfrag<BV>(wv[kc][0], wv[kc][1], 2 * i + 1);
                    const uint32_t a2 = vfrag<BV>(wv[kc][2], wv[kc][3], 2 * i);
                    const uint32_t a3 = vfrag<BV>(wv[kc][2], wv[kc][3], 2 * i + 1);
#pragma unroll
                    for (int hg = 0; hg < NG; hg++)
                        mma_f16(acc[hg][i], a0, a1, a2, a3, bp[hg][2 * kk], bp[hg][2 * kk + 1]);
                }
            }
        }
        __syncwarp();
    }

    // ---- this warp's partial: per head (M, L, O[d]) with O relative to 2^M
#pragma unroll
    for (int hg = 0; hg < NG; hg++) {
        float l = L[hg], mn = MN[hg];
#pragma unroll
        for (int o = 4; o < 32; o <<= 1) {
            l += __shfl_xor_sync(0xffffffffu, l, o);
            mn += __shfl_xor_sync(0xffffffffu, mn, o);
        }
        const int g = 4 * hg + c;
        const float rel = m[hg] == -INFINITY ? 0.0f : exp2f(mp[hg] - m[hg]);
#pragma unroll
        for (int i = 0; i < 8; i++)
#pragma unroll
            for (int r = 0; r < 2; r++) {
                const int d = 2 * i + r;
                const float raw = acc[hg][i][2 * r] + acc[hg][i][2 * r + 1];
                const float accn = raw * (1.0f / vfactor<BV>(d));
                sO[warp][g][16 * gq + d] = fmaf(rel, accn, mn);
            }
        if (gq == 0) {
            sM[warp][g] = m[hg];
            sL[warp][g] = l;
        }
    }
    __syncthreads();

    // ---- merge the warps; one slice writes the result, several meet in partials
    const int stride = D + 2;
    float *part = p.part + (((size_t)t * p.hkv + h) * p.nsplit) * hq_real * stride;
    for (int idx = threadIdx.x; idx < hq_real * D; idx += blockDim.x) {
        const int g = idx / D, d = idx % D;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < NW; w++) M = fmaxf(M, sM[w][g]);
        float Ls = 0.0f, O = 0.0f;
#pragma unroll
        for (int w = 0; w < NW; w++) {
            const float wt = sM[w][g] == -INFINITY ? 0.0f : exp2f(sM[w][g] - M);
            Ls += wt * sL[w][g];
            O += wt * sO[w][g][d];
        }
        if (nsp == 1) {
            // a head whose softmax sum is not positive stays zero (src/engine/mod.rs:483-485)
            p.out[(size_t)t * p.hq * D + (size_t)(h * hq_real + g) * D + d] = Ls > 0.0f ? O / Ls : 0.0f;
        } else {
            float *ps = part + ((size_t)split * hq_real + g) * stride;
            ps[d] = O;
            if (d == 0) {
                ps[D] = M;
                ps[D + 1] = Ls;
            }
        }
    }
    if (nsp == 1) return;
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
        unsigned *ctr = p.counters + (size_t)t * p.hkv + h;
        const unsigned prev = atomicAdd(ctr, 1u);
        is_last = prev == (unsigned)(nsp - 1);
        if (is_last) *ctr = 0u;
    }
    __syncthreads();
    if (!is_last) return;
    __threadfence();
    for (int idx = threadIdx.x; idx < nsp * hq_real; idx += blockDim.x) {
        const int s = idx / hq_real, g = idx % hq_real;
        sw[s][g] = __ldcg(part + ((size_t)s * hq_real + g) * stride + D);
        sls[s][g] = __ldcg(part + ((size_t)s * hq_real + g) * stride + D + 1);
    }
    __syncthreads();
    if (threadIdx.x < hq_real) {
        const int g = threadIdx.x;
        float M = -INFINITY;
        for (int s = 0; s < nsp; s++) M = fmaxf(M, sw[s][g]);
        float Ls = 0.0f;
        for (int s = 0; s < nsp; s++) {
            const float wt = sw[s][g] == -INFINITY ? 0.0f : exp2f(sw[s][g] - M);
            Ls += wt * sls[s][g];
            sw[s][g] = wt;
        }
        sMg[g] = M;
        sLg[g] = Ls;
    }
    __syncthreads();
    for (int idx = threadIdx.x; idx < hq_real * D; idx += blockDim.x) {
        const int g = idx / D, d = idx % D;
        float O = 0.0f;
        for (int s = 0; s < nsp; s++) O += sw[s][g] * __ldcg(part + ((size_t)s * hq_real + g) * stride + d);
        const float Ls = sLg[g];
        p.out[(size_t)t * p.hq * D + (size_t)(h * hq_real + g) * D + d] = Ls > 0.0f ? O / Ls : 0.0f;
    }
}

template <int BK, int BV, int NG>
cudaError_t launch_pk_t(const AttnParams &p, cudaStream_t st) {
    constexpr int TT = 32;
    constexpr int smem = kPkWarps * 2 * PkTile<BK, BV, TT>::BYTES;
    auto fn = k_attn_pk<BK, BV, NG>;
    cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(p.hkv, p.nsplit, p.m);
    cfg.blockDim = dim3(kPkWarps * 32);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = p.pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, fn, p);
}

template <int BK, int BV>
cudaError_t launch_pk_g(const AttnParams &p, cudaStream_t st) {
    return p.hq / p.hkv > 4 ? launch_pk_t<BK, BV, 2>(p, st) : launch_pk_t<BK, BV, 1>(p, st);
}

template <int BK>
cudaError_t launch_pk_v(const AttnParams &p, cudaStream_t st) {
    switch (p.bits_v) {
    case 2: return launch_pk_g<BK, 2>(p, st);
    case 3: return launch_pk_g<BK, 3>(p, st);
    case 4: return launch_pk_g<BK, 4>(p, st);
    case 6: return launch_pk_g<BK, 6>(p, st);
    case 8: return launch_pk_g<BK, 8>(p, st);
    }
    return cudaErrorInvalidValue;
}

bool bits_ok(int b) { return b == 2 || b == 3 || b == 4 || b == 6 || b == 8; }

}  // namespace

bool attention_pk_supported(const AttnParams &p) {
    const int G = p.hkv > 0 ? p.hq / p.hkv : 0;
    return p.head_dim == kPkD && (G == 1 || G == 2 || G == 4 || G == 8) && p.hq == G * p.hkv && bits_ok(p.bits_k) &&
           bits_ok(p.bits_v) && p.nsplit <= 64;
}

cudaError_t launch_attention_pk(const AttnParams &p, cudaStream_t st) {
    switch (p.bits_k) {
    case 2: return launch_pk_v<2>(p, st);
    case 3: return launch_pk_v<3>(p, st);
    case 4: return launch_pk_v<4>(p, st);
    case 6: return launch_pk_v<6>(p, st);
    case 8: return launch_pk_v<8>(p, st);
    }
    return cudaErrorInvalidValue;
}

}  // namespace nx
