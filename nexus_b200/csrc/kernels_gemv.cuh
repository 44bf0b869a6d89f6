#pragma once
// kernels_gemv.cuh -- dequant-fused GEMV for decode (m <= 4 tokens per pass).
//
// Replaces InferenceEngine::matvec (src/engine/mod.rs:775-801), which the
// reference runs on weights dequantized to f32 at load.  Here the weights stay
// in their block format in HBM (row-interleaved tiles, tiles.cuh) and are
// decoded in registers.
//
// Arithmetic.  Each token's input vector is re-expressed, per 256-element
// super-block s, as x_i ~= u_s * z_i with z_i a 16-bit integer
// (u_s = max|x|/32767), split as z = 256*h + l (h signed, l unsigned byte).
// A weight element of every supported format is (scale)*(small integer q) -
// (offset), so each super-block's contribution is
//     u_s * ( d * sum_j sc_j * sum_{i in j} q_i z_i  -  dmin * sum_j m_j * sum_{i in j} z_i )
// where the inner sums are exact 32-bit integer dot products (dp4a on four
// bytes at a time).  The only rounding beyond f32 accumulation is the 16-bit
// representation of x (|error| <= max|x|/65534 per super-block), which keeps
// per-output relative error near 1e-5, far inside the 1e-3 parity bound.
//
// Parallel layout.  One CTA per row group of 32 rows; lane i of every warp
// owns row 32g+i; the CTA's warps split the super-blocks and reduce through
// shared memory in a fixed order (deterministic).  Input preparation (optional
// RMSNorm, quantization of x) is done by each warp for its own super-blocks.
// Weight loads for the first super-block are issued before griddepcontrol.wait,
// so under programmatic dependent launch they overlap the previous kernel.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "common.cuh"
#include "kernels.h"
#include "tiles.cuh"

namespace nx {

template <int FMT>
struct Fmt;
template <>
struct Fmt<12> { static constexpr int C = 9; static constexpr bool AUX = false; };   // Q4_K
template <>
struct Fmt<2> { static constexpr int C = 9; static constexpr bool AUX = false; };    // Q4_0
template <>
struct Fmt<8> { static constexpr int C = 17; static constexpr bool AUX = false; };   // Q8_0
template <>
struct Fmt<10> { static constexpr int C = 5; static constexpr bool AUX = true; };    // Q2_K

// x of one token for one super-block, in shared memory
struct XSb {
    const uint4 *zh;  // 16 x uint4: signed high bytes of z for 256 elements
    const uint4 *zl;  // 16 x uint4: unsigned low bytes
    const int *sz;    // 16 ints: sum of z over each 16-element group
    float u;
};

__device__ __forceinline__ uint32_t byte_of(uint32_t w, int j) { return (w >> (8 * j)) & 0xffu; }

// Q4_K super-block (tiles.cuh): c[0] = d|dmin, scales; c[1..8] = qs
__device__ __forceinline__ float sb_dot_q4k(const uint4 *c, const XSb &x) {
    const uint32_t h0 = c[0].x;
    const float d = h2f_bits(h0), dmin = h2f_bits(h0 >> 16);
    const uint32_t s0 = c[0].y, s1 = c[0].z, s2 = c[0].w;
    // unpack_q4_k_scales (src/gguf/mod.rs:1547-1554), four sub-blocks per word
    const uint32_t scl = s0 & 0x3f3f3f3fu, mnl = s1 & 0x3f3f3f3fu;
    const uint32_t sch = (s2 & 0x0f0f0f0fu) | ((s0 >> 2) & 0x30303030u);
    const uint32_t mnh = ((s2 >> 4) & 0x0f0f0f0fu) | ((s1 >> 2) & 0x30303030u);
    int bh = 0, bl = 0;
#pragma unroll
    for (int cc = 0; cc < 8; cc++) {
        const uint4 q = c[1 + cc];
        const uint4 zhl = x.zh[cc], zll = x.zl[cc], zhh = x.zh[8 + cc], zlh = x.zl[8 + cc];
        int ah = 0, al = 0, ah2 = 0, al2 = 0;
#define NX_Q4K_STEP(W)                                              \
    {                                                               \
        const uint32_t lo = q.W & 0x0f0f0f0fu;                      \
        const uint32_t hi = (q.W >> 4) & 0x0f0f0f0fu;               \
        ah = dp4a_us(lo, zhl.W, ah);                                \
        al = dp4a_uu(lo, zll.W, al);                                \
        ah2 = dp4a_us(hi, zhh.W, ah2);                              \
        al2 = dp4a_uu(hi, zlh.W, al2);                              \
    }
        NX_Q4K_STEP(x) NX_Q4K_STEP(y) NX_Q4K_STEP(z) NX_Q4K_STEP(w)
#undef NX_Q4K_STEP
        const int j = cc >> 1;
        const int sl = (int)byte_of(scl, j), sh = (int)byte_of(sch, j);
        bh += sl * ah + sh * ah2;
        bl += sl * al + sh * al2;
    }
    const int4 z0 = reinterpret_cast<const int4 *>(x.sz)[0], z1 = reinterpret_cast<const int4 *>(x.sz)[1];
    const int4 z2 = reinterpret_cast<const int4 *>(x.sz)[2], z3 = reinterpret_cast<const int4 *>(x.sz)[3];
    const int mn = (int)byte_of(mnl, 0) * (z0.x + z0.y) + (int)byte_of(mnl, 1) * (z0.z + z0.w) +
                   (int)byte_of(mnl, 2) * (z1.x + z1.y) + (int)byte_of(mnl, 3) * (z1.z + z1.w) +
                   (int)byte_of(mnh, 0) * (z2.x + z2.y) + (int)byte_of(mnh, 1) * (z2.z + z2.w) +
                   (int)byte_of(mnh, 2) * (z3.x + z3.y) + (int)byte_of(mnh, 3) * (z3.z + z3.w);
    return x.u * (d * (256.0f * (float)bh + (float)bl) - dmin * (float)mn);
}

// Q8_0 super-block: c[0] = eight f16 scales, c[1+2b], c[2+2b] = qs of block b
__device__ __forceinline__ float sb_dot_q80(const uint4 *c, const XSb &x) {
    float acc = 0.0f;
    const uint32_t sw[4] = {c[0].x, c[0].y, c[0].z, c[0].w};
#pragma unroll
    for (int b = 0; b < 8; b++) {
        const uint4 q0 = c[1 + 2 * b], q1 = c[2 + 2 * b];
        const uint4 h0 = x.zh[2 * b], h1 = x.zh[2 * b + 1], l0 = x.zl[2 * b], l1 = x.zl[2 * b + 1];
        int ah = dp4a_ss(q0.x, h0.x, 0);
        ah = dp4a_ss(q0.y, h0.y, ah);
        ah = dp4a_ss(q0.z, h0.z, ah);
        ah = dp4a_ss(q0.w, h0.w, ah);
        ah = dp4a_ss(q1.x, h1.x, ah);
        ah = dp4a_ss(q1.y, h1.y, ah);
        ah = dp4a_ss(q1.z, h1.z, ah);
        ah = dp4a_ss(q1.w, h1.w, ah);
        int al = dp4a_su(q0.x, l0.x, 0);
        al = dp4a_su(q0.y, l0.y, al);
        al = dp4a_su(q0.z, l0.z, al);
        al = dp4a_su(q0.w, l0.w, al);
        al = dp4a_su(q1.x, l1.x, al);
        al = dp4a_su(q1.y, l1.y, al);
        al = dp4a_su(q1.z, l1.z, al);
        al = dp4a_su(q1.w, l1.w, al);
        const float db = h2f_bits(sw[b >> 1] >> (16 * (b & 1)));
        acc += db * (256.0f * (float)ah + (float)al);
    }
    return x.u * acc;
}

// Q4_0 super-block: c[0] = eight f16 scales, c[1+b] = qs of block b (q - 8)
__device__ __forceinline__ float sb_dot_q40(const uint4 *c, const XSb &x) {
    float acc = 0.0f;
    const uint32_t sw[4] = {c[0].x, c[0].y, c[0].z, c[0].w};
#pragma unroll
    for (int b = 0; b < 8; b++) {
        const uint4 q = c[1 + b];
        const uint4 hl = x.zh[2 * b], hh = x.zh[2 * b + 1], ll = x.zl[2 * b], lh = x.zl[2 * b + 1];
        int ah = 0, al = 0;
#define NX_Q40_STEP(W)                                  \
    {                                                   \
        const uint32_t lo = q.W & 0x0f0f0f0fu;          \
        const uint32_t hi = (q.W >> 4) & 0x0f0f0f0fu;   \
        ah = dp4a_us(lo, hl.W, ah);                     \
        ah = dp4a_us(hi, hh.W, ah);                     \
        al = dp4a_uu(lo, ll.W, al);                     \
        al = dp4a_uu(hi, lh.W, al);                     \
    }
        NX_Q40_STEP(x) NX_Q40_STEP(y) NX_Q40_STEP(z) NX_Q40_STEP(w)
#undef NX_Q40_STEP
        const int s32 = x.sz[2 * b] + x.sz[2 * b + 1];
        const float db = h2f_bits(sw[b >> 1] >> (16 * (b & 1)));
        acc += db * (256.0f * (float)ah + (float)(al - 8 * s32));
    }
    return x.u * acc;
}

// Q2_K super-block: c[0] = 16 scale bytes, c[1..4] = qs words (one per
// 16-element sub-block, crumb-planes ordered), aux = d | dmin << 16
__device__ __forceinline__ float sb_dot_q2k(const uint4 *c, uint32_t aux, const XSb &x) {
    const float d = h2f_bits(aux), dmin = h2f_bits(aux >> 16);
    const uint32_t scw[4] = {c[0].x, c[0].y, c[0].z, c[0].w};
    int bh = 0, bl = 0, mn = 0;
#pragma unroll
    for (int j = 0; j < 16; j++) {
        const uint4 qq = c[1 + (j >> 2)];
        const uint32_t qw = (j & 3) == 0 ? qq.x : (j & 3) == 1 ? qq.y : (j & 3) == 2 ? qq.z : qq.w;
        const uint4 h = x.zh[j], l = x.zl[j];
        const uint32_t p0 = qw & 0x03030303u, p1 = (qw >> 2) & 0x03030303u;
        const uint32_t p2 = (qw >> 4) & 0x03030303u, p3 = (qw >> 6) & 0x03030303u;
        int ah = dp4a_us(p0, h.x, 0);
        ah = dp4a_us(p1, h.y, ah);
        ah = dp4a_us(p2, h.z, ah);
        ah = dp4a_us(p3, h.w, ah);
        int al = dp4a_uu(p0, l.x, 0);
        al = dp4a_uu(p1, l.y, al);
        al = dp4a_uu(p2, l.z, al);
        al = dp4a_uu(p3, l.w, al);
        const uint32_t sb = byte_of(scw[j >> 2], j & 3);
        const int sc = (int)(sb & 15u), m = (int)(sb >> 4);
        bh += sc * ah;
        bl += sc * al;
        mn += m * x.sz[j];
    }
    return x.u * (d * (256.0f * (float)bh + (float)bl) - dmin * (float)mn);
}

template <int FMT>
__device__ __forceinline__ float sb_dot(const uint4 *c, uint32_t aux, const XSb &x) {
    if constexpr (FMT == 12) return sb_dot_q4k(c, x);
    else if constexpr (FMT == 8) return sb_dot_q80(c, x);
    else if constexpr (FMT == 2) return sb_dot_q40(c, x);
    else return sb_dot_q2k(c, aux, x);
}

// Shared-memory bytes of the prepared input of one token: zh[k], zl[k],
// sz[k/16], u[k/256], padded to 16 bytes so every token's image is aligned.
__host__ __device__ __forceinline__ size_t tok_smem_bytes(int k) {
    return ((size_t)2 * k + (size_t)4 * (k / 16) + (size_t)4 * (k / 256) + 15) / 16 * 16;
}

// Prepare super-block s of token t: optional RMSNorm, 16-bit quantization.
// One warp; lane handles elements 8*lane .. 8*lane+7 of the super-block.
__device__ __forceinline__ void prep_sb(const float *__restrict__ x, const float *__restrict__ nw, float rstd, int s,
                                        int lane, uint32_t *zh, uint32_t *zl, int *sz, float *u) {
    const float4 *xp = reinterpret_cast<const float4 *>(x + 256 * s + 8 * lane);
    float4 a = xp[0], b = xp[1];
    float v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
    if (nw) {
        const float4 *wp = reinterpret_cast<const float4 *>(nw + 256 * s + 8 * lane);
        float4 wa = wp[0], wb = wp[1];
        float w[8] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};
        // rms_norm: input[i] * rstd * weight[i] (src/kernel/mod.rs:206)
#pragma unroll
        for (int i = 0; i < 8; i++) v[i] = __fmul_rn(__fmul_rn(v[i], rstd), w[i]);
    }
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; i++) amax = fmaxf(amax, fabsf(v[i]));
    amax = warp_max(amax);
    const float inv = (amax > 0.0f && amax <= 3.0e38f) ? 32767.0f / amax : 0.0f;
    int z[8], psum = 0;
#pragma unroll
    for (int i = 0; i < 8; i++) {
        z[i] = __float2int_rn(v[i] * inv);
        psum += z[i];
    }
    uint32_t h0 = 0, h1 = 0, l0 = 0, l1 = 0;
#pragma unroll
    for (int i = 0; i < 4; i++) {
        h0 |= ((uint32_t)(z[i] >> 8) & 0xffu) << (8 * i);
        h1 |= ((uint32_t)(z[4 + i] >> 8) & 0xffu) << (8 * i);
        l0 |= ((uint32_t)z[i] & 0xffu) << (8 * i);
        l1 |= ((uint32_t)z[4 + i] & 0xffu) << (8 * i);
    }
    const int wi = 64 * s + 2 * lane;
    zh[wi] = h0;
    zh[wi + 1] = h1;
    zl[wi] = l0;
    zl[wi + 1] = l1;
    psum += __shfl_xor_sync(0xffffffffu, psum, 1);
    if ((lane & 1) == 0) sz[16 * s + (lane >> 1)] = psum;
    if (lane == 0) u[s] = amax / 32767.0f;
}

template <int FMT>
__device__ __forceinline__ void load_sb(uint4 (&c)[Fmt<FMT>::C], uint32_t &aux, const uint4 *__restrict__ base,
                                        const uint32_t *__restrict__ abase, int s) {
    constexpr int C = Fmt<FMT>::C;
    const uint4 *p = base + (size_t)s * C * 32;
#pragma unroll
    for (int i = 0; i < C; i++) c[i] = ld_stream(p + (size_t)i * 32);
    if constexpr (Fmt<FMT>::AUX) aux = ld_stream_u32(abase + (size_t)s * 32);
}

template <int FMT, int W, int M, int EPI>
__global__ void __launch_bounds__(W * 32) k_gemv(GemvParams p) {
    constexpr int C = Fmt<FMT>::C;
    extern __shared__ __align__(16) uint8_t smem[];
    const int g = blockIdx.x;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int k = p.k, n_sb = k >> 8;
    const int per = (n_sb + W - 1) / W;
    const int s0 = warp * per, s1 = min(n_sb, s0 + per);

    const size_t tok_bytes = tok_smem_bytes(k);
    float *red = reinterpret_cast<float *>(smem + tok_bytes * M);   // [W][M][32]
    float *misc = red + W * M * 32;                                  // [W*M] + [M]

    const uint4 *wbase = p.w_main + (size_t)g * n_sb * C * 32 + lane;
    const uint32_t *abase = Fmt<FMT>::AUX ? p.w_aux + (size_t)g * n_sb * 32 + lane : nullptr;

    // Prefetch the first super-block before waiting on the previous grid.
    uint4 cur[C];
    uint32_t aux_cur = 0;
    if (s0 < s1) load_sb<FMT>(cur, aux_cur, wbase, abase, s0);
    if (p.pdl) {
        pdl_launch_dependents();
        pdl_wait();
    }

    // Optional RMSNorm: every CTA reduces the full input row(s).
    float rstd[M];
#pragma unroll
    for (int t = 0; t < M; t++) rstd[t] = 1.0f;
    if (p.norm_w) {
#pragma unroll
        for (int t = 0; t < M; t++) {
            const float4 *xv = reinterpret_cast<const float4 *>(p.x + (size_t)t * p.x_stride);
            float ss = 0.0f;
            for (int i = threadIdx.x; i < k / 4; i += W * 32) {
                float4 v = xv[i];
                ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
            }
            ss = warp_sum(ss);
            if (lane == 0) misc[warp * M + t] = ss;
        }
        __syncthreads();
#pragma unroll
        for (int t = 0; t < M; t++) {
            float ss = 0.0f;
            for (int w = 0; w < W; w++) ss += misc[w * M + t];
            // rstd = 1 / sqrt(variance + eps) (src/kernel/mod.rs:202-203)
            rstd[t] = 1.0f / sqrtf(ss / (float)k + p.eps);
        }
    }

    // Each warp prepares x for exactly the super-blocks it consumes.
#pragma unroll
    for (int t = 0; t < M; t++) {
        uint8_t *tb = smem + tok_bytes * t;
        uint32_t *zh = reinterpret_cast<uint32_t *>(tb);
        uint32_t *zl = reinterpret_cast<uint32_t *>(tb + k);
        int *sz = reinterpret_cast<int *>(tb + 2 * k);
        float *u = reinterpret_cast<float *>(tb + 2 * k + 4 * (k / 16));
        const float *xt = p.x + (size_t)t * p.x_stride;
        for (int s = s0; s < s1; s++) prep_sb(xt, p.norm_w, rstd[t], s, lane, zh, zl, sz, u);
    }
    __syncwarp();

    float acc[M];
#pragma unroll
    for (int t = 0; t < M; t++) acc[t] = 0.0f;
    for (int s = s0; s < s1; s++) {
        uint4 nxt[C];
        uint32_t aux_nxt = 0;
        const bool more = s + 1 < s1;
        if (more) load_sb<FMT>(nxt, aux_nxt, wbase, abase, s + 1);
#pragma unroll
        for (int t = 0; t < M; t++) {
            const uint8_t *tb = smem + tok_bytes * t;
            XSb xs;
            xs.zh = reinterpret_cast<const uint4 *>(tb) + 16 * s;
            xs.zl = reinterpret_cast<const uint4 *>(tb + k) + 16 * s;
            xs.sz = reinterpret_cast<const int *>(tb + 2 * k) + 16 * s;
            xs.u = reinterpret_cast<const float *>(tb + 2 * k + 4 * (k / 16))[s];
            acc[t] += sb_dot<FMT>(cur, aux_cur, xs);
        }
        if (more) {
#pragma unroll
            for (int i = 0; i < C; i++) cur[i] = nxt[i];
            aux_cur = aux_nxt;
        }
    }

#pragma unroll
    for (int t = 0; t < M; t++) red[(warp * M + t) * 32 + lane] = acc[t];
    __syncthreads();
    if (warp != 0) return;

    const int row = 32 * g + lane;
#pragma unroll
    for (int t = 0; t < M; t++) {
        float tot = 0.0f;
        for (int w = 0; w < W; w++) tot += red[(w * M + t) * 32 + lane];
        if constexpr (EPI == EPI_STORE) {
            if (row < p.n) p.y[(size_t)t * p.y_stride + row] = tot;
        } else if constexpr (EPI == EPI_ADD) {
            if (row < p.n) {
                float *yp = p.y + (size_t)t * p.y_stride + row;
                *yp = *yp + tot;
            }
        } else if constexpr (EPI == EPI_SWIGLU) {
            // lanes 0..15: gate rows 16g+lane, lanes 16..31: the matching up rows
            const float up = __shfl_down_sync(0xffffffffu, tot, 16);
            const int i = 16 * g + lane;
            if (lane < 16 && 2 * i < p.n) {
                // (gate / (1 + exp(-gate))) * up  (src/engine/mod.rs:1139)
                p.y[(size_t)t * p.y_stride + i] = (tot / (1.0f + expf(-tot))) * up;
            }
        } else if constexpr (EPI == EPI_QKV) {
            const QkvEpilogue &q = p.qkv;
            const int D = q.head_dim, gph = D / 32;
            const int gq = q.hq * gph, gk = q.hkv * gph;
            const int kv_dim = q.hkv * D;
            const DevSeq &sq = q.seqs[t];
            const float other = __shfl_down_sync(0xffffffffu, tot, 16);
            float *kdst, *vdst;
            if (q.kv_scratch) {
                kdst = q.kv_scratch + (size_t)t * 2 * kv_dim;
                vdst = kdst + kv_dim;
            } else {
                const size_t base = (size_t)q.seq_ids[t] * q.seq_stride + (size_t)sq.slot * kv_dim;
                kdst = q.k_cache + base;
                vdst = q.v_cache + base;
            }
            if (g < gq + gk) {
                const bool isq = g < gq;
                const int gg = isq ? g : g - gq;
                const int head = gg / gph, i = gg % gph;
                if (lane < 16) {
                    const int d = 16 * i + lane;
                    const size_t ti = (size_t)sq.position * (D / 2) + d;
                    const float cs = q.rope_cos[ti], sn = q.rope_sin[ti];
                    // rope_single (src/kernel/mod.rs:267-268), separately rounded
                    const float r0 = __fsub_rn(__fmul_rn(tot, cs), __fmul_rn(other, sn));
                    const float r1 = __fadd_rn(__fmul_rn(tot, sn), __fmul_rn(other, cs));
                    float *dst = isq ? q.q_out + (size_t)t * q.hq * D + head * D : kdst + head * D;
                    dst[d] = r0;
                    dst[d + D / 2] = r1;
                }
            } else {
                const int r = 32 * (g - gq - gk) + lane;
                if (r < kv_dim) vdst[r] = tot;
            }
        } else if constexpr (EPI == EPI_ARGMAX) {
            if (row < p.n && p.y) p.y[(size_t)t * p.y_stride + row] = tot;
            // greedy_token: finite values only, larger value wins, ties -> larger index
            unsigned long long key = 0ull;
            if (row < p.n && isfinite(tot))
                key = ((unsigned long long)((unsigned)total_key(tot) ^ 0x80000000u) << 32) | (unsigned)row;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                unsigned long long other = __shfl_xor_sync(0xffffffffu, key, o);
                key = other > key ? other : key;
            }
            if (lane == 0 && key) atomicMax(&p.seqs[t].best, key);
        }
    }
}

// ---------------------------------------------------------------------------
template <int FMT, int W, int M, int EPI>
static cudaError_t launch_one(const GemvParams &p, cudaStream_t st) {
    const int groups = (p.n + 31) / 32;
    const size_t tok_bytes = tok_smem_bytes(p.k);
    const size_t smem = tok_bytes * M + (size_t)4 * W * M * 32 + (size_t)4 * (W * M + M);
    auto fn = k_gemv<FMT, W, M, EPI>;
    if (smem > 200 * 1024) return cudaErrorInvalidValue;
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
    }
    if (smem > 200 * 1024) return cudaErrorInvalidValue;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(groups);
    cfg.blockDim = dim3(W * 32);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = p.pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, fn, p);
}

template <int FMT, int M, int EPI>
static cudaError_t launch_w(const GemvParams &p, cudaStream_t st) {
    const int n_sb = p.k / 256;
    if (n_sb >= 8) return launch_one<FMT, 8, M, EPI>(p, st);
    if (n_sb >= 2) return launch_one<FMT, 4, M, EPI>(p, st);
    return launch_one<FMT, 1, M, EPI>(p, st);
}

template <int FMT, int M>
static cudaError_t launch_epi(const GemvParams &p, cudaStream_t st) {
    switch (p.epi) {
    case EPI_STORE: return launch_w<FMT, M, EPI_STORE>(p, st);
    case EPI_ADD: return launch_w<FMT, M, EPI_ADD>(p, st);
    case EPI_SWIGLU: return launch_w<FMT, M, EPI_SWIGLU>(p, st);
    case EPI_QKV: return launch_w<FMT, M, EPI_QKV>(p, st);
    case EPI_ARGMAX: return launch_w<FMT, M, EPI_ARGMAX>(p, st);
    default: return cudaErrorInvalidValue;
    }
}

template <int FMT>
cudaError_t launch_gemv_fmt(const GemvParams &p, cudaStream_t st) {
    switch (p.m) {
    case 1: return launch_epi<FMT, 1>(p, st);
    case 2: return launch_epi<FMT, 2>(p, st);
    case 4: return launch_epi<FMT, 4>(p, st);
    default: return cudaErrorInvalidValue;
    }
}

}  // namespace nx
