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
// Parallel layout.  The tile matrix is a sequence of items (row group g,
// super-block s) in group-major order, and that sequence is contiguous in
// memory.  Each CTA (one per SM) owns one contiguous run of items ("stream-K")
// and streams its bytes into a shared-memory ring with TMA bulk copies
// (cp.async.bulk + mbarrier transaction counts).  The first ring stages are
// issued before griddepcontrol.wait, so under programmatic dependent launch a
// GEMV streams its first weights while the previous kernel is still running.
// Lane i of every warp owns row 32g+i; the warps of a CTA take the items of a
// ring stage (P warps share an item, each taking 1/P of its blocks); warp 0
// sums item partials in item order and applies the epilogue when a row group
// ends.  A row group split between CTAs is finished by the last of them to
// arrive (self-resetting counter), which adds the per-CTA partials in CTA
// order -- deterministic, no float atomics.  The input is prepared (16-bit
// quantization, RMSNorm folded into the per-super-block scale) once per CTA.
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

// The sb_dot_* functions compute part `part` of P equal parts of one
// super-block's contribution; chunk i of the lane's row is c[32*i] (tile
// layout, in global memory or in a shared-memory copy of it).
#define NX_CH(i) c[32 * (i)]

// Q4_K super-block (tiles.cuh): chunk 0 = d|dmin, scales; chunks 1..8 = qs
template <int P>
__device__ __forceinline__ float sb_dot_q4k(const uint4 *c, const XSb &x, int part) {
    const uint4 c0 = NX_CH(0);
    const float d = h2f_bits(c0.x), dmin = h2f_bits(c0.x >> 16);
    const uint32_t s0 = c0.y, s1 = c0.z, s2 = c0.w;
    // unpack_q4_k_scales (src/gguf/mod.rs:1547-1554), four sub-blocks per word
    const uint32_t scl = s0 & 0x3f3f3f3fu, mnl = s1 & 0x3f3f3f3fu;
    const uint32_t sch = (s2 & 0x0f0f0f0fu) | ((s0 >> 2) & 0x30303030u);
    const uint32_t mnh = ((s2 >> 4) & 0x0f0f0f0fu) | ((s1 >> 2) & 0x30303030u);
    int bh = 0, bl = 0, mn = 0;
    constexpr int CPP = 8 / P;  // qs chunks per part (whole sub-block pairs)
#pragma unroll
    for (int k = 0; k < CPP; k++) {
        const int cc = part * CPP + k;
        const uint4 q = NX_CH(1 + cc);
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
        if ((cc & 1) == 0) {
            // min term of sub-blocks j and j + 4 (32 elements each)
            mn += (int)byte_of(mnl, j) * (x.sz[2 * j] + x.sz[2 * j + 1]) +
                  (int)byte_of(mnh, j) * (x.sz[8 + 2 * j] + x.sz[8 + 2 * j + 1]);
        }
    }
    return x.u * (d * (256.0f * (float)bh + (float)bl) - dmin * (float)mn);
}

// Q8_0 super-block: chunk 0 = eight f16 scales, chunks 1+2b, 2+2b = qs of block b
template <int P>
__device__ __forceinline__ float sb_dot_q80(const uint4 *c, const XSb &x, int part) {
    float acc = 0.0f;
    const uint4 c0 = NX_CH(0);
    const uint32_t sw[4] = {c0.x, c0.y, c0.z, c0.w};
    constexpr int BPP = 8 / P;
#pragma unroll
    for (int k = 0; k < BPP; k++) {
        const int b = part * BPP + k;
        const uint4 q0 = NX_CH(1 + 2 * b), q1 = NX_CH(2 + 2 * b);
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

// Q4_0 super-block: chunk 0 = eight f16 scales, chunk 1+b = qs of block b (q - 8)
template <int P>
__device__ __forceinline__ float sb_dot_q40(const uint4 *c, const XSb &x, int part) {
    float acc = 0.0f;
    const uint4 c0 = NX_CH(0);
    const uint32_t sw[4] = {c0.x, c0.y, c0.z, c0.w};
    constexpr int BPP = 8 / P;
#pragma unroll
    for (int k = 0; k < BPP; k++) {
        const int b = part * BPP + k;
        const uint4 q = NX_CH(1 + b);
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

// Q2_K super-block: chunk 0 = 16 scale bytes, chunks 1..4 = qs words (one per
// 16-element sub-block, bit-plane ordered), aux = d | dmin << 16
template <int P>
__device__ __forceinline__ float sb_dot_q2k(const uint4 *c, uint32_t aux, const XSb &x, int part) {
    const float d = h2f_bits(aux), dmin = h2f_bits(aux >> 16);
    const uint4 c0 = NX_CH(0);
    const uint32_t scw[4] = {c0.x, c0.y, c0.z, c0.w};
    int bh = 0, bl = 0, mn = 0;
    constexpr int JPP = 16 / P;
#pragma unroll
    for (int k = 0; k < JPP; k++) {
        const int j = part * JPP + k;
        const uint4 qq = NX_CH(1 + (j >> 2));
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
#undef NX_CH

template <int FMT, int P>
__device__ __forceinline__ float sb_dot(const uint4 *c, uint32_t aux, const XSb &x, int part) {
    if constexpr (FMT == 12) return sb_dot_q4k<P>(c, x, part);
    else if constexpr (FMT == 8) return sb_dot_q80<P>(c, x, part);
    else if constexpr (FMT == 2) return sb_dot_q40<P>(c, x, part);
    else return sb_dot_q2k<P>(c, aux, x, part);
}

// Shared-memory bytes of the prepared input of one token: zh[k], zl[k],
// sz[k/16], u[k/256], padded to 16 bytes so every token's image is aligned.
__host__ __device__ __forceinline__ size_t tok_smem_bytes(int k) {
    return ((size_t)2 * k + (size_t)4 * (k / 16) + (size_t)4 * (k / 256) + 15) / 16 * 16;
}

// Prepare super-block s of one token: 16-bit quantization of x (times the
// RMSNorm weight when fused).  One warp; lane handles elements 8*lane ..
// 8*lane+7.  The quantization is scale-invariant, so RMSNorm's rstd is not
// needed here: the caller multiplies u[s] by rstd once the sum of squares,
// accumulated in *ss, is known.  (x*rstd)*w and rstd*(x*w) agree to f32
// rounding, far below the 16-bit step.
__device__ __forceinline__ void prep_sb(const float *__restrict__ x, const float *__restrict__ nw, int s,
                                        int lane, uint32_t *zh, uint32_t *zl, int *sz, float *u, float *ss) {
    const float4 *xp = reinterpret_cast<const float4 *>(x + 256 * s + 8 * lane);
    float4 a = xp[0], b = xp[1];
    float v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
    for (int i = 0; i < 8; i++) *ss += v[i] * v[i];
    if (nw) {
        const float4 *wp = reinterpret_cast<const float4 *>(nw + 256 * s + 8 * lane);
        float4 wa = wp[0], wb = wp[1];
        float w[8] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};
#pragma unroll
        for (int i = 0; i < 8; i++) v[i] = v[i] * w[i];
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

// Epilogue for one row (lane) of row group g and token t.
template <int EPI>
__device__ __forceinline__ void gemv_epilogue(const GemvParams &p, int g, int t, int lane, float tot) {
    const int row = 32 * g + lane;
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


// Ring geometry per format: items (super-block tiles) per stage and warps per item.
template <int FMT>
struct Ring {
    static constexpr int C = Fmt<FMT>::C;
    static constexpr int ITEM_BYTES = C * 512;
    // ~18-20 KB per stage, 4 stages (about 74 KB in flight per CTA)
    static constexpr int IPS = FMT == 8 ? 2 : FMT == 10 ? 8 : 4;
    static constexpr int W = 8;
    static constexpr int P = W / IPS;  // warps sharing one item
    static constexpr int NST = 4;
    static constexpr int STAGE_BYTES = IPS * ITEM_BYTES;
};

constexpr unsigned kMbarSpinLimit = 1u << 20;

template <int FMT, int M, int EPI>
__global__ void __launch_bounds__(256, 1) k_gemv(GemvParams p) {
    using R = Ring<FMT>;
    constexpr int W = R::W, IPS = R::IPS, P = R::P, NST = R::NST;
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ unsigned long long full[NST];
    __shared__ int s_ok;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int k = p.k, n_sb = k >> 8;
    const int groups = (p.n + 31) / 32;
    const long long T = (long long)groups * n_sb;
    const int G = gridDim.x, c = blockIdx.x;
    const long long i0 = (long long)c * T / G, i1 = (long long)(c + 1) * T / G;
    const int nstages = (int)((i1 - i0 + IPS - 1) / IPS);

    uint8_t *ring = smem;                                              // NST * STAGE_BYTES
    uint32_t *aux_ring = reinterpret_cast<uint32_t *>(ring + NST * R::STAGE_BYTES);  // NST * IPS * 32 (Q2_K)
    uint8_t *xs = ring + NST * R::STAGE_BYTES + (Fmt<FMT>::AUX ? NST * IPS * 128 : 0);
    const size_t tok_bytes = tok_smem_bytes(k);
    float *red = reinterpret_cast<float *>(xs + tok_bytes * M);        // [W][M][32]
    float *misc = red + W * M * 32;                                    // [W*M]

    auto issue = [&](int st) {  // one thread: stage st into ring slot st % NST
        const long long a = i0 + (long long)st * IPS;
        const long long b = min(i1, a + IPS);
        const unsigned bytes = (unsigned)((b - a) * R::ITEM_BYTES);
        const unsigned abytes = Fmt<FMT>::AUX ? (unsigned)((b - a) * 128) : 0u;
        unsigned long long *bar = &full[st % NST];
        mbar_expect_tx(bar, bytes + abytes);
        tma_load_1d(ring + (size_t)(st % NST) * R::STAGE_BYTES,
                    reinterpret_cast<const uint8_t *>(p.w_main) + (size_t)a * R::ITEM_BYTES, bytes, bar);
        if constexpr (Fmt<FMT>::AUX)
            tma_load_1d(aux_ring + (size_t)(st % NST) * IPS * 32,
                        reinterpret_cast<const uint8_t *>(p.w_aux) + (size_t)a * 128, abytes, bar);
    };

    if (threadIdx.x == 0) {
        for (int i = 0; i < NST; i++) mbar_init(&full[i], 1);
        mbar_init_fence();
    }
    __syncthreads();
    // Stream the first stages of weights before waiting on the previous grid.
    if (threadIdx.x == 0)
        for (int st = 0; st < NST && st < nstages; st++) issue(st);
    if (p.pdl) {
        pdl_launch_dependents();
        pdl_wait();
    }

    // Prepare the whole input once (warp w takes super-blocks w, w+W, ...);
    // with a fused RMSNorm the sum of squares comes out of the same pass.
#pragma unroll
    for (int t = 0; t < M; t++) {
        uint8_t *tb = xs + tok_bytes * t;
        uint32_t *zh = reinterpret_cast<uint32_t *>(tb);
        uint32_t *zl = reinterpret_cast<uint32_t *>(tb + k);
        int *sz = reinterpret_cast<int *>(tb + 2 * k);
        float *u = reinterpret_cast<float *>(tb + 2 * k + 4 * (k / 16));
        const float *xt = p.x + (size_t)t * p.x_stride;
        float ss = 0.0f;
        for (int s = warp; s < n_sb; s += W) prep_sb(xt, p.norm_w, s, lane, zh, zl, sz, u, &ss);
        if (p.norm_w) {
            ss = warp_sum(ss);
            if (lane == 0) misc[warp * M + t] = ss;
        }
    }
    __syncthreads();
    if (p.norm_w) {
        // rstd = 1 / sqrt(variance + eps) (src/kernel/mod.rs:202-203), folded into u
#pragma unroll
        for (int t = 0; t < M; t++) {
            float ss = 0.0f;
            for (int w = 0; w < W; w++) ss += misc[w * M + t];
            const float rstd = 1.0f / sqrtf(ss / (float)k + p.eps);
            float *u = reinterpret_cast<float *>(xs + tok_bytes * t + 2 * k + 4 * (k / 16));
            for (int s = threadIdx.x; s < n_sb; s += W * 32) u[s] *= rstd;
        }
        __syncthreads();
    }

    // warp 0 state: running sum of the current row group
    int cur_g = -1;
    float gacc[M];
#pragma unroll
    for (int t = 0; t < M; t++) gacc[t] = 0.0f;

    auto flush = [&](int g) {  // warp 0: row group g is complete in this CTA's range
        const long long g0 = (long long)g * n_sb, g1 = g0 + n_sb;
        if (g0 >= i0 && g1 <= i1) {
#pragma unroll
            for (int t = 0; t < M; t++) gemv_epilogue<EPI>(p, g, t, lane, gacc[t]);
            return;
        }
        // shared with neighbouring CTAs: owner(i) = floor(((i+1)G - 1) / T)
        const int cf = (int)(((g0 + 1) * G - 1) / T), cl = (int)((g1 * G - 1) / T);
        const int slot = c - cf, count = cl - cf + 1;
        const size_t npad = (size_t)groups * 32;
        const int row = 32 * g + lane;
#pragma unroll
        for (int t = 0; t < M; t++) p.part[((size_t)slot * M + t) * npad + row] = gacc[t];
        __threadfence();
        __syncwarp();
        unsigned last = 0;
        if (lane == 0) {
            const unsigned prev = atomicAdd(&p.counters[g], 1u);
            last = prev == (unsigned)(count - 1);
            if (last) p.counters[g] = 0u;
        }
        if (__shfl_sync(0xffffffffu, last, 0)) {
            __threadfence();
#pragma unroll
            for (int t = 0; t < M; t++) {
                float sum = 0.0f;
                for (int sl = 0; sl < count; sl++) sum += __ldcg(p.part + ((size_t)sl * M + t) * npad + row);
                gemv_epilogue<EPI>(p, g, t, lane, sum);
            }
        }
    };

    const int it = warp / P, part = warp % P;
    for (int st = 0; st < nstages; st++) {
        // wait for the stage's bytes (bounded: a copy that never lands is reported)
        bool ok = true;
        {
            unsigned n = 0;
            while (!mbar_try_wait(&full[st % NST], (unsigned)((st / NST) & 1))) {
                if (++n > kMbarSpinLimit) {
                    ok = false;
                    break;
                }
            }
        }
        if (!__syncthreads_and(ok)) {
            if (threadIdx.x == 0 && p.err) atomicExch(p.err, 1);
            return;
        }
        const long long a = i0 + (long long)st * IPS;
        const int nit = (int)min((long long)IPS, i1 - a);
        float v[M];
#pragma unroll
        for (int t = 0; t < M; t++) v[t] = 0.0f;
        if (it < nit) {
            const long long item = a + it;
            const int s_sb = (int)(item % n_sb);
            const uint4 *cbase = reinterpret_cast<const uint4 *>(ring + (size_t)(st % NST) * R::STAGE_BYTES) +
                                 (size_t)it * R::C * 32 + lane;
            uint32_t auxw = 0;
            if constexpr (Fmt<FMT>::AUX) auxw = aux_ring[(size_t)(st % NST) * IPS * 32 + it * 32 + lane];
#pragma unroll
            for (int t = 0; t < M; t++) {
                const uint8_t *tb = xs + tok_bytes * t;
                XSb xsb;
                xsb.zh = reinterpret_cast<const uint4 *>(tb) + 16 * s_sb;
                xsb.zl = reinterpret_cast<const uint4 *>(tb + k) + 16 * s_sb;
                xsb.sz = reinterpret_cast<const int *>(tb + 2 * k) + 16 * s_sb;
                xsb.u = reinterpret_cast<const float *>(tb + 2 * k + 4 * (k / 16))[s_sb];
                v[t] = sb_dot<FMT, P>(cbase, auxw, xsb, part);
            }
        }
#pragma unroll
        for (int t = 0; t < M; t++) red[(warp * M + t) * 32 + lane] = v[t];
        fence_proxy_async_smem();
        __syncthreads();
        // every warp is done with ring slot st % NST: refill it
        if (threadIdx.x == 0 && st + NST < nstages) issue(st + NST);
        if (warp == 0) {
            for (int j = 0; j < nit; j++) {
                const int g = (int)((a + j) / n_sb);
                if (g != cur_g) {
                    if (cur_g >= 0) flush(cur_g);
                    cur_g = g;
#pragma unroll
                    for (int t = 0; t < M; t++) gacc[t] = 0.0f;
                }
#pragma unroll
                for (int t = 0; t < M; t++) {
                    float sv = 0.0f;
#pragma unroll
                    for (int q = 0; q < P; q++) sv += red[((j * P + q) * M + t) * 32 + lane];
                    gacc[t] += sv;
                }
            }
        }
        __syncthreads();
    }
    if (warp == 0 && cur_g >= 0) flush(cur_g);
}

// ---------------------------------------------------------------------------
template <int FMT, int M, int EPI>
static cudaError_t launch_fmt_m_epi(const GemvParams &pin, cudaStream_t st) {
    using R = Ring<FMT>;
    GemvParams p = pin;
    const int groups = (p.n + 31) / 32;
    const int n_sb = p.k / 256;
    const long long T = (long long)groups * n_sb;
    const size_t tok_bytes = tok_smem_bytes(p.k);
    const size_t smem = (size_t)R::NST * R::STAGE_BYTES + (Fmt<FMT>::AUX ? (size_t)R::NST * R::IPS * 128 : 0) +
                        tok_bytes * M + (size_t)4 * R::W * M * 32 + (size_t)4 * R::W * M;
    auto fn = k_gemv<FMT, M, EPI>;
    if (smem > 220 * 1024) return cudaErrorInvalidValue;
    cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    int dev = 0;
    cudaGetDevice(&dev);
    static int sm_count[16] = {};
    if (dev < 16 && sm_count[dev] == 0) cudaDeviceGetAttribute(&sm_count[dev], cudaDevAttrMultiProcessorCount, dev);
    int grid = dev < 16 && sm_count[dev] ? sm_count[dev] : 148;
    if ((long long)grid > T) grid = (int)T;
    // A row group spans at most ceil(n_sb / floor(T/grid)) + 1 CTAs; their
    // partials need scratch slots and the group a counter.
    auto max_share = [&](int gr) -> long long {
        const long long per = T / gr;
        return per >= n_sb ? 2 : (n_sb + per - 1) / per + 1;
    };
    while (grid > 1 && (!p.part || !p.counters || groups > p.counter_slots ||
                        (size_t)max_share(grid) * M * groups * 32 > p.part_floats)) {
        if (T % grid == 0 && (T / grid) % n_sb == 0) break;  // every CTA owns whole row groups
        grid = grid > 8 ? grid - grid / 8 : grid - 1;
    }
    if (grid < 1) grid = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(R::W * 32);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = p.pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, fn, p);
}

template <int FMT, int M>
static cudaError_t launch_epi(const GemvParams &p, cudaStream_t st) {
    switch (p.epi) {
    case EPI_STORE: return launch_fmt_m_epi<FMT, M, EPI_STORE>(p, st);
    case EPI_ADD: return launch_fmt_m_epi<FMT, M, EPI_ADD>(p, st);
    case EPI_SWIGLU: return launch_fmt_m_epi<FMT, M, EPI_SWIGLU>(p, st);
    case EPI_QKV: return launch_fmt_m_epi<FMT, M, EPI_QKV>(p, st);
    case EPI_ARGMAX: return launch_fmt_m_epi<FMT, M, EPI_ARGMAX>(p, st);
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
