#pragma once
// kernels_gemv.cuh -- dequant-fused GEMV for decode (m <= 4 tokens per pass).
//
// Replaces InferenceEngine::matvec (src/engine/mod.rs:775-801), which the
// reference runs on weights dequantized to f32 at load.  Here the weights stay
// in their block format in HBM (row-interleaved tiles, tiles.cuh) and are
// decoded in registers.
//
// Arithmetic.  Each token's input vector is re-expressed, per 256-element
// super-block s, as x_i ~= u_s * z_i with z_i a 24-bit integer
// (u_s = max|x|/(2^23-1)), split as z = 65536*h + 256*m + l (h signed, m and
// l unsigned bytes).
// A weight element of every supported format is (scale)*(small integer q) -
// (offset), so each super-block's contribution is
//     u_s * ( d * sum_j sc_j * sum_{i in j} q_i z_i  -  dmin * sum_j m_j * sum_{i in j} z_i )
// where the inner sums are exact 32-bit integer dot products (dp4a on four
// bytes at a time).  The only rounding beyond f32 accumulation is the 24-bit
// representation of x (|error| <= max|x|/(2^24-2) per super-block), so even
// heavy-tailed inputs (a few large elements setting a super-block's step, as
// in SwiGLU outputs) keep per-output errors near f32 rounding.
//
// Parallel layout.  An item is one (row group g of 32 rows, super-block s)
// tile: C*512 contiguous bytes (tiles.cuh).  Warps form teams of S warps; a
// team owns whole row groups and its S warps split each group's super-blocks.
// Every warp streams its own item sequence -- across the row groups its team
// owns -- through a private two-slot shared-memory ring filled by TMA bulk
// copies (cp.async.bulk + mbarrier), so a warp always has the next item in
// flight and no CTA-wide barrier sits in the main loop.  Lane i owns row
// 32g+i.  The S partial sums of a row group meet in shared memory behind a
// named barrier of the team, and the team's first warp adds them in warp
// order and applies the epilogue (deterministic).  CTAs are persistent, one
// per SM, and prepare the input (24-bit quantization, RMSNorm folded into
// the per-super-block scale) once.  The first ring slots are filled before
// griddepcontrol.wait, so under programmatic dependent launch a GEMV streams
// weights while the previous kernel finishes.
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
    const uint4 *zm;  // 16 x uint4: unsigned middle bytes
    const uint4 *zl;  // 16 x uint4: unsigned low bytes
    const int *sz;    // 16 ints: sum of z over each 16-element group
    float u;
};

__device__ __forceinline__ uint32_t byte_of(uint32_t w, int j) { return (w >> (8 * j)) & 0xffu; }

// The sb_dot_* functions compute part `part` of P equal parts of one
// super-block's contribution; chunk i of the lane's row is c[32*i] (tile
// layout, in global memory or in a shared-memory copy of it).
#define NX_CH(i) c[32 * (i)]

// Q4_K super-block (tiles.cuh): chunk 0 = d|dmin, scales; chunks 1..8 = qs.
// Low nibbles are masked in place; high nibbles are used in place as 16*q
// (one mask, no shift) and their sums carry a factor 16 removed at the end.
template <int P, int NB = 3>
__device__ __forceinline__ float sb_dot_q4k(const uint4 *c, const XSb &x, int part) {
    const uint4 c0 = NX_CH(0);
    const float d = h2f_bits(c0.x), dmin = h2f_bits(c0.x >> 16);
    const uint32_t s0 = c0.y, s1 = c0.z, s2 = c0.w;
    // unpack_q4_k_scales (src/gguf/mod.rs:1547-1554), four sub-blocks per word
    const uint32_t scl = s0 & 0x3f3f3f3fu, mnl = s1 & 0x3f3f3f3fu;
    const uint32_t sch = (s2 & 0x0f0f0f0fu) | ((s0 >> 2) & 0x30303030u);
    const uint32_t mnh = ((s2 >> 4) & 0x0f0f0f0fu) | ((s1 >> 2) & 0x30303030u);
    int bh = 0, bm = 0, bl = 0, bh16 = 0, bm16 = 0, bl16 = 0;
    float mn = 0.0f;
    constexpr int CPP = 8 / P;  // qs chunks per part (whole sub-block pairs)
#pragma unroll
    for (int k = 0; k < CPP; k++) {
        const int cc = part * CPP + k;
        const uint4 q = NX_CH(1 + cc);
        const uint4 zhl = x.zh[cc], zll = x.zl[cc];
        const uint4 zhh = x.zh[8 + cc], zlh = x.zl[8 + cc];
        uint4 zml = {}, zmh = {};
        if constexpr (NB == 3) {
            zml = x.zm[cc];
            zmh = x.zm[8 + cc];
        }
        int ah = 0, am = 0, al = 0, ah2 = 0, am2 = 0, al2 = 0;
#define NX_Q4K_STEP(W)                                              \
    {                                                               \
        const uint32_t lo = q.W & 0x0f0f0f0fu;                      \
        const uint32_t hi = q.W & 0xf0f0f0f0u;                      \
        ah = dp4a_us(lo, zhl.W, ah);                                \
        if constexpr (NB == 3) am = dp4a_uu(lo, zml.W, am);         \
        al = dp4a_uu(lo, zll.W, al);                                \
        ah2 = dp4a_us(hi, zhh.W, ah2);                              \
        if constexpr (NB == 3) am2 = dp4a_uu(hi, zmh.W, am2);       \
        al2 = dp4a_uu(hi, zlh.W, al2);                              \
    }
        NX_Q4K_STEP(x) NX_Q4K_STEP(y) NX_Q4K_STEP(z) NX_Q4K_STEP(w)
#undef NX_Q4K_STEP
        const int j = cc >> 1;
        const int sl = (int)byte_of(scl, j), sh = (int)byte_of(sch, j);
        bh += sl * ah;
        bm += sl * am;
        bl += sl * al;
        bh16 += sh * ah2;
        bm16 += sh * am2;
        bl16 += sh * al2;
        if ((cc & 1) == 0) {
            // min term of sub-blocks j and j + 4 (32 elements each); the z sums
            // reach 2^28, so their products with the mins are taken in f32
            mn += (float)byte_of(mnl, j) * (float)(x.sz[2 * j] + x.sz[2 * j + 1]) +
                  (float)byte_of(mnh, j) * (float)(x.sz[8 + 2 * j] + x.sz[8 + 2 * j + 1]);
        }
    }
    // |b*16| < 2^29 (16 * 63 * 8 chunks * 16 products of <= 15*255); the
    // factor 16 is exact in f32
    const float hsum = (float)bh + 0.0625f * (float)bh16;
    const float lsum = (float)bl + 0.0625f * (float)bl16;
    if constexpr (NB == 2) return x.u * (d * (256.0f * hsum + lsum) - dmin * mn);
    const float msum = (float)bm + 0.0625f * (float)bm16;
    return x.u * (d * (65536.0f * hsum + (256.0f * msum + lsum)) - dmin * mn);
}

// Q8_0 super-block: chunk 0 = eight f16 scales, chunks 1+2b, 2+2b = qs of block b
template <int P, int NB = 3>
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
        int am = 0;
        if constexpr (NB == 3) {
            const uint4 m0 = x.zm[2 * b], m1 = x.zm[2 * b + 1];
            am = dp4a_su(q0.x, m0.x, 0);
            am = dp4a_su(q0.y, m0.y, am);
            am = dp4a_su(q0.z, m0.z, am);
            am = dp4a_su(q0.w, m0.w, am);
            am = dp4a_su(q1.x, m1.x, am);
            am = dp4a_su(q1.y, m1.y, am);
            am = dp4a_su(q1.z, m1.z, am);
            am = dp4a_su(q1.w, m1.w, am);
        }
        int al = dp4a_su(q0.x, l0.x, 0);
        al = dp4a_su(q0.y, l0.y, al);
        al = dp4a_su(q0.z, l0.z, al);
        al = dp4a_su(q0.w, l0.w, al);
        al = dp4a_su(q1.x, l1.x, al);
        al = dp4a_su(q1.y, l1.y, al);
        al = dp4a_su(q1.z, l1.z, al);
        al = dp4a_su(q1.w, l1.w, al);
        const float db = h2f_bits(sw[b >> 1] >> (16 * (b & 1)));
        if constexpr (NB == 2) acc += db * (256.0f * (float)ah + (float)al);
        else acc += db * (65536.0f * (float)ah + (256.0f * (float)am + (float)al));
    }
    return x.u * acc;
}

// Half h of a Q8_0 super-block as the persistent step kernel stages it:
// chunk 0 = the eight f16 scales, chunks 1..8 = qs of blocks 4h..4h+3.
__device__ __forceinline__ float sb_dot_q80_half(const uint4 *c, const XSb &x, int h) {
    float acc = 0.0f;
    const uint4 c0 = NX_CH(0);
    // the scale words of blocks 4h..4h+3 (two f16 per word)
    const uint32_t sw[2] = {h ? c0.z : c0.x, h ? c0.w : c0.y};
#pragma unroll
    for (int k = 0; k < 4; k++) {
        const int b = 4 * h + k;
        const uint4 q0 = NX_CH(1 + 2 * k), q1 = NX_CH(2 + 2 * k);
        const uint4 h0 = x.zh[2 * b], h1 = x.zh[2 * b + 1], l0 = x.zl[2 * b], l1 = x.zl[2 * b + 1];
        const uint4 m0 = x.zm[2 * b], m1 = x.zm[2 * b + 1];
        int ah = dp4a_ss(q0.x, h0.x, 0);
        ah = dp4a_ss(q0.y, h0.y, ah);
        ah = dp4a_ss(q0.z, h0.z, ah);
        ah = dp4a_ss(q0.w, h0.w, ah);
        ah = dp4a_ss(q1.x, h1.x, ah);
        ah = dp4a_ss(q1.y, h1.y, ah);
        ah = dp4a_ss(q1.z, h1.z, ah);
        ah = dp4a_ss(q1.w, h1.w, ah);
        int am = dp4a_su(q0.x, m0.x, 0);
        am = dp4a_su(q0.y, m0.y, am);
        am = dp4a_su(q0.z, m0.z, am);
        am = dp4a_su(q0.w, m0.w, am);
        am = dp4a_su(q1.x, m1.x, am);
        am = dp4a_su(q1.y, m1.y, am);
        am = dp4a_su(q1.z, m1.z, am);
        am = dp4a_su(q1.w, m1.w, am);
        int al = dp4a_su(q0.x, l0.x, 0);
        al = dp4a_su(q0.y, l0.y, al);
        al = dp4a_su(q0.z, l0.z, al);
        al = dp4a_su(q0.w, l0.w, al);
        al = dp4a_su(q1.x, l1.x, al);
        al = dp4a_su(q1.y, l1.y, al);
        al = dp4a_su(q1.z, l1.z, al);
        al = dp4a_su(q1.w, l1.w, al);
        const float db = h2f_bits(sw[k >> 1] >> (16 * (k & 1)));
        acc += db * (65536.0f * (float)ah + (256.0f * (float)am + (float)al));
    }
    return x.u * acc;
}

// Q4_0 super-block: chunk 0 = eight f16 scales, chunk 1+b = qs of block b (q - 8)
template <int P, int NB = 3>
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
        uint4 ml = {}, mh = {};
        if constexpr (NB == 3) {
            ml = x.zm[2 * b];
            mh = x.zm[2 * b + 1];
        }
        int ah = 0, am = 0, al = 0;
#define NX_Q40_STEP(W)                                          \
    {                                                           \
        const uint32_t lo = q.W & 0x0f0f0f0fu;                  \
        const uint32_t hi = (q.W >> 4) & 0x0f0f0f0fu;           \
        ah = dp4a_us(lo, hl.W, ah);                             \
        ah = dp4a_us(hi, hh.W, ah);                             \
        if constexpr (NB == 3) am = dp4a_uu(lo, ml.W, am);      \
        if constexpr (NB == 3) am = dp4a_uu(hi, mh.W, am);      \
        al = dp4a_uu(lo, ll.W, al);                             \
        al = dp4a_uu(hi, lh.W, al);                             \
    }
        NX_Q40_STEP(x) NX_Q40_STEP(y) NX_Q40_STEP(z) NX_Q40_STEP(w)
#undef NX_Q40_STEP
        const int s32 = x.sz[2 * b] + x.sz[2 * b + 1];  // < 2^28
        const float db = h2f_bits(sw[b >> 1] >> (16 * (b & 1)));
        if constexpr (NB == 2) acc += db * (256.0f * (float)ah + ((float)al - 8.0f * (float)s32));
        else acc += db * (65536.0f * (float)ah + (256.0f * (float)am + ((float)al - 8.0f * (float)s32)));
    }
    return x.u * acc;
}

// Q2_K super-block: chunk 0 = 16 scale bytes, chunks 1..4 = qs words (one per
// 16-element sub-block, bit-plane ordered), aux = d | dmin << 16
template <int P, int NB = 3>
__device__ __forceinline__ float sb_dot_q2k(const uint4 *c, uint32_t aux, const XSb &x, int part) {
    const float d = h2f_bits(aux), dmin = h2f_bits(aux >> 16);
    const uint4 c0 = NX_CH(0);
    const uint32_t scw[4] = {c0.x, c0.y, c0.z, c0.w};
    int bh = 0, bm = 0, bl = 0;
    float mn = 0.0f;
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
        int am = 0;
        if constexpr (NB == 3) {
            const uint4 mm = x.zm[j];
            am = dp4a_uu(p0, mm.x, 0);
            am = dp4a_uu(p1, mm.y, am);
            am = dp4a_uu(p2, mm.z, am);
            am = dp4a_uu(p3, mm.w, am);
        }
        int al = dp4a_uu(p0, l.x, 0);
        al = dp4a_uu(p1, l.y, al);
        al = dp4a_uu(p2, l.z, al);
        al = dp4a_uu(p3, l.w, al);
        const uint32_t sb = byte_of(scw[j >> 2], j & 3);
        const int sc = (int)(sb & 15u), m = (int)(sb >> 4);
        bh += sc * ah;
        bm += sc * am;
        bl += sc * al;
        mn += (float)m * (float)x.sz[j];
    }
    if constexpr (NB == 2) return x.u * (d * (256.0f * (float)bh + (float)bl) - dmin * mn);
    return x.u * (d * (65536.0f * (float)bh + (256.0f * (float)bm + (float)bl)) - dmin * mn);
}
#undef NX_CH

template <int FMT, int P, int NB = 3>
__device__ __forceinline__ float sb_dot(const uint4 *c, uint32_t aux, const XSb &x, int part) {
    if constexpr (FMT == 12) return sb_dot_q4k<P, NB>(c, x, part);
    else if constexpr (FMT == 8) return sb_dot_q80<P, NB>(c, x, part);
    else if constexpr (FMT == 2) return sb_dot_q40<P, NB>(c, x, part);
    else return sb_dot_q2k<P, NB>(c, aux, x, part);
}

// Shared-memory bytes of the prepared input of one token: zh[k], zm[k] (24-bit
// inputs only), zl[k], sz[k/16], u[k/256], padded to 16 bytes so every
// token's image is aligned.  NB = bytes per input element (3: 24-bit, 2: 16-bit).
__host__ __device__ __forceinline__ size_t tok_smem_bytes(int k, int nb = 3) {
    return ((size_t)nb * k + (size_t)4 * (k / 16) + (size_t)4 * (k / 256) + 15) / 16 * 16;
}

// The planes of one token's prepared image (tok_smem_bytes layout).
struct TokPlanes {
    uint32_t *zh, *zm, *zl;
    int *sz;
    float *u;
};
template <int NB>
__device__ __forceinline__ TokPlanes tok_planes(uint8_t *tb, int k) {
    TokPlanes t;
    t.zh = reinterpret_cast<uint32_t *>(tb);
    t.zm = NB == 3 ? reinterpret_cast<uint32_t *>(tb + k) : nullptr;
    t.zl = reinterpret_cast<uint32_t *>(tb + (NB - 1) * k);
    t.sz = reinterpret_cast<int *>(tb + NB * k);
    t.u = reinterpret_cast<float *>(tb + NB * k + 4 * (k / 16));
    return t;
}

// Prepare super-block s of one token: 24-bit (NB = 3) or 16-bit (NB = 2)
// quantization of x (times the RMSNorm weight when fused) from the lane's 8
// values v (elements 8*lane .. 8*lane+7).  16-bit inputs serve matrices
// whose inputs are normalized (RMSNorm outputs, attention outputs): one dp4a
// fewer per four weights; heavy-tailed inputs (SwiGLU outputs) keep 24 bits.  The quantization is scale-invariant, so RMSNorm's
// rstd is not needed here: the caller multiplies u[s] by rstd once the sum of
// squares, accumulated in *ss, is known.  (x*rstd)*w and rstd*(x*w) agree to
// f32 rounding, far below the 24-bit step.
template <int NB = 3>
__device__ __forceinline__ void prep_sb_vals(float (&v)[8], const float (&w)[8], bool has_w, int s, int lane,
                                             uint32_t *zh, uint32_t *zm, uint32_t *zl, int *sz, float *u,
                                             float *ss) {
#pragma unroll
    for (int i = 0; i < 8; i++) *ss += v[i] * v[i];
    if (has_w) {
#pragma unroll
        for (int i = 0; i < 8; i++) v[i] = v[i] * w[i];
    }
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; i++) amax = fmaxf(amax, fabsf(v[i]));
    amax = warp_max(amax);
    constexpr int ZMAX = NB == 3 ? 8388607 : 32767;
    constexpr float FZMAX = (float)ZMAX;
    const float inv = (amax > 0.0f && amax <= 3.0e38f) ? FZMAX / amax : 0.0f;
    int z[8], psum = 0;
#pragma unroll
    for (int i = 0; i < 8; i++) {
        // v * inv can round to 2^23 (2^15) for the largest element; the top byte is signed
        z[i] = max(-ZMAX, min(ZMAX, __float2int_rn(v[i] * inv)));
        psum += z[i];
    }
    constexpr int HS = NB == 3 ? 16 : 8;  // shift of the signed top byte
    uint32_t h0 = 0, h1 = 0, m0 = 0, m1 = 0, l0 = 0, l1 = 0;
#pragma unroll
    for (int i = 0; i < 4; i++) {
        h0 |= ((uint32_t)(z[i] >> HS) & 0xffu) << (8 * i);
        h1 |= ((uint32_t)(z[4 + i] >> HS) & 0xffu) << (8 * i);
        m0 |= ((uint32_t)(z[i] >> 8) & 0xffu) << (8 * i);
        m1 |= ((uint32_t)(z[4 + i] >> 8) & 0xffu) << (8 * i);
        l0 |= ((uint32_t)z[i] & 0xffu) << (8 * i);
        l1 |= ((uint32_t)z[4 + i] & 0xffu) << (8 * i);
    }
    const int wi = 64 * s + 2 * lane;
    zh[wi] = h0;
    zh[wi + 1] = h1;
    if constexpr (NB == 3) {
        zm[wi] = m0;
        zm[wi + 1] = m1;
    }
    zl[wi] = l0;
    zl[wi + 1] = l1;
    psum += __shfl_xor_sync(0xffffffffu, psum, 1);
    if ((lane & 1) == 0) sz[16 * s + (lane >> 1)] = psum;
    if (lane == 0) u[s] = amax / FZMAX;
}

// One warp prepares super-blocks warp, warp + W, ... of one token.  All of a
// pass's loads are issued before any is used (one memory round trip per
// kPrepBatch super-blocks instead of one per super-block).
constexpr int kPrepBatch = 4;
template <int W, int NB = 3>
__device__ __forceinline__ float prep_token(const float *__restrict__ x, const float *__restrict__ nw, int n_sb,
                                            int warp, int lane, uint32_t *zh, uint32_t *zm, uint32_t *zl, int *sz,
                                            float *u) {
    float ss = 0.0f;
    for (int base = warp; base < n_sb; base += W * kPrepBatch) {
        float4 xa[kPrepBatch], xb[kPrepBatch], wa[kPrepBatch], wb[kPrepBatch];
#pragma unroll
        for (int i = 0; i < kPrepBatch; i++) {
            const int s = base + i * W;
            if (s < n_sb) {
                const float4 *xp = reinterpret_cast<const float4 *>(x + 256 * s + 8 * lane);
                xa[i] = __ldcg(xp);
                xb[i] = __ldcg(xp + 1);
                if (nw) {
                    const float4 *wp = reinterpret_cast<const float4 *>(nw + 256 * s + 8 * lane);
                    wa[i] = __ldg(wp);
                    wb[i] = __ldg(wp + 1);
                }
            }
        }
#pragma unroll
        for (int i = 0; i < kPrepBatch; i++) {
            const int s = base + i * W;
            if (s < n_sb) {
                float v[8] = {xa[i].x, xa[i].y, xa[i].z, xa[i].w, xb[i].x, xb[i].y, xb[i].z, xb[i].w};
                float w[8] = {1, 1, 1, 1, 1, 1, 1, 1};
                if (nw) {
                    w[0] = wa[i].x; w[1] = wa[i].y; w[2] = wa[i].z; w[3] = wa[i].w;
                    w[4] = wb[i].x; w[5] = wb[i].y; w[6] = wb[i].z; w[7] = wb[i].w;
                }
                prep_sb_vals<NB>(v, w, nw != nullptr, s, lane, zh, zm, zl, sz, u, &ss);
            }
        }
    }
    return ss;
}

// Epilogue for one row (lane) of row group g and token t.
template <int EPI>
__device__ __forceinline__ void gemv_epilogue(const GemvParams &p, int g, int t, int lane, float tot) {
    const int row = 32 * g + lane;
    if constexpr (EPI == EPI_STORE) {
        if (row < p.n) p.y[(size_t)t * p.y_stride + row] = tot;
    } else if constexpr (EPI == EPI_ADD) {
        if (row < p.n) {
            // read through L2: in the persistent step kernel another SM wrote
            // this row earlier in the same launch
            float *yp = p.y + (size_t)t * p.y_stride + row;
            *yp = __ldcg(yp) + tot;
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
            const size_t base = kv_phys(q.pages, q.seq_ids[t], sq.slot) * kv_dim;
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
            key = ((unsigned long long)((unsigned)total_key(tot) ^ 0x80000000u) << 32) | (unsigned)(row + p.row_offset);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            unsigned long long other = __shfl_xor_sync(0xffffffffu, key, o);
            key = other > key ? other : key;
        }
        if (lane == 0 && key) atomicMax(&p.seqs[t].best, key);
    }
}



template <int FMT>
struct Ring {
    static constexpr int C = Fmt<FMT>::C;
    static constexpr int ITEM_BYTES = C * 512;
    static constexpr int AUX_BYTES = Fmt<FMT>::AUX ? 128 : 0;
#ifndef NX_GEMV_WARPS
#define NX_GEMV_WARPS 16
#endif
#ifndef NX_GEMV_SLOTS
#define NX_GEMV_SLOTS 2
#endif
#ifndef NX_GEMV_WARPS_Q8
#define NX_GEMV_WARPS_Q8 8
#endif
    // warps per CTA: 16 (measured 556 vs 502 tok/s for the 8B-shape b = 1
    // step over 8); Q8_0 tiles are twice as large, so their rings hold 8
    static constexpr int W = FMT == 8 ? NX_GEMV_WARPS_Q8 : NX_GEMV_WARPS;
    static constexpr int NST = NX_GEMV_SLOTS;  // ring slots per warp
    static constexpr int SLOT_BYTES = ITEM_BYTES + AUX_BYTES;
};

constexpr unsigned kMbarSpinLimit = 1u << 20;

template <int FMT, int M, int EPI, int NB>
__global__ void __launch_bounds__(Ring<FMT>::W * 32, 1) k_gemv(GemvParams p) {
    using R = Ring<FMT>;
    constexpr int W = R::W, NST = R::NST;
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ unsigned long long full[W][NST];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int k = p.k, n_sb = k >> 8;
    const int groups = (p.n + 31) / 32;
    const int S = p.ksplit;             // warps per team (1, 2, 4 or 8)
    const int teams = W / S;
    const int team = warp / S, r = warp % S;
    const int total_teams = gridDim.x * teams;
    const int gteam = blockIdx.x * teams + team;
    // this warp's super-blocks of every group: [s0, s1)
    const int per = (n_sb + S - 1) / S;
    const int s0 = min(n_sb, r * per), s1 = min(n_sb, s0 + per);
    const int n_item = s1 - s0;
    const int my_groups = gteam < groups ? (groups - gteam + total_teams - 1) / total_teams : 0;
    const int n_total = my_groups * n_item;   // items this warp streams

    uint8_t *ring = smem + (size_t)warp * NST * R::SLOT_BYTES;
    uint8_t *xs = smem + (size_t)W * NST * R::SLOT_BYTES;
    const size_t tok_bytes = tok_smem_bytes(k, NB);
    float *red = reinterpret_cast<float *>(xs + tok_bytes * M);      // [W][2][M][32]
    float *misc = red + W * 2 * M * 32;                              // [W*M]

    auto item_addr = [&](int j, long long &item) {
        const int gi = j / n_item, si = j % n_item;
        const long long g = (long long)gteam + (long long)gi * total_teams;
        item = g * n_sb + s0 + si;
    };
    auto issue = [&](int j) {  // lane 0: item j of this warp into slot j % NST
        long long item;
        item_addr(j, item);
        unsigned long long *bar = &full[warp][j % NST];
        uint8_t *dst = ring + (size_t)(j % NST) * R::SLOT_BYTES;
        mbar_expect_tx(bar, R::ITEM_BYTES + R::AUX_BYTES);
        tma_load_1d(dst, reinterpret_cast<const uint8_t *>(p.w_main) + (size_t)item * R::ITEM_BYTES, R::ITEM_BYTES,
                    bar);
        if constexpr (Fmt<FMT>::AUX)
            tma_load_1d(dst + R::ITEM_BYTES, reinterpret_cast<const uint8_t *>(p.w_aux) + (size_t)item * 128, 128,
                        bar);
    };

    if (lane == 0) {
        for (int i = 0; i < NST; i++) mbar_init(&full[warp][i], 1);
        mbar_init_fence();
    }
    __syncwarp();
    // Stream the first items before waiting on the previous grid.
    if (lane == 0)
        for (int j = 0; j < NST && j < n_total; j++) issue(j);
    if (p.pdl) {
        pdl_launch_dependents();
        pdl_wait();
    }

    // Prepare the whole input once (warp w takes super-blocks w, w+W, ...);
    // with a fused RMSNorm the sum of squares comes out of the same pass.
#pragma unroll
    for (int t = 0; t < M; t++) {
        const TokPlanes tp = tok_planes<NB>(xs + tok_bytes * t, k);
        float ss = prep_token<W, NB>(p.x + (size_t)t * p.x_stride, p.norm_w, n_sb, warp, lane, tp.zh, tp.zm, tp.zl,
                                     tp.sz, tp.u);
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
            float *u = tok_planes<NB>(xs + tok_bytes * t, k).u;
            for (int s = threadIdx.x; s < n_sb; s += W * 32) u[s] *= rstd;
        }
        __syncthreads();
    }

    // All warps of a team run the same number of groups, so the team barrier
    // below is reached the same number of times by each of them.
    int j = 0;
    for (int gi = 0; gi < my_groups; gi++) {
        const int g = gteam + gi * total_teams;
        float acc[M];
#pragma unroll
        for (int t = 0; t < M; t++) acc[t] = 0.0f;
        for (int si = 0; si < n_item; si++, j++) {
            const int slot = j % NST;
            // bounded wait for the item's bytes: a copy that never lands is reported
            unsigned n = 0;
            bool ok = true;
            while (!mbar_try_wait(&full[warp][slot], (unsigned)((j / NST) & 1))) {
                if (++n > kMbarSpinLimit) {
                    ok = false;
                    break;
                }
            }
            if (!ok) {
                if (lane == 0 && p.err) atomicExch(p.err, 1);
                acc[0] = __int_as_float(0x7fc00000);  // NaN marks the row group as failed
                j = n_total;                            // stop issuing
                break;
            }
            const int s_sb = s0 + si;
            const uint4 *cbase = reinterpret_cast<const uint4 *>(ring + (size_t)slot * R::SLOT_BYTES) + lane;
            uint32_t auxw = 0;
            if constexpr (Fmt<FMT>::AUX)
                auxw = reinterpret_cast<const uint32_t *>(ring + (size_t)slot * R::SLOT_BYTES + R::ITEM_BYTES)[lane];
#pragma unroll
            for (int t = 0; t < M; t++) {
                const TokPlanes tp = tok_planes<NB>(xs + tok_bytes * t, k);
                XSb xsb;
                xsb.zh = reinterpret_cast<const uint4 *>(tp.zh) + 16 * s_sb;
                xsb.zm = NB == 3 ? reinterpret_cast<const uint4 *>(tp.zm) + 16 * s_sb : nullptr;
                xsb.zl = reinterpret_cast<const uint4 *>(tp.zl) + 16 * s_sb;
                xsb.sz = tp.sz + 16 * s_sb;
                xsb.u = tp.u[s_sb];
                acc[t] += sb_dot<FMT, 1, NB>(cbase, auxw, xsb, 0);
            }
            // every lane has consumed the slot's values: refill it with item j + NST
            __syncwarp();
            if (lane == 0 && j + NST < n_total) issue(j + NST);
        }
        if (S == 1) {
#pragma unroll
            for (int t = 0; t < M; t++) gemv_epilogue<EPI>(p, g, t, lane, acc[t]);
        } else {
            // team reduction: partials meet in shared memory, the team's first warp adds them in order
            float *tred = red + (size_t)(team * S) * 2 * M * 32;   // [S][2][M][32]
            const int buf = gi & 1;
#pragma unroll
            for (int t = 0; t < M; t++) tred[((r * 2 + buf) * M + t) * 32 + lane] = acc[t];
            asm volatile("bar.sync %0, %1;" ::"r"(1 + team), "r"(S * 32) : "memory");
            if (r == 0) {
#pragma unroll
                for (int t = 0; t < M; t++) {
                    float tot = 0.0f;
                    for (int q = 0; q < S; q++) tot += tred[((q * 2 + buf) * M + t) * 32 + lane];
                    gemv_epilogue<EPI>(p, g, t, lane, tot);
                }
            }
        }
    }
}

// ---------------------------------------------------------------------------
template <int FMT>
static size_t gemv_smem_bytes(int k, int m, int nb = 3) {
    using R = Ring<FMT>;
    return (size_t)R::W * R::NST * R::SLOT_BYTES + tok_smem_bytes(k, nb) * m + (size_t)4 * R::W * 2 * m * 32 +
           (size_t)4 * R::W * m;
}

// bytes per prepared input element: 16-bit inputs on request, else 24-bit
__host__ __device__ __forceinline__ int gemv_nb(const GemvParams &p) { return p.x_bits == 16 ? 2 : 3; }

template <int FMT, int M, int EPI, int NB>
static cudaError_t launch_fmt_m_epi(const GemvParams &pin, cudaStream_t st) {
    using R = Ring<FMT>;
    GemvParams p = pin;
    const int groups = (p.n + 31) / 32;
    const int n_sb = p.k / 256;
    const size_t smem = gemv_smem_bytes<FMT>(p.k, M, NB);
    auto fn = k_gemv<FMT, M, EPI, NB>;
    if (smem > 220 * 1024) return cudaErrorInvalidValue;
    cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    int dev = 0;
    cudaGetDevice(&dev);
    static int sm_count[16] = {};
    if (dev < 16 && sm_count[dev] == 0) cudaDeviceGetAttribute(&sm_count[dev], cudaDevAttrMultiProcessorCount, dev);
    const int sms = dev < 16 && sm_count[dev] ? sm_count[dev] : 148;
    // Team size: the smallest that gives every warp of the GPU a row group,
    // keeping at least two super-blocks per warp.  One CTA per team set of
    // row groups while they all fit at once (no tail imbalance); beyond that
    // the CTAs are persistent.
    int S = 1;
    while (S < R::W && (long long)groups * S < (long long)sms * R::W && n_sb >= 2 * S) S *= 2;
    p.ksplit = S;
    const int teams = R::W / S;
    int per_sm = 1;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, R::W * 32, smem);
    if (e != cudaSuccess) return e;
    if (per_sm < 1) per_sm = 1;
    int grid = (groups + teams - 1) / teams;
    if (grid > per_sm * sms) grid = per_sm * sms;
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

template <int FMT, int M, int NB>
static cudaError_t launch_epi_nb(const GemvParams &p, cudaStream_t st) {
    switch (p.epi) {
    case EPI_STORE: return launch_fmt_m_epi<FMT, M, EPI_STORE, NB>(p, st);
    case EPI_ADD: return launch_fmt_m_epi<FMT, M, EPI_ADD, NB>(p, st);
    case EPI_SWIGLU: return launch_fmt_m_epi<FMT, M, EPI_SWIGLU, NB>(p, st);
    case EPI_QKV: return launch_fmt_m_epi<FMT, M, EPI_QKV, NB>(p, st);
    case EPI_ARGMAX: return launch_fmt_m_epi<FMT, M, EPI_ARGMAX, NB>(p, st);
    default: return cudaErrorInvalidValue;
    }
}

template <int FMT, int M>
static cudaError_t launch_epi(const GemvParams &p, cudaStream_t st) {
    return gemv_nb(p) == 2 ? launch_epi_nb<FMT, M, 2>(p, st) : launch_epi_nb<FMT, M, 3>(p, st);
}

// Tokens [t0, t0 + m) of a batch: per-token pointers move, shared ones stay.
static GemvParams token_slice(const GemvParams &p, int t0, int m) {
    GemvParams q = p;
    q.m = m;
    q.x = p.x + (size_t)t0 * p.x_stride;
    if (p.y) q.y = p.y + (size_t)t0 * p.y_stride;
    if (p.seqs) q.seqs = p.seqs + t0;
    if (p.qkv.seqs) q.qkv.seqs = p.qkv.seqs + t0;
    if (p.qkv.seq_ids) q.qkv.seq_ids = p.qkv.seq_ids + t0;
    if (p.qkv.q_out) q.qkv.q_out = p.qkv.q_out + (size_t)t0 * p.qkv.hq * p.qkv.head_dim;
    if (p.qkv.kv_scratch) q.qkv.kv_scratch = p.qkv.kv_scratch + (size_t)t0 * 2 * p.qkv.hkv * p.qkv.head_dim;
    return q;
}

template <int FMT>
cudaError_t launch_gemv_fmt(const GemvParams &p, cudaStream_t st) {
    // A batch whose prepared inputs do not fit next to the weight rings runs
    // as two launches of half the tokens.
    if (p.m > 1 && gemv_smem_bytes<FMT>(p.k, p.m, gemv_nb(p)) > 220 * 1024) {
        const int h = p.m / 2;
        cudaError_t e = launch_gemv_fmt<FMT>(token_slice(p, 0, h), st);
        if (e != cudaSuccess) return e;
        return launch_gemv_fmt<FMT>(token_slice(p, h, p.m - h), st);
    }
    switch (p.m) {
    case 1: return launch_epi<FMT, 1>(p, st);
    case 2: return launch_epi<FMT, 2>(p, st);
    case 4: return launch_epi<FMT, 4>(p, st);
    default: {
        // other batch sizes: slices of 4, then 2, then 1 tokens
        if (p.m <= 0) return cudaErrorInvalidValue;
        for (int t0 = 0; t0 < p.m;) {
            const int r = p.m - t0, c = r >= 4 ? 4 : r >= 2 ? 2 : 1;
            cudaError_t e = launch_gemv_fmt<FMT>(token_slice(p, t0, c), st);
            if (e != cudaSuccess) return e;
            t0 += c;
        }
        return cudaSuccess;
    }
    }
}

}  // namespace nx
