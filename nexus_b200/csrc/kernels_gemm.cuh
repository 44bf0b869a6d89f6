// kernels_gemm.cuh -- dequant-to-shared-memory tcgen05 GEMM for batched
// decode and prefill (Y[m][n] = X[m][k] * W[n][k]^T over the row-interleaved
// weight tiles of tiles.cuh), used where the GEMV's per-token integer work
// would exceed the HBM budget (m >= 8).
//
// Exactness scheme for the super-block formats (Q4_K, Q2_K).  A weight is
// d*sc_j*q - dmin*m_j (src/gguf/mod.rs:1041-1049, 1076-1081) with integer
// q, sc_j, m_j.  The tensor cores multiply the exact small integers
//     A[r][k] = sc_j * q           (f16, <= 945: exact)
//     Amin[r][j] = m_j             (f16, <= 63: exact)
// with the activations split into two f16 halves x = hi + lo (22 significant
// bits), accumulating in f32 in TMEM per super-block:
//     D = sum_k A*x,  E = sum_j m_j * X_j  (X_j = sum of x over sub-block j)
// and the epilogue applies the per-row super-block scales in f32:
//     y += d*D - dmin*E.
// The activations are scaled per token by a power of two (kept in f16 range)
// and the scale is undone on output.  Everything beyond f32 rounding is the
// 2^-22 relative split of x, far inside the 1e-3 per-op bound.
// A tcgen05.mma of M=128, K=16 costs about the same issue time for any N up
// to 256, so the hi and lo halves of the tokens are stacked along N (one MMA
// of N = 2*NT per K step) rather than issued as two MMAs.
//
// Token tiles: 16 or 32 tokens; the block formats (Q8_0, Q4_0: no min term,
// no per-super-block epilogue scale) also run 64-token tiles (MMA N = 128),
// so a 64-token batch dequantizes every weight tile once.
// CTA roles (one CTA per SM, persistent over work units):
//   warps 0-7  dequantize (warp w: row group w&3 of the 128-row tile, half
//              w>>2 of each super-block) and run the epilogue (half w>>2 of
//              the token tile, TMEM lanes 32*(w&3)..)
//   warp 8     TMA bulk copies of the raw weight tiles (3-slot ring)
//   warp 9     TMEM allocation + TMA copies of the prepared activations
//   warp 10    tcgen05.mma issue (one thread)
// A work unit is (token tile, 128-row tile, K split); a super-block runs as 4
// quarter stages of 64 K (A: 128 x 64 f16 per stage in a 6-slot ring, B:
// NT*256 bytes per stage), so operands are staged ahead of the MMAs.  The
// super-block formats (Q4_K, Q2_K) keep A in tensor memory: the dequantizing
// warps write their 32 rows of a stage with one tcgen05.st (32 columns, two
// f16 per column) and the MMA reads A from there, which takes the 64 KB of
// dequantized A per super-block off shared memory (written once and read by
// every MMA); the block formats, whose 64-token tiles need all of tensor
// memory for accumulators, stage A in shared memory.  K-split partial sums
// meet in global scratch and the last CTA of a tile adds them in split order
// (deterministic) before the fused epilogue of kernels_gemv.cuh.
// Each warp signals a barrier once (after __syncwarp), so the arrival counts
// are warps, not threads.  Every wait is bounded: a wait that gives up sets the CTA's abort flag and
// the device error flag, later waits return at once, nothing new is issued,
// copies and MMAs in flight are waited for, and TMEM is freed before exit.
#pragma once
#include <cuda_fp16.h>

#include "kernels_gemv.cuh"

namespace nx {
namespace qg {

constexpr int kQuarters = 4;
constexpr int kDqWarps = 8;
constexpr int kThreads = (kDqWarps + 3) * 32;
constexpr unsigned kSpin = 1u << 22;

// Per-format scheme.  Super-block formats (Q4_K) multiply exact integers
// sc_j*q with a min operand and scale per super-block in the epilogue; the
// block formats (Q8_0) put the whole weight d*q into A as an exact f16 pair
// hi + lo (two MMAs per K step, no min term, no per-super-block scale).
template <int FMT>
struct GemmFmt;
#ifndef NX_Q4K_RAW_SLOTS
#define NX_Q4K_RAW_SLOTS 3
#endif
#ifndef NX_Q4K_STAGES
#define NX_Q4K_STAGES 6
#endif
template <>
struct GemmFmt<12> {  // Q4_K
    static constexpr bool MIN = true;
    static constexpr int A_MATS = 1;
    static constexpr int RAW_SLOTS = NX_Q4K_RAW_SLOTS, STAGES = NX_Q4K_STAGES;
};
template <>
struct GemmFmt<8> {  // Q8_0
    static constexpr bool MIN = false;
    static constexpr int A_MATS = 2;
    static constexpr int RAW_SLOTS = 2, STAGES = 3;
};
template <>
struct GemmFmt<10> {  // Q2_K: exact sc_j*q (<= 45) and sixteen 4-bit mins
    static constexpr bool MIN = true;
    static constexpr int A_MATS = 1;
    static constexpr int RAW_SLOTS = 4, STAGES = 6;
};
template <>
struct GemmFmt<2> {  // Q4_0: d*(q-8) as an exact f16 pair
    static constexpr bool MIN = false;
    static constexpr int A_MATS = 2;
    static constexpr int RAW_SLOTS = 3, STAGES = 3;
};

template <int FMT>
struct Raw {
    static constexpr int ITEM = Fmt<FMT>::C * 512;  // one row group x one super-block
    static constexpr int AUXB = Fmt<FMT>::AUX ? 128 : 0;
    static constexpr int SLOT = 4 * (ITEM + AUXB);  // four row groups
};

// Bytes of the prepared activations of one (token tile, super-block):
// 4 quarters x 8 K-chunks x 2NT rows (hi, lo) x 16 B, then the sub-block
// sums: 2 K-chunks x 2NT rows x 16 B (used by formats with a min term).
__host__ __device__ constexpr int bimg_sb_bytes(int nt) { return nt * 1088; }

// Shared memory: a ring of raw weight tiles (one super-block of 4 row
// groups per slot), a ring of quarter stages (the dequantized A matrix of 64 K
// and the prepared activations B of the same K; one full and one empty
// barrier per stage, signalled by the dequant warps and the B copy together),
// and two slots of the per-super-block min operands.
template <int FMT, int NT>
struct Smem {
    using GF = GemmFmt<FMT>;
    static constexpr int RSLOTS = GF::RAW_SLOTS, ASLOTS = GF::STAGES;
    static constexpr int BSLOTS = GF::STAGES;
    static constexpr int A_MAT = 8 * 128 * 16;          // one 128 x 64 f16 matrix
    static constexpr int A_BYTES = GF::A_MATS * A_MAT;  // one quarter stage
    // the super-block formats keep A in tensor memory (a_in_tmem): no
    // shared-memory A ring
    static constexpr int A_SMEM = GF::MIN ? 0 : A_BYTES;
    static constexpr int B_BYTES = NT * 256;
    static constexpr int AMIN_BYTES = 0;  // the min operand lives in tensor memory
    static constexpr int BMIN_BYTES = GF::MIN ? NT * 64 : 0;
    static constexpr int RAW = 0;
    static constexpr int A = RAW + RSLOTS * Raw<FMT>::SLOT;
    static constexpr int B = A + ASLOTS * A_SMEM;
    static constexpr int AMIN = B + BSLOTS * B_BYTES;
    static constexpr int BMIN = AMIN + 2 * AMIN_BYTES;
    static constexpr int TOTAL = BMIN + 2 * BMIN_BYTES + 1024;  // + alignment slack
};

struct GemmShape {
    int n_tt, n_rt, nsplit, n_sb, groups, mpad, npad;
};

__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
    // K-major, no swizzle: ((8 rows, n), 2 K-chunks) : ((16 B, SBO), LBO); version 1
    return (uint64_t)((saddr >> 4) & 0x3fffu) | ((uint64_t)((lbo >> 4) & 0x3fffu) << 16) |
           ((uint64_t)((sbo >> 4) & 0x3fffu) << 32) | (1ull << 46);
}
template <int N>
__device__ __forceinline__ constexpr uint32_t umma_idesc() {
    // D f32, A/B f16, both K-major, N, M = 128
    return (1u << 4) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
}
__device__ __forceinline__ void umma_f16(uint32_t dt, uint64_t ad, uint64_t bd, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %5, %5, %5}, p;\n}\n" ::"r"(dt),
        "l"(ad), "l"(bd), "r"(idesc), "r"(acc), "r"(0u)
        : "memory");
}
__device__ __forceinline__ void umma_commit(unsigned long long *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}
// Issue forms for a converged warp: one lane, chosen by elect.sync inside the
// same asm block, issues the instruction.  Issuing from a converged warp keeps
// the operands warp-uniform; a lone divergent thread issues several times slower.
__device__ __forceinline__ void umma_f16_w(uint32_t dt, uint64_t ad, uint64_t bd, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n .reg .pred p, q;\n elect.sync _|p, 0xffffffff;\n setp.ne.b32 q, %4, 0;\n"
        " @p tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %5, %5, %5}, q;\n}\n" ::"r"(dt),
        "l"(ad), "l"(bd), "r"(idesc), "r"(acc), "r"(0u)
        : "memory");
}
__device__ __forceinline__ void umma_commit_w(unsigned long long *bar) {
    asm volatile(
        "{\n .reg .pred p;\n elect.sync _|p, 0xffffffff;\n"
        " @p tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n}\n" ::"r"(smem_u32(bar))
        : "memory");
}
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void mbar_arrive(unsigned long long *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

template <int N>
__device__ __forceinline__ void tmem_ld(uint32_t taddr, float (&v)[N]);
template <>
__device__ __forceinline__ void tmem_ld<8>(uint32_t taddr, float (&v)[8]) {
    uint32_t r[8];
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                 : "r"(taddr));
#pragma unroll
    for (int i = 0; i < 8; i++) v[i] = __uint_as_float(r[i]);
}
template <>
__device__ __forceinline__ void tmem_ld<16>(uint32_t taddr, float (&v)[16]) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
#pragma unroll
    for (int i = 0; i < 16; i++) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Lane i of the warp writes v[0..31] to columns taddr.col .. +31 of TMEM lane
// taddr.lane + i (the warp's 32-lane quarter).
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&v)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
        "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
        "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]),
        "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]), "r"(v[16]),
        "r"(v[17]), "r"(v[18]), "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]), "r"(v[24]),
        "r"(v[25]), "r"(v[26]), "r"(v[27]), "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31])
        : "memory");
}
// Lane i of the warp writes v[0..7] to columns taddr.col .. +7 of TMEM lane taddr.lane + i.
__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t (&v)[8]) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(taddr), "r"(v[0]),
                 "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7])
                 : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// MMA whose A operand is in tensor memory (lane = row, two f16 of K per
// column), issued by an elected lane of a converged warp.
__device__ __forceinline__ void umma_f16_ts_w(uint32_t dt, uint32_t at, uint64_t bd, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n .reg .pred p, q;\n elect.sync _|p, 0xffffffff;\n setp.ne.b32 q, %4, 0;\n"
        " @p tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, {%5, %5, %5, %5}, q;\n}\n" ::"r"(dt),
        "r"(at), "l"(bd), "r"(idesc), "r"(acc), "r"(0u)
        : "memory");
}

// Bounded mbarrier wait; false once this CTA has given up (abort set).
__device__ __forceinline__ bool bwait(unsigned long long *bar, unsigned parity, volatile int *abort_flag, int *err) {
    unsigned n = 0;
    while (!mbar_try_wait(bar, parity)) {
        if ((++n & 255u) == 0) {
            if (*abort_flag) return false;
            if (n > kSpin) {
                *abort_flag = 1;
                if (err) atomicExch(err, 2);
                return false;
            }
        }
    }
    return true;
}

__device__ __forceinline__ uint32_t lop_or(uint32_t w, uint32_t mask) {
    // (w & mask) | 0x64006400: two f16 values 1024 + field
    uint32_t r;
    asm("lop3.b32 %0, %1, %2, %3, 0xea;" : "=r"(r) : "r"(w), "r"(mask), "r"(0x64006400u));
    return r;
}
__device__ __forceinline__ uint32_t hfma2u(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t r;
    asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(c));
    return r;
}
__device__ __forceinline__ uint32_t f16x2_splat(float v) {
    const uint32_t h = __half_as_ushort(__float2half_rn(v));
    return h | (h << 16);
}

// Work unit u -> (token tile, row tile, split) and the split's super-blocks.
__device__ __forceinline__ void unit_coords(const GemmShape &g, int u, int &tt, int &rt, int &ks, int &s0, int &s1) {
    ks = u % g.nsplit;
    const int tile = u / g.nsplit;
    rt = tile % g.n_rt;
    tt = tile / g.n_rt;
    const int per = g.n_sb / g.nsplit, rem = g.n_sb % g.nsplit;
    s0 = ks * per + min(ks, rem);
    s1 = s0 + per + (ks < rem ? 1 : 0);
}

// Q4_K dequantization of one quarter (qs bytes 32q..32q+31 of the row) into
// the A stage: K order inside a quarter: positions 0..31 are the low nibbles
// (sub-block q), 32..63 the high nibbles (sub-block q+4); within each 4-byte
// word the order is bytes 0,2,1,3 (the prepared activations use the same
// order, so the product is unchanged).  Exact f16 products:
// (1024+q)*sc - 1024*sc and (1024+16q)*(sc/16) - 64*sc.
// The quarter as 32 TMEM columns: K-chunk c (8 elements) in columns
// 4c..4c+3, two f16 per column, in the K order of the prepared activations.
__device__ __forceinline__ void dq_q4k_quarter_cols(const uint32_t (&w)[8], uint32_t sc_lo, uint32_t sc_hi,
                                                    uint32_t (&v)[32]) {
    const uint32_t ml = f16x2_splat((float)sc_lo), bl = f16x2_splat(-1024.0f * (float)sc_lo);
    const uint32_t mh = f16x2_splat((float)sc_hi * 0.0625f), bh = f16x2_splat(-64.0f * (float)sc_hi);
#pragma unroll
    for (int kc = 0; kc < 4; kc++) {
        const uint32_t w0 = w[2 * kc], w1 = w[2 * kc + 1];
        const uint32_t w0s = w0 >> 8, w1s = w1 >> 8;
        v[4 * kc + 0] = hfma2u(lop_or(w0, 0x000f000fu), ml, bl);
        v[4 * kc + 1] = hfma2u(lop_or(w0s, 0x000f000fu), ml, bl);
        v[4 * kc + 2] = hfma2u(lop_or(w1, 0x000f000fu), ml, bl);
        v[4 * kc + 3] = hfma2u(lop_or(w1s, 0x000f000fu), ml, bl);
        v[16 + 4 * kc + 0] = hfma2u(lop_or(w0, 0x00f000f0u), mh, bh);
        v[16 + 4 * kc + 1] = hfma2u(lop_or(w0s, 0x00f000f0u), mh, bh);
        v[16 + 4 * kc + 2] = hfma2u(lop_or(w1, 0x00f000f0u), mh, bh);
        v[16 + 4 * kc + 3] = hfma2u(lop_or(w1s, 0x00f000f0u), mh, bh);
    }
}

// Q8_0 dequantization of one quarter (blocks 2q and 2q+1 of the row, K in
// natural order) into the stage's hi and lo matrices: w = d*q exactly as
// hi + lo, hi = f16(d*q), lo = f16(d*q - hi) (one fma).
__device__ __forceinline__ void dq_q80_quarter(const uint32_t (&w)[16], uint32_t d01, uint8_t *a_row) {
    const uint32_t bias = 0x64806480u;  // f16x2 (1152, 1152): (1024 + (q ^ 0x80)) - 1152 = q
#pragma unroll
    for (int b = 0; b < 2; b++) {
        const uint32_t dh = (d01 >> (16 * b)) & 0xffffu;
        const uint32_t d2 = dh | (dh << 16);
#pragma unroll
        for (int kc = 0; kc < 4; kc++) {
            uint32_t hv[4], lv[4];
#pragma unroll
            for (int h = 0; h < 2; h++) {
                const uint32_t u = w[8 * b + 2 * kc + h] ^ 0x80808080u;
                uint32_t p01, p23;
                asm("prmt.b32 %0, %1, 0x64646464, 0x4140;" : "=r"(p01) : "r"(u));
                asm("prmt.b32 %0, %1, 0x64646464, 0x4342;" : "=r"(p23) : "r"(u));
                uint32_t q01, q23;
                asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(q01) : "r"(p01), "r"(bias));
                asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(q23) : "r"(p23), "r"(bias));
                uint32_t h01, h23;
                asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(h01) : "r"(q01), "r"(d2));
                asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(h23) : "r"(q23), "r"(d2));
                hv[2 * h] = h01;
                hv[2 * h + 1] = h23;
                lv[2 * h] = hfma2u(q01, d2, h01 ^ 0x80008000u);
                lv[2 * h + 1] = hfma2u(q23, d2, h23 ^ 0x80008000u);
            }
            const int chunk = 4 * b + kc;
            *reinterpret_cast<uint4 *>(a_row + chunk * 2048) = make_uint4(hv[0], hv[1], hv[2], hv[3]);
            *reinterpret_cast<uint4 *>(a_row + 16384 + chunk * 2048) = make_uint4(lv[0], lv[1], lv[2], lv[3]);
        }
    }
}

// Q2_K dequantization of one quarter (sub-blocks 4q..4q+3, one tile word
// each; bits 2k..2k+1 of byte b are element 16j+4k+b) into exact f16
// sc_j*q.  K order inside a sub-block: bit-plane k, bytes 0,2,1,3; as 32
// TMEM columns (K-chunk c in columns 4c..4c+3).
__device__ __forceinline__ void dq_q2k_quarter_cols(const uint32_t (&w)[4], uint32_t sc4, uint32_t (&v)[32]) {
#pragma unroll
    for (int jj = 0; jj < 4; jj++) {
        const float sc = (float)((sc4 >> (8 * jj)) & 0xfu);
        const uint32_t ms = f16x2_splat(sc), bs = f16x2_splat(-1024.0f * sc);
#pragma unroll
        for (int k = 0; k < 4; k++) {
            v[8 * jj + 2 * k] = hfma2u(lop_or(w[jj] >> (2 * k), 0x00030003u), ms, bs);
            v[8 * jj + 2 * k + 1] = hfma2u(lop_or(w[jj] >> (2 * k + 8), 0x00030003u), ms, bs);
        }
    }
}

// Q4_0 dequantization of one quarter (blocks 2q, 2q+1; element i of a block
// is the low nibble of byte i%16 for i < 16, else the high nibble) into the
// stage's hi and lo matrices: w = d*(q-8) exactly as hi + lo.  K order per
// block: low nibbles then high nibbles, bytes 0,2,1,3 inside each word.
__device__ __forceinline__ void dq_q40_quarter(const uint32_t (&w)[8], uint32_t d01, uint8_t *a_row) {
    const uint32_t bias = 0x64086408u;  // f16x2 (1032, 1032): (1024 + q) - 1032 = q - 8
#pragma unroll
    for (int b = 0; b < 2; b++) {
        const uint32_t dh = (d01 >> (16 * b)) & 0xffffu;
        const uint32_t d2 = dh | (dh << 16);
#pragma unroll
        for (int nib = 0; nib < 2; nib++) {
#pragma unroll
            for (int kc = 0; kc < 2; kc++) {
                uint32_t hv[4], lv[4];
#pragma unroll
                for (int h = 0; h < 2; h++) {
                    const uint32_t x = w[4 * b + 2 * kc + h] >> (4 * nib);
                    uint32_t q02 = lop_or(x, 0x000f000fu), q13 = lop_or(x >> 8, 0x000f000fu);
                    asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(q02) : "r"(q02), "r"(bias));
                    asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(q13) : "r"(q13), "r"(bias));
                    uint32_t h02, h13;
                    asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(h02) : "r"(q02), "r"(d2));
                    asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(h13) : "r"(q13), "r"(d2));
                    hv[2 * h] = h02;
                    hv[2 * h + 1] = h13;
                    lv[2 * h] = hfma2u(q02, d2, h02 ^ 0x80008000u);
                    lv[2 * h + 1] = hfma2u(q13, d2, h13 ^ 0x80008000u);
                }
                const int chunk = 4 * b + 2 * nib + kc;
                *reinterpret_cast<uint4 *>(a_row + chunk * 2048) = make_uint4(hv[0], hv[1], hv[2], hv[3]);
                *reinterpret_cast<uint4 *>(a_row + 16384 + chunk * 2048) = make_uint4(lv[0], lv[1], lv[2], lv[3]);
            }
        }
    }
}

template <int FMT, int NT, int EPI>
__global__ void __launch_bounds__(kThreads, 1)
    k_qgemm(GemvParams p, GemmShape g, const uint8_t *__restrict__ bimg, const float *__restrict__ tok_scale) {
    using GF = GemmFmt<FMT>;
    static_assert(NT == 16 || NT == 32 || (NT == 64 && !GF::MIN), "token tile");
    using S = Smem<FMT, NT>;
    using R = Raw<FMT>;
    constexpr int H = NT / 2;  // tokens per epilogue warp
    constexpr int NB = S::BSLOTS;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    constexpr int kRawSlots = S::RSLOTS, kASlots = S::ASLOTS;
    __shared__ unsigned long long raw_full[kRawSlots], raw_empty[kRawSlots];
    __shared__ unsigned long long st_full[kASlots], st_empty[kASlots];
    __shared__ unsigned long long mn_full[2], mn_empty[2];
    __shared__ unsigned long long acc_full[2], acc_empty[2], mma_done;
    __shared__ uint32_t tmem_base_s;
    __shared__ volatile int abort_s;
    __shared__ int last_s;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n_units = g.n_tt * g.n_rt * g.nsplit;
    // per accumulator buffer: D (2NT columns: hi tokens, lo tokens), E (2NT);
    // the super-block formats add their A stages (32 columns each) after the
    // accumulators; allocations are powers of two
    constexpr uint32_t kAccCols = 8 * NT;
    constexpr uint32_t kACol = kAccCols;  // first A stage column
    constexpr uint32_t kTmemCols = GF::MIN ? 512u : kAccCols;
    // and the two min-operand stages (8 columns each: K = 16 of one MMA)
    constexpr uint32_t kMinCol = kACol + 32 * S::ASLOTS;
    static_assert(!GF::MIN || kMinCol + 16 <= 512, "A stages exceed tensor memory");

    if (threadIdx.x == 0) {
        for (int i = 0; i < kRawSlots; i++) {
            mbar_init(&raw_full[i], 1);
            mbar_init(&raw_empty[i], kDqWarps);
        }
        for (int i = 0; i < kASlots; i++) {
            mbar_init(&st_full[i], 4 + 1);  // 4 dequant warps + the activation copy
            mbar_init(&st_empty[i], 1);
        }
        for (int i = 0; i < 2; i++) {
            mbar_init(&mn_full[i], 4 + 1);
            mbar_init(&mn_empty[i], 1);
            mbar_init(&acc_full[i], 1);
            mbar_init(&acc_empty[i], kDqWarps);
        }
        mbar_init(&mma_done, 1);
        abort_s = 0;
        mbar_init_fence();
    }
    if (warp == 9) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_base_s)),
                     "r"(kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_base_s;

    if (warp == 8) {
        // ---- raw weight tiles: 4 row groups of one super-block per slot (whole warp, elected issue) ----
        unsigned n = 0;
        bool ok = true;
        for (int u = blockIdx.x; u < n_units && ok; u += gridDim.x) {
            int tt, rt, ks, s0, s1;
            unit_coords(g, u, tt, rt, ks, s0, s1);
            for (int s = s0; s < s1; s++, n++) {
                const int slot = n % kRawSlots;
                ok = __all_sync(0xffffffffu, bwait(&raw_empty[slot], ((n / kRawSlots) & 1) ^ 1, &abort_s, p.err));
                if (!ok) break;
                const int ng = min(4, g.groups - 4 * rt);
                expect_tx_w(&raw_full[slot], (unsigned)(ng * (R::ITEM + R::AUXB)));
                uint8_t *dst = smem + S::RAW + slot * R::SLOT;
                for (int gi = 0; gi < ng; gi++) {
                    const size_t item = (size_t)(4 * rt + gi) * g.n_sb + s;
                    tma_load_1d_w(dst + gi * R::ITEM, reinterpret_cast<const uint8_t *>(p.w_main) + item * R::ITEM,
                                  R::ITEM, &raw_full[slot]);
                    if constexpr (R::AUXB > 0)
                        tma_load_1d_w(dst + 4 * R::ITEM + gi * R::AUXB,
                                      reinterpret_cast<const uint8_t *>(p.w_aux) + item * R::AUXB, R::AUXB,
                                      &raw_full[slot]);
                }
            }
        }
        // copies still in flight land before the CTA exits
        if (lane == 0) {
            for (int sl = 0; sl < kRawSlots; sl++) {
                if ((unsigned)sl < n) {
                    const unsigned fills = (n - 1 - sl) / kRawSlots + 1;
                    unsigned k = 0;
                    while (!mbar_try_wait(&raw_full[sl], (fills - 1) & 1) && ++k < kSpin) {
                    }
                }
            }
        }
    } else if (warp == 9) {
        // ---- prepared activations: one quarter per slot, sub-block sums per super-block ----
        if (p.pdl) pdl_wait();  // the image is the previous kernel's output
        unsigned n = 0, c = 0;
        bool ok = true;
        for (int u = blockIdx.x; u < n_units && ok; u += gridDim.x) {
            int tt, rt, ks, s0, s1;
            unit_coords(g, u, tt, rt, ks, s0, s1);
            for (int s = s0; s < s1 && ok; s++, n++) {
                const uint8_t *src = bimg + ((size_t)tt * g.n_sb + s) * bimg_sb_bytes(NT);
                for (int q = 0; q < kQuarters; q++, c++) {
                    const int slot = c % NB;
                    ok = __all_sync(0xffffffffu, bwait(&st_empty[slot], ((c / NB) & 1) ^ 1, &abort_s, p.err));
                    if (!ok) break;
                    expect_tx_w(&st_full[slot], S::B_BYTES);
                    tma_load_1d_w(smem + S::B + slot * S::B_BYTES, src + q * S::B_BYTES, S::B_BYTES, &st_full[slot]);
                    if (GF::MIN && q == 0) {
                        const int ms = n & 1;
                        ok = __all_sync(0xffffffffu, bwait(&mn_empty[ms], ((n >> 1) & 1) ^ 1, &abort_s, p.err));
                        if (!ok) break;
                        expect_tx_w(&mn_full[ms], S::BMIN_BYTES);
                        tma_load_1d_w(smem + S::BMIN + ms * S::BMIN_BYTES, src + kQuarters * S::B_BYTES,
                                      S::BMIN_BYTES, &mn_full[ms]);
                    }
                }
            }
        }
        // copies still in flight land before the CTA exits
        if (lane == 0) {
            for (int sl = 0; sl < NB; sl++) {
                if ((unsigned)sl < c) {
                    const unsigned fills = (c - 1 - sl) / NB + 1;
                    unsigned k = 0;
                    while (!mbar_try_wait(&st_full[sl], (fills - 1) & 1) && ++k < kSpin) {
                    }
                }
            }
            for (int ms = 0; ms < 2 && GF::MIN; ms++) {
                if ((unsigned)ms < n) {
                    const unsigned fills = (n - 1 - ms) / 2 + 1;
                    unsigned k = 0;
                    while (!mbar_try_wait(&mn_full[ms], (fills - 1) & 1) && ++k < kSpin) {
                    }
                }
            }
        }
    } else if (warp == 10) {
        // ---- MMA issue (whole warp, elected lane) ----
        constexpr uint32_t idesc = umma_idesc<2 * NT>();
        const uint32_t a0 = smem_u32(smem + S::A), b0 = smem_u32(smem + S::B);
        const uint32_t bmin0 = smem_u32(smem + S::BMIN);
        unsigned n = 0, c = 0, nu = 0;
        bool ok = true;
        for (int u = blockIdx.x; u < n_units && ok; u += gridDim.x, nu++) {
            int tt, rt, ks, s0, s1;
            unit_coords(g, u, tt, rt, ks, s0, s1);
            if constexpr (!GF::MIN) {
                // block formats: one accumulator per work unit
                const int ab = nu & 1;
                ok = __all_sync(0xffffffffu, bwait(&acc_empty[ab], ((nu >> 1) & 1) ^ 1, &abort_s, p.err));
                if (!ok) break;
                tc_fence_after();
            }
            for (int s = s0; s < s1 && ok; s++, n++) {
                const int ab = GF::MIN ? (int)(n & 1) : (int)(nu & 1);
                const uint32_t dcol = tmem + ab * 4 * NT, ecol = dcol + 2 * NT;
                if constexpr (GF::MIN) {
                    ok = __all_sync(0xffffffffu, bwait(&acc_empty[ab], ((n >> 1) & 1) ^ 1, &abort_s, p.err));
                    if (!ok) break;
                    tc_fence_after();
                }
                for (int q = 0; q < kQuarters; q++, c++) {
                    const int as = c % kASlots, bs = as;
                    ok = __all_sync(0xffffffffu, bwait(&st_full[as], (c / kASlots) & 1, &abort_s, p.err));
                    if (!ok) break;
                    tc_fence_after();
#pragma unroll
                    for (int kk = 0; kk < 4; kk++) {
                        const uint32_t bq = b0 + bs * S::B_BYTES + kk * 2 * NT * 32;
                        const uint64_t bd = umma_desc(bq, NT * 32, 128);
                        if constexpr (GF::MIN) {
                            // A in tensor memory: stage `as`, K step kk = 8 columns
                            umma_f16_ts_w(dcol, tmem + kACol + 32 * as + 8 * kk, bd, idesc, (q | kk) != 0);
                        } else {
#pragma unroll
                            for (int am = 0; am < GF::A_MATS; am++) {
                                const uint64_t ad =
                                    umma_desc(a0 + as * S::A_BYTES + am * S::A_MAT + kk * 2 * 2048, 2048, 128);
                                umma_f16_w(dcol, ad, bd, idesc, (q | kk | am) != 0 || s != s0);
                            }
                        }
                    }
                    umma_commit_w(&st_empty[as]);
                    if (GF::MIN && q == 0) {
                        const int ms = n & 1;
                        ok = __all_sync(0xffffffffu, bwait(&mn_full[ms], (n >> 1) & 1, &abort_s, p.err));
                        if (!ok) break;
                        tc_fence_after();
                        const uint32_t bm = bmin0 + ms * S::BMIN_BYTES;
                        umma_f16_ts_w(ecol, tmem + kMinCol + 8 * ms, umma_desc(bm, NT * 32, 128), idesc, 0);
                        umma_commit_w(&mn_empty[ms]);
                    }
                }
                if (GF::MIN && ok) umma_commit_w(&acc_full[ab]);
            }
            if (!GF::MIN && ok) umma_commit_w(&acc_full[nu & 1]);
        }
        // all MMAs issued so far have completed before TMEM is released
        umma_commit_w(&mma_done);
        if (lane == 0) {
            unsigned k = 0;
            while (!mbar_try_wait(&mma_done, 0) && ++k < kSpin) {
            }
        }
        __syncwarp();
    } else {
        // ---- dequantization + epilogue (warps 0-7) ----
        const int rg = warp & 3, half = warp >> 2;
        const int r = 32 * rg + lane;  // row inside the 128-row tile
        const uint32_t t_lane = (uint32_t)(32 * rg) << 16;
        unsigned n = 0;
        float pd = 0.0f, pdm = 0.0f;  // scales of the previous super-block
        // super-block formats: fold one super-block's D and E into acc with its scales
        auto epilogue_sb = [&](unsigned nn, float d, float dm, float (&acc)[H]) {
            if constexpr (!GF::MIN) return;
            const int ab = nn & 1;
            bwait(&acc_full[ab], (nn >> 1) & 1, &abort_s, p.err);
            __syncwarp();
            tc_fence_after();
            const uint32_t col = tmem + t_lane + ab * 4 * NT + half * H;
            constexpr int HM = GF::MIN ? H : 8;  // (block formats never get here)
            float dh[HM], dl[HM], eh[HM], el[HM];
            tmem_ld<HM>(col, dh);
            tmem_ld<HM>(col + NT, dl);
            tmem_ld<HM>(col + 2 * NT, eh);
            tmem_ld<HM>(col + 3 * NT, el);
            tmem_wait_ld();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acc_empty[ab]);
#pragma unroll
            for (int t = 0; t < HM; t++) acc[t] = fmaf(d, dh[t] + dl[t], fmaf(-dm, eh[t] + el[t], acc[t]));
        };
        // block formats: the accumulator of work unit nu (all its super-blocks)
        auto unit_acc = [&](unsigned nu, float (&acc)[H]) {
            const int ab = nu & 1;
            bwait(&acc_full[ab], (nu >> 1) & 1, &abort_s, p.err);
            __syncwarp();
            tc_fence_after();
            const uint32_t col = tmem + t_lane + ab * 4 * NT + half * H;
            constexpr int HC = H < 16 ? H : 16;
#pragma unroll
            for (int c0 = 0; c0 < H; c0 += HC) {
                float dh[HC], dl[HC];
                tmem_ld<HC>(col + c0, dh);
                tmem_ld<HC>(col + NT + c0, dl);
                tmem_wait_ld();
#pragma unroll
                for (int t = 0; t < HC; t++) acc[c0 + t] = dh[t] + dl[t];
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acc_empty[ab]);
        };
        // results of one work unit: the fused epilogue, or this split's partial
        // sums (the last split of the tile adds them in split order)
        bool waited = false;
        auto unit_output = [&](int tt, int rt, int ks, const float (&acc)[H]) {
            if (p.pdl && !waited) {
                pdl_wait();  // token scales, residuals and outputs follow the previous kernels
                waited = true;
            }
            const int grp = 4 * rt + rg;
            const int tok0 = tt * NT + half * H;
            if (g.nsplit == 1) {
                if (grp < g.groups) {
#pragma unroll
                    for (int t = 0; t < H; t++)
                        if (tok0 + t < p.m) gemv_epilogue<EPI>(p, grp, tok0 + t, lane, acc[t] * tok_scale[tok0 + t]);
                }
            } else {
                float *part = p.part + ((size_t)ks * g.mpad + tok0) * g.npad + 128 * rt + r;
#pragma unroll
                for (int t = 0; t < H; t++) __stcg(part + (size_t)t * g.npad, acc[t]);
                __threadfence();
                asm volatile("bar.sync 1, %0;" ::"r"(kDqWarps * 32) : "memory");
                if (threadIdx.x == 0) {
                    const unsigned tile = (unsigned)(tt * g.n_rt + rt);
                    last_s = atomicAdd(&p.counters[tile], 1u) == (unsigned)(g.nsplit - 1);
                    if (last_s) p.counters[tile] = 0;
                }
                asm volatile("bar.sync 1, %0;" ::"r"(kDqWarps * 32) : "memory");
                if (last_s) {
                    __threadfence();
                    if (grp < g.groups) {
                        const float *pp = p.part + (size_t)tok0 * g.npad + 128 * rt + r;
#pragma unroll
                        for (int t = 0; t < H; t++) {
                            float tot = 0.0f;
                            for (int k2 = 0; k2 < g.nsplit; k2++)
                                tot += __ldcg(pp + ((size_t)k2 * g.mpad + t) * g.npad);
                            if (tok0 + t < p.m) gemv_epilogue<EPI>(p, grp, tok0 + t, lane, tot * tok_scale[tok0 + t]);
                        }
                    }
                }
            }
        };
        // block formats finish a unit after dequantizing the next unit's first
        // super-block, so the MMAs of the unit's tail overlap that work
        bool pend = false;
        int p_tt = 0, p_rt = 0, p_ks = 0;
        unsigned p_nu = 0, nu = 0;
        auto finish_pending = [&]() {
            if (!pend) return;
            float acc[H];
            unit_acc(p_nu, acc);
            unit_output(p_tt, p_rt, p_ks, acc);
            pend = false;
        };
        for (int u = blockIdx.x; u < n_units; u += gridDim.x, nu++) {
            int tt, rt, ks, s0, s1;
            unit_coords(g, u, tt, rt, ks, s0, s1);
            float acc[H];
#pragma unroll
            for (int t = 0; t < H; t++) acc[t] = 0.0f;
            for (int s = s0; s < s1; s++, n++) {
                const int slot = n % kRawSlots;
                bwait(&raw_full[slot], (n / kRawSlots) & 1, &abort_s, p.err);
                const uint8_t *rawp = smem + S::RAW + slot * R::SLOT + rg * R::ITEM + lane * 16;
                float d = 1.0f, dm = 0.0f;
                if constexpr (FMT == 12) {
                    const uint4 c0 = *reinterpret_cast<const uint4 *>(rawp);
                    uint32_t wq[16];
#pragma unroll
                    for (int c = 0; c < 4; c++) {
                        const uint4 v = *reinterpret_cast<const uint4 *>(rawp + (1 + 4 * half + c) * 512);
                        wq[4 * c] = v.x;
                        wq[4 * c + 1] = v.y;
                        wq[4 * c + 2] = v.z;
                        wq[4 * c + 3] = v.w;
                    }
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&raw_empty[slot]);
                    d = h2f_bits(c0.x);
                    dm = h2f_bits(c0.x >> 16);
                    // unpack_q4_k_scales (src/gguf/mod.rs:1547-1554)
                    const uint32_t scl = c0.y & 0x3f3f3f3fu, mnl = c0.z & 0x3f3f3f3fu;
                    const uint32_t sch = (c0.w & 0x0f0f0f0fu) | ((c0.y >> 2) & 0x30303030u);
                    const uint32_t mnh = ((c0.w >> 4) & 0x0f0f0f0fu) | ((c0.z >> 2) & 0x30303030u);
#pragma unroll
                    for (int qq = 0; qq < 2; qq++) {
                        const int q = 2 * half + qq;
                        const unsigned c = 4 * n + q;
                        const int as = c % kASlots;
                        bwait(&st_empty[as], ((c / kASlots) & 1) ^ 1, &abort_s, p.err);
                        uint32_t w8[8];
#pragma unroll
                        for (int i = 0; i < 8; i++) w8[i] = wq[8 * qq + i];
                        uint32_t cols[32];
                        dq_q4k_quarter_cols(w8, byte_of(scl, q), byte_of(sch, q), cols);
                        tc_fence_after();  // the MMAs that read this stage have completed
                        tmem_st32(tmem + t_lane + kACol + 32 * as, cols);
                        tmem_wait_st();
                        tc_fence_before();
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&st_full[as]);
                        if (q == 0) {
                            // Amin row: m_0..m_7, then eight zeros
                            const int ms = n & 1;
                            bwait(&mn_empty[ms], ((n >> 1) & 1) ^ 1, &abort_s, p.err);
                            uint4 m0;
                            m0.x = __half_as_ushort(__float2half_rn((float)byte_of(mnl, 0))) |
                                   ((uint32_t)__half_as_ushort(__float2half_rn((float)byte_of(mnl, 1))) << 16);
                            m0.y = __half_as_ushort(__float2half_rn((float)byte_of(mnl, 2))) |
                                   ((uint32_t)__half_as_ushort(__float2half_rn((float)byte_of(mnl, 3))) << 16);
                            m0.z = __half_as_ushort(__float2half_rn((float)byte_of(mnh, 0))) |
                                   ((uint32_t)__half_as_ushort(__float2half_rn((float)byte_of(mnh, 1))) << 16);
                            m0.w = __half_as_ushort(__float2half_rn((float)byte_of(mnh, 2))) |
                                   ((uint32_t)__half_as_ushort(__float2half_rn((float)byte_of(mnh, 3))) << 16);
                            const uint32_t mc[8] = {m0.x, m0.y, m0.z, m0.w, 0u, 0u, 0u, 0u};
                            tc_fence_after();  // the min MMA that read this stage has completed
                            tmem_st8(tmem + t_lane + kMinCol + 8 * ms, mc);
                            tmem_wait_st();
                            tc_fence_before();
                            __syncwarp();
                            if (lane == 0) mbar_arrive(&mn_full[ms]);
                        }
                    }
                } else if constexpr (FMT == 10) {
                    // Q2_K: chunk 0 = sixteen scale bytes (sc | m << 4), chunk 1+q = the
                    // four sub-block words of quarter q, side word = d | dmin << 16
                    const uint4 c0 = *reinterpret_cast<const uint4 *>(rawp);
                    const uint4 qa = *reinterpret_cast<const uint4 *>(rawp + (1 + 2 * half) * 512);
                    const uint4 qb = *reinterpret_cast<const uint4 *>(rawp + (2 + 2 * half) * 512);
                    const uint32_t auxw = *reinterpret_cast<const uint32_t *>(
                        smem + S::RAW + slot * R::SLOT + 4 * R::ITEM + rg * R::AUXB + lane * 4);
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&raw_empty[slot]);
                    d = h2f_bits(auxw);
                    dm = h2f_bits(auxw >> 16);
                    const uint32_t scw[4] = {c0.x, c0.y, c0.z, c0.w};
#pragma unroll
                    for (int qq = 0; qq < 2; qq++) {
                        const int q = 2 * half + qq;
                        const unsigned c = 4 * n + q;
                        const int as = c % kASlots;
                        bwait(&st_empty[as], ((c / kASlots) & 1) ^ 1, &abort_s, p.err);
                        const uint4 wv = qq ? qb : qa;
                        const uint32_t w4[4] = {wv.x, wv.y, wv.z, wv.w};
                        uint32_t cols[32];
                        dq_q2k_quarter_cols(w4, scw[q] & 0x0f0f0f0fu, cols);
                        tc_fence_after();  // the MMAs that read this stage have completed
                        tmem_st32(tmem + t_lane + kACol + 32 * as, cols);
                        tmem_wait_st();
                        tc_fence_before();
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&st_full[as]);
                        if (q == 0) {
                            // Amin row: m_0..m_15 (the high nibbles of the scale bytes)
                            const int ms = n & 1;
                            bwait(&mn_empty[ms], ((n >> 1) & 1) ^ 1, &abort_s, p.err);
                            uint32_t mw[8];
#pragma unroll
                            for (int i = 0; i < 8; i++) {
                                const uint32_t sw = scw[i >> 1] >> (16 * (i & 1));
                                const float m0 = (float)((sw >> 4) & 0xfu), m1 = (float)((sw >> 12) & 0xfu);
                                mw[i] = __half_as_ushort(__float2half_rn(m0)) |
                                        ((uint32_t)__half_as_ushort(__float2half_rn(m1)) << 16);
                            }
                            tc_fence_after();  // the min MMA that read this stage has completed
                            tmem_st8(tmem + t_lane + kMinCol + 8 * ms, mw);
                            tmem_wait_st();
                            tc_fence_before();
                            __syncwarp();
                            if (lane == 0) mbar_arrive(&mn_full[ms]);
                        }
                    }
                } else if constexpr (FMT == 2) {
                    // Q4_0: chunk 0 = the eight block scales, chunk 1+b = qs of block b
                    const uint4 c0 = *reinterpret_cast<const uint4 *>(rawp);
                    uint32_t wq[16];
#pragma unroll
                    for (int c = 0; c < 4; c++) {
                        const uint4 v = *reinterpret_cast<const uint4 *>(rawp + (1 + 4 * half + c) * 512);
                        wq[4 * c] = v.x;
                        wq[4 * c + 1] = v.y;
                        wq[4 * c + 2] = v.z;
                        wq[4 * c + 3] = v.w;
                    }
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&raw_empty[slot]);
                    const uint32_t dsc[4] = {c0.x, c0.y, c0.z, c0.w};
#pragma unroll
                    for (int qq = 0; qq < 2; qq++) {
                        const int q = 2 * half + qq;
                        const unsigned c = 4 * n + q;
                        const int as = c % kASlots;
                        bwait(&st_empty[as], ((c / kASlots) & 1) ^ 1, &abort_s, p.err);
                        uint32_t w8[8];
#pragma unroll
                        for (int i = 0; i < 8; i++) w8[i] = wq[8 * qq + i];
                        dq_q40_quarter(w8, half ? dsc[2 + qq] : dsc[qq], smem + S::A + as * S::A_BYTES + r * 16);
                        fence_proxy_async_smem();
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&st_full[as]);
                    }
                } else {
                    // Q8_0: chunk 0 = the eight block scales, chunks 1+2b, 2+2b = qs of block b
                    const uint4 c0 = *reinterpret_cast<const uint4 *>(rawp);
                    uint32_t wq[32];
#pragma unroll
                    for (int c = 0; c < 8; c++) {
                        const uint4 v = *reinterpret_cast<const uint4 *>(rawp + (1 + 8 * half + c) * 512);
                        wq[4 * c] = v.x;
                        wq[4 * c + 1] = v.y;
                        wq[4 * c + 2] = v.z;
                        wq[4 * c + 3] = v.w;
                    }
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&raw_empty[slot]);
                    const uint32_t dsc[4] = {c0.x, c0.y, c0.z, c0.w};
#pragma unroll
                    for (int qq = 0; qq < 2; qq++) {
                        const int q = 2 * half + qq;
                        const unsigned c = 4 * n + q;
                        const int as = c % kASlots;
                        bwait(&st_empty[as], ((c / kASlots) & 1) ^ 1, &abort_s, p.err);
                        uint32_t w16[16];
#pragma unroll
                        for (int i = 0; i < 16; i++) w16[i] = wq[16 * qq + i];
                        dq_q80_quarter(w16, half ? dsc[2 + qq] : dsc[qq], smem + S::A + as * S::A_BYTES + r * 16);
                        fence_proxy_async_smem();
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&st_full[as]);
                    }
                }
                if constexpr (GF::MIN) {
                    if (s > s0) epilogue_sb(n - 1, pd, pdm, acc);
                    pd = d;
                    pdm = dm;
                } else if (s == s0) {
                    finish_pending();
                }
            }
            if constexpr (GF::MIN) {
                epilogue_sb(n - 1, pd, pdm, acc);
                unit_output(tt, rt, ks, acc);
            } else {
                pend = true;
                p_tt = tt;
                p_rt = rt;
                p_ks = ks;
                p_nu = nu;
            }
        }
        if constexpr (!GF::MIN) finish_pending();
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 9) {
        __syncwarp();
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
    }
}

}  // namespace qg
}  // namespace nx
