// kernels_gemm.cu -- activation preparation and launch of the tcgen05 GEMM
// (kernels_gemm.cuh) for batched decode and prefill.
#include <algorithm>

#include "kernels_gemm.cuh"

namespace nx {
namespace qg {

// Position of element e (0..255) of a Q4_K super-block inside its quarter
// stage: quarter e%128/32; low nibbles (e < 128) first, high nibbles second;
// inside a 4-byte word the byte order is 0,2,1,3 (see dq_q4k_quarter).
__device__ __forceinline__ void q4k_kpos(int e, int &quarter, int &pos) {
    const int b = e & 127, hi = e >> 7;
    quarter = b >> 5;
    const int i = (b & 31) >> 2, bw = b & 3;
    const int pw = ((bw & 1) << 1) | (bw >> 1);
    pos = hi * 32 + 4 * i + pw;
}

// 1024-thread CTAs, gridDim.y of them per token: optional RMSNorm
// ((x*rstd)*w, src/kernel/mod.rs:199-209), a power-of-two scale per token
// keeping |x| < 2^10 (so the 32-element sub-block sums stay below 2^15, well
// inside f16 range), the f16 hi/lo split, and the sub-block sums.  Every CTA
// of a token reads the whole row for its statistics (from L2; all of them
// get the same values) and then prepares its share of the super-blocks, four
// groups of 256 threads taking one super-block each at a time.  Image rows
// per quarter: tokens' hi halves (rows 0..NT-1), then lo halves (NT..2NT-1).
constexpr int kPrepThreads = 1024;
template <int FMT, int NT>
__global__ void __launch_bounds__(kPrepThreads) k_gemm_prep(const float *__restrict__ x, int x_stride,
                                                            const float *__restrict__ norm_w, float eps, int m, int k,
                                                            uint8_t *__restrict__ bimg, float *__restrict__ tok_scale,
                                                            int pdl) {
    if (pdl) {
        // the GEMM that follows may start its weight stream now; x is final
        // (and the previous GEMM has finished reading the image) after the wait
        pdl_launch_dependents();
        pdl_wait();
    }
    constexpr int NWP = kPrepThreads / 32;
    const int tok = blockIdx.x, tt = tok / NT, n = tok % NT;
    const int n_sb = k / 256;
    const int lane = threadIdx.x & 31;
    __shared__ float red_s[NWP], red_m[NWP];
    __shared__ float rstd_s, inv_s;
    const bool valid = tok < m;
    const float *xr = x + (size_t)tok * x_stride;
    if (valid) {
        float ss = 0.0f, mx = 0.0f;
        for (int i = threadIdx.x; i < k; i += kPrepThreads) {
            const float v = xr[i];
            ss += v * v;
            mx = fmaxf(mx, fabsf(norm_w ? v * norm_w[i] : v));
        }
        ss = warp_sum(ss);
        mx = warp_max(mx);
        if (lane == 0) {
            red_s[threadIdx.x >> 5] = ss;
            red_m[threadIdx.x >> 5] = mx;
        }
        __syncthreads();
        if (threadIdx.x == 0) {
            float s = 0.0f, M = 0.0f;
            for (int w = 0; w < NWP; w++) {
                s += red_s[w];
                M = fmaxf(M, red_m[w]);
            }
            const float rstd = norm_w ? 1.0f / sqrtf(s / (float)k + eps) : 1.0f;
            const float top = M * rstd;
            int e2 = 0;
            if (top > 0.0f && isfinite(top)) frexpf(top, &e2);
            // |x| < 2^e2 -> scaled by 2^(10-e2) stays below 2^10
            const float inv = top > 0.0f && isfinite(top) ? ldexpf(1.0f, 10 - e2) : 1.0f;
            rstd_s = rstd;
            inv_s = inv;
            if (blockIdx.y == 0) tok_scale[tok] = 1.0f / inv;
        }
        __syncthreads();
    }
    const float rstd = valid ? rstd_s : 1.0f, inv = valid ? inv_s : 1.0f;
    // thread tid of a 256-thread group handles element tid of its super-block
    const int tid = threadIdx.x & 255, warp = tid >> 5;
    for (int s = blockIdx.y * (kPrepThreads / 256) + (threadIdx.x >> 8); s < n_sb;
         s += gridDim.y * (kPrepThreads / 256)) {
        float v = 0.0f;
        if (valid) {
            v = xr[s * 256 + tid];
            if (norm_w) v = (v * rstd) * norm_w[s * 256 + tid];
            v *= inv;
        }
        const __half hi = __float2half_rn(v);
        const __half lo = __float2half_rn(v - __half2float(hi));
        uint8_t *base = bimg + ((size_t)tt * n_sb + s) * bimg_sb_bytes(NT);
        int q, pos;
        if constexpr (FMT == 12) {
            q4k_kpos(tid, q, pos);
        } else if constexpr (FMT == 10) {
            // Q2_K: sub-block j = tid/16 in quarter j/4; bit-plane k, bytes 0,2,1,3
            const int j = tid >> 4, i = tid & 15, k4 = i >> 2, b = i & 3;
            q = j >> 2;
            pos = 16 * (j & 3) + 4 * k4 + (((b & 1) << 1) | (b >> 1));
        } else if constexpr (FMT == 2) {
            // Q4_0: block tid/32 in quarter tid/64; low nibbles then high, bytes 0,2,1,3
            const int blk = tid >> 5, i = tid & 31, nib = i >> 4, wi = (i & 15) >> 2, b = i & 3;
            q = blk >> 1;
            pos = 32 * (blk & 1) + 16 * nib + 4 * wi + (((b & 1) << 1) | (b >> 1));
        } else {
            q = tid >> 6;  // natural K order
            pos = tid & 63;
        }
        // K-chunk (pos/8) of 2NT rows x 16 B; hi in row n, lo in row NT + n
        uint8_t *qb = base + q * NT * 256 + (pos >> 3) * NT * 32 + n * 16 + (pos & 7) * 2;
        *reinterpret_cast<__half *>(qb) = hi;
        *reinterpret_cast<__half *>(qb + NT * 16) = lo;
        if constexpr (!GemmFmt<FMT>::MIN) continue;
        uint8_t *mb = base + 4 * NT * 256;
        if constexpr (FMT == 10) {
            // Q2_K: sixteen 16-element sub-blocks, sums at K positions 0..15
            float sj = v;
#pragma unroll
            for (int o = 8; o > 0; o >>= 1) sj += __shfl_xor_sync(0xffffffffu, sj, o);
            if ((lane & 15) == 0) {
                const int j = tid >> 4;
                const __half sh = __float2half_rn(sj);
                const __half sl = __float2half_rn(sj - __half2float(sh));
                uint8_t *cb = mb + (j >> 3) * NT * 32 + n * 16 + (j & 7) * 2;
                *reinterpret_cast<__half *>(cb) = sh;
                *reinterpret_cast<__half *>(cb + NT * 16) = sl;
            }
            continue;
        }
        // sub-block sums (sub-block j = elements 32j..32j+31 = warp j): K
        // positions 0..7 of the min operand, positions 8..15 zero
        const float sj = warp_sum(v);
        if (lane == 0) {
            const __half sh = __float2half_rn(sj);
            const __half sl = __float2half_rn(sj - __half2float(sh));
            *reinterpret_cast<__half *>(mb + n * 16 + warp * 2) = sh;
            *reinterpret_cast<__half *>(mb + NT * 16 + n * 16 + warp * 2) = sl;
        }
        if (tid < 8) {
            *reinterpret_cast<__half *>(mb + NT * 32 + n * 16 + tid * 2) = __float2half_rn(0.0f);
            *reinterpret_cast<__half *>(mb + NT * 32 + NT * 16 + n * 16 + tid * 2) = __float2half_rn(0.0f);
        }
    }
}

static int sm_count_cached() {
    int dev = 0;
    cudaGetDevice(&dev);
    static int sm_count[16] = {};
    if (dev < 16 && sm_count[dev] == 0) cudaDeviceGetAttribute(&sm_count[dev], cudaDevAttrMultiProcessorCount, dev);
    return dev < 16 && sm_count[dev] ? sm_count[dev] : 148;
}

// Token tile of a GEMM: 16 or 32 tokens; 64 for the block formats (their
// 64-token tile fits the shared memory and needs no per-super-block
// epilogue) when the 128-row tiles alone cover the SMs.  Matrices with fewer
// row tiles fill the machine by splitting K, and there the shorter units of
// the 64-token tile measured slower than two 32-token passes.
static int token_tile(int fmt, int m, int n) {
    const bool min_term = fmt == 12 || fmt == 10;  // GemmFmt<fmt>::MIN
    if (m <= 16) return 16;
    if (m <= 32 || min_term || (n + 127) / 128 < sm_count_cached()) return 32;
    return 64;
}

// Tiles and K split of one GEMM: the split minimises waves x (super-blocks
// per unit + one for the pipeline fill).
static GemmShape plan(int m, int n, int k, int nt) {
    GemmShape g;
    g.n_sb = k / 256;
    g.groups = (n + 31) / 32;
    g.n_tt = (m + nt - 1) / nt;
    g.n_rt = (g.groups + 3) / 4;
    g.mpad = g.n_tt * nt;
    g.npad = g.n_rt * 128;
    const int sms = sm_count_cached();
    const long long units0 = (long long)g.n_tt * g.n_rt;
    int best = 1;
    long long best_cost = -1;
    for (int s = 1; s <= 16 && s <= g.n_sb; s++) {
        const long long waves = (units0 * s + sms - 1) / sms;
        const long long cost = waves * ((g.n_sb + s - 1) / s + 1);
        if (best_cost < 0 || cost < best_cost) {
            best_cost = cost;
            best = s;
        }
    }
    g.nsplit = best;
    return g;
}

template <int FMT, int NT, int EPI>
static cudaError_t launch_nt_epi(const GemvParams &p, const GemmScratch &sc, cudaStream_t st) {
    using S = Smem<FMT, NT>;
    GemmShape g = plan(p.m, p.n, p.k, NT);
    const int sms = sm_count_cached();
    const long long units0 = (long long)g.n_tt * g.n_rt;
    if (g.nsplit > 1) {
        if (!p.part || !p.counters || (size_t)g.nsplit * g.mpad * g.npad > p.part_floats ||
            units0 > (long long)p.counter_slots)
            g.nsplit = 1;
    }
    const size_t need = (size_t)g.n_tt * g.n_sb * bimg_sb_bytes(NT);
    if (!sc.bimg || need > sc.bimg_bytes || !sc.tok_scale || (size_t)g.mpad > sc.tok_scale_floats)
        return cudaErrorInvalidValue;
    // CTAs per token: one super-block per 256-thread group where the row allows
    dim3 pg(g.mpad, std::max(1, std::min(8, g.n_sb / (kPrepThreads / 256))));
    // programmatic dependent launch: the prep waits for the previous kernel;
    // the GEMM allocates TMEM and streams weights during the prep and waits
    // for it before reading the image or writing results
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t pc = {};
    pc.gridDim = pg;
    pc.blockDim = dim3(kPrepThreads);
    pc.stream = st;
    pc.attrs = attr;
    pc.numAttrs = p.pdl ? 1 : 0;
    cudaError_t e = cudaLaunchKernelEx(&pc, k_gemm_prep<FMT, NT>, p.x, p.x_stride, p.norm_w, p.eps, p.m, p.k, sc.bimg,
                                       sc.tok_scale, p.pdl);
    if (e != cudaSuccess) return e;
    auto fn = k_qgemm<FMT, NT, EPI>;
    e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, S::TOTAL);
    if (e != cudaSuccess) return e;
    const long long units = units0 * g.nsplit;
    cudaLaunchConfig_t gc = {};
    gc.gridDim = dim3((unsigned)(units < sms ? units : sms));
    gc.blockDim = dim3(kThreads);
    gc.dynamicSmemBytes = S::TOTAL;
    gc.stream = st;
    gc.attrs = attr;
    gc.numAttrs = p.pdl ? 1 : 0;
    return cudaLaunchKernelEx(&gc, fn, p, g, (const uint8_t *)sc.bimg, (const float *)sc.tok_scale);
}

template <int FMT, int NT>
static cudaError_t launch_nt(const GemvParams &p, const GemmScratch &sc, cudaStream_t st) {
    switch (p.epi) {
    case EPI_STORE: return launch_nt_epi<FMT, NT, EPI_STORE>(p, sc, st);
    case EPI_ADD: return launch_nt_epi<FMT, NT, EPI_ADD>(p, sc, st);
    case EPI_SWIGLU: return launch_nt_epi<FMT, NT, EPI_SWIGLU>(p, sc, st);
    case EPI_QKV: return launch_nt_epi<FMT, NT, EPI_QKV>(p, sc, st);
    case EPI_ARGMAX: return launch_nt_epi<FMT, NT, EPI_ARGMAX>(p, sc, st);
    default: return cudaErrorInvalidValue;
    }
}

template <int FMT>
static cudaError_t launch_fmt(const GemvParams &p, const GemmScratch &sc, cudaStream_t st) {
    const int nt = token_tile(FMT, p.m, p.n);
    if constexpr (!GemmFmt<FMT>::MIN) {
        if (nt == 64) return launch_nt<FMT, 64>(p, sc, st);
    }
    return nt == 16 ? launch_nt<FMT, 16>(p, sc, st) : launch_nt<FMT, 32>(p, sc, st);
}

}  // namespace qg

bool gemm_supported(int fmt) { return fmt == 12 || fmt == 8 || fmt == 10 || fmt == 2; }

GemmScratchSize gemm_scratch_size(int m, int n, int k) {
    // enough for either token tile a format may choose at this m
    GemmScratchSize z = {};
    for (int fmt : {12, 8}) {
        const int nt = qg::token_tile(fmt, m, n);
        const qg::GemmShape g = qg::plan(m, n, k, nt);
        z.bimg_bytes = std::max(z.bimg_bytes, (size_t)g.n_tt * g.n_sb * qg::bimg_sb_bytes(nt));
        z.tok_scale_floats = std::max(z.tok_scale_floats, (size_t)g.mpad);
        z.part_floats = std::max(z.part_floats, g.nsplit > 1 ? (size_t)g.nsplit * g.mpad * g.npad : (size_t)0);
        z.counter_slots = std::max(z.counter_slots, (size_t)g.n_tt * g.n_rt);
    }
    return z;
}

cudaError_t launch_gemm(const GemvParams &p, const GemmScratch &sc, cudaStream_t st) {
    if (!gemm_supported(p.fmt) || p.k % 256 != 0 || p.n <= 0 || p.m <= 0) return cudaErrorInvalidValue;
    switch (p.fmt) {
    case 12: return qg::launch_fmt<12>(p, sc, st);
    case 8: return qg::launch_fmt<8>(p, sc, st);
    case 10: return qg::launch_fmt<10>(p, sc, st);
    default: return qg::launch_fmt<2>(p, sc, st);
    }
}

}  // namespace nx
