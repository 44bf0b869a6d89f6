// kernels_step.cu -- a whole single-token decode step as one persistent kernel.
//
// Replaces the per-token layer loop of decode_with_cache
// (src/engine/mod.rs:1087-1146, + transformer_logits :1032-1044): for every
// layer RMSNorm -> Q|K|V -> RoPE -> KV append -> GQA attention -> o_proj +
// residual -> RMSNorm -> gate|up -> SwiGLU -> down + residual, then the output
// norm, the LM head and the greedy argmax.  The token's embedding row is
// decoded by k_embed just before this kernel.
//
// Why one kernel.  At batch 1 every matrix is read once per token, so the
// step is bound by HBM -- 4.48 GB per token for the Llama-3-8B shape -- but
// as a chain of 160 dependent kernels most of them are short (o_proj is 9 MB,
// 1.4 us of HBM time) and each pays its launch, ramp and drain.  Here one CTA
// per SM stays resident for the whole step; dependent phases are separated by
// a grid barrier, and every warp starts streaming the next matrix's weights
// into its shared-memory ring before it arrives at the barrier (weights do not
// depend on activations), so HBM keeps working across phase boundaries.
//
// Phases.  A matrix phase (the GEMV of kernels_gemv.cuh: every CTA prepares
// the 24-bit input planes once, with the RMSNorm folded in, and each warp
// dots its items with dp4a) splits the matrix's items -- (row group of 32
// rows, 256-column super-block) tiles, Q8_0 tiles in two halves -- evenly
// over the CTAs (CTA c of C takes [c*T/C, (c+1)*T/C)) and each CTA's share
// evenly over its warps.  A row group one warp holds is finished by that
// warp; the partials of a group held by several warps meet in shared memory
// and are added in warp order; a group crossing a CTA boundary leaves each
// CTA's sum in global memory and the CTA whose items complete it (an atomic
// item count per group) adds them in CTA order -- all deterministic -- and
// runs the fused epilogue (RoPE + KV append, residual add, SwiGLU, logits +
// argmax, chosen at run time so all phases of a format share one body of
// code).  The attention phase runs attn_block (attn_block.cuh) over
// (KV head, context slice) blocks spread over the CTAs.
//
// Measured (Llama-3-8B shape, b = 1): correct (the parity tests run it), but
// 3.7 ms per token against 1.8 ms for the kernel-per-op graph, so it is
// opt-in (NEXUS_CFG_PERSISTENT).  Timestamps per phase show ~11 us of fixed
// cost per phase -- ~3 us from the barrier to the phase's first instruction,
// 2-3 us (6 for k = 14336) of input preparation, ~2 us of partial sums and
// ~2.5 us of grid barrier -- while separate kernels under programmatic
// dependent launch overlap much of that with the previous kernel.  Pulling
// the next matrix into L2 during a phase made both paths slower.
//
// Shared memory per CTA: W warps x 2 ring slots of 4.5 KB (one Q4_K/Q4_0
// tile, a Q2_K tile and its side words, or half a Q8_0 tile), then the input
// planes of the widest matrix (during attention, attn_block's scratch), then
// a few words for the RMSNorm.
//
// Every wait is bounded: a weight copy that does not land or a grid barrier
// that does not complete sets the device error flag; CTAs then stop issuing,
// wait (bounded) for their copies in flight and exit.
#include <cuda_runtime.h>

#include <algorithm>

#include "attn_block.cuh"
#include "common.cuh"
#include "kernels.h"
#include "kernels_gemv.cuh"

namespace nx {
namespace step {

constexpr int kSlot = 9 * 512;          // ring slot bytes
constexpr int kNst = 2;                 // ring slots per warp
constexpr int kAttnTps = 64;            // attention: tokens per context slice, at least
constexpr unsigned kSpin = 1u << 21;    // bounded waits (mbarrier polls, barrier polls)

struct Geo {
    int n_sb;         // super-blocks per row
    int halves;       // items per super-block (2 for Q8_0)
    int groups;       // row groups of 32 rows
    long long items;  // groups * n_sb * halves
};

__device__ __forceinline__ Geo geo(const StepMat &w) {
    Geo g;
    g.n_sb = w.k >> 8;
    g.halves = w.fmt == 8 ? 2 : 1;
    g.groups = (w.n + 31) >> 5;
    g.items = (long long)g.groups * g.n_sb * g.halves;
    return g;
}

// this warp's item range of a matrix: [i0, i1)
__device__ __forceinline__ void warp_range(long long items, long long nw, long long gw, long long &i0,
                                           long long &i1) {
    i0 = gw * items / nw;
    i1 = (gw + 1) * items / nw;
}

struct Ring {
    uint8_t *slots;                 // this warp's kNst slots
    unsigned long long *full;       // one mbarrier per slot
    unsigned issued, waited;        // items loaded / consumed through the ring in this launch
    unsigned phase_base;            // `waited` when the current phase began
};

// lane 0: stage item `it` of matrix w into the next slot
__device__ __forceinline__ void issue(Ring &r, const StepMat &w, long long it) {
    const int slot = r.issued % kNst;
    uint8_t *dst = r.slots + slot * kSlot;
    unsigned long long *bar = &r.full[slot];
    const uint8_t *base = reinterpret_cast<const uint8_t *>(w.main);
    if (w.fmt == 8) {
        // half h of super-block tile it/2: the scale chunk, then 8 code chunks
        const long long t = it >> 1;
        const int h = (int)(it & 1);
        const uint8_t *tile = base + t * (17 * 512);
        mbar_expect_tx(bar, kSlot);
        tma_load_1d(dst, tile, 512, bar);
        tma_load_1d(dst + 512, tile + (1 + 8 * h) * 512, 8 * 512, bar);
    } else if (w.fmt == 10) {
        mbar_expect_tx(bar, 5 * 512 + 128);
        tma_load_1d(dst, base + it * (5 * 512), 5 * 512, bar);
        tma_load_1d(dst + 5 * 512, reinterpret_cast<const uint8_t *>(w.aux) + it * 128, 128, bar);
    } else {
        mbar_expect_tx(bar, kSlot);
        tma_load_1d(dst, base + it * kSlot, kSlot, bar);
    }
    r.issued++;
}

// lane 0: keep the ring full with this phase's remaining items, then the next
// phase's first ones (cur: n_cur items from c0; next: n_next items from n0)
__device__ __forceinline__ void top_up(Ring &r, const StepMat &cur, long long c0, long long n_cur,
                                       const StepMat *next, long long n0, long long n_next) {
    while (r.issued - r.waited < (unsigned)kNst) {
        const long long k = (long long)(r.issued - r.phase_base);
        if (k < n_cur) {
            issue(r, cur, c0 + k);
        } else if (next && k - n_cur < n_next && k - n_cur < kNst) {
            issue(r, *next, n0 + (k - n_cur));
        } else {
            break;
        }
    }
}

// bounded wait for the oldest slot; false when the copy never lands
__device__ __forceinline__ bool wait_slot(Ring &r) {
    const int slot = r.waited % kNst;
    const unsigned parity = (r.waited / kNst) & 1u;
    unsigned n = 0;
    while (!mbar_try_wait(&r.full[slot], parity))
        if (++n > kSpin) return false;
    r.waited++;
    return true;
}

// Grid barrier over the CTAs of the launch (all resident: cooperative launch).
// bar[0] counts arrivals, bar[1] is the generation; the last CTA to arrive
// resets the count and advances the generation.  False when it gave up (after
// about a second of polling) or the error flag is set.  `extra` > 0 is the
// fault-injection hook of the error path: the barrier then waits for CTAs that
// do not exist, every CTA gives up, sets the flag and leaves.
__device__ __forceinline__ bool grid_sync(unsigned *bar, int *err, unsigned extra) {
    __shared__ int s_ok;
    __syncthreads();
    if (threadIdx.x == 0) {
        volatile unsigned *gen = bar + 1;
        const unsigned g0 = *gen;
        __threadfence();
        const unsigned prev = atomicAdd(bar, 1u);
        int ok = 1;
        if (prev == gridDim.x - 1 + extra) {
            bar[0] = 0u;
            __threadfence();
            atomicAdd(bar + 1, 1u);
        } else {
            unsigned n = 0;
            while (*gen == g0) {
                if (++n > kSpin) {
                    ok = 0;
                    atomicExch(err, 1);
                    break;
                }
                __nanosleep(64);
            }
        }
        __threadfence();
        s_ok = ok && *(volatile int *)err == 0;
    }
    __syncthreads();
    return s_ok != 0;
}

struct Smem {
    uint8_t *xs;     // input planes (GEMV phases) / attention scratch
    float *misc;     // [W] RMSNorm partial sums
    float *red;      // [W][2][32] warp partials of shared row groups
};

template <int FMT>
__device__ __forceinline__ float dot_item(const uint8_t *slot, const XSb &x, int h, int lane) {
    const uint4 *c = reinterpret_cast<const uint4 *>(slot) + lane;
    if constexpr (FMT == 12) return sb_dot_q4k<1>(c, x, 0);
    else if constexpr (FMT == 2) return sb_dot_q40<1>(c, x, 0);
    else if constexpr (FMT == 8) return sb_dot_q80_half(c, x, h);
    else return sb_dot_q2k<1>(c, reinterpret_cast<const uint32_t *>(slot + 5 * 512)[lane], x, 0);
}

// The fused epilogue of row group g (gemv_epilogue), chosen at run time so
// that every matrix phase of a format shares one body of code.
__device__ __noinline__ void epilogue_rt(const GemvParams &gp, int epi, int g, int lane, float tot) {
    switch (epi) {
    case EPI_QKV: gemv_epilogue<EPI_QKV>(gp, g, 0, lane, tot); break;
    case EPI_ADD: gemv_epilogue<EPI_ADD>(gp, g, 0, lane, tot); break;
    case EPI_SWIGLU: gemv_epilogue<EPI_SWIGLU>(gp, g, 0, lane, tot); break;
    case EPI_ARGMAX: gemv_epilogue<EPI_ARGMAX>(gp, g, 0, lane, tot); break;
    default: gemv_epilogue<EPI_STORE>(gp, g, 0, lane, tot); break;
    }
}

// Item ranges.  CTA c of the grid takes items [c*T/C, (c+1)*T/C) of a matrix;
// warp w of the CTA takes [c0 + w*n/W, c0 + (w+1)*n/W) of the CTA's n items.
struct Split {
    long long c0, c1;  // this CTA's items
    long long i0, i1;  // this warp's items
};
template <int W>
__device__ __forceinline__ Split split_items(long long T, int warp) {
    Split s;
    const long long C = gridDim.x;
    s.c0 = (long long)blockIdx.x * T / C;
    s.c1 = ((long long)blockIdx.x + 1) * T / C;
    const long long n = s.c1 - s.c0;
    s.i0 = s.c0 + warp * n / W;
    s.i1 = s.c0 + (warp + 1) * n / W;
    return s;
}

// The CTA's row groups that more than one warp holds, or that other CTAs share:
// the warps' partials (red[w][0] = the warp's first group, red[w][1] = its
// last) are added in warp order; a group inside the CTA gets its epilogue,
// a group crossing a CTA boundary leaves the CTA's sum in global memory and
// the CTA whose items complete the group (an atomic item count per group) adds
// the CTAs' sums in CTA order and runs the epilogue.  Deterministic.
template <int W>
__device__ __noinline__ void finish_groups(const StepParams &sp, const GemvParams &gp, int epi, const float *red,
                                           const Split sp_, long long T, long long ipg, int warp, int lane) {
    const long long c0 = sp_.c0, c1 = sp_.c1, n = c1 - c0;
    if (n <= 0) return;
    const long long gA = c0 / ipg, gB = (c1 - 1) / ipg;
    const long long C = gridDim.x;
    for (long long g = gA + warp; g <= gB; g += W) {
        const long long lo = max(g * ipg, c0), hi = min((g + 1) * ipg, c1);
        const bool inside = lo == g * ipg && hi == (g + 1) * ipg;
        // warps of this CTA holding items of g: owner(lo) .. owner(hi - 1),
        // owner(i) = ((i - c0 + 1) * W - 1) / n
        const long long wf = ((lo - c0 + 1) * W - 1) / n, wl = ((hi - c0) * W - 1) / n;
        if (wf == wl && inside) continue;  // one warp held the whole group and finished it
        float tot = 0.0f;
        for (long long w = wf; w <= wl; w++) {
            const long long s0 = c0 + w * n / W, s1 = c0 + (w + 1) * n / W;
            if (s1 <= s0) continue;
            tot += red[((int)w * 2 + (s0 / ipg == g ? 0 : 1)) * 32 + lane];
        }
        if (inside) {
            epilogue_rt(gp, epi, (int)g, lane, tot);
            continue;
        }
        const int cs = g == gA ? 0 : 1;
        sp.gpart[((size_t)blockIdx.x * 2 + cs) * 32 + lane] = tot;
        __threadfence();
        __syncwarp();
        unsigned last = 0;
        if (lane == 0) {
            const unsigned mine = (unsigned)(hi - lo);
            last = atomicAdd(&sp.gcounters[g], mine) + mine == (unsigned)ipg;
        }
        last = __shfl_sync(0xffffffffu, last, 0);
        if (!last) continue;
        __threadfence();
        // CTAs holding items of g: owner((g*ipg)) .. owner((g+1)*ipg - 1), owner(i) = ((i + 1) * C - 1) / T
        const long long cf = ((g * ipg + 1) * C - 1) / T, cl = (((g + 1) * ipg) * C - 1) / T;
        float all = 0.0f;
        for (long long c = cf; c <= cl; c++) {
            const long long s0 = c * T / C, s1 = (c + 1) * T / C;
            if (s1 <= s0) continue;
            all += __ldcg(&sp.gpart[((size_t)c * 2 + (s0 / ipg == g ? 0 : 1)) * 32 + lane]);
        }
        if (lane == 0) sp.gcounters[g] = 0u;
        epilogue_rt(gp, epi, (int)g, lane, all);
    }
}

// One matrix phase (every thread of the CTA calls it).  The ring state comes
// in and goes out by value so it stays in registers across the hot loop.  A
// wait that gives up sets the error flag, which the next grid barrier reports
// to every CTA.
template <int W, int FMT>
__device__ __noinline__ Ring gemv_phase(const StepParams &sp, const GemvParams &gp, const int epi, const StepMat w,
                                        const StepMat nxt, const bool has_next, Ring r, const Smem sm) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const Geo G = geo(w);
    const int k = w.k, n_sb = G.n_sb;
    const Split it_ = split_items<W>(G.items, warp);
    const long long i0 = it_.i0, i1 = it_.i1;
    long long n0 = 0, n1 = 0;
    if (has_next) {
        const Split nx = split_items<W>(geo(nxt).items, warp);
        n0 = nx.i0;
        n1 = nx.i1;
    }
    // the ring may still be loading this phase's first items: start on the input
    // ---- input planes (24-bit x per super-block), RMSNorm folded into u ----
    uint8_t *tb = sm.xs;
    uint32_t *zh = reinterpret_cast<uint32_t *>(tb);
    uint32_t *zm = reinterpret_cast<uint32_t *>(tb + k);
    uint32_t *zl = reinterpret_cast<uint32_t *>(tb + 2 * k);
    int *sz = reinterpret_cast<int *>(tb + 3 * k);
    float *u = reinterpret_cast<float *>(tb + 3 * k + 4 * (k / 16));
    const float *norm_w = gp.norm_w;
    float ss = prep_token<W>(gp.x, norm_w, n_sb, warp, lane, zh, zm, zl, sz, u);
    if (norm_w) {
        ss = warp_sum(ss);
        if (lane == 0) sm.misc[warp] = ss;
    }
    __syncthreads();
    if (norm_w) {
        float tot = 0.0f;
        for (int i = 0; i < W; i++) tot += sm.misc[i];
        // rstd = 1 / sqrt(variance + eps) (src/kernel/mod.rs:202-203)
        const float rstd = 1.0f / sqrtf(tot / (float)k + gp.eps);
        for (int s = threadIdx.x; s < n_sb; s += W * 32) u[s] *= rstd;
        __syncthreads();
    }

    // ---- this warp's items ----
    r.phase_base = r.waited;
    const long long ipg = (long long)n_sb * G.halves;
    const StepMat *nptr = has_next ? &nxt : nullptr;
    float acc = 0.0f;
    long long gcur = -1;
    bool ok = true;
    const long long gfirst = i0 / ipg;
    auto close_group = [&](long long g, float a) {
        if (i0 <= g * ipg && (g + 1) * ipg <= i1) epilogue_rt(gp, epi, (int)g, lane, a);  // the warp's own group
        else sm.red[(warp * 2 + (g == gfirst ? 0 : 1)) * 32 + lane] = a;
    };
    if (lane == 0) top_up(r, w, i0, i1 - i0, nptr, n0, n1 - n0);
    for (long long it = i0; it < i1; it++) {
        if (!wait_slot(r)) {
            ok = false;
            break;
        }
        const long long g = it / ipg;
        const int rem = (int)(it % ipg);
        const int s_sb = rem / G.halves, h = rem % G.halves;
        if (g != gcur) {
            if (gcur >= 0) close_group(gcur, acc);
            gcur = g;
            acc = 0.0f;
        }
        XSb xsb;
        xsb.zh = reinterpret_cast<const uint4 *>(zh) + 16 * s_sb;
        xsb.zm = reinterpret_cast<const uint4 *>(zm) + 16 * s_sb;
        xsb.zl = reinterpret_cast<const uint4 *>(zl) + 16 * s_sb;
        xsb.sz = sz + 16 * s_sb;
        xsb.u = u[s_sb];
        acc += dot_item<FMT>(r.slots + ((r.waited - 1) % kNst) * kSlot, xsb, h, lane);
        __syncwarp();
        if (lane == 0) top_up(r, w, i0, i1 - i0, nptr, n0, n1 - n0);
    }
    if (ok && gcur >= 0) close_group(gcur, acc);
    // every lane learns what lane 0 issued (the failure path drains it)
    r.issued = __shfl_sync(0xffffffffu, r.issued, 0);
    if (!ok && lane == 0) atomicExch(sp.err, 1);
    __syncthreads();
    if (ok) finish_groups<W>(sp, gp, epi, sm.red, it_, G.items, ipg, warp, lane);
    return r;
}

template <int W>
__device__ __forceinline__ Ring gemv_fmt(const StepParams &sp, const GemvParams &gp, int epi, const StepMat &w,
                                         const StepMat *next, Ring r, const Smem &sm) {
    const StepMat nx = next ? *next : w;
    switch (w.fmt) {
    case 12: return gemv_phase<W, 12>(sp, gp, epi, w, nx, next != nullptr, r, sm);
    case 8: return gemv_phase<W, 8>(sp, gp, epi, w, nx, next != nullptr, r, sm);
    case 2: return gemv_phase<W, 2>(sp, gp, epi, w, nx, next != nullptr, r, sm);
    default: return gemv_phase<W, 10>(sp, gp, epi, w, nx, next != nullptr, r, sm);
    }
}

// L2 prefetch of a small read-only vector (the next phase's RMSNorm weights)
// while the grid barrier is pending.
__device__ __forceinline__ void prefetch_l2(const void *p, size_t bytes) {
    const char *c = static_cast<const char *>(p);
    for (size_t off = (size_t)threadIdx.x * 128; off < bytes; off += (size_t)blockDim.x * 128)
        asm volatile("prefetch.global.L2 [%0];" ::"l"(c + off));
}

template <int W, int G>
__device__ __noinline__ void attn_phase(const StepParams &sp, const StepLayer &L, uint8_t *smem) {
    AttnParams a = {};
    a.hq = sp.hq;
    a.hkv = sp.hkv;
    a.head_dim = sp.head_dim;
    a.m = 1;
    a.q = sp.q;
    a.out = sp.attn;
    a.scale = 1.0f / sqrtf((float)sp.head_dim);
    a.k_cache = L.k_cache;
    a.v_cache = L.v_cache;
    a.pages = sp.pages;
    a.seqs = sp.seqs;
    a.seq_ids = sp.seq_ids;
    a.kv_dim = sp.hkv * sp.head_dim;
    a.nsplit = sp.attn_nsplit;
    a.part = sp.attn_part;
    a.counters = sp.attn_counters;
    auto &sa = *reinterpret_cast<AttnSmem<4, G, W> *>(smem);
    const int blocks = a.hkv * a.nsplit;
    for (int vb = blockIdx.x; vb < blocks; vb += gridDim.x) {
        attn_block<4, G, W, kAttnTps>(a, vb % a.hkv, vb / a.hkv, 0, sa);
        __syncthreads();
    }
}

// Bytes k_decode_step keeps for the input planes and the attention scratch.
template <int W, int G>
__host__ __device__ __forceinline__ size_t x_region_bytes(int kmax) {
    size_t xb = tok_smem_bytes(kmax);
    if (sizeof(AttnSmem<4, G, W>) > xb) xb = sizeof(AttnSmem<4, G, W>);
    return (xb + 127) / 128 * 128;
}

template <int W, int G>
__global__ void __launch_bounds__(W * 32, 1) k_decode_step(StepParams sp) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ unsigned long long full[W][kNst];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    Ring r;
    r.slots = smem + (size_t)warp * kNst * kSlot;
    r.full = full[warp];
    r.issued = r.waited = r.phase_base = 0;
    Smem sm;
    sm.xs = smem + (size_t)W * kNst * kSlot;
    sm.misc = reinterpret_cast<float *>(
        sm.xs + x_region_bytes<W, G>(max(sp.hidden, max(sp.hq * sp.head_dim, sp.ffn))));
    sm.red = sm.misc + 32;
    if (lane == 0) {
        for (int i = 0; i < kNst; i++) mbar_init(&full[warp][i], 1);
        mbar_init_fence();
    }
    __syncwarp();

    const int H = sp.hidden, D = sp.head_dim;
    const StepLayer *layers = sp.layers;
    bool ok = true;
    {
        // the first matrix's first items
        const Split s0 = split_items<W>(geo(layers[0].qkv).items, warp);
        if (lane == 0) top_up(r, layers[0].qkv, s0.i0, s0.i1 - s0.i0, nullptr, 0, 0);
    }
    for (int l = 0; l < sp.num_layers && ok; l++) {
        const StepLayer &L = layers[l];
        // attn_norm -> Q|K|V -> RoPE -> K, V into the cache
        GemvParams g = {};
        g.n = L.qkv.n;
        g.k = H;
        g.m = 1;
        g.x = sp.x_hidden;
        g.x_stride = H;
        g.norm_w = L.attn_norm;
        g.eps = sp.eps;
        g.qkv.hq = sp.hq;
        g.qkv.hkv = sp.hkv;
        g.qkv.head_dim = D;
        g.qkv.q_out = sp.q;
        g.qkv.rope_cos = sp.rope_cos;
        g.qkv.rope_sin = sp.rope_sin;
        g.qkv.k_cache = L.k_cache;
        g.qkv.v_cache = L.v_cache;
        g.qkv.pages = sp.pages;
        g.qkv.seqs = sp.seqs;
        g.qkv.seq_ids = sp.seq_ids;
        r = gemv_fmt<W>(sp, g, EPI_QKV, L.qkv, &L.o, r, sm);
        if (!(ok = grid_sync(sp.bar, sp.err, sp.bar_extra))) break;
        attn_phase<W, G>(sp, L, sm.xs);
        if (!(ok = grid_sync(sp.bar, sp.err, sp.bar_extra))) break;
        // o_proj + residual
        GemvParams o = {};
        o.n = H;
        o.k = sp.hq * D;
        o.m = 1;
        o.x = sp.attn;
        o.x_stride = o.k;
        o.y = sp.x_hidden;
        o.y_stride = H;
        r = gemv_fmt<W>(sp, o, EPI_ADD, L.o, &L.gateup, r, sm);
        prefetch_l2(L.ffn_norm, (size_t)H * 4);
        if (!(ok = grid_sync(sp.bar, sp.err, sp.bar_extra))) break;
        // ffn_norm -> gate|up -> SwiGLU
        GemvParams gu = {};
        gu.n = L.gateup.n;
        gu.k = H;
        gu.m = 1;
        gu.x = sp.x_hidden;
        gu.x_stride = H;
        gu.norm_w = L.ffn_norm;
        gu.eps = sp.eps;
        gu.y = sp.gated;
        gu.y_stride = sp.ffn;
        r = gemv_fmt<W>(sp, gu, EPI_SWIGLU, L.gateup, &L.down, r, sm);
        if (!(ok = grid_sync(sp.bar, sp.err, sp.bar_extra))) break;
        // down + residual
        GemvParams dn = {};
        dn.n = H;
        dn.k = sp.ffn;
        dn.m = 1;
        dn.x = sp.gated;
        dn.x_stride = sp.ffn;
        dn.y = sp.x_hidden;
        dn.y_stride = H;
        r = gemv_fmt<W>(sp, dn, EPI_ADD, L.down, l + 1 < sp.num_layers ? &layers[l + 1].qkv : &sp.head, r, sm);
        prefetch_l2(l + 1 < sp.num_layers ? layers[l + 1].attn_norm : sp.out_norm, (size_t)H * 4);
        ok = grid_sync(sp.bar, sp.err, sp.bar_extra);
    }
    if (ok) {
        // output norm -> LM head -> logits + greedy argmax (transformer_logits, greedy_token)
        GemvParams hd = {};
        hd.n = sp.head.n;
        hd.k = H;
        hd.m = 1;
        hd.x = sp.x_hidden;
        hd.x_stride = H;
        hd.norm_w = sp.out_norm;
        hd.eps = sp.eps;
        hd.y = sp.logits;
        hd.y_stride = sp.head.n;
        hd.seqs = sp.seqs;
        r = gemv_fmt<W>(sp, hd, EPI_ARGMAX, sp.head, nullptr, r, sm);
        ok = grid_sync(sp.bar, sp.err, sp.bar_extra);
    }
    if (ok) {
        if (blockIdx.x == 0 && threadIdx.x == 0) {
            // next token = argmax; the sequence advances by one (k_advance).
            // Read through L2: other SMs' atomics wrote `best` in this launch.
            DevSeq s = sp.seqs[0];
            s.best = __ldcg(&sp.seqs[0].best);
            const uint32_t tok = (uint32_t)(s.best & 0xffffffffull);
            sp.out_tokens[0] = tok;
            s.token = tok;
            s.position += 1;
            // the next slot of the sequence's ring of max_seq slots
            s.slot = s.slot + 1 == sp.max_seq ? 0u : s.slot + 1;
            s.seq_len = s.seq_len < sp.max_seq ? s.seq_len + 1 : sp.max_seq;
            sp.seqs[0] = s;
        }
        return;
    }
    // failure: no more copies; wait (bounded) for the ones in flight
    r.issued = __shfl_sync(0xffffffffu, r.issued, 0);
    while (r.waited < r.issued)
        if (!wait_slot(r)) break;
}

}  // namespace step

namespace {
using StepFn = void (*)(StepParams);

// (warps, query heads per KV head) pairs with a kernel: 16 warps for G <= 4,
// 8 warps for every G (G = 8 at 16 warps would not fit attn_block's scratch)
StepFn step_kernel(int W, int G) {
    if (W == 16) {
        switch (G) {
        case 1: return step::k_decode_step<16, 1>;
        case 2: return step::k_decode_step<16, 2>;
        case 4: return step::k_decode_step<16, 4>;
        default: return nullptr;
        }
    }
    switch (G) {
    case 1: return step::k_decode_step<8, 1>;
    case 2: return step::k_decode_step<8, 2>;
    case 4: return step::k_decode_step<8, 4>;
    case 8: return step::k_decode_step<8, 8>;
    default: return nullptr;
    }
}

size_t x_region(int W, int G, int kmax) {
    if (W == 16)
        return G == 1 ? step::x_region_bytes<16, 1>(kmax) : G == 2 ? step::x_region_bytes<16, 2>(kmax)
                                                                   : step::x_region_bytes<16, 4>(kmax);
    return G == 1 ? step::x_region_bytes<8, 1>(kmax)
                  : G == 2 ? step::x_region_bytes<8, 2>(kmax)
                           : G == 4 ? step::x_region_bytes<8, 4>(kmax) : step::x_region_bytes<8, 8>(kmax);
}
}  // namespace

cudaError_t step_plan(const StepParams &p, int device, StepLaunch *out) {
    if (p.head_dim != 128 || p.hkv <= 0 || p.hq % p.hkv) return cudaErrorNotSupported;
    const int G = p.hq / p.hkv;
    if (G != 1 && G != 2 && G != 4 && G != 8) return cudaErrorNotSupported;
    if (p.hidden % 256 || p.ffn % 256 || (p.hq * p.head_dim) % 256) return cudaErrorNotSupported;
    const int kmax = std::max(p.hidden, std::max(p.hq * p.head_dim, p.ffn));
    int sms = 0, optin = 0;
    cudaError_t e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, device);
    if (e != cudaSuccess) return e;
#ifndef NX_STEP_WARPS
#define NX_STEP_WARPS 16
#endif
    for (int W : {NX_STEP_WARPS, 8}) {
        StepFn fn = step_kernel(W, G);
        if (!fn) continue;
        // ring | input planes or attention scratch | RMSNorm sums
        const size_t smem = (size_t)W * step::kNst * step::kSlot + x_region(W, G, kmax) + 4 * 32 + 4 * W * 2 * 32;
        if (smem + 1024 > (size_t)optin) continue;  // + the kernel's static shared memory
        e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        int per_sm = 0;
        e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, W * 32, smem);
        if (e != cudaSuccess) return e;
        if (per_sm < 1) continue;
        out->warps = W;
        out->grid = sms;
        out->smem = smem;
        return cudaSuccess;
    }
    return cudaErrorNotSupported;
}

size_t step_gpart_floats(const StepLaunch &l) { return (size_t)l.grid * 2 * 32; }

cudaError_t launch_decode_step(const StepParams &p, const StepLaunch &l, cudaStream_t st) {
    StepFn fn = step_kernel(l.warps, p.hkv > 0 ? p.hq / p.hkv : 0);
    if (!fn) return cudaErrorNotSupported;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(l.grid);
    cfg.blockDim = dim3(l.warps * 32);
    cfg.dynamicSmemBytes = l.smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, fn, p);
}

}  // namespace nx
