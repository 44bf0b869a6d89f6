// kernels_quant.cu -- bit-exact block-format kernels for sm_100a.
//
// Compiled with -fmad=false: every multiply and add below is rounded on its
// own, as in the reference (src/gguf/mod.rs:1049,1081 compute
// ((d*sc)*q) - (dmin*m) with four roundings).  Division is IEEE (prec-div).
//
//   dequant_raw   : GGUF blocks -> f32   (GgufReader::tensor_bytes_to_f32)
//   quantize      : f32 -> GGUF blocks   (QuantEngine::quantize_weights)
//   repack_tiles  : GGUF blocks -> row-interleaved tiles (tiles.cuh)
//   dequant_tiles : tiles -> f32, the inverse view (same bits as dequant_raw)
#include <cuda_runtime.h>

#include "common.cuh"
#include "kernels.h"
#include "quant_math.cuh"
#include "tiles.cuh"

namespace nx {

// one thread per output element
__global__ void k_dequant_raw(int fmt, const uint8_t *__restrict__ blocks, size_t n,
                              float *__restrict__ out) {
    size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    size_t stride = (size_t)gridDim.x * blockDim.x;
    int be = block_elems(fmt), bb = block_bytes(fmt);
    for (; i < n; i += stride) {
        size_t b = i / be;
        int j = (int)(i % be);
        out[i] = dequant_elem(fmt, blocks + b * bb, j);
    }
}

// one thread per block
__global__ void k_quantize(int fmt, const float *__restrict__ x, size_t n, uint8_t *__restrict__ out) {
    size_t b = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    int be = block_elems(fmt), bb = block_bytes(fmt);
    size_t nblocks = (n + be - 1) / be;
    if (b >= nblocks) return;
    float v[256];
    size_t s = b * be;
    int len = (int)((n - s) < (size_t)be ? (n - s) : (size_t)be);
    for (int i = 0; i < be; i++) v[i] = i < len ? x[s + i] : 0.0f;
    uint8_t *o = out + b * bb;
    if (fmt == Q8_0) quantize_block_q8_0(v, len, o);
    else if (fmt == Q4_0) quantize_block_q4_0(v, len, o);
    else if (fmt == Q4_K) quantize_block_q4_k(v, o);
    else if (fmt == Q2_K) quantize_block_q2_k(v, o);
}

// Copy 16 bytes from an unaligned byte source.
__device__ __forceinline__ uint4 load16(const uint8_t *p) {
    uint32_t w[4];
    for (int k = 0; k < 4; k++)
        w[k] = (uint32_t)p[4 * k] | ((uint32_t)p[4 * k + 1] << 8) | ((uint32_t)p[4 * k + 2] << 16) |
               ((uint32_t)p[4 * k + 3] << 24);
    return make_uint4(w[0], w[1], w[2], w[3]);
}

// One thread per (row, super-block).  Rows >= n are zero-filled.
__global__ void k_repack_tiles(int fmt, const uint8_t *__restrict__ raw, int n, int k,
                               uint4 *__restrict__ main, uint32_t *__restrict__ aux) {
    int sb_per_row = k / 256;
    int groups = (n + 31) / 32;
    long long t = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= (long long)groups * 32 * sb_per_row) return;
    int s = (int)(t % sb_per_row);
    int row = (int)(t / sb_per_row);
    int g = row / 32, lane = row % 32;
    TileGeom geo = tile_geom(fmt);
    uint4 *dst = main + ((size_t)(g * sb_per_row + s) * geo.chunks) * 32 + lane;
    uint32_t *adst = aux ? aux + (size_t)(g * sb_per_row + s) * 32 + lane : nullptr;
    if (row >= n) {
        for (int c = 0; c < geo.chunks; c++) dst[(size_t)c * 32] = make_uint4(0, 0, 0, 0);
        if (adst) *adst = 0;
        return;
    }
    size_t elem0 = (size_t)row * k + (size_t)s * 256;  // first element of this super-block
    if (fmt == Q4_K) {
        const uint8_t *b = raw + (elem0 / 256) * 144;
        for (int c = 0; c < 9; c++) dst[(size_t)c * 32] = load16(b + 16 * c);
    } else if (fmt == Q4_0 || fmt == Q8_0) {
        int bb = fmt == Q4_0 ? 18 : 34;
        const uint8_t *b0 = raw + (elem0 / 32) * bb;
        uint32_t sc[4];
        for (int i = 0; i < 4; i++) {
            const uint8_t *x0 = b0 + (size_t)(2 * i) * bb, *x1 = b0 + (size_t)(2 * i + 1) * bb;
            sc[i] = (uint32_t)x0[0] | ((uint32_t)x0[1] << 8) | ((uint32_t)x1[0] << 16) | ((uint32_t)x1[1] << 24);
        }
        dst[0] = make_uint4(sc[0], sc[1], sc[2], sc[3]);
        for (int blk = 0; blk < 8; blk++) {
            const uint8_t *qs = b0 + (size_t)blk * bb + 2;
            if (fmt == Q4_0) {
                dst[(size_t)(1 + blk) * 32] = load16(qs);
            } else {
                dst[(size_t)(1 + 2 * blk) * 32] = load16(qs);
                dst[(size_t)(2 + 2 * blk) * 32] = load16(qs + 16);
            }
        }
    } else if (fmt == Q2_K) {
        const uint8_t *b = raw + (elem0 / 256) * 84;
        dst[0] = load16(b);
        const uint8_t *qs = b + 16;
        uint32_t words[16];
        for (int j = 0; j < 16; j++) {
            uint32_t w = 0;
            for (int bi = 0; bi < 4; bi++)
                for (int kk = 0; kk < 4; kk++) {
                    int e = 16 * j + 4 * kk + bi;
                    uint32_t q = (qs[e / 4] >> ((e % 4) * 2)) & 3u;
                    w |= q << (8 * bi + 2 * kk);
                }
            words[j] = w;
        }
        for (int c = 0; c < 4; c++)
            dst[(size_t)(1 + c) * 32] = make_uint4(words[4 * c], words[4 * c + 1], words[4 * c + 2], words[4 * c + 3]);
        *adst = (uint32_t)b[80] | ((uint32_t)b[81] << 8) | ((uint32_t)b[82] << 16) | ((uint32_t)b[83] << 24);
    }
}

// Rebuild the reference block bytes of one super-block from its tile and decode
// element j with the reference formula.  One thread per element.
__global__ void k_dequant_tiles(int fmt, const uint4 *__restrict__ main, const uint32_t *__restrict__ aux,
                                int n, int k, float *__restrict__ out) {
    long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (long long)n * k) return;
    int row = (int)(i / k), col = (int)(i % k);
    int s = col / 256, j = col % 256;
    int sb_per_row = k / 256;
    int g = row / 32, lane = row % 32;
    TileGeom geo = tile_geom(fmt);
    const uint4 *src = main + ((size_t)(g * sb_per_row + s) * geo.chunks) * 32 + lane;
    auto byte_of = [&](int c, int b) -> uint8_t {
        uint4 v = src[(size_t)c * 32];
        uint32_t w = b < 4 ? v.x : b < 8 ? v.y : b < 12 ? v.z : v.w;
        return (uint8_t)(w >> (8 * (b & 3)));
    };
    uint8_t blk[144];
    if (fmt == Q4_K) {
        for (int c = 0; c < 9; c++)
            for (int b = 0; b < 16; b++) blk[16 * c + b] = byte_of(c, b);
        out[i] = dequant_elem(Q4_K, blk, j);
    } else if (fmt == Q4_0 || fmt == Q8_0) {
        int sub = j / 32;
        blk[0] = byte_of(0, 2 * sub);
        blk[1] = byte_of(0, 2 * sub + 1);
        if (fmt == Q4_0) {
            for (int b = 0; b < 16; b++) blk[2 + b] = byte_of(1 + sub, b);
        } else {
            for (int b = 0; b < 16; b++) blk[2 + b] = byte_of(1 + 2 * sub, b);
            for (int b = 0; b < 16; b++) blk[18 + b] = byte_of(2 + 2 * sub, b);
        }
        out[i] = dequant_elem(fmt, blk, j % 32);
    } else if (fmt == Q2_K) {
        for (int b = 0; b < 16; b++) blk[b] = byte_of(0, b);
        // only the crumb of element j is needed: dequant_elem reads no other
        const int jj = j / 16, r = j % 16, kk = r / 4, bi = r % 4;
        const uint8_t q = (byte_of(1 + jj / 4, 4 * (jj % 4) + bi) >> (2 * kk)) & 3u;
        blk[16 + j / 4] = (uint8_t)(q << ((j % 4) * 2));
        uint32_t a = aux[(size_t)(g * sb_per_row + s) * 32 + lane];
        blk[80] = (uint8_t)a;
        blk[81] = (uint8_t)(a >> 8);
        blk[82] = (uint8_t)(a >> 16);
        blk[83] = (uint8_t)(a >> 24);
        out[i] = dequant_elem(Q2_K, blk, j);
    }
}

// ---------------------------------------------------------------------------
// launchers
// ---------------------------------------------------------------------------
static int grid_for(size_t n, int threads) {
    size_t g = (n + threads - 1) / threads;
    if (g > (size_t)148 * 64) g = (size_t)148 * 64;
    return (int)(g ? g : 1);
}

cudaError_t launch_dequant_raw(int fmt, const uint8_t *blocks, size_t n, float *out, cudaStream_t st) {
    if (n == 0) return cudaSuccess;
    k_dequant_raw<<<grid_for(n, 256), 256, 0, st>>>(fmt, blocks, n, out);
    return cudaGetLastError();
}

cudaError_t launch_quantize(int fmt, const float *x, size_t n, uint8_t *out, cudaStream_t st) {
    size_t be = (size_t)block_elems(fmt);
    size_t nb = (n + be - 1) / be;
    if (nb == 0) return cudaSuccess;
    int threads = 64;
    k_quantize<<<(unsigned)((nb + threads - 1) / threads), threads, 0, st>>>(fmt, x, n, out);
    return cudaGetLastError();
}

cudaError_t launch_repack_tiles(int fmt, const uint8_t *raw, int n, int k, uint4 *main, uint32_t *aux,
                                cudaStream_t st) {
    long long total = (long long)((n + 31) / 32) * 32 * (k / 256);
    if (total == 0) return cudaSuccess;
    int threads = 128;
    k_repack_tiles<<<(unsigned)((total + threads - 1) / threads), threads, 0, st>>>(fmt, raw, n, k, main, aux);
    return cudaGetLastError();
}

cudaError_t launch_dequant_tiles(int fmt, const uint4 *main, const uint32_t *aux, int n, int k, float *out,
                                 cudaStream_t st) {
    long long total = (long long)n * k;
    if (total == 0) return cudaSuccess;
    int threads = 256;
    k_dequant_tiles<<<(unsigned)((total + threads - 1) / threads), threads, 0, st>>>(fmt, main, aux, n, k, out);
    return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// decode-step kernels that must round like the reference
// ---------------------------------------------------------------------------

// Token embedding row (src/engine/mod.rs:1090-1097): row token % rows, decoded
// with the reference formula.  One thread per block of the row: the block's
// bytes are loaded first (independent loads), then decoded.  Also clears the
// step's argmax accumulator.
__global__ void k_embed(EmbedParams p) {
    const int t = blockIdx.x;
    if (p.pdl) {
        asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
        asm volatile("griddepcontrol.wait;" ::: "memory");
    }
    const uint32_t token = p.seqs[t].token;
    const size_t row = p.vocab_rows ? (size_t)token % p.vocab_rows : 0;
    const int be = block_elems(p.fmt), bb = block_bytes(p.fmt);
    float *__restrict__ out = p.out + (size_t)t * p.hidden;
    const size_t e0 = row * (size_t)p.hidden;
    if (e0 % be == 0 && p.hidden % be == 0) {
        const int nblk = p.hidden / be;
        const uint8_t *__restrict__ base = p.table + (e0 / be) * bb;
        for (int b = threadIdx.x; b < nblk; b += blockDim.x) {
            uint8_t blk[144];
            const uint8_t *src = base + (size_t)b * bb;
#pragma unroll 16
            for (int i = 0; i < bb; i++) blk[i] = src[i];
            for (int j = 0; j < be; j++) out[b * be + j] = dequant_elem(p.fmt, blk, j);
        }
    } else {
        for (int i = threadIdx.x; i < p.hidden; i += blockDim.x) {
            const size_t e = e0 + i;
            out[i] = dequant_elem(p.fmt, p.table + (e / be) * bb, (int)(e % be));
        }
    }
    if (threadIdx.x == 0) p.seqs[t].best = 0ull;
}

cudaError_t launch_embed(const EmbedParams &p, cudaStream_t st) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(p.m);
    cfg.blockDim = dim3(256);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = p.pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, k_embed, p);
}

// PackedKvBuffer::add (src/engine/mod.rs:209-232) for one stream of one token:
// grid (m, 2 streams), 256 threads.  min/max over kv_dim values, scale =
// (max-min)/levels (1.0 when the range is <= 1e-8), q = round((v-min)/scale)
// clamped, written LSB-first at bit offset i*bits.
__global__ void k_kv_pack(KvPackParams p) {
    const int t = blockIdx.x, which = blockIdx.y;
    extern __shared__ unsigned words[];
    __shared__ float smin[8], smax[8];
    if (p.pdl) {
        asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
        asm volatile("griddepcontrol.wait;" ::: "memory");
    }
    const int bits = which ? p.bits_v : p.bits_k;
    const size_t bpt = which ? p.pk_bpt_v : p.pk_bpt_k;
    const float *v = p.kv_scratch + ((size_t)t * 2 + which) * p.kv_dim;
    float mn = INFINITY, mx = -INFINITY;
    for (int i = threadIdx.x; i < p.kv_dim; i += blockDim.x) {
        mn = fminf(mn, v[i]);
        mx = fmaxf(mx, v[i]);
    }
    for (int o = 16; o > 0; o >>= 1) {
        mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    }
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    if (lane == 0) {
        smin[warp] = mn;
        smax[warp] = mx;
    }
    const int nwords = (int)((bpt + 3) / 4);
    for (int i = threadIdx.x; i < nwords; i += blockDim.x) words[i] = 0u;
    __syncthreads();
    mn = smin[0];
    mx = smax[0];
    for (int w = 1; w < nw; w++) {
        mn = fminf(mn, smin[w]);
        mx = fmaxf(mx, smax[w]);
    }
    const unsigned levels = (1u << bits) - 1u;
    const float scale = fabsf(mx - mn) > 1e-8f ? (mx - mn) / (float)levels : 1.0f;
    for (int i = threadIdx.x; i < p.kv_dim; i += blockDim.x) {
        const float qf = rclamp(roundf((v[i] - mn) / scale), 0.0f, (float)levels);
        const unsigned q = (qf == qf && qf > 0.0f) ? (unsigned)qf : 0u;
        const unsigned bit = (unsigned)i * bits;
        atomicOr(&words[bit >> 5], q << (bit & 31));
        if ((bit & 31) + bits > 32) atomicOr(&words[(bit >> 5) + 1], q >> (32 - (bit & 31)));
    }
    __syncthreads();
    const DevSeq sq = p.seqs[t];
    const uint32_t sid = p.seq_ids[t];
    const size_t ph = kv_phys(p.pages, sid, sq.slot);
    uint8_t *dst = (which ? p.vp_data : p.kp_data) + ph * bpt;
    const uint8_t *src = reinterpret_cast<const uint8_t *>(words);
    for (size_t i = threadIdx.x; i < bpt; i += blockDim.x) dst[i] = src[i];
    if (threadIdx.x == 0) {
        (which ? p.vp_min : p.kp_min)[ph] = mn;
        (which ? p.vp_scale : p.kp_scale)[ph] = scale;
    }
}

cudaError_t launch_kv_pack(const KvPackParams &p, cudaStream_t st) {
    size_t bpt = p.pk_bpt_k > p.pk_bpt_v ? p.pk_bpt_k : p.pk_bpt_v;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(p.m, 2);
    cfg.blockDim = dim3(256);
    cfg.dynamicSmemBytes = (bpt + 7) / 4 * 4 + 8;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = p.pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, k_kv_pack, p);
}

// Advance every sequence of a device-chained decode step: the next input token
// is this step's greedy argmax (0 when no logit was finite), positions move by
// one, and the KV slot moves to the next slot of the sequence's ring of
// `ring` slots (a full cache drops its oldest token, KvCache::add,
// src/engine/mod.rs:410-426), attending over at most `ring` tokens.
__global__ void k_advance(DevSeq *seqs, int m, uint32_t *out_tokens, uint32_t ring) {
    const int t = threadIdx.x;
    if (t >= m) return;
    asm volatile("griddepcontrol.wait;" ::: "memory");
    DevSeq s = seqs[t];
    const uint32_t tok = (uint32_t)(s.best & 0xffffffffull);
    out_tokens[t] = tok;
    s.token = tok;
    s.position += 1;
    s.slot = s.slot + 1 == ring ? 0u : s.slot + 1;
    s.seq_len = s.seq_len < ring ? s.seq_len + 1 : ring;
    seqs[t] = s;
}

cudaError_t launch_advance(DevSeq *seqs, int m, uint32_t *out_tokens, uint32_t ring, int pdl, cudaStream_t st) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(1);
    cfg.blockDim = dim3(32 * ((m + 31) / 32));
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, k_advance, seqs, m, out_tokens, ring);
}

}  // namespace nx
