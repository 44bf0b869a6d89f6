// kernels_attn.cu -- GQA decode attention over the KV cache (float or packed).
//
// Replaces KvCache::attention_decode (src/engine/mod.rs:452-499): for query
// head qh, kv head kvh = qh / (Hq/Hkv); s_t = (q . k_t) * (1/sqrt(D));
// o = sum_t softmax(s)_t * v_t.  Packed caches are read directly in their
// low-bit form: value = min_t + q * scale_t (PackedKvBuffer::value_at,
// src/engine/mod.rs:252-256), one (min, scale) per token across all KV heads.
//
// Split-context ("flash decoding") layout: grid (Hkv, nsplit, batch).  Each
// CTA owns one KV head, a contiguous slice of at least kTokensPerSplit tokens
// of the context, and all G query heads sharing that KV head, so every K/V
// element is read from HBM once.  The slice count adapts to the context
// length (CTAs beyond it exit), so short contexts use few, full slices
// (16-token slices that fill every SM twice measured slower at b = 1: the
// kernel is bound by its chain of dependent memory round trips, and more
// slices lengthen the merge).
// Eight warps stride over the slice; each warp issues the loads of kBatch
// tokens before using any of them (one memory round trip per batch); lane i
// holds head_dim/32 dims of each row.  Warps keep an online softmax per query
// head, are merged in shared memory, and slices are merged by the last CTA to
// finish (an atomic counter per (sequence, KV head), reset by that CTA).
#include <cuda_runtime.h>
#include <math.h>

#include "attn_block.cuh"
#include "common.cuh"
#include "kernels.h"

namespace nx {

constexpr int kAttnWarps = 8;
constexpr int kTokensPerSplit = NX_ATTN_TPS;  // a slice holds at least this many tokens

template <int VEC, int G>
__global__ void __launch_bounds__(kAttnWarps * 32, G <= 4 ? 2 : 1) k_attn(AttnParams p) {
    __shared__ AttnSmem<VEC, G, kAttnWarps> sm;
    if (p.pdl) {
        pdl_launch_dependents();
        pdl_wait();
    }
    attn_block<VEC, G, kAttnWarps, kTokensPerSplit>(p, blockIdx.x, blockIdx.y, blockIdx.z, sm);
}

template <int VEC, int G>
static cudaError_t launch_attn_t(const AttnParams &p, cudaStream_t st) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(p.hkv, p.nsplit, p.m);
    cfg.blockDim = dim3(kAttnWarps * 32);
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
    if (p.hkv <= 0 || p.hq % p.hkv != 0 || p.nsplit < 1 || p.nsplit > 64) return cudaErrorInvalidValue;
    if (p.bits_k > 0 && attention_pk_supported(p)) return launch_attention_pk(p, st);
    switch (p.head_dim) {
    case 32: return launch_attn_g<1>(p, st);
    case 64: return launch_attn_g<2>(p, st);
    case 128: return launch_attn_g<4>(p, st);
    default: return cudaErrorInvalidValue;
    }
}

}  // namespace nx
