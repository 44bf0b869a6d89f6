// kernels.h -- launch interfaces of the sm_100a kernels (host side).
#pragma once
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace nx {

// ---- kernels_quant.cu (bit-exact, -fmad=false) ----
cudaError_t launch_dequant_raw(int fmt, const uint8_t *blocks, size_t n, float *out, cudaStream_t st);
cudaError_t launch_quantize(int fmt, const float *x, size_t n, uint8_t *out, cudaStream_t st);
cudaError_t launch_repack_tiles(int fmt, const uint8_t *raw, int n, int k, uint4 *main, uint32_t *aux,
                                cudaStream_t st);
cudaError_t launch_dequant_tiles(int fmt, const uint4 *main, const uint32_t *aux, int n, int k, float *out,
                                 cudaStream_t st);

// ---- kernels_gemv.cu ----
enum GemvEpilogue : int {
    EPI_STORE = 0,   // y[t][row] = dot
    EPI_ADD = 1,     // y[t][row] += dot            (residual add)
    EPI_SWIGLU = 2,  // tile rows: 16 gate rows then 16 up rows per group -> y[t][i] = silu(g)*u
    EPI_QKV = 3,     // fused Q|K|V with RoPE; K,V written to the KV destination
    EPI_ARGMAX = 4   // logits (optional) + greedy argmax via a packed 64-bit atomic max
};

// Per-step values read by the kernels on the device (so one captured graph
// serves every decode step).  One entry per sequence in the batch.
struct DevSeq {
    uint32_t token;         // input token of this step
    uint32_t position;      // RoPE position (the token's index in the sequence)
    uint32_t slot;          // KV slot written this step (= cached tokens before it)
    uint32_t seq_len;       // tokens attended over (= slot + 1)
    unsigned long long best;  // packed argmax accumulator of the head
};

// Paged KV cache (Scheduler::allocate_kv_pages, src/scheduler.rs:333-361):
// token `tok` of the sequence in cache row `sid` lives at physical token
// slot table[sid * per_seq + (tok >> shift)] * 2^shift + (tok & (2^shift - 1))
// of the per-layer pool; table == nullptr means one contiguous sequence
// (physical slot = tok), as the op-level entry points pass it.
struct KvPages {
    const uint32_t *table;  // [rows][per_seq] page ids
    uint32_t per_seq;       // table entries per cache row
    uint32_t shift;         // log2(tokens per page)
};

struct QkvEpilogue {
    int hq, hkv, head_dim;      // heads and dims (head_dim/2 a multiple of 16)
    float *q_out;               // [m][hq*head_dim]
    const float *rope_cos;      // [max_pos][head_dim/2] host-computed table
    const float *rope_sin;
    // KV destinations: the float cache pool [pages*page_tokens][kv_dim]
    // (k_cache/v_cache, addressed through `pages`) or, when kv_scratch is set,
    // the new K/V rows go to kv_scratch[m][2][kv_dim]
    float *k_cache, *v_cache;
    KvPages pages;
    float *kv_scratch;
    const DevSeq *seqs;         // [m]
    const uint32_t *seq_ids;    // [m] cache row of each batch entry
};

// Decode attention: a context slice holds at least this many tokens (the
// step's slice count per (sequence, KV head) is sized with it).
#ifndef NX_ATTN_TPS
#define NX_ATTN_TPS 64
#endif

struct GemvParams {
    int fmt;
    const uint4 *w_main;
    const uint32_t *w_aux;
    int n;        // valid output rows of the tile matrix
    int k;        // input columns (multiple of 256)
    int m;        // tokens
    const float *x;     // [m][x_stride]
    int x_stride;
    const float *norm_w;  // fused RMSNorm weights (nullptr = none)
    float eps;
    int epi;
    float *y;           // [m][y_stride]
    int y_stride;
    QkvEpilogue qkv;
    DevSeq *seqs;       // EPI_ARGMAX: best accumulators per token
    int pdl;            // 1: launched with programmatic stream serialization
    // K-split scratch (optional; without it the GEMV never splits K)
    float *part;            // [S][m][groups*32] partial row sums
    size_t part_floats;     // capacity of part
    unsigned *counters;     // [groups] arrival counters, zero on entry and exit
    int counter_slots;      // capacity of counters
    int ksplit;             // warps per row group (set by the launcher)
    int nst;                // weight ring slots per warp (set by the launcher)
    int *err;               // device flag set when a bounded wait gives up (may be NULL)
    int row_offset;         // EPI_ARGMAX: global index of local row 0 (vocab slice of a rank)
    int x_bits;             // GEMV input precision: 16 (normalized inputs) or 24 (default, 0)
};

cudaError_t launch_gemv(const GemvParams &p, cudaStream_t st);

// ---- kernels_gemm.cu: tcgen05 GEMM for m >= 8 (same weights, epilogues and
// K-split scratch fields of GemvParams) ----
struct GemmScratch {
    uint8_t *bimg;            // prepared activations (f16 hi/lo in the MMA layout)
    size_t bimg_bytes;
    float *tok_scale;         // per-token power-of-two scales
    size_t tok_scale_floats;
};
struct GemmScratchSize {
    size_t bimg_bytes, tok_scale_floats, part_floats, counter_slots;
};
bool gemm_supported(int fmt);
GemmScratchSize gemm_scratch_size(int m, int n, int k);
cudaError_t launch_gemm(const GemvParams &p, const GemmScratch &sc, cudaStream_t st);

// ---- kernels_attn.cu ----
struct AttnParams {
    int hq, hkv, head_dim, m;
    const float *q;          // [m][hq*head_dim]
    float *out;              // [m][hq*head_dim]
    float scale;             // 1/sqrt(head_dim)
    // float cache pool [slots][kv_dim]
    const float *k_cache, *v_cache;
    // packed cache pool (bits_k > 0): per physical slot, bytes + min + scale
    int bits_k, bits_v;
    const uint8_t *kp_data, *vp_data;
    const float *kp_min, *kp_scale, *vp_min, *vp_scale;
    size_t pk_bpt_k, pk_bpt_v;     // bytes per token
    KvPages pages;           // token -> physical slot of either cache
    const DevSeq *seqs;
    const uint32_t *seq_ids;
    int kv_dim;
    int nsplit;              // splits of the context per (sequence, kv head)
    float *part;             // scratch [m][hkv][nsplit][G][head_dim + 2]
    unsigned *counters;      // [m][hkv], zero on entry, left zero on exit
    int pdl;
};
cudaError_t launch_attention(const AttnParams &p, cudaStream_t st);
// packed-cache attention on the tensor cores (kernels_attn_pk.cu): head_dim
// 128, G in {1, 2, 4, 8}, bits in {2, 3, 4, 6, 8}; launch_attention routes there
bool attention_pk_supported(const AttnParams &p);
cudaError_t launch_attention_pk(const AttnParams &p, cudaStream_t st);
// causal attention for m consecutive tokens of one sequence (seqs[0].slot is
// the first token's slot) on the tensor cores (kernels_attn_prefill.cu):
// float cache, head_dim 128, G in {1, 2, 4, 8}
bool attention_prefill_supported(const AttnParams &p);
cudaError_t launch_attention_prefill(const AttnParams &p, cudaStream_t st);

// packed KV append (PackedKvBuffer::add, src/engine/mod.rs:209-232) for m tokens
struct KvPackParams {
    int m, kv_dim, bits_k, bits_v;
    const float *kv_scratch;      // [m][2][kv_dim]
    uint8_t *kp_data, *vp_data;
    float *kp_min, *kp_scale, *vp_min, *vp_scale;
    size_t pk_bpt_k, pk_bpt_v;
    KvPages pages;
    const DevSeq *seqs;
    const uint32_t *seq_ids;
    int pdl;
};
cudaError_t launch_kv_pack(const KvPackParams &p, cudaStream_t st);
// device-chained decode: next token = argmax, positions advance by one
cudaError_t launch_advance(DevSeq *seqs, int m, uint32_t *out_tokens, uint32_t ring, int pdl, cudaStream_t st);

// ---- kernels_step.cu: the single-token decode step as one persistent kernel ----
// One matrix in the tile layout (tiles.cuh): fmt, tiles, Q2_K side words, rows, columns.
struct StepMat {
    int fmt;
    const uint4 *main;
    const uint32_t *aux;
    int n, k;
};
struct StepLayer {
    StepMat qkv, o, gateup, down;   // fused Q|K|V (RoPE pairs in lanes i, i+16), o_proj, gate|up, down
    const float *attn_norm, *ffn_norm;
    float *k_cache, *v_cache;       // float KV page pools
};
struct StepParams {
    const StepLayer *layers;        // device array
    int num_layers;
    StepMat head;
    const float *out_norm;
    int hidden, hq, hkv, head_dim, ffn;
    float eps;
    const float *rope_cos, *rope_sin;
    float *x_hidden, *q, *attn, *gated;
    float *logits;                  // head outputs (nullptr: argmax only)
    DevSeq *seqs;                   // one sequence
    const uint32_t *seq_ids;
    KvPages pages;
    uint32_t *out_tokens;           // [0] = next token
    int *err;                       // set when a bounded wait gives up
    float *attn_part;               // [hkv][attn_nsplit][G][head_dim + 2]
    unsigned *attn_counters;        // [hkv], zero between launches
    int attn_nsplit;
    uint32_t max_seq;               // KV ring slots per sequence (the cache keeps the last max_seq tokens)
    float *gpart;                   // [grid * warps][2][32] partial row sums of shared row groups
    unsigned *gcounters;            // [max row groups], zero between launches
    unsigned *bar;                  // grid barrier: arrivals, generation
    unsigned bar_extra;             // 0; 1 = fault injection: barriers wait for one CTA too many
};
struct StepLaunch {
    int warps, grid;
    size_t smem;
};
// Fills the launch shape for the model, or returns cudaErrorNotSupported when
// the step kernel does not cover it (head_dim 128, G in {1, 2, 4, 8}, widths
// multiples of 256, shared memory within the SM).
cudaError_t step_plan(const StepParams &p, int device, StepLaunch *out);
size_t step_gpart_floats(const StepLaunch &l);
cudaError_t launch_decode_step(const StepParams &p, const StepLaunch &l, cudaStream_t st);

// ---- kernels_peer.cu: one-shot all-reduce over NVLink peer memory (TP) ----
constexpr int kPeerMaxRanks = 8;
constexpr int kPeerCtas = 32;
struct PeerReduce {
    float *bufs[kPeerMaxRanks][2];   // every rank's two staging buffers (peer mappings for the others)
    unsigned *flags[kPeerMaxRanks];  // every rank's epoch flags [kPeerCtas][2]
    unsigned *epoch;                 // this rank's epoch per CTA [kPeerCtas]
    int rank, world;
    size_t max_floats;               // capacity of one staging buffer
    int *err;                        // set when a peer's flag never arrives
};
// x[0..n) <- the sum over ranks of every rank's x (rank order, bit-identical on all ranks)
cudaError_t launch_peer_allreduce(const PeerReduce &pr, float *x, size_t n, cudaStream_t st);

// ---- kernels_misc.cu ----
// embedding row gather with bit-exact dequantization; also resets seqs[t].best
struct EmbedParams {
    int fmt, m, hidden;
    size_t vocab_rows;
    const uint8_t *table;   // raw GGUF blocks
    float *out;             // [m][hidden]
    DevSeq *seqs;
    int pdl;
};
cudaError_t launch_embed(const EmbedParams &p, cudaStream_t st);

cudaError_t launch_rms_norm(const float *x, const float *w, float *out, int rows, int n, float eps, cudaStream_t st);
cudaError_t launch_layer_norm(const float *x, const float *w, const float *b, float *out, int rows, int n,
                              float eps, cudaStream_t st);
cudaError_t launch_softmax(const float *x, float *out, int rows, int n, cudaStream_t st);
cudaError_t launch_binary(int op, const float *a, const float *b, float *out, size_t n, cudaStream_t st);
cudaError_t launch_matmul_f32(const float *a, const float *b, float *c, int m, int n, int k, int transpose_b,
                              cudaStream_t st);
cudaError_t launch_rope(float *x, int heads, int head_dim, int position, float base, cudaStream_t st);
cudaError_t launch_argmax(const float *x, size_t n, unsigned long long *best, cudaStream_t st);

}  // namespace nx
