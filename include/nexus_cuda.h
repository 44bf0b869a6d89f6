/*
 * nexus_cuda.h -- C ABI of the B200 (sm_100a) CUDA backend for Nexus.
 *
 * This library fills the "unavailable" CUDA capability slot of the reference
 * (luen-eth/Nexus, Rust).  Every entry point is plain C: pointers, sizes and
 * status codes, no C++ or torch types.  Citations are paths in the reference
 * project, naming the interface each entry point replaces.
 *
 * Conventions
 *   - Every function returns an int status (NEXUS_OK = 0) unless noted.
 *     Once the CUDA backend is selected there is no CPU fallback: a failure is
 *     reported, never silently rerouted (contrast src/engine/mod.rs:1160-1166).
 *   - Handles are opaque and owned by the library; *_destroy frees them.
 *   - Caller buffers are borrowed for the duration of the call only.
 *   - Host pointers unless a name or flag says "device".
 *   - One in-flight call per model handle; different handles may be used from
 *     different threads (the reference's Backend is Send + Sync,
 *     src/backend/mod.rs:75).
 */
#ifndef NEXUS_CUDA_H
#define NEXUS_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define NEXUS_CUDA_ABI_VERSION 1

/* ---- status codes (replace io::Result / Result<_, String>) ---- */
enum {
    NEXUS_OK = 0,
    NEXUS_E_INVALID = 1,            /* bad argument or shape */
    NEXUS_E_UNSUPPORTED_FORMAT = 2, /* tensor type not handled on this path */
    NEXUS_E_OOM = 3,                /* device or host allocation failed */
    NEXUS_E_CUDA = 4,               /* CUDA runtime error */
    NEXUS_E_COMM = 5,               /* NCCL / peer communication error */
    NEXUS_E_TIMEOUT = 6,            /* a bounded device wait gave up */
    NEXUS_E_IO = 7,                 /* file open/read/map failed */
    NEXUS_E_MISSING_TENSOR = 8,     /* a required GGUF tensor is absent */
    NEXUS_E_TRUNCATED = 9,          /* payload shorter than its block count */
    NEXUS_E_UNAVAILABLE = 10        /* no usable sm_100 device */
};

/* ---- weight formats: GGUF type ids (GgufDataType::id, src/gguf/mod.rs:104-151)
 *      and the QuantFormat subset the backend handles (src/quant/mod.rs:16-31) ---- */
enum {
    NEXUS_FMT_F32 = 0,
    NEXUS_FMT_F16 = 1,
    NEXUS_FMT_Q4_0 = 2,
    NEXUS_FMT_Q8_0 = 8,
    NEXUS_FMT_Q2_K = 10,
    NEXUS_FMT_Q4_K = 12,
    NEXUS_FMT_BF16 = 28
};

/* ======================================================================== */
/* Backend selection and the Backend trait (src/backend/mod.rs:75-96)        */
/* ======================================================================== */

/* Replaces BackendFactory::unavailable_capability(BackendType::Cuda)
 * (src/backend/mod.rs:222-240): 1 when an sm_100 device is present. */
int nexus_cuda_is_available(void);

/* BackendCapabilities (src/backend/mod.rs:25-31).  Strings are static. */
typedef struct {
    int available;
    int device_count;
    const char *backend;              /* "cuda" (BackendType::name, :34-41) */
    const char *features[16];
    int n_features;
    const char *supported_ops[16];    /* same names as src/backend/cpu.rs:128-136 */
    int n_supported_ops;
} nexus_cuda_caps;
int nexus_cuda_capabilities(nexus_cuda_caps *caps);

/* Backend construction (BackendFactory::create(Some(BackendType::Cuda)),
 * src/backend/mod.rs:190-214, with the InferenceConfig knobs the device needs,
 * src/engine/mod.rs:65-98). */
typedef struct {
    int device;            /* first CUDA ordinal */
    int tp;                /* tensor-parallel degree, 1 = single GPU */
    uint32_t kv_bits_k;    /* 0 = float KV (KvQuantType::None); else packed key bits */
    uint32_t kv_bits_v;    /* packed value bits (KvQuantType::val_bits, src/quant/mod.rs:150) */
    uint32_t max_batch;    /* largest decode_batch the model will see (>= 1) */
    uint32_t max_seq_len;  /* 0 = GGUF llama.context_length (src/engine/mod.rs:561); KV tokens
                              kept per sequence: a full cache drops its oldest token
                              (KvCache::add, src/engine/mod.rs:410-426); positions run to
                              4 * max_seq_len */
    uint32_t page_tokens;  /* KV page size in tokens, a power of two <= 4096; 0 = 16 (the
                              scheduler's page size, src/scheduler.rs:333-361) */
    uint32_t max_pages;    /* KV pages in the pool per rank; 0 = max_batch * ceil(max_seq_len /
                              page_tokens) (every sequence can hold max_seq_len tokens) */
    uint32_t flags;        /* NEXUS_CFG_* */
    uint32_t tp_timeout_ms; /* tensor parallelism: how long nexus_cuda_tp_init waits for every
                               rank to join before it gives up with NEXUS_E_COMM; 0 = 120 s */
} nexus_cuda_config;

#define NEXUS_CFG_NO_GRAPH 0x1u  /* launch kernels directly instead of a CUDA graph */
#define NEXUS_CFG_NO_PDL 0x2u    /* no programmatic dependent launch between kernels */
#define NEXUS_CFG_PERSISTENT 0x4u /* single-token steps on the persistent whole-step kernel
                                     (one launch per token) instead of the kernel-per-op graph */
#define NEXUS_CFG_GEMV_16BIT 0x10u /* steps of 1-7 tokens: the GEMVs whose inputs are normalized
                                    (q/k/v, o_proj, gate/up, the head) read them as 16-bit instead of
                                    24-bit integers (one dp4a fewer per four weights; down keeps 24
                                    bits).  About 8% faster at b = 1 on the 8B shape, but its logits
                                    then differ from the reference's by ~2e-3, the edge of the
                                    2e-3 bound; off by default */
#define NEXUS_CFG_NCCL_ALLREDUCE 0x8u /* tensor parallelism: NCCL for every all-reduce instead of
                                        the one-shot peer-memory all-reduce of the hidden state */
#define NEXUS_CFG_FAULT_STALL_BARRIER 0x100u /* fault injection for tests of the error path: the
                                     persistent step kernel's grid barrier waits for a CTA that does
                                     not exist, so every step gives up after its bounded wait (about
                                     a second) and returns NEXUS_E_TIMEOUT; the context stays usable */

typedef struct nexus_cuda_backend nexus_cuda_backend;

/* Fills cfg with defaults (device 0, tp 1, float KV, max_batch 1, page 16). */
void nexus_cuda_config_default(nexus_cuda_config *cfg);
int nexus_cuda_backend_create(const nexus_cuda_config *cfg, nexus_cuda_backend **out);
int nexus_cuda_backend_destroy(nexus_cuda_backend *b);
/* Backend::name (src/backend/mod.rs:77): returns "cuda" */
const char *nexus_cuda_backend_name(const nexus_cuda_backend *b);
/* Backend::memory_info / MemoryInfo (src/backend/mod.rs:86,99-104) */
int nexus_cuda_memory_info(nexus_cuda_backend *b, size_t *total, size_t *free_bytes,
                           size_t *used);
/* Backend::synchronize (src/backend/mod.rs:95) */
int nexus_cuda_synchronize(nexus_cuda_backend *b);
/* Last error message for this backend (thread-local when b is NULL). */
const char *nexus_cuda_last_error(const nexus_cuda_backend *b);

/* ---- Tensor parallelism (one process per GPU) ----
 * No counterpart in the reference, which has no multi-GPU path; these give
 * BackendFactory::create(Some(Cuda)) (src/backend/mod.rs:206-213) a
 * multi-GPU form.  Rank 0 creates an id, the launcher shares it with every
 * rank (e.g. over torch.distributed), and each rank calls tp_init on its
 * backend before nexus_cuda_model_load.  Layers are then sharded: query/KV
 * heads, FFN rows and LM-head rows per rank; o_proj and down are column
 * slices whose partial sums meet in one all-reduce per sublayer (over peer
 * memory, or NCCL, loaded at tp_init).  Every rank must make the same model
 * calls in the same order.  tp_init returns NEXUS_E_COMM when not every rank
 * joined within tp_timeout_ms (the group is then torn down on this rank). */
#define NEXUS_TP_ID_BYTES 128
int nexus_cuda_tp_unique_id(void *id, size_t id_bytes);
int nexus_cuda_tp_init(nexus_cuda_backend *b, int rank, int world, const void *id, size_t id_bytes);
/* How the hidden-state all-reduces of a tensor-parallel backend run:
 * NEXUS_TP_NONE (not initialised or world 1), NEXUS_TP_NCCL, or
 * NEXUS_TP_PEER -- one kernel per all-reduce over NVLink peer memory (CUDA IPC
 * mapped staging buffers and flags, bounded waits), set up at tp_init unless
 * NEXUS_CFG_NCCL_ALLREDUCE is given or a peer cannot be mapped.  The sampled
 * logits' all-gather runs on NCCL either way. */
#define NEXUS_TP_NONE 0
#define NEXUS_TP_NCCL 1
#define NEXUS_TP_PEER 2
int nexus_cuda_tp_allreduce_kind(const nexus_cuda_backend *b);

/* The slice of a model one rank holds (host-only arithmetic, no device). */
typedef struct nexus_tp_slice {
    uint32_t q_head_begin, q_heads;    /* query heads */
    uint32_t kv_head_begin, kv_heads;  /* KV heads (each rank's query heads use only its own) */
    uint32_t ffn_begin, ffn_rows;      /* gate/up rows = down columns */
    uint32_t vocab_begin, vocab_rows;  /* LM-head rows */
} nexus_tp_slice;
/* NEXUS_E_INVALID when the shapes do not split (heads divisible by world,
 * column slices whole 256-element super-blocks, vocab rows whole 32-row groups). */
int nexus_tp_plan(uint32_t num_heads, uint32_t num_kv_heads, uint32_t head_dim, uint32_t ff_dim,
                  uint32_t vocab_rows, int rank, int world, nexus_tp_slice *out);

/* ---- KernelOp (src/backend/mod.rs:118-183) executed by Backend::execute ---- */
enum {
    NEXUS_OP_MATMUL = 0,      /* C[m,n] = A[m,k] @ B  (B is [n,k] when transpose_b, else [k,n]) */
    NEXUS_OP_ATTENTION = 1,   /* GQA decode attention, see nexus_op fields */
    NEXUS_OP_LAYER_NORM = 2,  /* layer_norm, src/kernel/mod.rs:212-231 */
    NEXUS_OP_RMS_NORM = 3,    /* rms_norm, src/kernel/mod.rs:199-209 */
    NEXUS_OP_ADD = 4,
    NEXUS_OP_MUL = 5,
    NEXUS_OP_SOFTMAX = 6,     /* softmax over rows of length n, src/kernel/mod.rs:234-255 */
    NEXUS_OP_QUANTIZE = 7,    /* QuantEngine::quantize_weights, src/quant/mod.rs:623-640 */
    NEXUS_OP_DEQUANTIZE = 8,  /* GgufReader::tensor_bytes_to_f32, src/gguf/mod.rs:902-956 */
    NEXUS_OP_QMATVEC = 9,     /* Y[m,n] = X[m,k] @ W[n,k]^T with W in a block format */
    NEXUS_OP_ROPE = 10,       /* rope_single over every head, src/kernel/mod.rs:258-271 */
    NEXUS_OP_ARGMAX = 11,     /* greedy_token, src/engine/mod.rs:809-817 */
    NEXUS_OP_KV_QUANTIZE = 12, /* PackedKvBuffer::add of one vector, src/engine/mod.rs:209-232:
                                 a = len floats, k = bits; out = ceil(len*bits/8) packed bytes
                                 followed by the f32 min and f32 scale */
    NEXUS_OP_ATTENTION_PACKED = 13 /* KvCache::attention_decode over packed buffers
                                 (src/engine/mod.rs:452-499 with KvCacheBuffer::Quantized):
                                 a = q (m*k floats); b = keys, c = values, each n rows of
                                 ceil(kv_heads*k*bits/8) bytes (PackedKvBuffer layout,
                                 src/engine/mod.rs:187-232) followed by n f32 mins and n f32
                                 scales; format = bits_k | bits_v << 8 (1..8 each) */
};

typedef struct {
    int kind;          /* NEXUS_OP_* */
    int device_ptrs;   /* 1: pointers are device pointers on the backend's device */
    const void *a;     /* MATMUL A / norm input / quantize input / dequant blocks / QMATVEC X /
                          ATTENTION q / SOFTMAX input / ADD,MUL lhs / ROPE in-out / ARGMAX logits */
    const void *b;     /* MATMUL B / norm weight / QMATVEC W blocks / ATTENTION keys / ADD,MUL rhs */
    const void *c;     /* ATTENTION values / LAYER_NORM bias (may be NULL) */
    void *out;         /* written output (ARGMAX: one uint32) */
    size_t m, n, k;    /* MATMUL/QMATVEC dims; norms and softmax: m rows of n;
                          ATTENTION: m = q heads, n = seq_len, k = head_dim; ROPE: m heads of k;
                          DEQUANTIZE: m = bytes available at `a` (0 = exactly the block count) */
    size_t len;        /* element count for ADD/MUL/QUANTIZE/DEQUANTIZE/ARGMAX */
    size_t kv_heads;   /* ATTENTION: KV heads (GQA group = m / kv_heads) */
    size_t position;   /* ROPE position */
    float scale;       /* ATTENTION score scale (0 = 1/sqrt(head_dim)); ROPE base */
    float eps;         /* norm epsilon */
    int format;        /* NEXUS_FMT_* for QUANTIZE/DEQUANTIZE/QMATVEC */
    int transpose_b;   /* MATMUL: 1 = B is [n,k] (the doc's A @ B^T, src/backend/mod.rs:119);
                          0 = B is [k,n] (what CpuBackend::matmul computes, src/backend/cpu.rs:24-38) */
} nexus_op;

/* Backend::execute (src/backend/mod.rs:92).  Unlike the CPU backend, which
 * discards its results (src/backend/cpu.rs:140-157), the output is written. */
int nexus_cuda_execute(nexus_cuda_backend *b, const nexus_op *op);

/* ======================================================================== */
/* Quantized weights resident on the device (for the GEMV sweep and callers  */
/* that manage their own matrices)                                           */
/* ======================================================================== */
typedef struct nexus_cuda_qweight nexus_cuda_qweight;
/* Uploads rows x cols elements of GGUF blocks (row-major, cols % 256 == 0 for
 * K-quants and Q4_0/Q8_0) and repacks them into the device tile layout. */
int nexus_cuda_qweight_create(nexus_cuda_backend *b, int format, size_t rows, size_t cols,
                              const void *blocks, size_t nbytes, nexus_cuda_qweight **out);
int nexus_cuda_qweight_destroy(nexus_cuda_qweight *w);
/* Y[m, rows] = X[m, cols] @ W^T on device pointers, on the backend's stream.
 * Asynchronous: call nexus_cuda_synchronize before reading Y on the host. */
int nexus_cuda_qmatvec_device(nexus_cuda_qweight *w, const float *x_dev, size_t m, float *y_dev);
/* Same with host buffers (copies inside, synchronous). */
int nexus_cuda_qmatvec_host(nexus_cuda_qweight *w, const float *x, size_t m, float *y);
/* Bit-exact dequantization of the stored weight back to f32 (rows*cols floats, host). */
int nexus_cuda_qweight_dequantize(nexus_cuda_qweight *w, float *out);
/* Device bytes of the repacked weight (the GEMV's algorithmic weight traffic). */
size_t nexus_cuda_qweight_bytes(const nexus_cuda_qweight *w);
/* Times `iters` GEMV launches on device buffers: each launch is bracketed by
 * CUDA events on the backend stream, and flush_bytes of a scratch buffer are
 * written between launches so every launch starts with a cold L2.  avg_ms is
 * the mean launch time. */
int nexus_cuda_qmatvec_bench(nexus_cuda_qweight *w, const float *x_dev, size_t m, float *y_dev, int iters,
                             size_t flush_bytes, float *avg_ms);

/* ======================================================================== */
/* Engine-level calls: the real hot boundary.  InferenceEngine               */
/* (src/engine/mod.rs:503-1238) calls these instead of its own matvec loop.  */
/* ======================================================================== */
typedef struct nexus_cuda_model nexus_cuda_model;

typedef struct {
    uint32_t num_layers, hidden_size, ff_dim, num_heads, num_kv_heads, head_dim;
    uint32_t vocab_rows;   /* logits length (output head rows) */
    uint32_t max_seq_len;
    float rope_freq_base;
    float rms_norm_eps;
    uint64_t weight_bytes; /* device bytes of all streamed weights (per decode step) */
    int body_format;       /* format of blk.*.attn_q (for reporting) */
    uint32_t max_batch;    /* sequences (nexus_cuda_config.max_batch) */
    uint32_t page_tokens;  /* KV page size in tokens */
    uint32_t max_pages;    /* KV pages in the pool (per rank) */
} nexus_cuda_model_info;

/* InferenceEngine::load_model (src/engine/mod.rs:539-692): mmaps the GGUF,
 * uploads raw blocks (no f32 materialization) and repacks them on the device. */
int nexus_cuda_model_load(nexus_cuda_backend *b, const char *gguf_path, nexus_cuda_model **out);
int nexus_cuda_model_free(nexus_cuda_model *m);
int nexus_cuda_model_get_info(const nexus_cuda_model *m, nexus_cuda_model_info *info);

/* Sequences: ids in [0, max_batch).  Every sequence owns a KV cache. */
/* KvCache::clear for one sequence (src/engine/mod.rs:437-441) */
int nexus_cuda_seq_reset(nexus_cuda_model *m, uint32_t seq_id);
/* tokens currently cached for a sequence (KvCache::seq_len) */
int nexus_cuda_seq_len(nexus_cuda_model *m, uint32_t seq_id, uint32_t *len);

/* decode_with_cache(token, position) (src/engine/mod.rs:1087-1146).
 * logits (vocab_rows floats) may be NULL; argmax (greedy_token) may be NULL. */
int nexus_cuda_decode(nexus_cuda_model *m, uint32_t seq_id, uint32_t token, uint32_t position,
                      float *logits, uint32_t *argmax);

/* prefill(tokens) (src/engine/mod.rs:1149-1170): clears the sequence's cache
 * and runs every token; logits/argmax are those of the last token. */
int nexus_cuda_prefill(nexus_cuda_model *m, uint32_t seq_id, const uint32_t *tokens, size_t n,
                       float *logits, uint32_t *argmax);

/* generate with greedy sampling (generate_with_config_streaming at
 * temperature 0, src/engine/mod.rs:1196-1238): out gets n + max_tokens ids. */
int nexus_cuda_generate(nexus_cuda_model *m, uint32_t seq_id, const uint32_t *prompt, size_t n,
                        size_t max_tokens, uint32_t *out);

/* generate_with_draft_tokens with greedy sampling (src/engine/mod.rs:1244-1291):
 * out gets n + max_tokens ids, the prompt then the greedy continuation (the
 * same tokens as nexus_cuda_generate); *accepted / *rejected count the
 * positions p < min(n_draft, max_tokens) where draft[p] equals / differs from
 * the generated token.  Each window of up to `window` tokens (0 = 8) -- the
 * next verified token followed by the draft tokens after it -- is checked in
 * one multi-token forward step (the reference decodes one token per call); the
 * cache keeps the tokens up to the first rejected draft.  Stop sequences are
 * not handled (greedy runs to max_tokens). */
int nexus_cuda_generate_with_draft(nexus_cuda_model *m, uint32_t seq_id, const uint32_t *prompt, size_t n,
                                   const uint32_t *draft, size_t n_draft, size_t max_tokens, uint32_t window,
                                   uint32_t *out, uint32_t *accepted, uint32_t *rejected);

/* KV pages.  The KV cache of every layer is a pool of max_pages pages of
 * page_tokens tokens (nexus_cuda_config); token t of a sequence lives in page
 * page_ids[t / page_tokens] of its list, at slot t % page_tokens.  A sequence
 * without a list uses the library's own pages [seq_id * P, (seq_id + 1) * P),
 * P = ceil(max_seq_len / page_tokens), when the pool has them.  A page belongs
 * to at most one sequence.
 *
 * Binds a request's page list (Scheduler::allocate_kv_pages,
 * src/scheduler.rs:333-361, ceil((prompt + max_tokens) / 16) ids) to seq_id
 * before its prefill.  The pages of tokens already cached must keep their
 * place (the list may only extend or end after them); ids must be below
 * max_pages and listed once; a page of another sequence is refused.
 * n_pages = 0 releases the sequence's pages and clears its cache. */
int nexus_cuda_seq_set_pages(nexus_cuda_model *m, uint32_t seq_id, const uint32_t *page_ids,
                             uint32_t n_pages);

/* One decode step for a batch of sequences (Scheduler::decode_batch items,
 * src/scheduler.rs:108-115,207-229).  page_ids (n_pages entries) is the
 * sequence's KV page list, ScheduledDecode.kv_pages: it is bound as by
 * nexus_cuda_seq_set_pages and must cover the token this step writes; NULL
 * keeps the sequence's current list. */
typedef struct {
    uint32_t seq_id;
    uint32_t token;
    uint32_t position;
    uint32_t n_pages;
    const uint32_t *page_ids;
} nexus_decode_item;
int nexus_cuda_decode_batch(nexus_cuda_model *m, const nexus_decode_item *items, size_t n,
                            uint32_t *out_tokens, float *out_logits);

/* ---- Request scheduler (src/scheduler.rs:126-365), host only ----
 * FIFO admission of up to max_batch_size running requests, each given
 * ceil((prompt_len + max_tokens) / page_size_tokens) KV page ids (at least
 * one) while at most max_kv_pages are in use (0 = no limit, Scheduler::new).
 * Request ids are the caller's.  Unlike the reference, whose page ids come
 * from a counter that never goes back, a released id is reused (smallest
 * first): the ids name pages of the device KV pool.  A request needs at least
 * one token (the reference would keep an empty one running without ever
 * giving it a decode item).  Arrays returned through a pointer stay valid
 * until the next call on the scheduler.  Buffers too small for the result
 * give NEXUS_E_INVALID with the needed count in *n and change nothing. */
typedef struct nexus_scheduler nexus_scheduler;
/* ScheduledDecode (src/scheduler.rs:106-115); position = the request's token
 * count, so `token` is its token number position - 1 */
typedef struct {
    uint64_t id;
    uint32_t token;
    uint32_t position;
    uint32_t generated;
    uint32_t prompt_len;
    uint32_t n_pages;
    const uint32_t *kv_pages;
} nexus_scheduled_decode;
/* Message of the calling thread's last scheduler call that failed (every
 * failure of a nexus_scheduler_* call, and the scheduler-side checks of
 * nexus_cuda_serve_step, return NEXUS_E_INVALID with a message here). */
const char *nexus_scheduler_last_error(void);
/* Scheduler::with_kv_pages (:152-166) */
int nexus_scheduler_create(uint32_t max_batch_size, uint32_t page_size_tokens, uint32_t max_kv_pages,
                           nexus_scheduler **out);
int nexus_scheduler_destroy(nexus_scheduler *s);
/* Scheduler::add_request (:169-172); NEXUS_E_INVALID for a used id or no tokens */
int nexus_scheduler_add_request(nexus_scheduler *s, uint64_t id, const uint32_t *tokens, size_t n,
                                uint32_t max_tokens);
/* Scheduler::get_next_batch (:175-179): ids of the requests admitted now */
int nexus_scheduler_get_next_batch(nexus_scheduler *s, uint64_t *ids, size_t max, size_t *n);
/* Scheduler::decode_batch (:207-229): admits pending work, then one item per running request */
int nexus_scheduler_decode_batch(nexus_scheduler *s, nexus_scheduled_decode *items, size_t max, size_t *n);
/* Scheduler::append_generated (:232-251); *found = 0 when id is not running */
int nexus_scheduler_append_generated(nexus_scheduler *s, uint64_t id, uint32_t token, int *found);
/* Scheduler::step (:254-281): ids of the requests that advanced */
int nexus_scheduler_step(nexus_scheduler *s, uint64_t *ids, size_t max, size_t *n);
/* Scheduler::get_completed (:284-287): takes the completed requests' ids */
int nexus_scheduler_get_completed(nexus_scheduler *s, uint64_t *ids, size_t max, size_t *n);
/* Scheduler::complete_request (:290-314) */
int nexus_scheduler_complete_request(nexus_scheduler *s, uint64_t id, int *found);
/* Scheduler::stats (:317-322) */
int nexus_scheduler_stats(nexus_scheduler *s, size_t *pending, size_t *running, size_t *completed);
/* Scheduler::kv_page_stats (:324-331): pages in use, max_kv_pages (0 = no limit) */
int nexus_scheduler_kv_page_stats(nexus_scheduler *s, size_t *used, size_t *max_pages);
/* Scheduler::kv_allocation (:333-335): NEXUS_E_INVALID when the request holds no pages */
int nexus_scheduler_kv_allocation(nexus_scheduler *s, uint64_t id, uint32_t *page_ids, size_t max, size_t *n,
                                  size_t *capacity_tokens);
/* Request::tokens of a pending, running or completed (not yet taken) request:
 * the prompt followed by the generated tokens */
int nexus_scheduler_tokens(nexus_scheduler *s, uint64_t id, uint32_t *out, size_t max, size_t *n);

/* ---- Continuous batching (no counterpart: the reference server runs one
 * generate_with_config per request behind the engine mutex,
 * src/server/mod.rs:407,416, and never calls decode_batch) ----
 * One tick: pending requests are admitted (Scheduler::fill_running, :182-204)
 * and each new one gets a free device sequence with its page ids bound
 * (nexus_cuda_seq_set_pages) and all but its last prompt token prefilled;
 * then one nexus_cuda_decode_batch step runs every running request's decode
 * item and each greedy token is appended (append_generated).  A request's
 * tokens equal greedy nexus_cuda_generate(prompt, max_tokens) run alone.
 * One event per request that produced a token or ended in this tick: its
 * id, the token, its index among the request's generated tokens, done = 1
 * when the request completed, status NEXUS_E_INVALID for a request the model
 * cannot hold (prompt_len + max_tokens - 1 > max_seq_len), which ends without
 * tokens, or the status of a failed page binding or prefill for a request
 * that could not be set up (it ends too; the backend's last error says why).  The scheduler's page size must equal the model's page_tokens,
 * max_kv_pages must be set and within the model's pool, max_batch_size within
 * its max_batch and max_events >= max_batch_size.  From its first tick the
 * scheduler owns every sequence of the model (their pages are released
 * then); requests cancelled with nexus_scheduler_complete_request give their
 * sequence back at the next tick. */
typedef struct {
    uint64_t request_id;
    uint32_t token;
    uint32_t index;
    uint32_t done;
    int32_t status;
} nexus_serve_event;
int nexus_cuda_serve_step(nexus_cuda_model *m, nexus_scheduler *s, nexus_serve_event *events, size_t max_events,
                          size_t *n_events);

/* Device time of the last decode/prefill call in milliseconds (CUDA events). */
int nexus_cuda_last_step_ms(const nexus_cuda_model *m, float *ms);

/* Per-kernel profile of `steps` single-token decode steps of sequence seq_id
 * (continuing from its current length, greedy tokens fed back): every kernel
 * launch is bracketed by CUDA events on the launching stream, no graph.  One
 * record per kernel role; bytes = algorithmic bytes per launch (weights read
 * + activations read and written).  The KV cache advances by `steps`. */
typedef struct {
    char name[24];       /* embed, qkv, kv_pack, attention, o_proj, gate_up, down, head, advance */
    uint32_t launches;
    float total_ms;
    double bytes_per_launch;
} nexus_kernel_profile;
int nexus_cuda_profile_decode(nexus_cuda_model *m, uint32_t seq_id, uint32_t token, uint32_t steps,
                              nexus_kernel_profile *out, int max_out, int *n_out);

/* GQA decode attention that allocates nothing (no counterpart in the
 * reference).  For callers that cannot allocate device memory while they
 * run -- serving loops that cannot take the device-wide synchronization of
 * cudaMalloc/cudaFree, and embedders whose device memory is all handed to
 * their own pool.  Same computation as
 * nexus_cuda_execute with NEXUS_OP_ATTENTION on device pointers: q is
 * num_q_heads*head_dim floats, k/v are seq_len rows of num_kv_heads*head_dim
 * floats, out is num_q_heads*head_dim floats, all device memory owned by the
 * caller; scale 0 means 1/sqrt(head_dim).  Its scratch lives in one fixed
 * 1 MiB device array per GPU, held until the process exits; shapes needing
 * more return NEXUS_E_INVALID.  All calls share that array: calls that
 * overlap on the GPU race, so order them on one stream.  The first call on a
 * device looks up the array's address and should come before any stream
 * capture.  Synchronous on the backend's stream; the calling thread's current
 * device is left as it was.  num_q_heads must be a nonzero multiple of
 * num_kv_heads. */
int nexus_cuda_attention_noalloc(nexus_cuda_backend *b, const float *q_dev, const float *k_dev,
                                 const float *v_dev, float *out_dev, size_t num_q_heads,
                                 size_t num_kv_heads, size_t head_dim, size_t seq_len, float scale);

/* ======================================================================== */
/* Host utilities (the reference's converter and quantizers)                 */
/* ======================================================================== */

/* QuantEngine::quantize_weights on the host (src/quant/mod.rs:623-640);
 * returns bytes written or 0 for an unsupported format. */
size_t nexus_quantize_host(int format, const float *x, size_t n, uint8_t *out);
/* bytes for n elements (GgufDataType::bytes_per_element, src/gguf/mod.rs:246-291) */
size_t nexus_format_bytes(int format, size_t n);

/* Seeded synthetic LLaMA-style GGUF v3 writer following nexus-convert's file
 * conventions (tools/nexus-convert/main.rs:190-383): blk.N.* names, [out,in]
 * shapes, llama.* keys, 32-byte alignment; weights N(0, std^2) from a
 * counter-based generator, norms 1.0 quantized with norm_format. */
typedef struct {
    uint32_t num_layers, hidden_size, num_heads, num_kv_heads, ff_dim, vocab_size;
    uint32_t context_length;
    float rope_theta;       /* written as llama.rope.freq_base */
    float weight_std;       /* 0.02 */
    uint64_t seed;
    int attn_format;        /* q/k/v/o */
    int ffn_format;         /* gate/up/down */
    int embd_format;        /* token_embd */
    int head_format;        /* output (LM head); -1 = no output.weight (tied) */
    int norm_format;        /* attn_norm/ffn_norm/output_norm */
    int threads;            /* generator threads (0 = all cores) */
    uint32_t repeat_chunks; /* 0 = every element drawn; n = each tensor repeats its first
                               n * 65536 drawn elements (quick generation of very large
                               models; the kernels' work is unchanged) */
} nexus_synth_config;
int nexus_synth_model_write(const char *path, const nexus_synth_config *cfg);

#ifdef __cplusplus
}
#endif
#endif /* NEXUS_CUDA_H */
