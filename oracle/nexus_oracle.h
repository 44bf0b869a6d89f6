/*
 * nexus_oracle.h -- CPU restatement of the reference (luen-eth/Nexus, Rust)
 * quantized decode path.  TEST INFRASTRUCTURE ONLY: the parity checker and the
 * timed CPU baseline.  Nothing in the shipped library links or calls this code.
 *
 * Every function follows the reference's operation order so that, compiled
 * with -O2 -ffp-contract=off and no fast-math, results are bit-identical to
 * the reference's CPU path on the same GGUF file.  Citations are paths inside
 * the reference project.
 *
 * Pinning: the reference is Rust and cannot be built in this environment (no
 * cargo/rustc).  This restatement is pinned against the known-answer tests in
 * the reference's own inline test modules (transcribed as fixtures under
 * tests/golden/), see tests/test_oracle_kat.py.
 */
#ifndef NEXUS_ORACLE_H
#define NEXUS_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* GGUF tensor type ids (src/gguf/mod.rs:104-151). */
enum {
    ORC_F32 = 0,
    ORC_F16 = 1,
    ORC_Q4_0 = 2,
    ORC_Q8_0 = 8,
    ORC_Q2_K = 10,
    ORC_Q4_K = 12,
    ORC_BF16 = 28
};

/* Status codes. */
enum {
    ORC_OK = 0,
    ORC_E_TRUNCATED = -1,
    ORC_E_UNSUPPORTED = -2,
    ORC_E_INVALID = -3,
    ORC_E_IO = -4,
    ORC_E_MISSING_TENSOR = -5,
    ORC_E_SHAPE = -6,
    ORC_E_NOMEM = -7
};

/* ---- half (f16) conversion: `half` crate 2.7.1, IEEE binary16, RNE ---- */
uint16_t orc_f32_to_f16(float x);
float orc_f16_to_f32(uint16_t h);

/* ---- block formats ---- */
/* bytes for n elements (GgufDataType::bytes_per_element, src/gguf/mod.rs:246-291) */
size_t orc_type_size(int type, size_t n);
/* QuantEngine::quantize_weights (src/quant/mod.rs:623-640); returns bytes written
 * (0 for an unsupported type).  out must hold orc_type_size(type, n) bytes. */
size_t orc_quantize(int type, const float *x, size_t n, uint8_t *out);
/* GgufReader::tensor_bytes_to_f32 (src/gguf/mod.rs:902-956) */
int orc_dequantize(int type, const uint8_t *data, size_t data_len, size_t n, float *out);
/* Elements [start, start+count) of the flat dequantized tensor.  Values are the
 * same bits as orc_dequantize's (each element depends only on its own block). */
void orc_dequantize_range(int type, const uint8_t *data, size_t start, size_t count, float *out);

/* ---- transformer kernels (src/kernel/mod.rs) ---- */
void orc_rms_norm(const float *x, const float *w, size_t n, float eps, float *out);
void orc_rope_single(float *x, size_t position, size_t head_dim, float base);
/* InferenceEngine::matvec (src/engine/mod.rs:775-801) on f32 weights */
void orc_matvec(const float *w, size_t rows, size_t cols, const float *x, float *y);
/* the same matvec over a quantized tensor, dequantizing each row on the fly;
 * rows are split over `threads` threads (each row's result is unchanged). */
int orc_qmatvec(int type, const uint8_t *w, size_t rows, size_t cols, const float *x,
                float *y, int threads);
/* greedy_token (src/engine/mod.rs:809-817): argmax over finite values, last max wins */
uint32_t orc_greedy(const float *logits, size_t n);
/* softmax (src/kernel/mod.rs:234-255) */
void orc_softmax(const float *x, size_t n, float *out);

/* ---- packed low-bit KV stream (PackedKvBuffer, src/engine/mod.rs:187-313) ---- */
typedef struct orc_packed_kv orc_packed_kv;
orc_packed_kv *orc_packed_kv_new(uint32_t bits, size_t head_dim, size_t max_seq_len);
void orc_packed_kv_free(orc_packed_kv *b);
void orc_packed_kv_add(orc_packed_kv *b, size_t position, const float *values);
float orc_packed_kv_value_at(const orc_packed_kv *b, size_t position, size_t dim);
void orc_packed_kv_get_all(const orc_packed_kv *b, size_t seq_len, float *out);
void orc_packed_kv_shift_left(orc_packed_kv *b, size_t seq_len);
/* raw views for parity with device packed KV */
const uint8_t *orc_packed_kv_data(const orc_packed_kv *b);
const float *orc_packed_kv_mins(const orc_packed_kv *b);
const float *orc_packed_kv_scales(const orc_packed_kv *b);
size_t orc_packed_kv_bytes_per_token(const orc_packed_kv *b);

/* ---- GGUF (src/gguf/mod.rs:1091-1358) ---- */
typedef struct {
    char name[256];
    uint32_t n_dims;
    uint64_t shape[4];
    int type;
    uint64_t offset; /* relative to tensor data section */
} orc_tensor_info;

typedef struct orc_gguf orc_gguf;
int orc_gguf_open(const char *path, orc_gguf **out);
void orc_gguf_close(orc_gguf *g);
size_t orc_gguf_tensor_count(const orc_gguf *g);
const orc_tensor_info *orc_gguf_tensor(const orc_gguf *g, size_t i);
/* pointer to the tensor's bytes in the mapped file, NULL if out of bounds */
const uint8_t *orc_gguf_tensor_data(const orc_gguf *g, const orc_tensor_info *t);
uint64_t orc_gguf_data_offset(const orc_gguf *g);
/* metadata lookups; return 1 if found */
int orc_gguf_get_usize(const orc_gguf *g, const char *key, uint64_t *out);
int orc_gguf_get_f32(const orc_gguf *g, const char *key, float *out);

/* ---- decode engine (InferenceEngine, src/engine/mod.rs:503-1238) ---- */
typedef struct {
    uint32_t num_layers, hidden_size, ff_dim, num_heads, num_kv_heads, head_dim;
    uint32_t vocab_rows; /* rows of the output head (logits length) */
    uint32_t max_seq_len;
    float rope_freq_base;
    float rms_norm_eps;
    uint32_t kv_bits_k, kv_bits_v; /* 0 = float KV */
} orc_model_info;

typedef struct orc_model orc_model;
/* kv_bits_k/kv_bits_v = 0 selects the float KV cache (KvQuantType::None);
 * otherwise the packed buffer with those bit widths.  threads splits matvec
 * rows (results unchanged).  max_seq_len_override 0 = GGUF context_length. */
int orc_model_load(const char *path, uint32_t kv_bits_k, uint32_t kv_bits_v, int threads,
                   uint32_t max_seq_len_override, orc_model **out);
void orc_model_free(orc_model *m);
void orc_model_get_info(const orc_model *m, orc_model_info *info);
void orc_model_set_threads(orc_model *m, int threads);
/* InferenceConfig::rms_norm_eps override (tests use 0.0, src/engine/mod.rs:1728) */
void orc_model_set_eps(orc_model *m, float eps);
/* decode_with_cache: logits has vocab_rows entries */
int orc_model_decode(orc_model *m, uint32_t token, size_t position, float *logits);
/* prefill: clears the KV cache, runs every prompt token; logits of the last */
int orc_model_prefill(orc_model *m, const uint32_t *tokens, size_t n, float *logits);
/* greedy generate: out receives n + max_tokens ids (prompt then generated) */
int orc_model_generate(orc_model *m, const uint32_t *prompt, size_t n, size_t max_tokens,
                       uint32_t *out);
size_t orc_model_seq_len(const orc_model *m, uint32_t layer);
/* hidden state after the last decode (before the output norm), hidden_size floats */
const float *orc_model_last_hidden(const orc_model *m);

/* prefill with a layer-major schedule (every token through layer l before
 * layer l+1): the same logits and KV cache bits as orc_model_prefill, much
 * faster for long prompts.  n must not exceed max_seq_len. */
int orc_model_prefill_batched(orc_model *m, const uint32_t *tokens, size_t n, float *logits);

/* ---- seeded synthetic GGUF writer (same bytes as nexus_synth_model_write) ---- */
typedef struct {
    uint32_t num_layers, hidden_size, num_heads, num_kv_heads, ff_dim, vocab_size;
    uint32_t context_length;
    float rope_theta;
    float weight_std;
    uint64_t seed;
    int attn_format, ffn_format, embd_format, head_format, norm_format;
    int threads;
    uint32_t repeat_chunks;
} orc_synth_config;
int orc_synth_write(const char *path, const orc_synth_config *cfg);

#ifdef __cplusplus
}
#endif
#endif
