/*
 * nexus_oracle.c -- CPU restatement of the reference's quantized decode path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity oracle and the timed CPU
 * baseline ("port").  Only tests/, __graft_entry__.smoke() and bench.py's CPU
 * legs load it; the shipped library (nexus_b200/) never does.
 *
 * Build: see oracle/Makefile (-O2 -ffp-contract=off, no fast-math), so every
 * a*b+c below is two separately rounded operations, as in the Rust reference.
 *
 * Reference: luen-eth/Nexus (Rust).  Citations are file:line in that project.
 */
#define _GNU_SOURCE
#include "nexus_oracle.h"

#include <fcntl.h>
#include <math.h>
#include <pthread.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

/* ------------------------------------------------------------------------ */
/* f16 <-> f32 (`half` 2.7.1, Cargo.lock:629-631; f32_to_f16 is IEEE RNE,    */
/* NaN keeps the top mantissa bits and sets the quiet bit)                   */
/* ------------------------------------------------------------------------ */
uint16_t orc_f32_to_f16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t exp = (x >> 23) & 0xffu;
    uint32_t man = x & 0x7fffffu;
    if (exp == 0xffu) {
        if (man == 0) return (uint16_t)(sign | 0x7c00u);
        return (uint16_t)(sign | 0x7c00u | 0x0200u | (man >> 13));
    }
    int e = (int)exp - 127 + 15;
    if (e >= 0x1f) return (uint16_t)(sign | 0x7c00u);
    if (e <= 0) {
        if (e < -10) return (uint16_t)sign;
        man |= 0x800000u;
        int shift = 14 - e;
        uint32_t hm = man >> shift;
        uint32_t rem = man & ((1u << shift) - 1u);
        uint32_t halfway = 1u << (shift - 1);
        if (rem > halfway || (rem == halfway && (hm & 1u))) hm++;
        return (uint16_t)(sign | hm);
    }
    uint32_t hm = man >> 13;
    uint32_t rem = man & 0x1fffu;
    uint32_t h = sign | ((uint32_t)e << 10) | hm;
    if (rem > 0x1000u || (rem == 0x1000u && (hm & 1u))) h++;
    return (uint16_t)h;
}

float orc_f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1fu;
    uint32_t man = h & 0x3ffu;
    uint32_t x;
    if (exp == 0) {
        if (man == 0) {
            x = sign;
        } else {
            int e = -1;
            do {
                e++;
                man <<= 1;
            } while (!(man & 0x400u));
            x = sign | ((uint32_t)(127 - 15 - e) << 23) | ((man & 0x3ffu) << 13);
        }
    } else if (exp == 0x1f) {
        x = sign | 0x7f800000u | (man << 13);
    } else {
        x = sign | ((exp + 112u) << 23) | (man << 13);
    }
    float f;
    memcpy(&f, &x, 4);
    return f;
}

static inline float ld_f16(const uint8_t *p) { return orc_f16_to_f32((uint16_t)(p[0] | (p[1] << 8))); }
static inline void st_f16(uint8_t *p, float v) {
    uint16_t h = orc_f32_to_f16(v);
    p[0] = (uint8_t)(h & 0xff);
    p[1] = (uint8_t)(h >> 8);
}

/* Rust `f as uN` / `f as iN`: saturating, NaN -> 0 */
static inline uint32_t sat_u32(float v) {
    if (!(v == v) || v <= 0.0f) return 0;
    if (v >= 4294967295.0f) return 4294967295u;
    return (uint32_t)v;
}
static inline uint8_t sat_u8(float v) {
    if (!(v == v) || v <= 0.0f) return 0;
    if (v >= 255.0f) return 255;
    return (uint8_t)v;
}
static inline int32_t sat_i32(float v) {
    if (!(v == v)) return 0;
    if (v <= -2147483648.0f) return INT32_MIN;
    if (v >= 2147483647.0f) return INT32_MAX;
    return (int32_t)v;
}
static inline int8_t sat_i8(float v) {
    if (!(v == v)) return 0;
    if (v <= -128.0f) return -128;
    if (v >= 127.0f) return 127;
    return (int8_t)v;
}
/* Rust f32::clamp: NaN passes through */
static inline float rclamp(float v, float lo, float hi) {
    if (v < lo) v = lo;
    if (v > hi) v = hi;
    return v;
}

/* ------------------------------------------------------------------------ */
/* sizes                                                                     */
/* ------------------------------------------------------------------------ */
static size_t div_ceil(size_t a, size_t b) { return (a + b - 1) / b; }

size_t orc_type_size(int type, size_t n) {
    switch (type) {
    case ORC_F32: return n * 4;
    case ORC_F16:
    case ORC_BF16: return n * 2;
    case ORC_Q4_0: return div_ceil(n, 32) * 18;
    case ORC_Q8_0: return div_ceil(n, 32) * 34;
    case ORC_Q2_K: return div_ceil(n, 256) * 84;
    case ORC_Q4_K: return div_ceil(n, 256) * 144;
    default: return 0;
    }
}

/* ------------------------------------------------------------------------ */
/* quantizers (src/quant/mod.rs)                                             */
/* ------------------------------------------------------------------------ */

/* quantize_q8_0, src/quant/mod.rs:669-687 */
static size_t quantize_q8_0(const float *data, size_t n, uint8_t *out) {
    size_t o = 0;
    for (size_t c = 0; c < n; c += 32) {
        size_t len = n - c < 32 ? n - c : 32;
        float max_abs = 0.0f;
        for (size_t i = 0; i < len; i++) max_abs = fmaxf(max_abs, fabsf(data[c + i]));
        float scale = max_abs > 0.0f ? max_abs / 127.0f : 0.0f;
        st_f16(out + o, scale);
        o += 2;
        for (size_t i = 0; i < 32; i++) {
            float value = i < len ? data[c + i] : 0.0f;
            int8_t q = 0;
            if (scale > 0.0f) q = sat_i8(rclamp(roundf(value / scale), -128.0f, 127.0f));
            out[o++] = (uint8_t)q;
        }
    }
    return o;
}

/* quantize_symmetric_4bit, src/quant/mod.rs:746-753 */
static uint8_t quantize_symmetric_4bit(float value, float scale) {
    if (scale > 0.0f) {
        int32_t q = sat_i32(rclamp(roundf(value / scale), -8.0f, 7.0f));
        return (uint8_t)(q + 8);
    }
    return 8;
}

/* quantize_q4_0, src/quant/mod.rs:705-720 */
static size_t quantize_q4_0(const float *data, size_t n, uint8_t *out) {
    size_t o = 0;
    for (size_t c = 0; c < n; c += 32) {
        size_t len = n - c < 32 ? n - c : 32;
        float max_abs = 0.0f;
        for (size_t i = 0; i < len; i++) max_abs = fmaxf(max_abs, fabsf(data[c + i]));
        float scale = max_abs > 0.0f ? max_abs / 7.0f : 0.0f;
        st_f16(out + o, scale);
        o += 2;
        for (size_t i = 0; i < 16; i++) {
            float lo_v = i < len ? data[c + i] : 0.0f;
            float hi_v = i + 16 < len ? data[c + i + 16] : 0.0f;
            uint8_t lo = quantize_symmetric_4bit(lo_v, scale);
            uint8_t hi = quantize_symmetric_4bit(hi_v, scale);
            out[o++] = (uint8_t)((lo & 0x0f) | ((hi & 0x0f) << 4));
        }
    }
    return o;
}

/* quantize_u6 / quantize_u4, src/quant/mod.rs:1117-1131 */
static uint8_t quantize_uN(float value, float scale, float hi) {
    if (scale > 0.0f && value > 0.0f) return sat_u8(rclamp(roundf(value / scale), 1.0f, hi));
    return 0;
}

/* quantize_q4_k_value / quantize_q2_k_value, src/quant/mod.rs:1133-1151 */
static uint8_t quantize_kq_value(float value, float d, float dmin, uint8_t scale_q, uint8_t min_q,
                                 float hi) {
    float scale = d * (float)scale_q;
    float offset = dmin * (float)min_q;
    if (scale > 0.0f) return sat_u8(rclamp(roundf((value + offset) / scale), 0.0f, hi));
    return 0;
}

/* pack_q4_k_scales, src/quant/mod.rs:1153-1161 */
static void pack_q4_k_scales(const uint8_t *scales, const uint8_t *mins, uint8_t *out) {
    for (int i = 0; i < 4; i++) {
        out[i] = (uint8_t)((scales[i] & 0x3f) | ((scales[i + 4] >> 4) << 6));
        out[i + 4] = (uint8_t)((mins[i] & 0x3f) | ((mins[i + 4] >> 4) << 6));
        out[i + 8] = (uint8_t)((scales[i + 4] & 0x0f) | ((mins[i + 4] & 0x0f) << 4));
    }
}

/* unpack_q4_k_scales, src/gguf/mod.rs:1547-1554 */
static void unpack_q4_k_scales(const uint8_t *packed, uint8_t *scales, uint8_t *mins) {
    for (int i = 0; i < 4; i++) {
        scales[i] = packed[i] & 0x3f;
        mins[i] = packed[i + 4] & 0x3f;
        scales[i + 4] = (uint8_t)((packed[i + 8] & 0x0f) | ((packed[i] >> 6) << 4));
        mins[i + 4] = (uint8_t)((packed[i + 8] >> 4) | ((packed[i + 4] >> 6) << 4));
    }
}

/* quantize_q4_k, src/quant/mod.rs:756-818 */
static size_t quantize_q4_k(const float *data, size_t n, uint8_t *out) {
    size_t o = 0;
    for (size_t c = 0; c < n; c += 256) {
        size_t len = n - c < 256 ? n - c : 256;
        float block[256];
        memset(block, 0, sizeof(block));
        memcpy(block, data + c, len * sizeof(float));
        float sub_scales[8], sub_offsets[8];
        for (int sub = 0; sub < 8; sub++) {
            const float *v = block + sub * 32;
            float mn = INFINITY, mx = -INFINITY;
            for (int i = 0; i < 32; i++) mn = fminf(mn, v[i]);
            for (int i = 0; i < 32; i++) mx = fmaxf(mx, v[i]);
            float offset = mn < 0.0f ? -mn : 0.0f;
            float scale = fmaxf((mx + offset) / 15.0f, 0.0f);
            sub_scales[sub] = scale;
            sub_offsets[sub] = offset;
        }
        float max_scale = 0.0f, max_offset = 0.0f;
        for (int s = 0; s < 8; s++) max_scale = fmaxf(max_scale, sub_scales[s]);
        for (int s = 0; s < 8; s++) max_offset = fmaxf(max_offset, sub_offsets[s]);
        float d = max_scale > 0.0f ? max_scale / 63.0f : 0.0f;
        float dmin = max_offset > 0.0f ? max_offset / 63.0f : 0.0f;
        uint8_t scales[8], mins[8];
        for (int s = 0; s < 8; s++) {
            scales[s] = quantize_uN(sub_scales[s], d, 63.0f);
            mins[s] = quantize_uN(sub_offsets[s], dmin, 63.0f);
        }
        st_f16(out + o, d);
        st_f16(out + o + 2, dmin);
        pack_q4_k_scales(scales, mins, out + o + 4);
        uint8_t *qs = out + o + 16;
        for (int i = 0; i < 128; i++) {
            uint8_t lo = quantize_kq_value(block[i], d, dmin, scales[i / 32], mins[i / 32], 15.0f);
            uint8_t hi = quantize_kq_value(block[i + 128], d, dmin, scales[(i + 128) / 32],
                                           mins[(i + 128) / 32], 15.0f);
            qs[i] = (uint8_t)((lo & 0x0f) | ((hi & 0x0f) << 4));
        }
        o += 144;
    }
    return o;
}

/* quantize_q2_k, src/quant/mod.rs:851-911 */
static size_t quantize_q2_k(const float *data, size_t n, uint8_t *out) {
    size_t o = 0;
    for (size_t c = 0; c < n; c += 256) {
        size_t len = n - c < 256 ? n - c : 256;
        float block[256];
        memset(block, 0, sizeof(block));
        memcpy(block, data + c, len * sizeof(float));
        float sub_scales[16], sub_offsets[16];
        for (int sub = 0; sub < 16; sub++) {
            const float *v = block + sub * 16;
            float mn = INFINITY, mx = -INFINITY;
            for (int i = 0; i < 16; i++) mn = fminf(mn, v[i]);
            for (int i = 0; i < 16; i++) mx = fmaxf(mx, v[i]);
            float offset = mn < 0.0f ? -mn : 0.0f;
            float scale = fmaxf((mx + offset) / 3.0f, 0.0f);
            sub_scales[sub] = scale;
            sub_offsets[sub] = offset;
        }
        float max_scale = 0.0f, max_offset = 0.0f;
        for (int s = 0; s < 16; s++) max_scale = fmaxf(max_scale, sub_scales[s]);
        for (int s = 0; s < 16; s++) max_offset = fmaxf(max_offset, sub_offsets[s]);
        float d = max_scale > 0.0f ? max_scale / 15.0f : 0.0f;
        float dmin = max_offset > 0.0f ? max_offset / 15.0f : 0.0f;
        uint8_t *scales = out + o;
        uint8_t *qs = out + o + 16;
        memset(qs, 0, 64);
        for (int s = 0; s < 16; s++) {
            uint8_t sq = quantize_uN(sub_scales[s], d, 15.0f);
            uint8_t mq = quantize_uN(sub_offsets[s], dmin, 15.0f);
            scales[s] = (uint8_t)((sq & 0x0f) | ((mq & 0x0f) << 4));
        }
        for (int i = 0; i < 256; i++) {
            uint8_t packed = scales[i / 16];
            uint8_t q = quantize_kq_value(block[i], d, dmin, packed & 0x0f, packed >> 4, 3.0f);
            qs[i / 4] |= (uint8_t)((q & 0x03) << ((i % 4) * 2));
        }
        st_f16(out + o + 80, d);
        st_f16(out + o + 82, dmin);
        o += 84;
    }
    return o;
}

size_t orc_quantize(int type, const float *x, size_t n, uint8_t *out) {
    switch (type) {
    case ORC_F32: memcpy(out, x, n * 4); return n * 4;
    case ORC_F16:
        for (size_t i = 0; i < n; i++) st_f16(out + 2 * i, x[i]);
        return n * 2;
    case ORC_Q8_0: return quantize_q8_0(x, n, out);
    case ORC_Q4_0: return quantize_q4_0(x, n, out);
    case ORC_Q4_K: return quantize_q4_k(x, n, out);
    case ORC_Q2_K: return quantize_q2_k(x, n, out);
    default: return 0;
    }
}

/* ------------------------------------------------------------------------ */
/* dequantizers (src/gguf/mod.rs:962-1088)                                   */
/* ------------------------------------------------------------------------ */

/* decode one whole block of `type` starting at `blk` into out[0..block_elems) */
static void dequant_block(int type, const uint8_t *blk, float *out) {
    switch (type) {
    case ORC_Q8_0: { /* dequantize_q8_0, :962-984 */
        float d = ld_f16(blk);
        for (int i = 0; i < 32; i++) out[i] = (float)(int8_t)blk[2 + i] * d;
        break;
    }
    case ORC_Q4_0: { /* dequantize_q4_0, :986-1019 */
        float d = ld_f16(blk);
        const uint8_t *qs = blk + 2;
        for (int i = 0; i < 16; i++) out[i] = (float)(int8_t)((int8_t)(qs[i] & 0x0f) - 8) * d;
        for (int i = 0; i < 16; i++) out[16 + i] = (float)(int8_t)((int8_t)(qs[i] >> 4) - 8) * d;
        break;
    }
    case ORC_Q4_K: { /* dequantize_q4_k, :1021-1056 */
        float d = ld_f16(blk);
        float dmin = ld_f16(blk + 2);
        uint8_t scales[8], mins[8];
        unpack_q4_k_scales(blk + 4, scales, mins);
        const uint8_t *qs = blk + 16;
        for (int i = 0; i < 256; i++) {
            uint8_t packed = qs[i % 128];
            uint8_t q = i < 128 ? (packed & 0x0f) : (packed >> 4);
            int sub = i / 32;
            out[i] = d * (float)scales[sub] * (float)q - dmin * (float)mins[sub];
        }
        break;
    }
    case ORC_Q2_K: { /* dequantize_q2_k, :1058-1088 */
        const uint8_t *scales = blk;
        const uint8_t *qs = blk + 16;
        float d = ld_f16(blk + 80);
        float dmin = ld_f16(blk + 82);
        for (int i = 0; i < 256; i++) {
            uint8_t q = (qs[i / 4] >> ((i % 4) * 2)) & 0x03;
            uint8_t packed = scales[i / 16];
            float scale = (float)(packed & 0x0f);
            float mn = (float)(packed >> 4);
            out[i] = d * scale * (float)q - dmin * mn;
        }
        break;
    }
    default: break;
    }
}

static int block_geom(int type, size_t *elems, size_t *bytes) {
    switch (type) {
    case ORC_Q8_0: *elems = 32; *bytes = 34; return 1;
    case ORC_Q4_0: *elems = 32; *bytes = 18; return 1;
    case ORC_Q4_K: *elems = 256; *bytes = 144; return 1;
    case ORC_Q2_K: *elems = 256; *bytes = 84; return 1;
    case ORC_F32: *elems = 1; *bytes = 4; return 1;
    case ORC_F16:
    case ORC_BF16: *elems = 1; *bytes = 2; return 1;
    default: return 0;
    }
}

void orc_dequantize_range(int type, const uint8_t *data, size_t start, size_t count, float *out) {
    if (type == ORC_F32) {
        memcpy(out, data + start * 4, count * 4);
        return;
    }
    if (type == ORC_F16) {
        for (size_t i = 0; i < count; i++) out[i] = ld_f16(data + 2 * (start + i));
        return;
    }
    if (type == ORC_BF16) {
        for (size_t i = 0; i < count; i++) {
            const uint8_t *p = data + 2 * (start + i);
            uint32_t b = (uint32_t)(p[0] | (p[1] << 8)) << 16;
            memcpy(&out[i], &b, 4);
        }
        return;
    }
    size_t be, bb;
    if (!block_geom(type, &be, &bb)) return;
    float tmp[256];
    size_t i = start, end = start + count, o = 0;
    while (i < end) {
        size_t b = i / be, off = i % be;
        dequant_block(type, data + b * bb, tmp);
        size_t take = be - off;
        if (take > end - i) take = end - i;
        memcpy(out + o, tmp + off, take * sizeof(float));
        o += take;
        i += take;
    }
}

int orc_dequantize(int type, const uint8_t *data, size_t data_len, size_t n, float *out) {
    size_t be, bb;
    if (!block_geom(type, &be, &bb)) return ORC_E_UNSUPPORTED;
    if (data_len < orc_type_size(type, n)) return ORC_E_TRUNCATED;
    orc_dequantize_range(type, data, 0, n, out);
    return ORC_OK;
}

/* ------------------------------------------------------------------------ */
/* kernels (src/kernel/mod.rs)                                               */
/* ------------------------------------------------------------------------ */

/* rms_norm, src/kernel/mod.rs:199-209 */
void orc_rms_norm(const float *x, const float *w, size_t n, float eps, float *out) {
    float sum = 0.0f;
    for (size_t i = 0; i < n; i++) sum += x[i] * x[i];
    float variance = sum / (float)n;
    float rstd = 1.0f / sqrtf(variance + eps);
    for (size_t i = 0; i < n; i++) out[i] = x[i] * rstd * w[i];
}

/* rope_single, src/kernel/mod.rs:258-271 */
void orc_rope_single(float *x, size_t position, size_t head_dim, float base) {
    size_t half = head_dim / 2;
    for (size_t d = 0; d < half; d++) {
        float inv_freq = (float)position / powf(base, 2.0f * (float)d / (float)head_dim);
        float c = cosf(inv_freq);
        float s = sinf(inv_freq);
        float x0 = x[d];
        float x1 = x[d + half];
        x[d] = x0 * c - x1 * s;
        x[d + half] = x0 * s + x1 * c;
    }
}

/* matvec, src/engine/mod.rs:775-801 */
void orc_matvec(const float *w, size_t rows, size_t cols, const float *x, float *y) {
    for (size_t r = 0; r < rows; r++) {
        float sum = 0.0f;
        const float *row = w + r * cols;
        for (size_t c = 0; c < cols; c++) sum += row[c] * x[c];
        y[r] = sum;
    }
}

typedef struct {
    int type;
    const uint8_t *w;
    size_t r0, r1, cols;
    const float *x;
    float *y;
} qmv_job;

static void *qmv_worker(void *arg) {
    qmv_job *j = (qmv_job *)arg;
    float *row = (float *)malloc(j->cols * sizeof(float));
    if (!row) return (void *)1;
    for (size_t r = j->r0; r < j->r1; r++) {
        orc_dequantize_range(j->type, j->w, r * j->cols, j->cols, row);
        float sum = 0.0f;
        for (size_t c = 0; c < j->cols; c++) sum += row[c] * j->x[c];
        j->y[r] = sum;
    }
    free(row);
    return NULL;
}

int orc_qmatvec(int type, const uint8_t *w, size_t rows, size_t cols, const float *x, float *y,
                int threads) {
    size_t be, bb;
    if (!block_geom(type, &be, &bb)) return ORC_E_UNSUPPORTED;
    if (threads < 1) threads = 1;
    if ((size_t)threads > rows) threads = rows ? (int)rows : 1;
    if (threads == 1) {
        qmv_job j = {type, w, 0, rows, cols, x, y};
        return qmv_worker(&j) ? ORC_E_NOMEM : ORC_OK;
    }
    pthread_t tid[256];
    qmv_job jobs[256];
    if (threads > 256) threads = 256;
    size_t per = rows / threads, extra = rows % threads, r = 0;
    for (int t = 0; t < threads; t++) {
        size_t n = per + ((size_t)t < extra ? 1 : 0);
        jobs[t] = (qmv_job){type, w, r, r + n, cols, x, y};
        r += n;
        pthread_create(&tid[t], NULL, qmv_worker, &jobs[t]);
    }
    int rc = ORC_OK;
    for (int t = 0; t < threads; t++) {
        void *ret;
        pthread_join(tid[t], &ret);
        if (ret) rc = ORC_E_NOMEM;
    }
    return rc;
}

/* f32::total_cmp key: orders -0.0 below +0.0 */
static inline int32_t total_key(float v) {
    int32_t b;
    memcpy(&b, &v, 4);
    return b ^ (int32_t)(((uint32_t)(b >> 31)) >> 1);
}

/* greedy_token, src/engine/mod.rs:809-817: finite values only, max_by keeps the last max */
uint32_t orc_greedy(const float *logits, size_t n) {
    int found = 0;
    int32_t best = 0;
    uint32_t idx = 0;
    for (size_t i = 0; i < n; i++) {
        if (!isfinite(logits[i])) continue;
        int32_t k = total_key(logits[i]);
        if (!found || k >= best) {
            best = k;
            idx = (uint32_t)i;
            found = 1;
        }
    }
    return found ? idx : 0;
}

/* softmax, src/kernel/mod.rs:234-255 */
void orc_softmax(const float *x, size_t n, float *out) {
    float mx = -INFINITY;
    for (size_t i = 0; i < n; i++) mx = fmaxf(mx, x[i]);
    float sum = 0.0f;
    for (size_t i = 0; i < n; i++) {
        out[i] = expf(x[i] - mx);
        sum += out[i];
    }
    if (sum > 0.0f)
        for (size_t i = 0; i < n; i++) out[i] /= sum;
}

/* ------------------------------------------------------------------------ */
/* PackedKvBuffer (src/engine/mod.rs:187-313)                                */
/* ------------------------------------------------------------------------ */
struct orc_packed_kv {
    uint8_t *data;
    float *mins;
    float *scales;
    uint32_t bits;
    size_t head_dim;
    size_t bytes_per_token;
    size_t max_seq_len;
};

orc_packed_kv *orc_packed_kv_new(uint32_t bits, size_t head_dim, size_t max_seq_len) {
    orc_packed_kv *b = (orc_packed_kv *)calloc(1, sizeof(*b));
    if (!b) return NULL;
    b->bits = bits;
    b->head_dim = head_dim;
    b->bytes_per_token = div_ceil(head_dim * bits, 8);
    b->max_seq_len = max_seq_len;
    b->data = (uint8_t *)calloc(b->bytes_per_token * max_seq_len + 1, 1);
    b->mins = (float *)calloc(max_seq_len + 1, sizeof(float));
    b->scales = (float *)malloc((max_seq_len + 1) * sizeof(float));
    if (!b->data || !b->mins || !b->scales) {
        orc_packed_kv_free(b);
        return NULL;
    }
    for (size_t i = 0; i < max_seq_len; i++) b->scales[i] = 1.0f;
    return b;
}

void orc_packed_kv_free(orc_packed_kv *b) {
    if (!b) return;
    free(b->data);
    free(b->mins);
    free(b->scales);
    free(b);
}

/* write_bits, :288-299 */
static void pk_write_bits(orc_packed_kv *b, size_t token_start, size_t index, uint32_t value) {
    size_t bit_offset = index * b->bits;
    for (uint32_t bit = 0; bit < b->bits; bit++) {
        if (((value >> bit) & 1u) == 0) continue;
        size_t absolute = token_start * 8 + bit_offset + bit;
        b->data[absolute / 8] |= (uint8_t)(1u << (absolute % 8));
    }
}

/* read_bits, :301-312 */
static uint32_t pk_read_bits(const orc_packed_kv *b, size_t token_start, size_t index) {
    size_t bit_offset = index * b->bits;
    uint32_t value = 0;
    for (uint32_t bit = 0; bit < b->bits; bit++) {
        size_t absolute = token_start * 8 + bit_offset + bit;
        uint32_t bv = (b->data[absolute / 8] >> (absolute % 8)) & 1u;
        value |= bv << bit;
    }
    return value;
}

/* add, :209-232 */
void orc_packed_kv_add(orc_packed_kv *b, size_t position, const float *values) {
    uint32_t levels = (1u << b->bits) - 1u;
    float mn = INFINITY, mx = -INFINITY;
    for (size_t i = 0; i < b->head_dim; i++) mn = fminf(mn, values[i]);
    for (size_t i = 0; i < b->head_dim; i++) mx = fmaxf(mx, values[i]);
    float scale = fabsf(mx - mn) > 1e-8f ? (mx - mn) / (float)levels : 1.0f;
    b->mins[position] = mn;
    b->scales[position] = scale;
    size_t start = position * b->bytes_per_token;
    memset(b->data + start, 0, b->bytes_per_token);
    for (size_t i = 0; i < b->head_dim; i++) {
        uint32_t q = sat_u32(rclamp(roundf((values[i] - mn) / scale), 0.0f, (float)levels));
        pk_write_bits(b, start, i, q);
    }
}

/* value_at, :252-256 */
float orc_packed_kv_value_at(const orc_packed_kv *b, size_t position, size_t dim) {
    size_t start = position * b->bytes_per_token;
    uint32_t q = pk_read_bits(b, start, dim) & ((1u << b->bits) - 1u);
    return b->mins[position] + (float)q * b->scales[position];
}

/* get_all, :234-250 */
void orc_packed_kv_get_all(const orc_packed_kv *b, size_t seq_len, float *out) {
    for (size_t p = 0; p < seq_len; p++)
        for (size_t d = 0; d < b->head_dim; d++)
            out[p * b->head_dim + d] = orc_packed_kv_value_at(b, p, d);
}

/* shift_left, :258-274 */
void orc_packed_kv_shift_left(orc_packed_kv *b, size_t seq_len) {
    if (seq_len <= 1) return;
    size_t bytes = (seq_len - 1) * b->bytes_per_token;
    memmove(b->data, b->data + b->bytes_per_token, bytes);
    memset(b->data + bytes, 0, b->bytes_per_token);
    memmove(b->mins, b->mins + 1, (seq_len - 1) * sizeof(float));
    memmove(b->scales, b->scales + 1, (seq_len - 1) * sizeof(float));
    b->mins[seq_len - 1] = 0.0f;
    b->scales[seq_len - 1] = 1.0f;
}

static void orc_packed_kv_clear(orc_packed_kv *b) {
    memset(b->data, 0, b->bytes_per_token * b->max_seq_len);
    memset(b->mins, 0, b->max_seq_len * sizeof(float));
    for (size_t i = 0; i < b->max_seq_len; i++) b->scales[i] = 1.0f;
}

const uint8_t *orc_packed_kv_data(const orc_packed_kv *b) { return b->data; }
const float *orc_packed_kv_mins(const orc_packed_kv *b) { return b->mins; }
const float *orc_packed_kv_scales(const orc_packed_kv *b) { return b->scales; }
size_t orc_packed_kv_bytes_per_token(const orc_packed_kv *b) { return b->bytes_per_token; }

/* ------------------------------------------------------------------------ */
/* GGUF reader (GgufReader::parse_from_bytes, src/gguf/mod.rs:1091-1358)     */
/* ------------------------------------------------------------------------ */
enum { VT_U8 = 0, VT_I8, VT_U16, VT_I16, VT_U32, VT_I32, VT_F32, VT_BOOL, VT_STR, VT_ARR, VT_U64, VT_I64, VT_F64 };

typedef struct {
    char key[128];
    int vtype;
    uint64_t u;
    int64_t i;
    double f;
} orc_kv;

struct orc_gguf {
    const uint8_t *map;
    size_t len;
    uint32_t version;
    orc_kv *kvs;
    size_t n_kv;
    orc_tensor_info *tensors;
    size_t n_tensors;
    uint64_t alignment;
    uint64_t data_offset;
};

static int rd_u32(const uint8_t *d, size_t len, size_t *pos, uint32_t *v) {
    if (*pos + 4 > len) return 0;
    memcpy(v, d + *pos, 4);
    *pos += 4;
    return 1;
}
static int rd_u64(const uint8_t *d, size_t len, size_t *pos, uint64_t *v) {
    if (*pos + 8 > len) return 0;
    memcpy(v, d + *pos, 8);
    *pos += 8;
    return 1;
}

/* read_value_from_bytes, src/gguf/mod.rs:1359-1538.  Scalar values are kept;
 * arrays are skipped with the reference's byte accounting (I32/F32/String
 * arrays exactly; any other element type is assumed 4 bytes wide, :1533-1536). */
static int rd_value(const uint8_t *d, size_t len, size_t *pos, int vt, orc_kv *kv) {
    switch (vt) {
    case VT_BOOL:
    case VT_U8:
        if (*pos + 1 > len) return 0;
        kv->u = d[*pos];
        kv->i = vt == VT_U8 ? (int64_t)d[*pos] : (int64_t)(d[*pos] != 0);
        *pos += 1;
        return 1;
    case VT_I8:
        if (*pos + 1 > len) return 0;
        kv->i = (int8_t)d[*pos];
        *pos += 1;
        return 1;
    case VT_U16:
    case VT_I16: {
        if (*pos + 2 > len) return 0;
        uint16_t v;
        memcpy(&v, d + *pos, 2);
        kv->u = v;
        kv->i = vt == VT_I16 ? (int16_t)v : v;
        *pos += 2;
        return 1;
    }
    case VT_U32:
    case VT_I32:
    case VT_F32: {
        uint32_t v;
        if (!rd_u32(d, len, pos, &v)) return 0;
        kv->u = v;
        kv->i = (int32_t)v;
        float f;
        memcpy(&f, &v, 4);
        kv->f = f;
        return 1;
    }
    case VT_U64:
    case VT_I64:
    case VT_F64: {
        uint64_t v;
        if (!rd_u64(d, len, pos, &v)) return 0;
        kv->u = v;
        kv->i = (int64_t)v;
        double f;
        memcpy(&f, &v, 8);
        kv->f = f;
        return 1;
    }
    case VT_STR: {
        uint64_t sl;
        if (!rd_u64(d, len, pos, &sl)) return 0;
        if (sl > len - *pos) return 0;
        *pos += sl;
        return 1;
    }
    case VT_ARR: {
        uint32_t at;
        uint64_t n;
        if (!rd_u32(d, len, pos, &at) || !rd_u64(d, len, pos, &n)) return 0;
        if (at > VT_F64) return 0;
        if (at == VT_STR) {
            for (uint64_t k = 0; k < n; k++) {
                uint64_t sl;
                if (!rd_u64(d, len, pos, &sl)) return 0;
                if (sl > len - *pos) return 0;
                *pos += sl;
            }
        } else {
            if (n > (len - *pos) / 4) return 0;
            *pos += n * 4;
        }
        return 1;
    }
    default: return 0;
    }
}

int orc_gguf_open(const char *path, orc_gguf **out) {
    *out = NULL;
    int fd = open(path, O_RDONLY);
    if (fd < 0) return ORC_E_IO;
    struct stat st;
    if (fstat(fd, &st) != 0) {
        close(fd);
        return ORC_E_IO;
    }
    size_t len = (size_t)st.st_size;
    const uint8_t *d = len ? (const uint8_t *)mmap(NULL, len, PROT_READ, MAP_PRIVATE, fd, 0) : NULL;
    close(fd);
    if (len && d == MAP_FAILED) return ORC_E_IO;
    orc_gguf *g = (orc_gguf *)calloc(1, sizeof(*g));
    g->map = d;
    g->len = len;
    size_t pos = 0;
    int rc = ORC_E_TRUNCATED;
    uint64_t tc, kc;
    if (len < 8 || memcmp(d, "GGUF", 4) != 0) {
        rc = ORC_E_INVALID;
        goto fail;
    }
    pos = 4;
    if (!rd_u32(d, len, &pos, &g->version)) goto fail;
    if (g->version != 2 && g->version != 3) {
        rc = ORC_E_INVALID;
        goto fail;
    }
    if (!rd_u64(d, len, &pos, &tc) || !rd_u64(d, len, &pos, &kc)) goto fail;
    if (kc > len || tc > len) goto fail;
    g->kvs = (orc_kv *)calloc(kc ? kc : 1, sizeof(orc_kv));
    g->tensors = (orc_tensor_info *)calloc(tc ? tc : 1, sizeof(orc_tensor_info));
    for (uint64_t k = 0; k < kc; k++) {
        uint64_t kl;
        uint32_t vt;
        if (!rd_u64(d, len, &pos, &kl) || kl > len - pos) goto fail;
        orc_kv *kv = &g->kvs[g->n_kv];
        size_t cp = kl < sizeof(kv->key) - 1 ? kl : sizeof(kv->key) - 1;
        memcpy(kv->key, d + pos, cp);
        pos += kl;
        if (!rd_u32(d, len, &pos, &vt)) goto fail;
        if (vt > VT_F64) {
            rc = ORC_E_INVALID;
            goto fail;
        }
        kv->vtype = (int)vt;
        if (!rd_value(d, len, &pos, (int)vt, kv)) goto fail;
        /* HashMap insert: a later duplicate key replaces an earlier one */
        size_t j;
        for (j = 0; j < g->n_kv; j++)
            if (strcmp(g->kvs[j].key, kv->key) == 0) break;
        if (j < g->n_kv) g->kvs[j] = *kv;
        else g->n_kv++;
    }
    for (uint64_t t = 0; t < tc; t++) {
        uint64_t nl;
        if (!rd_u64(d, len, &pos, &nl) || nl > len - pos) goto fail;
        orc_tensor_info *ti = &g->tensors[g->n_tensors];
        size_t cp = nl < sizeof(ti->name) - 1 ? nl : sizeof(ti->name) - 1;
        memcpy(ti->name, d + pos, cp);
        pos += nl;
        if (!rd_u32(d, len, &pos, &ti->n_dims)) goto fail;
        for (uint32_t k = 0; k < ti->n_dims; k++) {
            uint64_t dim;
            if (!rd_u64(d, len, &pos, &dim)) goto fail;
            if (k < 4) ti->shape[k] = dim;
        }
        if (ti->n_dims > 4) {
            rc = ORC_E_UNSUPPORTED;
            goto fail;
        }
        uint32_t ty;
        if (!rd_u32(d, len, &pos, &ty)) goto fail;
        ti->type = (int)ty;
        if (!rd_u64(d, len, &pos, &ti->offset)) goto fail;
        g->n_tensors++;
    }
    g->alignment = 32;
    for (size_t j = 0; j < g->n_kv; j++) {
        if (strcmp(g->kvs[j].key, "general.alignment") == 0 &&
            (g->kvs[j].vtype == VT_U32 || g->kvs[j].vtype == VT_U64))
            g->alignment = g->kvs[j].u;
    }
    if (g->alignment < 1) g->alignment = 1;
    g->data_offset = div_ceil(pos, g->alignment) * g->alignment;
    *out = g;
    return ORC_OK;
fail:
    orc_gguf_close(g);
    return rc;
}

void orc_gguf_close(orc_gguf *g) {
    if (!g) return;
    if (g->map && g->len) munmap((void *)g->map, g->len);
    free(g->kvs);
    free(g->tensors);
    free(g);
}

size_t orc_gguf_tensor_count(const orc_gguf *g) { return g->n_tensors; }
const orc_tensor_info *orc_gguf_tensor(const orc_gguf *g, size_t i) {
    return i < g->n_tensors ? &g->tensors[i] : NULL;
}
uint64_t orc_gguf_data_offset(const orc_gguf *g) { return g->data_offset; }

static size_t tensor_elems(const orc_tensor_info *t) {
    size_t n = 1;
    for (uint32_t k = 0; k < t->n_dims; k++) n *= (size_t)t->shape[k];
    return n;
}

const uint8_t *orc_gguf_tensor_data(const orc_gguf *g, const orc_tensor_info *t) {
    size_t bytes = orc_type_size(t->type, tensor_elems(t));
    uint64_t off = g->data_offset + t->offset;
    if (off > g->len || bytes > g->len - off) return NULL;
    return g->map + off;
}

static const orc_kv *find_kv(const orc_gguf *g, const char *key) {
    for (size_t j = 0; j < g->n_kv; j++)
        if (strcmp(g->kvs[j].key, key) == 0) return &g->kvs[j];
    return NULL;
}

/* ModelMetadata::get_usize, src/gguf/mod.rs:511-520: U64, U32, non-negative I64/I32 */
int orc_gguf_get_usize(const orc_gguf *g, const char *key, uint64_t *out) {
    const orc_kv *kv = find_kv(g, key);
    if (!kv) return 0;
    if (kv->vtype == VT_U64 || kv->vtype == VT_U32) {
        *out = kv->u;
        return 1;
    }
    if ((kv->vtype == VT_I64 || kv->vtype == VT_I32) && kv->i >= 0) {
        *out = (uint64_t)kv->i;
        return 1;
    }
    return 0;
}

int orc_gguf_get_f32(const orc_gguf *g, const char *key, float *out) {
    const orc_kv *kv = find_kv(g, key);
    if (!kv || kv->vtype != VT_F32) return 0;
    *out = (float)kv->f;
    return 1;
}

/* ------------------------------------------------------------------------ */
/* decode engine (src/engine/mod.rs)                                         */
/* ------------------------------------------------------------------------ */
typedef struct {
    int present;
    int type;
    const uint8_t *data;
    size_t elems;
} orc_wt;

typedef struct {
    orc_wt attn_norm, q, k, v, o, ffn_norm, gate, up, down;
    /* KvCache, :387-450 */
    float *kf, *vf;          /* float streams [max_seq][kv_dim] */
    orc_packed_kv *kp, *vp;  /* packed streams */
    size_t seq_len;
} orc_layer;

struct orc_model {
    orc_gguf *g;
    orc_model_info info;
    orc_layer *layers;
    orc_wt embd, out_norm, out_head;
    int threads;
    float *hidden, *normed, *q, *k, *v, *attn, *tmp, *gate, *up, *scores, *rowbuf;
    float *norm_tmp;
};

static orc_wt find_tensor(const orc_gguf *g, const char *const *names, size_t n_names,
                          size_t cap) {
    orc_wt w = {0, 0, NULL, 0};
    for (size_t k = 0; k < n_names; k++) {
        for (size_t i = 0; i < g->n_tensors; i++) {
            const orc_tensor_info *t = &g->tensors[i];
            if (strcmp(t->name, names[k]) != 0) continue;
            size_t be, bb;
            size_t elems = tensor_elems(t);
            /* load_model skips empty, over-cap and unsupported tensors (:600-650) */
            if (elems == 0 || (cap && elems > cap) || !block_geom(t->type, &be, &bb)) continue;
            const uint8_t *p = orc_gguf_tensor_data(g, t);
            if (!p) continue;
            w.present = 1;
            w.type = t->type;
            w.data = p;
            w.elems = elems;
            return w;
        }
    }
    return w;
}

/* layer_tensor_names, src/engine/mod.rs:709-733 */
static orc_wt layer_tensor(const orc_gguf *g, uint32_t layer, const char *role, const char *hf) {
    char a[160], b[160], c[160];
    snprintf(a, sizeof a, "blk.%u.%s.weight", layer, role);
    snprintf(b, sizeof b, "model.layers.%u.%s.weight", layer, hf);
    snprintf(c, sizeof c, "layers.%u.%s.weight", layer, hf);
    const char *names[3] = {a, b, c};
    return find_tensor(g, names, 3, 0);
}


void orc_model_free(orc_model *m) {
    if (!m) return;
    if (m->layers) {
        for (uint32_t l = 0; l < m->info.num_layers; l++) {
            free(m->layers[l].kf);
            free(m->layers[l].vf);
            orc_packed_kv_free(m->layers[l].kp);
            orc_packed_kv_free(m->layers[l].vp);
        }
        free(m->layers);
    }
    free(m->hidden);
    free(m->normed);
    free(m->q);
    free(m->k);
    free(m->v);
    free(m->attn);
    free(m->tmp);
    free(m->gate);
    free(m->up);
    free(m->scores);
    free(m->rowbuf);
    free(m->norm_tmp);
    orc_gguf_close(m->g);
    free(m);
}

/* load_model, src/engine/mod.rs:539-692 (metadata defaults :551-562) */
int orc_model_load(const char *path, uint32_t kv_bits_k, uint32_t kv_bits_v, int threads,
                   uint32_t max_seq_len_override, orc_model **out) {
    *out = NULL;
    orc_gguf *g;
    int rc = orc_gguf_open(path, &g);
    if (rc) return rc;
    orc_model *m = (orc_model *)calloc(1, sizeof(*m));
    m->g = g;
    m->threads = threads < 1 ? 1 : threads;
    uint64_t v;
    orc_model_info *I = &m->info;
    I->num_layers = orc_gguf_get_usize(g, "llama.block_count", &v) ? (uint32_t)v : 32;
    I->hidden_size = orc_gguf_get_usize(g, "llama.embedding_length", &v) ? (uint32_t)v : 4096;
    I->ff_dim = orc_gguf_get_usize(g, "llama.feed_forward_length", &v) ? (uint32_t)v : 11008;
    I->num_heads = orc_gguf_get_usize(g, "llama.attention.head_count", &v) ? (uint32_t)v : 32;
    I->num_kv_heads =
        orc_gguf_get_usize(g, "llama.attention.head_count_kv", &v) ? (uint32_t)v : I->num_heads;
    float fb;
    /* rope_freq_base, src/gguf/mod.rs:569-571 */
    I->rope_freq_base = orc_gguf_get_f32(g, "llama.rope.freq_base", &fb) ? fb : 1000000.0f;
    /* InferenceConfig::default().rms_norm_eps, src/engine/mod.rs:94 (GGUF key ignored) */
    I->rms_norm_eps = 1e-5f;
    if (I->num_heads == 0 || I->hidden_size == 0) {
        orc_model_free(m);
        return ORC_E_INVALID;
    }
    I->head_dim = I->hidden_size / I->num_heads;
    I->max_seq_len = orc_gguf_get_usize(g, "llama.context_length", &v) ? (uint32_t)v : 4096;
    if (max_seq_len_override) I->max_seq_len = max_seq_len_override;
    I->kv_bits_k = kv_bits_k;
    I->kv_bits_v = kv_bits_v;

    static const char *embd_names[] = {"token_embd.weight", "token_embd",
                                       "model.embed_tokens.weight", "transformer.wte.weight"};
    static const char *onorm_names[] = {"output_norm.weight", "norm.weight", "model.norm.weight",
                                        "transformer.ln_f.weight"};
    static const char *head_names[] = {"output.weight", "lm_head.weight",
                                       "model.embed_tokens.weight", "token_embd.weight"};
    m->embd = find_tensor(g, embd_names, 4, 0);
    m->out_norm = find_tensor(g, onorm_names, 4, 0);
    m->out_head = find_tensor(g, head_names, 4, 0);
    size_t H = I->hidden_size;
    I->vocab_rows = m->out_head.present ? (uint32_t)(m->out_head.elems / H) : (uint32_t)H;

    size_t kv_dim = (size_t)I->num_kv_heads * I->head_dim;
    m->layers = (orc_layer *)calloc(I->num_layers ? I->num_layers : 1, sizeof(orc_layer));
    for (uint32_t l = 0; l < I->num_layers; l++) {
        orc_layer *L = &m->layers[l];
        L->attn_norm = layer_tensor(g, l, "attn_norm", "input_layernorm");
        L->q = layer_tensor(g, l, "attn_q", "self_attn.q_proj");
        L->k = layer_tensor(g, l, "attn_k", "self_attn.k_proj");
        L->v = layer_tensor(g, l, "attn_v", "self_attn.v_proj");
        L->o = layer_tensor(g, l, "attn_output", "self_attn.o_proj");
        L->ffn_norm = layer_tensor(g, l, "ffn_norm", "post_attention_layernorm");
        L->gate = layer_tensor(g, l, "ffn_gate", "mlp.gate_proj");
        L->up = layer_tensor(g, l, "ffn_up", "mlp.up_proj");
        L->down = layer_tensor(g, l, "ffn_down", "mlp.down_proj");
        /* KvCache::new(num_kv_heads*head_dim, max_seq_len, kv_quant), :593-597 */
        if (kv_bits_k == 0) {
            L->kf = (float *)calloc((size_t)I->max_seq_len * kv_dim + 1, sizeof(float));
            L->vf = (float *)calloc((size_t)I->max_seq_len * kv_dim + 1, sizeof(float));
            if (!L->kf || !L->vf) {
                orc_model_free(m);
                return ORC_E_NOMEM;
            }
        } else {
            L->kp = orc_packed_kv_new(kv_bits_k, kv_dim, I->max_seq_len);
            L->vp = orc_packed_kv_new(kv_bits_v, kv_dim, I->max_seq_len);
            if (!L->kp || !L->vp) {
                orc_model_free(m);
                return ORC_E_NOMEM;
            }
        }
    }
    size_t F = I->ff_dim, Q = (size_t)I->num_heads * I->head_dim;
    size_t big = H > F ? H : F;
    if (Q > big) big = Q;
    if (I->vocab_rows > big) big = I->vocab_rows;
    m->hidden = (float *)calloc(H, sizeof(float));
    m->normed = (float *)calloc(H, sizeof(float));
    m->q = (float *)calloc(Q + 1, sizeof(float));
    m->k = (float *)calloc(kv_dim + 1, sizeof(float));
    m->v = (float *)calloc(kv_dim + 1, sizeof(float));
    m->attn = (float *)calloc(Q + 1, sizeof(float));
    m->tmp = (float *)calloc(big, sizeof(float));
    m->gate = (float *)calloc(F + 1, sizeof(float));
    m->up = (float *)calloc(F + 1, sizeof(float));
    m->scores = (float *)calloc((size_t)I->max_seq_len + 1, sizeof(float));
    m->rowbuf = (float *)calloc(big, sizeof(float));
    m->norm_tmp = (float *)calloc(H, sizeof(float));
    *out = m;
    return ORC_OK;
}

void orc_model_get_info(const orc_model *m, orc_model_info *info) { *info = m->info; }
void orc_model_set_threads(orc_model *m, int threads) { m->threads = threads < 1 ? 1 : threads; }
void orc_model_set_eps(orc_model *m, float eps) { m->info.rms_norm_eps = eps; }
size_t orc_model_seq_len(const orc_model *m, uint32_t layer) {
    return layer < m->info.num_layers ? m->layers[layer].seq_len : 0;
}
const float *orc_model_last_hidden(const orc_model *m) { return m->hidden; }

/* Self::matvec with the shape checks of :775-793 */
static int wmatvec(orc_model *m, const orc_wt *w, size_t rows, size_t cols, const float *x,
                   float *y) {
    if (!w->present) return ORC_E_MISSING_TENSOR;
    if (w->elems < rows * cols) return ORC_E_SHAPE;
    return orc_qmatvec(w->type, w->data, rows, cols, x, y, m->threads);
}

static int wnorm(const orc_wt *w, size_t n, const float *x, float eps, float *out, float *tmp) {
    if (!w->present) return ORC_E_MISSING_TENSOR;
    if (w->elems < n) return ORC_E_SHAPE;
    orc_dequantize_range(w->type, w->data, 0, n, tmp);
    orc_rms_norm(x, tmp, n, eps, out);
    return ORC_OK;
}

/* KvCache::add + shift, :410-426 */
static void kv_add(orc_model *m, orc_layer *L, const float *k, const float *v) {
    size_t kv_dim = (size_t)m->info.num_kv_heads * m->info.head_dim;
    if (L->seq_len >= m->info.max_seq_len) {
        if (L->kf) {
            size_t total = L->seq_len * kv_dim;
            memmove(L->kf, L->kf + kv_dim, (total - kv_dim) * sizeof(float));
            memset(L->kf + total - kv_dim, 0, kv_dim * sizeof(float));
            memmove(L->vf, L->vf + kv_dim, (total - kv_dim) * sizeof(float));
            memset(L->vf + total - kv_dim, 0, kv_dim * sizeof(float));
        } else {
            orc_packed_kv_shift_left(L->kp, L->seq_len);
            orc_packed_kv_shift_left(L->vp, L->seq_len);
        }
        L->seq_len -= 1;
    }
    if (L->kf) {
        memcpy(L->kf + L->seq_len * kv_dim, k, kv_dim * sizeof(float));
        memcpy(L->vf + L->seq_len * kv_dim, v, kv_dim * sizeof(float));
    } else {
        orc_packed_kv_add(L->kp, L->seq_len, k);
        orc_packed_kv_add(L->vp, L->seq_len, v);
    }
    L->seq_len += 1;
}

static inline float kv_value(const orc_layer *L, int is_v, size_t token, size_t dim,
                             size_t kv_dim) {
    if (L->kf) return (is_v ? L->vf : L->kf)[token * kv_dim + dim];
    return orc_packed_kv_value_at(is_v ? L->vp : L->kp, token, dim);
}

/* KvCache::attention_decode, :452-499 */
static void attention_decode(orc_model *m, const orc_layer *L, const float *q, float *out) {
    size_t D = m->info.head_dim, Hq = m->info.num_heads, Hkv = m->info.num_kv_heads;
    size_t kv_dim = Hkv * D;
    size_t group = Hq / Hkv;
    if (group < 1) group = 1;
    float scale = 1.0f / sqrtf((float)D);
    memset(out, 0, Hq * D * sizeof(float));
    float *scores = m->scores;
    for (size_t qh = 0; qh < Hq; qh++) {
        size_t kvh = qh / group;
        if (kvh > Hkv - 1) kvh = Hkv - 1;
        for (size_t t = 0; t < L->seq_len; t++) {
            float score = 0.0f;
            for (size_t d = 0; d < D; d++)
                score += q[qh * D + d] * kv_value(L, 0, t, kvh * D + d, kv_dim);
            scores[t] = score * scale;
        }
        float mx = -INFINITY;
        for (size_t t = 0; t < L->seq_len; t++) mx = fmaxf(mx, scores[t]);
        float sum_exp = 0.0f;
        for (size_t t = 0; t < L->seq_len; t++) {
            scores[t] = expf(scores[t] - mx);
            sum_exp += scores[t];
        }
        if (sum_exp <= 0.0f) continue;
        for (size_t d = 0; d < D; d++) {
            float ws = 0.0f;
            size_t dim = kvh * D + d;
            for (size_t t = 0; t < L->seq_len; t++)
                ws += (scores[t] / sum_exp) * kv_value(L, 1, t, dim, kv_dim);
            out[qh * D + d] = ws;
        }
    }
}

/* decode_with_cache, src/engine/mod.rs:1087-1146 (+ transformer_logits :1032-1044) */
int orc_model_decode(orc_model *m, uint32_t token, size_t position, float *logits) {
    orc_model_info *I = &m->info;
    size_t H = I->hidden_size, D = I->head_dim, F = I->ff_dim;
    size_t Q = (size_t)I->num_heads * D, kv_dim = (size_t)I->num_kv_heads * D;
    float eps = I->rms_norm_eps;
    int rc;
    if (!m->embd.present) return ORC_E_MISSING_TENSOR;
    size_t vocab_rows = m->embd.elems / H;
    if (vocab_rows < 1) vocab_rows = 1;
    size_t start = ((size_t)token % vocab_rows) * H;
    if (start + H > m->embd.elems) return ORC_E_SHAPE;
    orc_dequantize_range(m->embd.type, m->embd.data, start, H, m->hidden);

    for (uint32_t l = 0; l < I->num_layers; l++) {
        orc_layer *L = &m->layers[l];
        if ((rc = wnorm(&L->attn_norm, H, m->hidden, eps, m->normed, m->norm_tmp))) return rc;
        if ((rc = wmatvec(m, &L->q, Q, H, m->normed, m->q))) return rc;
        if ((rc = wmatvec(m, &L->k, kv_dim, H, m->normed, m->k))) return rc;
        if ((rc = wmatvec(m, &L->v, kv_dim, H, m->normed, m->v))) return rc;
        /* apply_rope_heads, :1026-1030 */
        for (size_t h = 0; h + D <= Q; h += D) orc_rope_single(m->q + h, position, D, I->rope_freq_base);
        for (size_t h = 0; h + D <= kv_dim; h += D)
            orc_rope_single(m->k + h, position, D, I->rope_freq_base);
        kv_add(m, L, m->k, m->v);
        attention_decode(m, L, m->q, m->attn);
        if ((rc = wmatvec(m, &L->o, H, H, m->attn, m->tmp))) return rc;
        for (size_t i = 0; i < H; i++) m->hidden[i] += m->tmp[i];

        if ((rc = wnorm(&L->ffn_norm, H, m->hidden, eps, m->normed, m->norm_tmp))) return rc;
        if ((rc = wmatvec(m, &L->gate, F, H, m->normed, m->gate))) return rc;
        if ((rc = wmatvec(m, &L->up, F, H, m->normed, m->up))) return rc;
        for (size_t i = 0; i < F; i++) m->gate[i] = (m->gate[i] / (1.0f + expf(-m->gate[i]))) * m->up[i];
        if ((rc = wmatvec(m, &L->down, H, F, m->gate, m->tmp))) return rc;
        for (size_t i = 0; i < H; i++) m->hidden[i] += m->tmp[i];
    }

    /* transformer_logits: output norm (default ones) then head matvec */
    if (m->out_norm.present && m->out_norm.elems >= H) {
        orc_dequantize_range(m->out_norm.type, m->out_norm.data, 0, H, m->norm_tmp);
    } else {
        for (size_t i = 0; i < H; i++) m->norm_tmp[i] = 1.0f;
    }
    orc_rms_norm(m->hidden, m->norm_tmp, H, eps, m->normed);
    if (m->out_head.present) {
        size_t rows = m->out_head.elems / H;
        return orc_qmatvec(m->out_head.type, m->out_head.data, rows, H, m->normed, logits,
                           m->threads);
    }
    memcpy(logits, m->normed, H * sizeof(float));
    return ORC_OK;
}

static void kv_clear(orc_model *m) {
    size_t kv_dim = (size_t)m->info.num_kv_heads * m->info.head_dim;
    for (uint32_t l = 0; l < m->info.num_layers; l++) {
        orc_layer *L = &m->layers[l];
        if (L->kf) {
            memset(L->kf, 0, (size_t)m->info.max_seq_len * kv_dim * sizeof(float));
            memset(L->vf, 0, (size_t)m->info.max_seq_len * kv_dim * sizeof(float));
        } else {
            orc_packed_kv_clear(L->kp);
            orc_packed_kv_clear(L->vp);
        }
        L->seq_len = 0;
    }
}

/* prefill, src/engine/mod.rs:1149-1170.  The reference falls back to a
 * stateless smoke decode when a tensor is missing; this restatement returns
 * the error instead (the CUDA backend never falls back). */
int orc_model_prefill(orc_model *m, const uint32_t *tokens, size_t n, float *logits) {
    if (n == 0) return ORC_OK;
    kv_clear(m);
    for (size_t p = 0; p < n; p++) {
        int rc = orc_model_decode(m, tokens[p], p, logits);
        if (rc) return rc;
    }
    return ORC_OK;
}

/* generate_with_config_streaming with temperature 0, src/engine/mod.rs:1196-1238 */
int orc_model_generate(orc_model *m, const uint32_t *prompt, size_t n, size_t max_tokens,
                       uint32_t *out) {
    size_t V = m->info.vocab_rows;
    float *logits = (float *)calloc(V + 1, sizeof(float));
    if (!logits) return ORC_E_NOMEM;
    memcpy(out, prompt, n * sizeof(uint32_t));
    int rc = orc_model_prefill(m, prompt, n, logits);
    size_t have_logits = n > 0 ? V : 0;
    for (size_t i = 0; rc == ORC_OK && i < max_tokens; i++) {
        uint32_t next = have_logits ? orc_greedy(logits, have_logits) : 0;
        out[n + i] = next;
        size_t position = n + i;
        rc = orc_model_decode(m, next, position, logits);
        have_logits = V;
    }
    free(logits);
    return rc;
}

/* ------------------------------------------------------------------------ */
/* Layer-major prefill (a faster schedule of orc_model_prefill, same bits)   */
/* ------------------------------------------------------------------------ */
/* The reference prefill (src/engine/mod.rs:1149-1170) runs decode_with_cache
 * once per prompt token.  Token p at layer l reads only the layer-l K/V of
 * tokens 0..p, so running every token through layer l before layer l+1 gives
 * the same values as long as each token's own arithmetic is unchanged: every
 * matvec row below is the same sequential f32 sum (mul then add, in column
 * order), merely computed for a tile of tokens at once (one dequantized row,
 * many tokens), and attention for token p runs over exactly p + 1 cached
 * positions.  Used to produce parity fixtures at long contexts; the result is
 * checked bit for bit against orc_model_prefill by tests/test_oracle_batched.py. */

#define ORC_TT 32 /* tokens per tile of the batched matvec */
typedef float orc_v8 __attribute__((vector_size(32)));

typedef struct {
    int type;
    const uint8_t *w;
    size_t rows, cols, nt;
    const float *xt; /* [cols][nt]: token-minor copy of the inputs */
    float *y;        /* [nt][y_stride] */
    size_t y_stride;
    size_t r0, r1;
    int rc;
} qmm_job;

__attribute__((target_clones("avx512f", "avx2", "default")))
static void qmm_rows(qmm_job *j, float *row) {
    const size_t nt = j->nt, K = j->cols;
    for (size_t r = j->r0; r < j->r1; r++) {
        orc_dequantize_range(j->type, j->w, r * K, K, row);
        for (size_t t0 = 0; t0 < nt; t0 += ORC_TT) {
            const size_t tn = nt - t0 < ORC_TT ? nt - t0 : ORC_TT;
            if (tn == ORC_TT) {
                orc_v8 a0 = {0}, a1 = {0}, a2 = {0}, a3 = {0};
                for (size_t c = 0; c < K; c++) {
                    const float *xp = j->xt + c * nt + t0;
                    orc_v8 x0, x1, x2, x3;
                    memcpy(&x0, xp, 32);
                    memcpy(&x1, xp + 8, 32);
                    memcpy(&x2, xp + 16, 32);
                    memcpy(&x3, xp + 24, 32);
                    const float wv = row[c];
                    /* sum += w * x: a separately rounded product, then the add */
                    a0 = a0 + wv * x0;
                    a1 = a1 + wv * x1;
                    a2 = a2 + wv * x2;
                    a3 = a3 + wv * x3;
                }
                float acc[ORC_TT];
                memcpy(acc, &a0, 32);
                memcpy(acc + 8, &a1, 32);
                memcpy(acc + 16, &a2, 32);
                memcpy(acc + 24, &a3, 32);
                for (size_t t = 0; t < ORC_TT; t++) j->y[(t0 + t) * j->y_stride + r] = acc[t];
            } else {
                for (size_t t = 0; t < tn; t++) {
                    float sum = 0.0f;
                    for (size_t c = 0; c < K; c++) sum += row[c] * j->xt[c * nt + t0 + t];
                    j->y[(t0 + t) * j->y_stride + r] = sum;
                }
            }
        }
    }
}

static void *qmm_worker(void *arg) {
    qmm_job *j = (qmm_job *)arg;
    float *row = (float *)malloc(j->cols * sizeof(float));
    if (!row) {
        j->rc = ORC_E_NOMEM;
        return NULL;
    }
    qmm_rows(j, row);
    free(row);
    return NULL;
}

/* Y[t][r] = sum_c W[r][c] * X[t][c] for nt tokens; rows split over threads. */
static int orc_qmatmul(int type, const uint8_t *w, size_t rows, size_t cols, const float *x,
                       size_t x_stride, size_t nt, float *y, size_t y_stride, int threads) {
    size_t be, bb;
    if (!block_geom(type, &be, &bb)) return ORC_E_UNSUPPORTED;
    float *xt = (float *)malloc(cols * nt * sizeof(float) + 64);
    if (!xt) return ORC_E_NOMEM;
    for (size_t t = 0; t < nt; t++)
        for (size_t c = 0; c < cols; c++) xt[c * nt + t] = x[t * x_stride + c];
    if (threads < 1) threads = 1;
    if (threads > 256) threads = 256;
    if ((size_t)threads > rows) threads = rows ? (int)rows : 1;
    pthread_t tid[256];
    qmm_job jobs[256];
    size_t per = rows / threads, extra = rows % threads, r = 0;
    for (int t = 0; t < threads; t++) {
        size_t n = per + ((size_t)t < extra ? 1 : 0);
        jobs[t] = (qmm_job){type, w, rows, cols, nt, xt, y, y_stride, r, r + n, ORC_OK};
        r += n;
        pthread_create(&tid[t], NULL, qmm_worker, &jobs[t]);
    }
    int rc = ORC_OK;
    for (int t = 0; t < threads; t++) {
        pthread_join(tid[t], NULL);
        if (jobs[t].rc) rc = jobs[t].rc;
    }
    free(xt);
    return rc;
}

static int bmatmul(orc_model *m, const orc_wt *w, size_t rows, size_t cols, const float *x,
                   size_t x_stride, size_t nt, float *y, size_t y_stride) {
    if (!w->present) return ORC_E_MISSING_TENSOR;
    if (w->elems < rows * cols) return ORC_E_SHAPE;
    return orc_qmatmul(w->type, w->data, rows, cols, x, x_stride, nt, y, y_stride, m->threads);
}

/* attention_decode (:452-499) for one query head over `len` cached positions */
static void attention_head(const orc_model *m, const orc_layer *L, size_t len, const float *q,
                           size_t qh, float *scores, float *out) {
    size_t D = m->info.head_dim, Hq = m->info.num_heads, Hkv = m->info.num_kv_heads;
    size_t kv_dim = Hkv * D;
    size_t group = Hq / Hkv;
    if (group < 1) group = 1;
    float scale = 1.0f / sqrtf((float)D);
    size_t kvh = qh / group;
    if (kvh > Hkv - 1) kvh = Hkv - 1;
    for (size_t d = 0; d < D; d++) out[qh * D + d] = 0.0f;
    for (size_t t = 0; t < len; t++) {
        float score = 0.0f;
        for (size_t d = 0; d < D; d++) score += q[qh * D + d] * kv_value(L, 0, t, kvh * D + d, kv_dim);
        scores[t] = score * scale;
    }
    float mx = -INFINITY;
    for (size_t t = 0; t < len; t++) mx = fmaxf(mx, scores[t]);
    float sum_exp = 0.0f;
    for (size_t t = 0; t < len; t++) {
        scores[t] = expf(scores[t] - mx);
        sum_exp += scores[t];
    }
    if (sum_exp <= 0.0f) return;
    for (size_t d = 0; d < D; d++) {
        float ws = 0.0f;
        size_t dim = kvh * D + d;
        for (size_t t = 0; t < len; t++) ws += (scores[t] / sum_exp) * kv_value(L, 1, t, dim, kv_dim);
        out[qh * D + d] = ws;
    }
}

typedef struct {
    const orc_model *m;
    const orc_layer *L;
    const float *q;  /* [n][Q] */
    float *out;      /* [n][Q] */
    size_t p0, n, Q;
    size_t w, nw;    /* this worker takes (token, head) pairs w, w + nw, ... */
} attn_job;

static void *attn_worker(void *arg) {
    attn_job *j = (attn_job *)arg;
    size_t Hq = j->m->info.num_heads;
    float *scores = (float *)malloc((j->p0 + j->n + 1) * sizeof(float));
    if (!scores) return (void *)1;
    for (size_t i = j->w; i < j->n * Hq; i += j->nw) {
        size_t t = i / Hq, qh = i % Hq;
        attention_head(j->m, j->L, j->p0 + t + 1, j->q + t * j->Q, qh, scores, j->out + t * j->Q);
    }
    free(scores);
    return NULL;
}

/* orc_model_prefill with a layer-major schedule: identical logits and KV. */
int orc_model_prefill_batched(orc_model *m, const uint32_t *tokens, size_t n, float *logits) {
    if (n == 0) return ORC_OK;
    orc_model_info *I = &m->info;
    if (n > I->max_seq_len) return ORC_E_INVALID; /* no shift-on-full in this schedule */
    kv_clear(m);
    size_t H = I->hidden_size, D = I->head_dim, F = I->ff_dim;
    size_t Q = (size_t)I->num_heads * D, kv_dim = (size_t)I->num_kv_heads * D;
    float eps = I->rms_norm_eps;
    int rc = ORC_OK;
    if (!m->embd.present) return ORC_E_MISSING_TENSOR;
    size_t vocab_rows = m->embd.elems / H;
    if (vocab_rows < 1) vocab_rows = 1;
    float *hid = (float *)malloc(n * H * sizeof(float));
    float *nrm = (float *)malloc(n * H * sizeof(float));
    float *qb = (float *)malloc(n * Q * sizeof(float));
    float *kb = (float *)malloc(n * kv_dim * sizeof(float));
    float *vb = (float *)malloc(n * kv_dim * sizeof(float));
    float *ab = (float *)malloc(n * Q * sizeof(float));
    float *tb = (float *)malloc(n * H * sizeof(float));
    float *gb = (float *)malloc(n * F * sizeof(float));
    float *ub = (float *)malloc(n * F * sizeof(float));
    float *wn = (float *)malloc(H * sizeof(float));
    if (!hid || !nrm || !qb || !kb || !vb || !ab || !tb || !gb || !ub || !wn) {
        rc = ORC_E_NOMEM;
        goto done;
    }
    for (size_t p = 0; p < n; p++) {
        size_t start = ((size_t)tokens[p] % vocab_rows) * H;
        if (start + H > m->embd.elems) {
            rc = ORC_E_SHAPE;
            goto done;
        }
        orc_dequantize_range(m->embd.type, m->embd.data, start, H, hid + p * H);
    }
    for (uint32_t l = 0; l < I->num_layers && rc == ORC_OK; l++) {
        orc_layer *L = &m->layers[l];
        for (size_t p = 0; p < n && rc == ORC_OK; p++)
            rc = wnorm(&L->attn_norm, H, hid + p * H, eps, nrm + p * H, wn);
        if (!rc) rc = bmatmul(m, &L->q, Q, H, nrm, H, n, qb, Q);
        if (!rc) rc = bmatmul(m, &L->k, kv_dim, H, nrm, H, n, kb, kv_dim);
        if (!rc) rc = bmatmul(m, &L->v, kv_dim, H, nrm, H, n, vb, kv_dim);
        if (rc) break;
        for (size_t p = 0; p < n; p++) {
            for (size_t h = 0; h + D <= Q; h += D) orc_rope_single(qb + p * Q + h, p, D, I->rope_freq_base);
            for (size_t h = 0; h + D <= kv_dim; h += D)
                orc_rope_single(kb + p * kv_dim + h, p, D, I->rope_freq_base);
            kv_add(m, L, kb + p * kv_dim, vb + p * kv_dim);
        }
        {
            int nw = m->threads < 1 ? 1 : (m->threads > 256 ? 256 : m->threads);
            pthread_t tid[256];
            attn_job jobs[256];
            for (int w = 0; w < nw; w++) {
                jobs[w] = (attn_job){m, L, qb, ab, 0, n, Q, (size_t)w, (size_t)nw};
                pthread_create(&tid[w], NULL, attn_worker, &jobs[w]);
            }
            for (int w = 0; w < nw; w++) {
                void *ret;
                pthread_join(tid[w], &ret);
                if (ret) rc = ORC_E_NOMEM;
            }
        }
        if (!rc) rc = bmatmul(m, &L->o, H, H, ab, Q, n, tb, H);
        if (rc) break;
        for (size_t i = 0; i < n * H; i++) hid[i] += tb[i];
        for (size_t p = 0; p < n && rc == ORC_OK; p++)
            rc = wnorm(&L->ffn_norm, H, hid + p * H, eps, nrm + p * H, wn);
        if (!rc) rc = bmatmul(m, &L->gate, F, H, nrm, H, n, gb, F);
        if (!rc) rc = bmatmul(m, &L->up, F, H, nrm, H, n, ub, F);
        if (rc) break;
        for (size_t i = 0; i < n * F; i++) gb[i] = (gb[i] / (1.0f + expf(-gb[i]))) * ub[i];
        rc = bmatmul(m, &L->down, H, F, gb, F, n, tb, H);
        if (rc) break;
        for (size_t i = 0; i < n * H; i++) hid[i] += tb[i];
    }
    if (rc == ORC_OK) {
        /* the last token's logits, as decode_with_cache returns them */
        memcpy(m->hidden, hid + (n - 1) * H, H * sizeof(float));
        if (m->out_norm.present && m->out_norm.elems >= H) {
            orc_dequantize_range(m->out_norm.type, m->out_norm.data, 0, H, m->norm_tmp);
        } else {
            for (size_t i = 0; i < H; i++) m->norm_tmp[i] = 1.0f;
        }
        orc_rms_norm(m->hidden, m->norm_tmp, H, eps, m->normed);
        if (m->out_head.present) {
            size_t rows = m->out_head.elems / H;
            rc = orc_qmatvec(m->out_head.type, m->out_head.data, rows, H, m->normed, logits, m->threads);
        } else {
            memcpy(logits, m->normed, H * sizeof(float));
        }
    }
done:
    free(hid);
    free(nrm);
    free(qb);
    free(kb);
    free(vb);
    free(ab);
    free(tb);
    free(gb);
    free(ub);
    free(wn);
    return rc;
}

/* ------------------------------------------------------------------------ */
/* Seeded synthetic GGUF writer (test infrastructure)                        */
/* ------------------------------------------------------------------------ */
/* Writes the same bytes as the shipped library's nexus_synth_model_write for
 * the same configuration (checked by tests/test_oracle_batched.py), so the
 * CPU-only legs (bench.py --impl reference) can produce their model file
 * without loading the CUDA library.  File conventions follow nexus-convert
 * (tools/nexus-convert/main.rs:190-383): blk.N.* tensor names sorted, [out,in]
 * shapes, llama.* metadata keys sorted, general.alignment 32.  Element i of a
 * tensor is a counter-based normal draw: pair p = i/2,
 * r = splitmix64(splitmix64(seed ^ fnv1a(name)) + p), u1 = ((r>>40)+1)/2^24,
 * u2 = (r & 0xffffff)/2^24, z = sqrt(-2 ln u1) * (cos|sin)(2 pi u2) for even|odd i. */
static uint64_t orc_splitmix64(uint64_t x) {
    x += 0x9e3779b97f4a7c15ull;
    x = (x ^ (x >> 30)) * 0xbf58476d1ce4e5b9ull;
    x = (x ^ (x >> 27)) * 0x94d049bb133111ebull;
    return x ^ (x >> 31);
}

static uint64_t orc_fnv1a(const char *s) {
    uint64_t h = 0xcbf29ce484222325ull;
    for (; *s; s++) {
        h ^= (unsigned char)*s;
        h *= 0x100000001b3ull;
    }
    return h;
}

static void orc_gen_normal(uint64_t seed, uint64_t stream, size_t start, size_t count, float stdv,
                           float *out) {
    uint64_t base = orc_splitmix64(seed ^ stream);
    for (size_t k = 0; k < count; k++) {
        size_t i = start + k;
        uint64_t r = orc_splitmix64(base + (uint64_t)(i / 2));
        float u1 = (float)((r >> 40) + 1) * (1.0f / 16777216.0f);
        float u2 = (float)(r & 0xffffffu) * (1.0f / 16777216.0f);
        float rad = sqrtf(-2.0f * logf(u1));
        float ang = 6.28318530717958647692f * u2;
        float z = (i & 1) ? rad * sinf(ang) : rad * cosf(ang);
        out[k] = stdv * z;
    }
}

typedef struct {
    char name[96];
    uint32_t n_dims;
    uint64_t shape[2];
    int type;
    int ones;
} syn_tensor;

static int syn_cmp(const void *a, const void *b) {
    return strcmp(((const syn_tensor *)a)->name, ((const syn_tensor *)b)->name);
}

typedef struct {
    uint8_t *p;
    size_t n, cap;
} syn_buf;

static void sb_put(syn_buf *b, const void *src, size_t n) {
    if (b->n + n > b->cap) {
        b->cap = (b->n + n) * 2 + 256;
        b->p = (uint8_t *)realloc(b->p, b->cap);
    }
    memcpy(b->p + b->n, src, n);
    b->n += n;
}
static void sb_u32(syn_buf *b, uint32_t v) { sb_put(b, &v, 4); }
static void sb_u64(syn_buf *b, uint64_t v) { sb_put(b, &v, 8); }
static void sb_str(syn_buf *b, const char *s) {
    sb_u64(b, strlen(s));
    sb_put(b, s, strlen(s));
}

typedef struct {
    const orc_synth_config *cfg;
    const syn_tensor *t;
    uint64_t stream;
    size_t n, drawn, be, bb;
    uint8_t *buf;
    int tid, nt;
} syn_job;

#define SYN_CH 65536
static void *syn_worker(void *arg) {
    syn_job *j = (syn_job *)arg;
    float *vals = (float *)malloc(SYN_CH * sizeof(float));
    if (!vals) return (void *)1;
    for (size_t c = (size_t)j->tid; c < j->drawn; c += (size_t)j->nt) {
        size_t s = c * SYN_CH, cnt = j->n - s < SYN_CH ? j->n - s : SYN_CH;
        if (j->t->ones) {
            for (size_t i = 0; i < cnt; i++) vals[i] = 1.0f;
        } else {
            orc_gen_normal(j->cfg->seed, j->stream, s, cnt, j->cfg->weight_std, vals);
        }
        orc_quantize(j->t->type, vals, cnt, j->buf + s / j->be * j->bb);
    }
    free(vals);
    return NULL;
}

int orc_synth_write(const char *path, const orc_synth_config *C) {
    const int fmts[4] = {C->attn_format, C->ffn_format, C->embd_format, C->norm_format};
    size_t be, bb;
    if (C->num_heads == 0 || C->hidden_size % C->num_heads) return ORC_E_INVALID;
    for (int i = 0; i < 4; i++)
        if (!block_geom(fmts[i], &be, &bb) || fmts[i] == ORC_BF16) return ORC_E_UNSUPPORTED;
    if (C->head_format >= 0 && (!block_geom(C->head_format, &be, &bb) || C->head_format == ORC_BF16))
        return ORC_E_UNSUPPORTED;
    uint64_t H = C->hidden_size, F = C->ff_dim, V = C->vocab_size;
    uint64_t D = H / C->num_heads, KV = (uint64_t)C->num_kv_heads * D;
    size_t nts = 3 + (size_t)C->num_layers * 9;
    syn_tensor *ts = (syn_tensor *)calloc(nts, sizeof(syn_tensor));
    if (!ts) return ORC_E_NOMEM;
    size_t k = 0;
#define SYN_ADD(nm, d0, d1, nd, ty, on)                                     \
    do {                                                                    \
        snprintf(ts[k].name, sizeof ts[k].name, "%s", nm);                  \
        ts[k].n_dims = nd;                                                  \
        ts[k].shape[0] = d0;                                                \
        ts[k].shape[1] = d1;                                                \
        ts[k].type = ty;                                                    \
        ts[k].ones = on;                                                    \
        k++;                                                                \
    } while (0)
    SYN_ADD("token_embd.weight", V, H, 2, C->embd_format, 0);
    SYN_ADD("output_norm.weight", H, 0, 1, C->norm_format, 1);
    if (C->head_format >= 0) SYN_ADD("output.weight", V, H, 2, C->head_format, 0);
    for (uint32_t l = 0; l < C->num_layers; l++) {
        char nm[96];
#define SYN_L(role, d0, d1, nd, ty, on)                        \
    snprintf(nm, sizeof nm, "blk.%u.%s.weight", l, role);     \
    SYN_ADD(nm, d0, d1, nd, ty, on)
        SYN_L("attn_norm", H, 0, 1, C->norm_format, 1);
        SYN_L("attn_q", H, H, 2, C->attn_format, 0);
        SYN_L("attn_k", KV, H, 2, C->attn_format, 0);
        SYN_L("attn_v", KV, H, 2, C->attn_format, 0);
        SYN_L("attn_output", H, H, 2, C->attn_format, 0);
        SYN_L("ffn_norm", H, 0, 1, C->norm_format, 1);
        SYN_L("ffn_gate", F, H, 2, C->ffn_format, 0);
        SYN_L("ffn_up", F, H, 2, C->ffn_format, 0);
        SYN_L("ffn_down", H, F, 2, C->ffn_format, 0);
#undef SYN_L
    }
#undef SYN_ADD
    nts = k;
    qsort(ts, nts, sizeof(syn_tensor), syn_cmp);

    const uint64_t ALIGN = 32;
    syn_buf hb = {0};
    sb_put(&hb, "GGUF", 4);
    sb_u32(&hb, 3);
    sb_u64(&hb, nts);
    sb_u64(&hb, 12);
    /* metadata in key order; value types: 4 = u32, 6 = f32, 8 = string */
    sb_str(&hb, "general.alignment"); sb_u32(&hb, 4); sb_u32(&hb, (uint32_t)ALIGN);
    sb_str(&hb, "general.architecture"); sb_u32(&hb, 8); sb_str(&hb, "llama");
    sb_str(&hb, "general.name"); sb_u32(&hb, 8); sb_str(&hb, "nexus-synthetic");
    sb_str(&hb, "llama.attention.head_count"); sb_u32(&hb, 4); sb_u32(&hb, C->num_heads);
    sb_str(&hb, "llama.attention.head_count_kv"); sb_u32(&hb, 4); sb_u32(&hb, C->num_kv_heads);
    {
        float eps = 1e-5f;
        uint32_t u;
        memcpy(&u, &eps, 4);
        sb_str(&hb, "llama.attention.layer_norm_rms_epsilon"); sb_u32(&hb, 6); sb_u32(&hb, u);
    }
    sb_str(&hb, "llama.block_count"); sb_u32(&hb, 4); sb_u32(&hb, C->num_layers);
    sb_str(&hb, "llama.context_length"); sb_u32(&hb, 4); sb_u32(&hb, C->context_length);
    sb_str(&hb, "llama.embedding_length"); sb_u32(&hb, 4); sb_u32(&hb, C->hidden_size);
    sb_str(&hb, "llama.feed_forward_length"); sb_u32(&hb, 4); sb_u32(&hb, C->ff_dim);
    {
        uint32_t u;
        memcpy(&u, &C->rope_theta, 4);
        sb_str(&hb, "llama.rope.freq_base"); sb_u32(&hb, 6); sb_u32(&hb, u);
    }
    sb_str(&hb, "llama.vocab_size"); sb_u32(&hb, 4); sb_u32(&hb, C->vocab_size);
    uint64_t off = 0;
    uint64_t *sizes = (uint64_t *)calloc(nts, sizeof(uint64_t));
    for (size_t i = 0; i < nts; i++) {
        sb_str(&hb, ts[i].name);
        sb_u32(&hb, ts[i].n_dims);
        for (uint32_t d = 0; d < ts[i].n_dims; d++) sb_u64(&hb, ts[i].shape[d]);
        sb_u32(&hb, (uint32_t)ts[i].type);
        sb_u64(&hb, off);
        uint64_t n = ts[i].shape[0] * (ts[i].n_dims > 1 ? ts[i].shape[1] : 1);
        sizes[i] = orc_type_size(ts[i].type, n);
        off += (sizes[i] + ALIGN - 1) / ALIGN * ALIGN;
    }
    while (hb.n % ALIGN) {
        uint8_t z = 0;
        sb_put(&hb, &z, 1);
    }
    int rc = ORC_OK;
    FILE *fp = fopen(path, "wb");
    if (!fp) rc = ORC_E_IO;
    if (!rc && fwrite(hb.p, 1, hb.n, fp) != hb.n) rc = ORC_E_IO;
    int threads = C->threads > 0 ? C->threads : (int)sysconf(_SC_NPROCESSORS_ONLN);
    if (threads < 1) threads = 1;
    if (threads > 256) threads = 256;
    for (size_t i = 0; !rc && i < nts; i++) {
        const syn_tensor *t = &ts[i];
        size_t n = (size_t)(t->shape[0] * (t->n_dims > 1 ? t->shape[1] : 1));
        size_t padded = (size_t)((sizes[i] + ALIGN - 1) / ALIGN * ALIGN);
        uint8_t *buf = (uint8_t *)calloc(padded ? padded : 1, 1);
        if (!buf) {
            rc = ORC_E_NOMEM;
            break;
        }
        block_geom(t->type, &be, &bb);
        size_t nchunks = (n + SYN_CH - 1) / SYN_CH;
        size_t drawn = C->repeat_chunks ? (nchunks < C->repeat_chunks ? nchunks : C->repeat_chunks) : nchunks;
        int nt = (size_t)threads < drawn ? threads : (int)drawn;
        if (nt < 1) nt = 1;
        pthread_t tid[256];
        syn_job jobs[256];
        for (int w = 0; w < nt; w++) {
            jobs[w] = (syn_job){C, t, orc_fnv1a(t->name), n, drawn, be, bb, buf, w, nt};
            pthread_create(&tid[w], NULL, syn_worker, &jobs[w]);
        }
        for (int w = 0; w < nt; w++) {
            void *ret;
            pthread_join(tid[w], &ret);
            if (ret) rc = ORC_E_NOMEM;
        }
        for (size_t c = drawn; c < nchunks; c++) {
            size_t s = c * SYN_CH, cnt = n - s < SYN_CH ? n - s : SYN_CH, src = (c % drawn) * SYN_CH;
            memcpy(buf + s / be * bb, buf + src / be * bb, cnt / be * bb);
        }
        if (!rc && fwrite(buf, 1, padded, fp) != padded) rc = ORC_E_IO;
        free(buf);
    }
    if (fp && fclose(fp) != 0) rc = ORC_E_IO;
    free(sizes);
    free(hb.p);
    free(ts);
    return rc;
}
