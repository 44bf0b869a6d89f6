// quant_math.cuh -- block-format arithmetic shared by host and device code.
//
// These routines restate the reference's quantizers and dequantizers
// (src/quant/mod.rs:669-911,1117-1161 and src/gguf/mod.rs:962-1088,1547-1554)
// so that, with multiply-add contraction disabled (-fmad=false on the device
// translation unit that includes this header, -ffp-contract=off on the host),
// every value is bit-identical to the reference.  f16 conversion is IEEE
// binary16 with round-to-nearest-even, as the `half` crate (2.7.1) does.
#pragma once
#include <stdint.h>
#include <string.h>
#include <math.h>

#ifdef __CUDACC__
#define NX_HD __host__ __device__ __forceinline__
#else
#define NX_HD inline
#endif

namespace nx {

enum Format : int {
    F32 = 0, F16 = 1, Q4_0 = 2, Q8_0 = 8, Q2_K = 10, Q4_K = 12, BF16 = 28
};

NX_HD uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
NX_HD float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

// f32 -> f16 bits, IEEE round-to-nearest-even (half::f16::from_f32).
NX_HD uint16_t f32_to_f16(float f) {
    uint32_t x = f2u(f);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t exp = (x >> 23) & 0xffu;
    uint32_t man = x & 0x7fffffu;
    if (exp == 0xffu) {
        if (man == 0) return (uint16_t)(sign | 0x7c00u);
        return (uint16_t)(sign | 0x7e00u | (man >> 13));
    }
    int e = (int)exp - 112;
    if (e >= 31) return (uint16_t)(sign | 0x7c00u);
    if (e <= 0) {
        if (e < -10) return (uint16_t)sign;
        man |= 0x800000u;
        int shift = 14 - e;
        uint32_t hm = man >> shift;
        uint32_t rem = man & ((1u << shift) - 1u);
        uint32_t half = 1u << (shift - 1);
        if (rem > half || (rem == half && (hm & 1u))) hm++;
        return (uint16_t)(sign | hm);
    }
    uint32_t hm = man >> 13;
    uint32_t rem = man & 0x1fffu;
    uint32_t h = sign | ((uint32_t)e << 10) | hm;
    if (rem > 0x1000u || (rem == 0x1000u && (hm & 1u))) h++;
    return (uint16_t)h;
}

// f16 bits -> f32 (exact).
NX_HD float f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1fu;
    uint32_t man = h & 0x3ffu;
    uint32_t x;
    if (exp == 0) {
        if (man == 0) {
            x = sign;
        } else {
            uint32_t e = 113;
            while (!(man & 0x400u)) { man <<= 1; e--; }
            x = sign | (e << 23) | ((man & 0x3ffu) << 13);
        }
    } else if (exp == 0x1f) {
        x = sign | 0x7f800000u | (man << 13);
    } else {
        x = sign | ((exp + 112u) << 23) | (man << 13);
    }
    return u2f(x);
}

NX_HD float ld_f16(const uint8_t *p) { return f16_to_f32((uint16_t)(p[0] | (p[1] << 8))); }
NX_HD void st_f16(uint8_t *p, float v) {
    uint16_t h = f32_to_f16(v);
    p[0] = (uint8_t)(h & 0xff);
    p[1] = (uint8_t)(h >> 8);
}

// Rust float->int `as` casts saturate and map NaN to 0.
NX_HD uint8_t sat_u8(float v) {
    if (!(v == v) || v <= 0.0f) return 0;
    if (v >= 255.0f) return 255;
    return (uint8_t)v;
}
NX_HD int8_t sat_i8(float v) {
    if (!(v == v)) return 0;
    if (v <= -128.0f) return -128;
    if (v >= 127.0f) return 127;
    return (int8_t)v;
}
NX_HD int32_t sat_i32(float v) {
    if (!(v == v)) return 0;
    if (v <= -2147483648.0f) return INT32_MIN;
    if (v >= 2147483647.0f) return INT32_MAX;
    return (int32_t)v;
}
// Rust f32::clamp keeps NaN.
NX_HD float rclamp(float v, float lo, float hi) {
    if (v < lo) v = lo;
    if (v > hi) v = hi;
    return v;
}

// Block geometry: elements and bytes per block.
NX_HD int block_elems(int fmt) {
    return (fmt == Q4_K || fmt == Q2_K) ? 256 : (fmt == Q8_0 || fmt == Q4_0) ? 32 : 1;
}
NX_HD int block_bytes(int fmt) {
    switch (fmt) {
    case Q4_K: return 144;
    case Q2_K: return 84;
    case Q8_0: return 34;
    case Q4_0: return 18;
    case F32: return 4;
    case F16: case BF16: return 2;
    default: return 0;
    }
}
NX_HD bool format_supported(int fmt) { return block_bytes(fmt) != 0; }
NX_HD size_t format_bytes(int fmt, size_t n) {
    size_t be = (size_t)block_elems(fmt), bb = (size_t)block_bytes(fmt);
    return (n + be - 1) / be * bb;
}

// ---------------------------------------------------------------------------
// quantizers: one block from `len` valid values (rest zero / as the reference)
// ---------------------------------------------------------------------------

// quantize_q8_0, src/quant/mod.rs:669-687
NX_HD void quantize_block_q8_0(const float *v, int len, uint8_t *out) {
    float max_abs = 0.0f;
    for (int i = 0; i < len; i++) max_abs = fmaxf(max_abs, fabsf(v[i]));
    float scale = max_abs > 0.0f ? max_abs / 127.0f : 0.0f;
    st_f16(out, scale);
    for (int i = 0; i < 32; i++) {
        float value = i < len ? v[i] : 0.0f;
        int8_t q = 0;
        if (scale > 0.0f) q = sat_i8(rclamp(roundf(value / scale), -128.0f, 127.0f));
        out[2 + i] = (uint8_t)q;
    }
}

// quantize_symmetric_4bit / quantize_q4_0, src/quant/mod.rs:705-753
NX_HD uint8_t q4_0_sym(float value, float scale) {
    if (scale > 0.0f) {
        int32_t q = sat_i32(rclamp(roundf(value / scale), -8.0f, 7.0f));
        return (uint8_t)(q + 8);
    }
    return 8;
}
NX_HD void quantize_block_q4_0(const float *v, int len, uint8_t *out) {
    float max_abs = 0.0f;
    for (int i = 0; i < len; i++) max_abs = fmaxf(max_abs, fabsf(v[i]));
    float scale = max_abs > 0.0f ? max_abs / 7.0f : 0.0f;
    st_f16(out, scale);
    for (int i = 0; i < 16; i++) {
        uint8_t lo = q4_0_sym(i < len ? v[i] : 0.0f, scale);
        uint8_t hi = q4_0_sym(i + 16 < len ? v[i + 16] : 0.0f, scale);
        out[2 + i] = (uint8_t)((lo & 0x0f) | ((hi & 0x0f) << 4));
    }
}

// quantize_u6 / quantize_u4, src/quant/mod.rs:1117-1131
NX_HD uint8_t quantize_un(float value, float scale, float hi) {
    if (scale > 0.0f && value > 0.0f) return sat_u8(rclamp(roundf(value / scale), 1.0f, hi));
    return 0;
}
// quantize_q4_k_value / quantize_q2_k_value, src/quant/mod.rs:1133-1151
NX_HD uint8_t quantize_kq(float value, float d, float dmin, uint8_t sq, uint8_t mq, float hi) {
    float scale = d * (float)sq;
    float offset = dmin * (float)mq;
    if (scale > 0.0f) return sat_u8(rclamp(roundf((value + offset) / scale), 0.0f, hi));
    return 0;
}

// quantize_q4_k, src/quant/mod.rs:756-818 (v holds 256 values, zero padded)
NX_HD void quantize_block_q4_k(const float *block, uint8_t *out) {
    float sub_scales[8], sub_offsets[8];
    for (int sub = 0; sub < 8; sub++) {
        const float *v = block + sub * 32;
        float mn = INFINITY, mx = -INFINITY;
        for (int i = 0; i < 32; i++) mn = fminf(mn, v[i]);
        for (int i = 0; i < 32; i++) mx = fmaxf(mx, v[i]);
        float offset = mn < 0.0f ? -mn : 0.0f;
        sub_scales[sub] = fmaxf((mx + offset) / 15.0f, 0.0f);
        sub_offsets[sub] = offset;
    }
    float max_scale = 0.0f, max_offset = 0.0f;
    for (int s = 0; s < 8; s++) max_scale = fmaxf(max_scale, sub_scales[s]);
    for (int s = 0; s < 8; s++) max_offset = fmaxf(max_offset, sub_offsets[s]);
    float d = max_scale > 0.0f ? max_scale / 63.0f : 0.0f;
    float dmin = max_offset > 0.0f ? max_offset / 63.0f : 0.0f;
    uint8_t sc[8], mn[8];
    for (int s = 0; s < 8; s++) {
        sc[s] = quantize_un(sub_scales[s], d, 63.0f);
        mn[s] = quantize_un(sub_offsets[s], dmin, 63.0f);
    }
    st_f16(out, d);
    st_f16(out + 2, dmin);
    // pack_q4_k_scales, src/quant/mod.rs:1153-1161
    for (int i = 0; i < 4; i++) {
        out[4 + i] = (uint8_t)((sc[i] & 0x3f) | ((sc[i + 4] >> 4) << 6));
        out[8 + i] = (uint8_t)((mn[i] & 0x3f) | ((mn[i + 4] >> 4) << 6));
        out[12 + i] = (uint8_t)((sc[i + 4] & 0x0f) | ((mn[i + 4] & 0x0f) << 4));
    }
    for (int i = 0; i < 128; i++) {
        uint8_t lo = quantize_kq(block[i], d, dmin, sc[i / 32], mn[i / 32], 15.0f);
        uint8_t hi = quantize_kq(block[i + 128], d, dmin, sc[(i + 128) / 32], mn[(i + 128) / 32], 15.0f);
        out[16 + i] = (uint8_t)((lo & 0x0f) | ((hi & 0x0f) << 4));
    }
}

// quantize_q2_k, src/quant/mod.rs:851-911 (v holds 256 values, zero padded)
NX_HD void quantize_block_q2_k(const float *block, uint8_t *out) {
    float sub_scales[16], sub_offsets[16];
    for (int sub = 0; sub < 16; sub++) {
        const float *v = block + sub * 16;
        float mn = INFINITY, mx = -INFINITY;
        for (int i = 0; i < 16; i++) mn = fminf(mn, v[i]);
        for (int i = 0; i < 16; i++) mx = fmaxf(mx, v[i]);
        float offset = mn < 0.0f ? -mn : 0.0f;
        sub_scales[sub] = fmaxf((mx + offset) / 3.0f, 0.0f);
        sub_offsets[sub] = offset;
    }
    float max_scale = 0.0f, max_offset = 0.0f;
    for (int s = 0; s < 16; s++) max_scale = fmaxf(max_scale, sub_scales[s]);
    for (int s = 0; s < 16; s++) max_offset = fmaxf(max_offset, sub_offsets[s]);
    float d = max_scale > 0.0f ? max_scale / 15.0f : 0.0f;
    float dmin = max_offset > 0.0f ? max_offset / 15.0f : 0.0f;
    uint8_t *scales = out, *qs = out + 16;
    for (int i = 0; i < 64; i++) qs[i] = 0;
    for (int s = 0; s < 16; s++) {
        uint8_t sq = quantize_un(sub_scales[s], d, 15.0f);
        uint8_t mq = quantize_un(sub_offsets[s], dmin, 15.0f);
        scales[s] = (uint8_t)((sq & 0x0f) | ((mq & 0x0f) << 4));
    }
    for (int i = 0; i < 256; i++) {
        uint8_t p = scales[i / 16];
        uint8_t q = quantize_kq(block[i], d, dmin, p & 0x0f, p >> 4, 3.0f);
        qs[i / 4] |= (uint8_t)((q & 0x03) << ((i % 4) * 2));
    }
    st_f16(out + 80, d);
    st_f16(out + 82, dmin);
}

// ---------------------------------------------------------------------------
// dequantizers (src/gguf/mod.rs:962-1088): element j of one block
// ---------------------------------------------------------------------------
// unpack_q4_k_scales, src/gguf/mod.rs:1547-1554, for one sub-block
NX_HD void q4k_scale_min(const uint8_t *packed, int sub, uint8_t *sc, uint8_t *mn) {
    if (sub < 4) {
        *sc = packed[sub] & 0x3f;
        *mn = packed[sub + 4] & 0x3f;
    } else {
        int i = sub - 4;
        *sc = (uint8_t)((packed[i + 8] & 0x0f) | ((packed[i] >> 6) << 4));
        *mn = (uint8_t)((packed[i + 8] >> 4) | ((packed[i + 4] >> 6) << 4));
    }
}

NX_HD float dequant_elem(int fmt, const uint8_t *blk, int j) {
    switch (fmt) {
    case Q8_0: return (float)(int8_t)blk[2 + j] * ld_f16(blk);
    case Q4_0: {
        uint8_t p = blk[2 + (j & 15)];
        int q = j < 16 ? (p & 0x0f) : (p >> 4);
        return (float)(q - 8) * ld_f16(blk);
    }
    case Q4_K: {
        float d = ld_f16(blk), dmin = ld_f16(blk + 2);
        uint8_t sc, mn;
        q4k_scale_min(blk + 4, j / 32, &sc, &mn);
        uint8_t p = blk[16 + (j & 127)];
        uint8_t q = j < 128 ? (p & 0x0f) : (p >> 4);
        return d * (float)sc * (float)q - dmin * (float)mn;
    }
    case Q2_K: {
        uint8_t q = (blk[16 + j / 4] >> ((j % 4) * 2)) & 0x03;
        uint8_t p = blk[j / 16];
        float d = ld_f16(blk + 80), dmin = ld_f16(blk + 82);
        return d * (float)(p & 0x0f) * (float)q - dmin * (float)(p >> 4);
    }
    case F32: { float f; memcpy(&f, blk, 4); return f; }
    case F16: return ld_f16(blk);
    case BF16: return u2f((uint32_t)(blk[0] | (blk[1] << 8)) << 16);
    default: return 0.0f;
    }
}

}  // namespace nx
