/*
 * ah_oracle.c — CPU restatement of agent_harness's quantized-weight hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity oracle: only tests/,
 * __graft_entry__.smoke() and bench.py's CPU-baseline leg may load it, and only
 * as the checker (or the timed CPU baseline), never as a product code path.
 *
 * It restates the *scalar* semantics of the reference (Rust) code, which are the
 * defined semantics of each format (the reference's AVX-512 twins diverge from
 * them; those are restated separately, as-is, in ah_oracle_avx512.c for timing).
 * Every function cites the reference file:line it follows.  The reference is
 * Rust; Rust never contracts a*b+c into an FMA, so this file must be compiled
 * with -ffp-contract=off (oracle/Makefile does).
 *
 * Pinned against: the reference's own known-answer tests
 * (formats/gguf.rs:681-721, models/quantization.rs:536-583), numpy's IEEE
 * float16 conversion over all 65536 half values, and an independent numpy
 * restatement of every formula (tests/test_oracle.py).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define OR_API __attribute__((visibility("default")))

static inline float bits_f32(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
static inline uint32_t f32_bits(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }

/* Rust `f32 as i32`: saturating, NaN -> 0. */
static inline int32_t rust_f32_as_i32(float v) {
    if (v != v) return 0;
    if (v >= 2147483647.0f) return INT32_MAX;
    if (v <= -2147483648.0f) return INT32_MIN;
    return (int32_t)v;
}

/* ------------------------------------------------------------------------- */
/* f16 / bf16                                                                 */
/* ------------------------------------------------------------------------- */

/* formats/gguf.rs:93-120 `f16_to_f32` — IEEE-correct, NaN canonicalised to
 * f32::NAN (0x7FC00000) with the sign applied afterwards (`-val`). */
OR_API float or_f16_to_f32(uint16_t bits) {
    uint32_t sign = (bits >> 15) & 1u;
    uint32_t exp = (bits >> 10) & 0x1Fu;
    uint32_t mant = bits & 0x3FFu;
    float val;
    if (exp == 0) {
        if (mant == 0) {
            val = 0.0f;
        } else {
            float m = (float)mant / 1024.0f;
            val = m * ldexpf(1.0f, -14);           /* 2f32.powi(-14): exact */
        }
    } else if (exp == 0x1F) {
        val = (mant == 0) ? bits_f32(0x7F800000u) : bits_f32(0x7FC00000u);
    } else {
        float m = 1.0f + (float)mant / 1024.0f;
        val = m * ldexpf(1.0f, (int)exp - 15);     /* exact power of two */
    }
    return sign ? -val : val;
}

/* formats/gguf.rs:124-126 `bf16_to_f32`. */
OR_API float or_bf16_to_f32(uint16_t bits) { return bits_f32((uint32_t)bits << 16); }

/* models/avx512_kernel.rs:258-281 `f16_to_f32_scalar`, restated as-is including
 * its defects (sign shifted by 24 instead of 16; subnormal exponent off by one;
 * u32 wrap-around in release builds).  Used only to document the divergence. */
OR_API float or_f16_to_f32_scalar_asis(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u);
    uint32_t exp = (uint32_t)((h >> 10) & 0x1Fu);
    uint32_t mant = (uint32_t)(h & 0x03FFu);
    if (exp == 0) {
        if (mant == 0) return bits_f32(sign << 24);
        uint32_t m = mant;
        int32_t e = 0;
        while ((m & 0x0400u) == 0) { m <<= 1; e -= 1; }
        m &= 0x03FFu;
        uint32_t biased = (uint32_t)(127u - 15u + (uint32_t)e);
        return bits_f32((sign << 24) | (biased << 23) | (m << 13));
    } else if (exp == 0x1F) {
        return bits_f32((sign << 24) | 0x7F800000u | (mant << 13));
    }
    uint32_t biased = exp - 15u + 127u;
    return bits_f32((sign << 24) | (biased << 23) | (mant << 13));
}

/* f32 -> f16, IEEE round-to-nearest-even.  The reference has no f32->f16
 * conversion (parity unpinned); this is the builder's definition, checked
 * against numpy astype(float16).  NaN -> sign | 0x7E00 | top payload bits. */
OR_API uint16_t or_f32_to_f16(float f) {
    uint32_t x = f32_bits(f);
    uint16_t sign = (uint16_t)((x >> 16) & 0x8000u);
    uint32_t absx = x & 0x7FFFFFFFu;
    if (absx > 0x7F800000u) {                       /* NaN */
        return (uint16_t)(sign | 0x7E00u | ((absx >> 13) & 0x3FFu));
    }
    if (absx >= 0x477FF000u) {                      /* rounds to >= 65520 -> inf */
        return (uint16_t)(sign | 0x7C00u);
    }
    int32_t e = (int32_t)(absx >> 23) - 127;
    uint32_t mant = absx & 0x7FFFFFu;
    if (e >= -14) {                                 /* normal half */
        uint32_t he = (uint32_t)(e + 15);
        uint32_t hm = mant >> 13;
        uint32_t rem = mant & 0x1FFFu;
        uint32_t h = (he << 10) | hm;
        if (rem > 0x1000u || (rem == 0x1000u && (hm & 1u))) h += 1;
        return (uint16_t)(sign | h);
    }
    if (e < -25) return sign;                       /* below half the smallest subnormal */
    /* subnormal half: value = full * 2^(e-23); in units of 2^-24 that is
     * full * 2^(e+1), i.e. full >> (-1-e) with the remainder rounded RNE. */
    uint32_t full = mant | 0x800000u;
    int shift = -1 - (int)e;                        /* 14 .. 24 */
    uint32_t hm = full >> shift;
    uint32_t rem = full & ((1u << shift) - 1u);
    uint32_t half = 1u << (shift - 1);
    if (rem > half || (rem == half && (hm & 1u))) hm += 1;
    return (uint16_t)(sign | hm);
}

OR_API void or_f16_array_to_f32(const uint16_t* src, float* dst, int64_t n) {
    for (int64_t i = 0; i < n; ++i) dst[i] = or_f16_to_f32(src[i]);
}
OR_API void or_bf16_array_to_f32(const uint16_t* src, float* dst, int64_t n) {
    for (int64_t i = 0; i < n; ++i) dst[i] = or_bf16_to_f32(src[i]);
}
OR_API void or_f32_array_to_f16(const float* src, uint16_t* dst, int64_t n) {
    for (int64_t i = 0; i < n; ++i) dst[i] = or_f32_to_f16(src[i]);
}

/* ------------------------------------------------------------------------- */
/* GGUF block dequantisation                                                  */
/* ------------------------------------------------------------------------- */

/* formats/gguf.rs:434-535 `GGUFFile::dequantize_to_f32`.  Returns the number of
 * f32 values the reference's Vec would hold, or -1 where the reference panics
 * (Q4_0 with a truncated block: it indexes raw[off+2+i] unchecked, :489). */
OR_API int64_t or_dequantize_to_f32(const uint8_t* raw, int64_t raw_len, uint32_t dtype,
                                    int64_t element_count, float* out) {
    int64_t k = 0;
    switch (dtype) {
    case 0: /* F32, :443-447 — chunks_exact, ignores element_count */
        for (int64_t i = 0; i + 4 <= raw_len; i += 4) { float f; memcpy(&f, raw + i, 4); out[k++] = f; }
        return k;
    case 1: /* F16, :449-453 */
        for (int64_t i = 0; i + 2 <= raw_len; i += 2)
            out[k++] = or_f16_to_f32((uint16_t)(raw[i] | (raw[i + 1] << 8)));
        return k;
    case 30: /* BF16, :455-459 */
        for (int64_t i = 0; i + 2 <= raw_len; i += 2)
            out[k++] = or_bf16_to_f32((uint16_t)(raw[i] | (raw[i + 1] << 8)));
        return k;
    case 8: { /* Q8_0, :460-479 */
        const int64_t be = 32, bs = 34;
        int64_t nb = (element_count + be - 1) / be;
        for (int64_t b = 0; b < nb; ++b) {
            int64_t off = b * bs;
            if (off + 2 > raw_len) break;
            float d = or_f16_to_f32((uint16_t)(raw[off] | (raw[off + 1] << 8)));
            for (int64_t i = 0; i < be; ++i) {
                int64_t idx = b * be + i;
                if (idx >= element_count) break;
                int64_t q_off = off + 2 + i;
                if (q_off >= raw_len) break;
                float q = (float)(int8_t)raw[q_off];
                out[k++] = d * q;
            }
        }
        return k;
    }
    case 2: { /* Q4_0, :480-502 — byte i: low nibble -> elem 2i, high -> 2i+1 */
        const int64_t be = 32, bs = 18;
        int64_t nb = (element_count + be - 1) / be;
        for (int64_t b = 0; b < nb; ++b) {
            int64_t off = b * bs;
            if (off + 2 > raw_len) break;
            if (off + 2 + 16 > raw_len) return -1;  /* reference panics (slice index) */
            float d = or_f16_to_f32((uint16_t)(raw[off] | (raw[off + 1] << 8)));
            for (int64_t i = 0; i < 16; ++i) {
                uint8_t byte = raw[off + 2 + i];
                float q0 = (float)(int8_t)(byte & 0x0F) - 8.0f;
                float q1 = (float)(int8_t)(byte >> 4) - 8.0f;
                int64_t idx0 = b * be + i * 2, idx1 = idx0 + 1;
                if (idx0 < element_count) out[k++] = d * q0;
                if (idx1 < element_count) out[k++] = d * q1;
            }
        }
        return k;
    }
    case 13: { /* Q6_K "approximate, for stats" branch, :503-529 */
        const int64_t be = 256, bs = 210;
        int64_t nb = (element_count + be - 1) / be;
        for (int64_t b = 0; b < nb; ++b) {
            int64_t off = b * bs;
            if (off + bs > raw_len) break;
            float d = or_f16_to_f32((uint16_t)(raw[off] | (raw[off + 1] << 8)));
            for (int64_t i = 0; i < be; ++i) {
                int64_t idx = b * be + i;
                if (idx >= element_count) break;
                int64_t q_off = off + 4 + 2 + (i % 128);
                if (q_off < raw_len) out[k++] = ((float)(int8_t)raw[q_off]) * d / 127.0f;
                else out[k++] = 0.0f;
            }
        }
        return k;
    }
    default: /* :530-533 unknown type: zeros */
        for (int64_t i = 0; i < element_count; ++i) out[i] = 0.0f;
        return element_count;
    }
}

/* ------------------------------------------------------------------------- */
/* Engine INT4 format (f32 scales SoA + linear nibbles)                       */
/* ------------------------------------------------------------------------- */

/* models/quantization.rs:423-435 */
OR_API int64_t or_packed_bytes(int64_t n) { return (n + 1) / 2; }
OR_API int64_t or_n_groups(int64_t n, int64_t gs) { return (n + gs - 1) / gs; }
OR_API int64_t or_quantized_bytes(int64_t n, int64_t gs) { return or_n_groups(n, gs) * 4 + or_packed_bytes(n); }

/* models/quantization.rs:369-404 `quantize` (duplicate at inference/math.rs:223-253).
 * `packed` has or_packed_bytes(n) bytes and is zeroed here (the reference
 * allocates it zeroed and ORs nibbles in). */
OR_API void or_quantize_q4(const float* w, int64_t n, int64_t group_size, float* scales, uint8_t* packed) {
    int64_t gs = group_size < 1 ? 1 : group_size;
    int64_t ng = (n + gs - 1) / gs;
    memset(packed, 0, (size_t)((n + 1) / 2));
    for (int64_t g = 0; g < ng; ++g) {
        int64_t start = g * gs, end = start + gs < n ? start + gs : n;
        float max_abs = 0.0f;
        for (int64_t i = start; i < end; ++i) max_abs = fmaxf(max_abs, fabsf(w[i]));
        float scale = max_abs > 0.0f ? max_abs / 7.0f : 0.0f;
        float inv_scale = scale > 0.0f ? 1.0f / scale : 0.0f;
        scales[g] = scale;
        for (int64_t idx = start; idx < end; ++idx) {
            int32_t q = scale > 0.0f ? rust_f32_as_i32(roundf(w[idx] * inv_scale)) : 0;
            int32_t clamped = (q < -8 ? -8 : (q > 7 ? 7 : q)) + 8;
            if (idx % 2 == 0) packed[idx / 2] |= (uint8_t)clamped;
            else packed[idx / 2] |= (uint8_t)(clamped << 4);
        }
    }
}

/* models/quantization.rs:407-420 `dequant_weight` */
OR_API float or_dequant_weight(const float* scales, const uint8_t* packed, int64_t index, int64_t group_size) {
    int64_t gs = group_size < 1 ? 1 : group_size;
    float scale = scales[index / gs];
    uint8_t nib = (index % 2 == 0) ? (packed[index / 2] & 0x0F) : ((packed[index / 2] >> 4) & 0x0F);
    return ((float)nib - 8.0f) * scale;
}

/* models/quantization.rs:439-454 `dequant_layer`, scalar branch :444-452 (the
 * defined semantics; the AVX-512 branch permutes lanes and skips the tail). */
OR_API void or_dequant_layer(const float* scales, const uint8_t* packed, float* result, int64_t n, int64_t group_size) {
    for (int64_t i = 0; i < n; ++i) {
        int64_t gi = i / group_size;
        uint8_t nib = (i % 2 == 0) ? (packed[i / 2] & 0x0F) : ((packed[i / 2] >> 4) & 0x0F);
        result[i] = ((float)nib - 8.0f) * scales[gi];
    }
}

/* ------------------------------------------------------------------------- */
/* Builder quantisers for the BASELINE block formats (no reference quantiser  */
/* exists; the dequant side is pinned by formats/gguf.rs:459-502).            */
/* ------------------------------------------------------------------------- */

/* Q8_0 {u16 d; i8 qs[32]} (types/dtype.rs:77-83): d = f16(absmax/127),
 * q = clamp(round(w * (1/d)), -127, 127); a partial last block is zero-padded. */
OR_API void or_quantize_q8_0(const float* w, int64_t n, uint8_t* blocks) {
    int64_t nb = (n + 31) / 32;
    for (int64_t b = 0; b < nb; ++b) {
        float amax = 0.0f;
        for (int64_t i = 0; i < 32; ++i) { int64_t j = b * 32 + i; if (j < n) amax = fmaxf(amax, fabsf(w[j])); }
        uint16_t d16 = or_f32_to_f16(amax / 127.0f);
        float d = or_f16_to_f32(d16);
        float id = d != 0.0f ? 1.0f / d : 0.0f;
        uint8_t* blk = blocks + b * 34;
        blk[0] = (uint8_t)(d16 & 0xFF); blk[1] = (uint8_t)(d16 >> 8);
        for (int64_t i = 0; i < 32; ++i) {
            int64_t j = b * 32 + i;
            int32_t q = 0;
            if (j < n) { q = rust_f32_as_i32(roundf(w[j] * id)); q = q < -127 ? -127 : (q > 127 ? 127 : q); }
            blk[2 + i] = (uint8_t)(int8_t)q;
        }
    }
}

/* Q4_0 {u16 d; u8 qs[16]} (types/dtype.rs:69-75) with the reference's nibble
 * order (formats/gguf.rs:488-497: low nibble = element 2i, high = 2i+1):
 * d = f16(absmax/8), q = clamp(round(w * (1/d)) + 8, 0, 15). */
OR_API void or_quantize_q4_0(const float* w, int64_t n, uint8_t* blocks) {
    int64_t nb = (n + 31) / 32;
    for (int64_t b = 0; b < nb; ++b) {
        float amax = 0.0f;
        for (int64_t i = 0; i < 32; ++i) { int64_t j = b * 32 + i; if (j < n) amax = fmaxf(amax, fabsf(w[j])); }
        uint16_t d16 = or_f32_to_f16(amax / 8.0f);
        float d = or_f16_to_f32(d16);
        float id = d != 0.0f ? 1.0f / d : 0.0f;
        uint8_t* blk = blocks + b * 18;
        blk[0] = (uint8_t)(d16 & 0xFF); blk[1] = (uint8_t)(d16 >> 8);
        for (int64_t i = 0; i < 16; ++i) {
            int32_t q[2];
            for (int t = 0; t < 2; ++t) {
                int64_t j = b * 32 + 2 * i + t;
                int32_t v = 8;
                if (j < n) { v = rust_f32_as_i32(roundf(w[j] * id)) + 8; v = v < 0 ? 0 : (v > 15 ? 15 : v); }
                q[t] = v;
            }
            blk[2 + i] = (uint8_t)(q[0] | (q[1] << 4));
        }
    }
}

/* ------------------------------------------------------------------------- */
/* GEMV                                                                       */
/* ------------------------------------------------------------------------- */

/* inference/math.rs:382-418 `gemv_4bit_parallel_worker_scalar`: per row a
 * sequential f32 sum in element order; w = (nib - 8) * scale, sum += w * x[j]. */
OR_API void or_gemv_4bit_worker_scalar(float* out, const float* scales, const uint8_t* packed, const float* x,
                                       int64_t row_start, int64_t row_end, int64_t cols, int64_t group_size) {
    int64_t gs = group_size < 1 ? 1 : group_size;
    int64_t n_gpr = (cols + gs - 1) / gs;
    #pragma omp parallel for schedule(static)
    for (int64_t i = row_start; i < row_end; ++i) {
        const float* rs = scales + i * n_gpr;
        int64_t row_offset = i * cols;
        float sum = 0.0f;
        for (int64_t g = 0; g < n_gpr; ++g) {
            float scale = rs[g];
            int64_t j0 = g * gs, j1 = j0 + gs < cols ? j0 + gs : cols;
            for (int64_t j = j0; j < j1; ++j) {
                int64_t lin = row_offset + j;
                uint8_t nib = (lin & 1) == 0 ? (packed[lin >> 1] & 0x0F) : ((packed[lin >> 1] >> 4) & 0x0F);
                float w = ((float)nib - 8.0f) * scale;
                sum += w * x[j];
            }
        }
        out[i - row_start] = sum;
    }
}

/* inference/math.rs:255-295 `gemv_4bit_into` (empty -> zeros, :264-267).  The
 * row split across threads does not change any row's result, so the scalar
 * worker over all rows is the parity oracle. */
OR_API void or_gemv_4bit_into(float* out, const float* scales, const uint8_t* packed, const float* x,
                              int64_t rows, int64_t cols, int64_t group_size) {
    if (rows == 0 || cols == 0 || x == NULL) { for (int64_t i = 0; i < rows; ++i) out[i] = 0.0f; return; }
    or_gemv_4bit_worker_scalar(out, scales, packed, x, 0, rows, cols, group_size);
}

/* Q4_0-block GEMV: the scalar worker's semantics (math.rs:405-414) with each
 * block's scale taken as gguf f16_to_f32(d) (formats/gguf.rs:486).  `out` rows,
 * `x` cols (cols % 32 == 0), weights row-major AoS blocks. */
OR_API void or_gemv_q4_0(float* out, const uint8_t* blocks, const float* x, int64_t rows, int64_t cols) {
    int64_t nb = cols / 32;
    #pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; ++r) {
        const uint8_t* rb = blocks + r * nb * 18;
        float sum = 0.0f;
        for (int64_t b = 0; b < nb; ++b) {
            const uint8_t* blk = rb + b * 18;
            float scale = or_f16_to_f32((uint16_t)(blk[0] | (blk[1] << 8)));
            for (int64_t j = 0; j < 32; ++j) {
                uint8_t byte = blk[2 + (j >> 1)];
                uint8_t nib = (j & 1) == 0 ? (byte & 0x0F) : (byte >> 4);
                float w = ((float)nib - 8.0f) * scale;
                sum += w * x[b * 32 + j];
            }
        }
        out[r] = sum;
    }
}

/* Batched Q4_0 GEMM oracle: C[m][n] = the scalar GEMV of row n of W against
 * A[m] (the reference prefills token by token with GEMV, inference/mod.rs:550).
 * A is f32 [M][K]; C is f32 [M][N]. */
OR_API void or_gemm_q4_0(float* c, const uint8_t* blocks, const float* a, int64_t m, int64_t n, int64_t k) {
    int64_t nb = k / 32;
    #pragma omp parallel for schedule(static) collapse(2)
    for (int64_t i = 0; i < m; ++i) {
        for (int64_t r = 0; r < n; ++r) {
            const uint8_t* rb = blocks + r * nb * 18;
            const float* x = a + i * k;
            float sum = 0.0f;
            for (int64_t b = 0; b < nb; ++b) {
                const uint8_t* blk = rb + b * 18;
                float scale = or_f16_to_f32((uint16_t)(blk[0] | (blk[1] << 8)));
                for (int64_t j = 0; j < 32; ++j) {
                    uint8_t byte = blk[2 + (j >> 1)];
                    uint8_t nib = (j & 1) == 0 ? (byte & 0x0F) : (byte >> 4);
                    float w = ((float)nib - 8.0f) * scale;
                    sum += w * x[b * 32 + j];
                }
            }
            c[i * n + r] = sum;
        }
    }
}

/* inference/math.rs:13-22 `gemv_serial_into` (f32 weights). */
OR_API void or_gemv_f32(float* out, const float* w, const float* x, int64_t rows, int64_t cols) {
    #pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < rows; ++i) {
        const float* row = w + i * cols;
        float sum = 0.0f;
        for (int64_t j = 0; j < cols; ++j) sum += row[j] * x[j];
        out[i] = sum;
    }
}

/* ------------------------------------------------------------------------- */
/* Element-wise math                                                          */
/* ------------------------------------------------------------------------- */

/* inference/math.rs:53-63 */
OR_API void or_rms_norm_into(float* out, const float* x, const float* weight, int64_t n, float eps) {
    float ss = 0.0f;
    for (int64_t i = 0; i < n; ++i) ss += x[i] * x[i];
    float inv = 1.0f / sqrtf((ss / (float)n) + eps);
    for (int64_t i = 0; i < n; ++i) out[i] = x[i] * inv * weight[i];
}

/* inference/math.rs:87-95 */
OR_API float or_sigmoid(float x) {
    if (x >= 0.0f) return 1.0f / (1.0f + expf(-x));
    float e = expf(x);
    return e / (1.0f + e);
}
/* inference/math.rs:82-85 */
OR_API float or_silu(float x) { return x * or_sigmoid(x); }

/* inference/math.rs:106-117 */
OR_API void or_softmax(float* x, int64_t n) {
    float mx = -INFINITY;
    for (int64_t i = 0; i < n; ++i) mx = fmaxf(mx, x[i]);
    float sum = 0.0f;
    for (int64_t i = 0; i < n; ++i) { x[i] = expf(x[i] - mx); sum += x[i]; }
    float inv = 1.0f / sum;
    for (int64_t i = 0; i < n; ++i) x[i] *= inv;
}

/* inference/math.rs:119-151 `rope_multi`, applied to one head's slice (the
 * per-head use of inference/attention.rs:126-139). */
OR_API void or_rope_multi(float* x, int64_t len, int64_t pos, const int32_t* sections, float freq_base) {
    int64_t total_d = 0;
    for (int s = 0; s < 4; ++s) if (sections[s] > 0) total_d += sections[s];
    if (total_d == 0) return;
    int64_t offset = 0, freq_idx = 0;
    for (int s = 0; s < 4; ++s) {
        int64_t d = sections[s] <= 0 ? 0 : sections[s];
        if (d == 0) continue;
        for (int64_t t = 0; t < d; ++t) {
            int64_t dim_idx = offset + 2 * (freq_idx - offset / 2);
            if (dim_idx + 1 >= len) break;
            float theta = (float)pos * powf(freq_base, -((float)freq_idx) / ((float)total_d));
            float sn = sinf(theta), cs = cosf(theta);
            float x0 = x[dim_idx], x1 = x[dim_idx + 1];
            x[dim_idx] = x0 * cs - x1 * sn;
            x[dim_idx + 1] = x0 * sn + x1 * cs;
            freq_idx += 1;
        }
        offset += 2 * d;
    }
}

/* inference/sampling.rs:4-14 — first strict maximum wins. */
OR_API uint32_t or_argmax(const float* logits, int64_t n) {
    uint32_t best = 0;
    float best_val = -INFINITY;
    for (int64_t i = 0; i < n; ++i) if (logits[i] > best_val) { best_val = logits[i]; best = (uint32_t)i; }
    return best;
}

/* inference/sampling.rs:17-64 `sample` with the uniform draw r given (the
 * reference draws it from a clock-seeded xorshift): p_i = exp((v_i - max) /
 * T) over every logit, the top_k indices by p (descending; equal p in index
 * order, which the reference's unstable selection leaves unspecified), the
 * sum over them in that order, then the CDF scan.  top_k >= 1. */
static const float* or_sample_p;
static int or_sample_cmp(const void* a, const void* b) {
    const int64_t ia = *(const int64_t*)a, ib = *(const int64_t*)b;
    const float pa = or_sample_p[ia], pb = or_sample_p[ib];
    if (pa > pb) return -1;
    if (pa < pb) return 1;
    return ia < ib ? -1 : (ia > ib ? 1 : 0);
}
OR_API uint32_t or_sample(const float* logits, int64_t n, float temperature, int64_t top_k, float r) {
    if (n == 0) return 0;
    float max_logit = -INFINITY;
    for (int64_t i = 0; i < n; ++i) max_logit = fmaxf(max_logit, logits[i]);
    const float inv_temp = 1.0f / temperature;
    float* probs = (float*)malloc(sizeof(float) * (size_t)n);
    int64_t* idx = (int64_t*)malloc(sizeof(int64_t) * (size_t)n);
    for (int64_t i = 0; i < n; ++i) {
        probs[i] = expf((logits[i] - max_logit) * inv_temp);
        idx[i] = i;
    }
    const int64_t k = top_k < n ? top_k : n;
    or_sample_p = probs;
    qsort(idx, (size_t)n, sizeof(int64_t), or_sample_cmp);
    float sum = 0.0f;
    for (int64_t j = 0; j < k; ++j) sum += probs[idx[j]];
    uint32_t pick = (uint32_t)idx[k - 1];
    if (sum == 0.0f) {
        pick = (uint32_t)idx[0];
    } else {
        const float inv = 1.0f / sum;
        float cdf = 0.0f;
        for (int64_t j = 0; j < k; ++j) {
            cdf += probs[idx[j]] * inv;
            if (r < cdf) { pick = (uint32_t)idx[j]; break; }
        }
    }
    free(probs);
    free(idx);
    return pick;
}

/* inference/ffn.rs:155-174 `swiglu_4bit_into` on the engine INT4 format. */
OR_API void or_swiglu_4bit_into(float* out, const float* input,
                                const float* gs_, const uint8_t* gp, const float* us, const uint8_t* up,
                                const float* ds, const uint8_t* dp, int64_t n_embd, int64_t n_ff, int64_t group_size,
                                float* sg, float* su, float* sa) {
    or_gemv_4bit_into(sg, gs_, gp, input, n_ff, n_embd, group_size);
    or_gemv_4bit_into(su, us, up, input, n_ff, n_embd, group_size);
    for (int64_t i = 0; i < n_ff; ++i) sa[i] = or_silu(sg[i]) * su[i];
    or_gemv_4bit_into(out, ds, dp, sa, n_embd, n_ff, group_size);
}

/* ------------------------------------------------------------------------- */
/* Llama-shaped decoder (inference/mod.rs:333-545 with per-head RoPE)          */
/* ------------------------------------------------------------------------- */

typedef struct {
    int64_t n_layer, n_embd, n_ff, n_head, n_head_kv, head_dim, vocab, max_seq;
    float rope_base, eps;
    const uint16_t* tok_embd;        /* [vocab][n_embd] f16 */
    const uint16_t* attn_norm;       /* [n_layer][n_embd] f16 */
    const uint16_t* ffn_norm;        /* [n_layer][n_embd] f16 */
    const uint16_t* out_norm;        /* [n_embd] f16 */
    const uint8_t* const* wq;        /* per layer, Q4_0 blocks, [n_embd][n_embd] */
    const uint8_t* const* wk;        /* [n_kv*hd][n_embd] */
    const uint8_t* const* wv;
    const uint8_t* const* wo;        /* [n_embd][n_head*hd] */
    const uint8_t* const* wg;        /* [n_ff][n_embd] */
    const uint8_t* const* wu;
    const uint8_t* const* wd;        /* [n_embd][n_ff] */
    const uint8_t* lm_head;          /* [vocab][n_embd] */
    uint16_t* k_cache;               /* [n_layer][n_kv][max_seq][hd] f16 */
    uint16_t* v_cache;
    float* k_cache_f32;              /* the same rows as f32 (or_f16_to_f32 of the stored bits), */
    float* v_cache_f32;              /* converted once at append instead of at every read */
    int64_t engine;                  /* 0: projections are Q4_0 blocks; 1: each points at quantize()'s
                                      * output, scales [rows*cols/32] f32 then packed [rows*cols/2] */
} or_model;

/* y = W x for one projection in the model's format: Q4_0 blocks, or the
 * engine format through the scalar gemv_4bit worker (inference/math.rs:382-418). */
static void model_mv(const or_model* m, float* out, const uint8_t* w, const float* x, int64_t rows, int64_t cols) {
    if (!m->engine) {
        or_gemv_q4_0(out, w, x, rows, cols);
        return;
    }
    const float* scales = (const float*)w;
    const uint8_t* packed = w + (size_t)rows * (cols / 32) * 4;
    or_gemv_4bit_worker_scalar(out, scales, packed, x, 0, rows, cols, 32);
}

static void f16_row(const uint16_t* src, float* dst, int64_t n) { for (int64_t i = 0; i < n; ++i) dst[i] = or_f16_to_f32(src[i]); }

/* One decoder step for `token` at position `pos`; logits -> `logits[vocab]`.
 * K/V are stored rounded to f16 (the f16 KV cache of the decode configs). */
OR_API int or_model_forward(const or_model* m, int32_t token, int64_t pos, float* logits) {
    int64_t d = m->n_embd, hd = m->head_dim, nkv = m->n_head_kv, nh = m->n_head, ff = m->n_ff;
    int64_t dkv = nkv * hd, dq = nh * hd;
    if (token < 0 || token >= m->vocab || pos < 0 || pos >= m->max_seq) return -1;
    float* hidden = malloc(sizeof(float) * d);
    float* normed = malloc(sizeof(float) * d);
    float* nw = malloc(sizeof(float) * (d > ff ? d : ff));
    float* q = malloc(sizeof(float) * dq);
    float* k = malloc(sizeof(float) * dkv);
    float* v = malloc(sizeof(float) * dkv);
    float* att = malloc(sizeof(float) * dq);
    float* tmp = malloc(sizeof(float) * d);
    float* g = malloc(sizeof(float) * ff);
    float* u = malloc(sizeof(float) * ff);
    float* scores = malloc(sizeof(float) * (pos + 1));
    int32_t sections[4] = { (int32_t)(hd / 2), 0, 0, 0 };   /* inference/config.rs:170-172 defaults */
    f16_row(m->tok_embd + (int64_t)token * d, hidden, d);
    for (int64_t il = 0; il < m->n_layer; ++il) {
        f16_row(m->attn_norm + il * d, nw, d);
        or_rms_norm_into(normed, hidden, nw, d, m->eps);
        model_mv(m, q, m->wq[il], normed, dq, d);
        model_mv(m, k, m->wk[il], normed, dkv, d);
        model_mv(m, v, m->wv[il], normed, dkv, d);
        for (int64_t h = 0; h < nh; ++h) or_rope_multi(q + h * hd, hd, pos, sections, m->rope_base);
        for (int64_t h = 0; h < nkv; ++h) or_rope_multi(k + h * hd, hd, pos, sections, m->rope_base);
        uint16_t* kc = m->k_cache + il * nkv * m->max_seq * hd;
        uint16_t* vc = m->v_cache + il * nkv * m->max_seq * hd;
        float* kf = m->k_cache_f32 + il * nkv * m->max_seq * hd;
        float* vf = m->v_cache_f32 + il * nkv * m->max_seq * hd;
        for (int64_t h = 0; h < nkv; ++h)
            for (int64_t e = 0; e < hd; ++e) {
                const int64_t at = (h * m->max_seq + pos) * hd + e;
                kc[at] = or_f32_to_f16(k[h * hd + e]);
                vc[at] = or_f32_to_f16(v[h * hd + e]);
                kf[at] = or_f16_to_f32(kc[at]);
                vf[at] = or_f16_to_f32(vc[at]);
            }
        float scale = 1.0f / sqrtf((float)hd);
        for (int64_t h = 0; h < nh; ++h) {
            int64_t kvh = nkv > 0 ? h * nkv / nh : 0;
            const float* qh = q + h * hd;
            float max_s = -INFINITY;
            for (int64_t p = 0; p <= pos; ++p) {
                const float* kr = kf + (kvh * m->max_seq + p) * hd;
                float dot = 0.0f;
                for (int64_t e = 0; e < hd; ++e) dot += qh[e] * kr[e];
                scores[p] = dot * scale;
                if (scores[p] > max_s) max_s = scores[p];
            }
            float sum_exp = 0.0f;
            for (int64_t p = 0; p <= pos; ++p) { scores[p] = expf(scores[p] - max_s); sum_exp += scores[p]; }
            float inv = 1.0f / sum_exp;
            /* acc[e] sums scores[p] * v[p][e] over p in ascending order, as a
             * loop over p per e would; positions outer keeps the reads row-wise */
            float* acc = att + h * hd;
            for (int64_t e = 0; e < hd; ++e) acc[e] = 0.0f;
            for (int64_t p = 0; p <= pos; ++p) {
                const float* vr = vf + (kvh * m->max_seq + p) * hd;
                const float sp = scores[p];
                for (int64_t e = 0; e < hd; ++e) acc[e] += sp * vr[e];
            }
            for (int64_t e = 0; e < hd; ++e) acc[e] *= inv;
        }
        model_mv(m, tmp, m->wo[il], att, d, dq);
        for (int64_t i = 0; i < d; ++i) hidden[i] += tmp[i];
        f16_row(m->ffn_norm + il * d, nw, d);
        or_rms_norm_into(normed, hidden, nw, d, m->eps);
        model_mv(m, g, m->wg[il], normed, ff, d);
        model_mv(m, u, m->wu[il], normed, ff, d);
        for (int64_t i = 0; i < ff; ++i) g[i] = or_silu(g[i]) * u[i];
        model_mv(m, tmp, m->wd[il], g, d, ff);
        for (int64_t i = 0; i < d; ++i) hidden[i] += tmp[i];
    }
    f16_row(m->out_norm, nw, d);
    or_rms_norm_into(normed, hidden, nw, d, m->eps);
    model_mv(m, logits, m->lm_head, normed, m->vocab, d);
    free(hidden); free(normed); free(nw); free(q); free(k); free(v); free(att); free(tmp); free(g); free(u); free(scores);
    return 0;
}
