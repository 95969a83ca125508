/*
 * ah_oracle_avx512.c — the reference's AVX-512 CPU kernels restated as-is, with
 * the same intrinsic sequence, for TIMING ONLY (the CPU baseline that bench.py
 * reports beside the GPU figures and times in its reference arm).
 *
 * TEST INFRASTRUCTURE: only tests/ and bench.py's CPU legs may load this.
 *
 * These kernels do not compute the formats' defined semantics (the reference's
 * unpacklo/hi_epi8 interleave works within 128-bit lanes, so weights come out
 * lane-permuted; the f16 path reads 4 x i32 lanes from 8 packed u16).  They are
 * kept exactly so their cost is the reference's cost; parity is always checked
 * against the scalar restatement in ah_oracle.c.
 */
#include <immintrin.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define OR_API __attribute__((visibility("default")))

float or_f16_to_f32_scalar_asis(uint16_t h);
void or_gemv_4bit_worker_scalar(float* out, const float* scales, const uint8_t* packed, const float* x,
                                int64_t row_start, int64_t row_end, int64_t cols, int64_t group_size);

/* inference/math.rs:316-380 `gemv_4bit_parallel_worker_avx512` */
OR_API void or_avx_gemv_4bit_worker(float* out, const float* gscales, const uint8_t* gpacked, const float* x,
                                    int64_t row_start, int64_t row_end, int64_t cols) {
    int64_t n_gpr = cols / 32, chunks_128 = cols / 128;
    __m512 v_offset = _mm512_set1_ps(-8.0f);
    __m512i v_mask_low = _mm512_set1_epi8(0x0F);
    for (int64_t i = row_start; i < row_end; ++i) {
        const float* rs = gscales + i * n_gpr;
        int64_t row_off = (i * cols) / 2;
        __m512 acc = _mm512_setzero_ps();
        for (int64_t c = 0; c < chunks_128; ++c) {
            int64_t bo = row_off + c * 64, xo = c * 128, go = c * 4;
            __m512i raw = _mm512_loadu_si512((const void*)(gpacked + bo));
            __m512i be = _mm512_and_si512(raw, v_mask_low);
            __m512i bodd = _mm512_and_si512(_mm512_srli_epi16(raw, 4), v_mask_low);
            __m512i lin0 = _mm512_unpacklo_epi8(be, bodd);
            __m512i lin1 = _mm512_unpackhi_epi8(be, bodd);
#define AH_W(src, lane, s) _mm512_fmadd_ps(_mm512_add_ps(_mm512_cvtepi32_ps(_mm512_cvtepu8_epi32(lane)), v_offset), s, _mm512_setzero_ps())
            __m512 s0 = _mm512_set1_ps(rs[go]);
            acc = _mm512_fmadd_ps(AH_W(lin0, _mm512_castsi512_si128(lin0), s0), _mm512_loadu_ps(x + xo), acc);
            acc = _mm512_fmadd_ps(AH_W(lin0, _mm512_extracti32x4_epi32(lin0, 1), s0), _mm512_loadu_ps(x + xo + 16), acc);
            __m512 s1 = _mm512_set1_ps(rs[go + 1]);
            acc = _mm512_fmadd_ps(AH_W(lin0, _mm512_extracti32x4_epi32(lin0, 2), s1), _mm512_loadu_ps(x + xo + 32), acc);
            acc = _mm512_fmadd_ps(AH_W(lin0, _mm512_extracti32x4_epi32(lin0, 3), s1), _mm512_loadu_ps(x + xo + 48), acc);
            __m512 s2 = _mm512_set1_ps(rs[go + 2]);
            acc = _mm512_fmadd_ps(AH_W(lin1, _mm512_castsi512_si128(lin1), s2), _mm512_loadu_ps(x + xo + 64), acc);
            acc = _mm512_fmadd_ps(AH_W(lin1, _mm512_extracti32x4_epi32(lin1, 1), s2), _mm512_loadu_ps(x + xo + 80), acc);
            __m512 s3 = _mm512_set1_ps(rs[go + 3]);
            acc = _mm512_fmadd_ps(AH_W(lin1, _mm512_extracti32x4_epi32(lin1, 2), s3), _mm512_loadu_ps(x + xo + 96), acc);
            acc = _mm512_fmadd_ps(AH_W(lin1, _mm512_extracti32x4_epi32(lin1, 3), s3), _mm512_loadu_ps(x + xo + 112), acc);
#undef AH_W
        }
        out[i - row_start] = _mm512_reduce_add_ps(acc);
    }
}

typedef struct {
    float* out; const float* scales; const uint8_t* packed; const float* x;
    int64_t row_start, row_end, cols, gs;
} gemv_job;

/* inference/math.rs:297-314 `gemv_4bit_worker_dispatch` */
static void gemv_dispatch(gemv_job* j) {
    if (j->gs == 32 && j->cols % 128 == 0)
        or_avx_gemv_4bit_worker(j->out, j->scales, j->packed, j->x, j->row_start, j->row_end, j->cols);
    else
        or_gemv_4bit_worker_scalar(j->out, j->scales, j->packed, j->x, j->row_start, j->row_end, j->cols, j->gs);
}
static void* gemv_thread(void* p) { gemv_dispatch((gemv_job*)p); return NULL; }

/* inference/math.rs:255-295 `gemv_4bit_into`: serial at <= 1e6 elements,
 * otherwise min(available_parallelism, 32) scoped threads spawned per call over
 * contiguous row chunks (`nthreads` stands in for available_parallelism). */
OR_API void or_avx_gemv_4bit_into(float* out, const float* scales, const uint8_t* packed, const float* x,
                                  int64_t rows, int64_t cols, int64_t gs, int nthreads) {
    if (rows == 0 || cols == 0) { for (int64_t i = 0; i < rows; ++i) out[i] = 0.0f; return; }
    if (rows * cols <= 1000000) {
        gemv_job j = { out, scales, packed, x, 0, rows, cols, gs };
        gemv_dispatch(&j);
        return;
    }
    int nt = nthreads < 1 ? 1 : (nthreads > 32 ? 32 : nthreads);
    int64_t chunk = (rows + nt - 1) / nt;
    pthread_t th[32];
    gemv_job jobs[32];
    int started = 0;
    int64_t start = 0;
    for (int t = 0; t < nt; ++t) {
        int64_t end = (int64_t)(t + 1) * chunk < rows ? (int64_t)(t + 1) * chunk : rows;
        if (start >= end) continue;
        jobs[started] = (gemv_job){ out + start, scales, packed, x, start, end, cols, gs };
        pthread_create(&th[started], NULL, gemv_thread, &jobs[started]);
        started++;
        start = end;
    }
    for (int t = 0; t < started; ++t) pthread_join(th[t], NULL);
}

/* Batched form for the prefill-GEMM CPU baseline: the reference prefills token
 * by token (inference/mod.rs:550), i.e. one gemv_4bit_into per token row. */
OR_API void or_avx_gemm_rows(float* c, const float* scales, const uint8_t* packed, const float* a,
                             int64_t m, int64_t n, int64_t k, int nthreads) {
    for (int64_t i = 0; i < m; ++i) or_avx_gemv_4bit_into(c + i * n, scales, packed, a + i * k, n, k, 32, nthreads);
}

/* models/quantization.rs:456-530 `dequant_layer_avx512` (the n % 128 tail is
 * never written, as in the reference). */
OR_API void or_avx_dequant_layer(const float* scales, const uint8_t* packed, float* result, int64_t n) {
    int64_t chunks = n / 128;
    __m512 v_offset = _mm512_set1_ps(-8.0f);
    __m512i v_mask_low = _mm512_set1_epi8(0x0F);
    for (int64_t c = 0; c < chunks; ++c) {
        int64_t bo = c * 64, fo = c * 128, go = c * 4;
        __m512i raw = _mm512_loadu_si512((const void*)(packed + bo));
        __m512i be = _mm512_and_si512(raw, v_mask_low);
        __m512i bodd = _mm512_and_si512(_mm512_srli_epi16(raw, 4), v_mask_low);
        __m512i lin0 = _mm512_unpacklo_epi8(be, bodd);
        __m512i lin1 = _mm512_unpackhi_epi8(be, bodd);
#define AH_ST(off, lane, s) _mm512_storeu_ps(result + fo + (off), _mm512_fmadd_ps(_mm512_add_ps(_mm512_cvtepi32_ps(_mm512_cvtepu8_epi32(lane)), v_offset), s, _mm512_setzero_ps()))
        __m512 s0 = _mm512_set1_ps(scales[go]);
        AH_ST(0, _mm512_castsi512_si128(lin0), s0);
        AH_ST(16, _mm512_extracti32x4_epi32(lin0, 1), s0);
        __m512 s1 = _mm512_set1_ps(scales[go + 1]);
        AH_ST(32, _mm512_extracti32x4_epi32(lin0, 2), s1);
        AH_ST(48, _mm512_extracti32x4_epi32(lin0, 3), s1);
        __m512 s2 = _mm512_set1_ps(scales[go + 2]);
        AH_ST(64, _mm512_castsi512_si128(lin1), s2);
        AH_ST(80, _mm512_extracti32x4_epi32(lin1, 1), s2);
        __m512 s3 = _mm512_set1_ps(scales[go + 3]);
        AH_ST(96, _mm512_extracti32x4_epi32(lin1, 2), s3);
        AH_ST(112, _mm512_extracti32x4_epi32(lin1, 3), s3);
#undef AH_ST
    }
}

/* models/avx512_kernel.rs:161-177 `f16_128_to_f32` */
static inline __m128 f16_128_to_f32(__m128i v) {
    __m128i sign_part = _mm_slli_epi32(_mm_and_si128(v, _mm_set1_epi32(0x8000)), 16);
    __m128i exp_mant = _mm_slli_epi32(_mm_and_si128(v, _mm_set1_epi32(0x7FFF)), 13);
    __m128i combined = _mm_or_si128(sign_part, exp_mant);
    __m128i biased = _mm_add_epi32(combined, _mm_set1_epi32(112 << 23));
    return _mm_castsi128_ps(biased);
}

/* models/avx512_kernel.rs:137-155 `avx512_f16_to_f32`.  `src` must have 4 u16 of
 * readable slack past n (the reference reads them, :147). */
OR_API void or_avx_f16_to_f32(const uint16_t* src, float* out, int64_t n) {
    int64_t chunks = n / 8;
    for (int64_t c = 0; c < chunks; ++c) {
        int64_t o = c * 8;
        __m128i lo = _mm_loadu_si128((const __m128i*)(src + o));
        __m128i hi = _mm_loadu_si128((const __m128i*)(src + o + 4));
        _mm_storeu_ps(out + o, f16_128_to_f32(lo));
        _mm_storeu_ps(out + o + 4, f16_128_to_f32(hi));
    }
}

/* models/avx512_kernel.rs:212-232 `f16_bytes_to_f32`: stages the bytes into a
 * fresh u16 Vec (:218), converts with the AVX kernel, tail via the scalar
 * converter.  `out` has n_bytes/2 floats; returns the element count. */
OR_API int64_t or_avx_f16_bytes_to_f32(const uint8_t* src, int64_t n_bytes, float* out) {
    int64_t n = n_bytes / 2;
    if (n == 0) return 0;
    uint16_t* u16s = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)(n + 8));
    for (int64_t i = 0; i < n; ++i) u16s[i] = (uint16_t)(src[2 * i] | (src[2 * i + 1] << 8));
    memset(u16s + n, 0, 8 * sizeof(uint16_t));
    or_avx_f16_to_f32(u16s, out, n);
    for (int64_t i = n - n % 8; i < n; ++i) out[i] = or_f16_to_f32_scalar_asis(u16s[i]);
    free(u16s);
    return n;
}

/* models/avx512_kernel.rs:181-208 `avx512_bf16_to_f32` + :236-255 `bf16_bytes_to_f32`. */
OR_API int64_t or_avx_bf16_bytes_to_f32(const uint8_t* src, int64_t n_bytes, float* out) {
    int64_t n = n_bytes / 2;
    if (n == 0) return 0;
    uint16_t* u16s = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)(n + 8));
    for (int64_t i = 0; i < n; ++i) u16s[i] = (uint16_t)(src[2 * i] | (src[2 * i + 1] << 8));
    int64_t chunks = n / 8;
    for (int64_t c = 0; c < chunks; ++c) {
        int64_t o = c * 8;
        __m256i v = _mm256_loadu_si256((const __m256i*)(u16s + o));
        __m128i lo = _mm256_castsi256_si128(v);
        __m128i hi = _mm256_extracti128_si256(v, 1);
        _mm_storeu_ps(out + o, _mm_castsi128_ps(_mm_slli_epi32(lo, 16)));
        _mm_storeu_ps(out + o + 4, _mm_castsi128_ps(_mm_slli_epi32(hi, 16)));
    }
    for (int64_t i = n - n % 8; i < n; ++i) {
        uint32_t b = (uint32_t)u16s[i] << 16;
        memcpy(&out[i], &b, 4);
    }
    free(u16s);
    return n;
}
