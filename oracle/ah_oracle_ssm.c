/*
 * ah_oracle_ssm.c — CPU restatement of agent_harness's gated delta-net SSM
 * block (inference/ssm.rs:171-296), one token step.
 *
 * TEST INFRASTRUCTURE ONLY, like ah_oracle.c: loaded by tests/ as the checker,
 * never by the product.
 *
 * Follows the reference literally, with its helpers from inference/math.rs:
 * gemv_serial_into (:13-22, sequential f32 sum per row), rms_norm_into
 * (:53-63), l2_norm (:71-80), silu / sigmoid (:83-96), softplus (:98-104) and
 * conv1d_depthwise_into (:165-190).  Compiled with -ffp-contract=off.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define OR_API __attribute__((visibility("default")))

static void gemv_rows(float* out, const float* w, const float* x, int64_t rows, int64_t cols) {
    for (int64_t i = 0; i < rows; ++i) {
        float sum = 0.0f;
        for (int64_t j = 0; j < cols; ++j) sum += w[i * cols + j] * x[j];
        out[i] = sum;
    }
}

static float sigmoid_r(float x) {
    if (x >= 0.0f) return 1.0f / (1.0f + expf(-x));
    const float e = expf(x);
    return e / (1.0f + e);
}
static float silu_r(float x) { return x * sigmoid_r(x); }
static float softplus_r(float x) { return x > 20.0f ? x : logf(1.0f + expf(x)); }

static void l2_norm_r(float* x, int64_t n, float eps) {
    float norm = 0.0f;
    for (int64_t i = 0; i < n; ++i) norm += x[i] * x[i];
    const float s = sqrtf(norm);
    const float inv = 1.0f / (s > eps ? s : eps);  /* norm.sqrt().max(eps) */
    for (int64_t i = 0; i < n; ++i) x[i] *= inv;
}

/* SsmBlock::forward.  Weights row-major f32: wqkv [conv_dim][n_embd],
 * wqkv_gate [value_dim][n_embd], conv1d [conv_dim][d_conv], dt_bias, a,
 * alpha [dt_rank][n_embd], beta [dt_rank][n_embd], norm [head_v_dim],
 * out [n_embd][value_dim].  State: conv_state [(d_conv-1)][conv_dim],
 * ssm_state [dt_rank][head_v_dim][head_k_dim], updated in place.
 * Returns 0, or -1 when head_k_dim != head_v_dim (the reference asserts). */
OR_API int or_ssm_forward(int64_t n_embd, int64_t d_state, int64_t n_group, int64_t dt_rank, int64_t d_inner,
                          int64_t d_conv, float eps, const float* wqkv, const float* wqkv_gate, const float* conv1d,
                          const float* dt_bias, const float* a, const float* alpha, const float* beta_w,
                          const float* norm_w, const float* w_out, float* conv_state, float* ssm_state,
                          const float* input, float* out) {
    const int64_t hk = d_state, nk = n_group, key_dim = hk * nk;
    const int64_t hv = d_inner / dt_rank, nv = dt_rank, value_dim = hv * nv;
    const int64_t conv_dim = key_dim * 2 + value_dim;
    if (hk != hv) return -1;
    float* qkv = malloc(sizeof(float) * conv_dim);
    float* z = malloc(sizeof(float) * value_dim);
    float* braw = malloc(sizeof(float) * nv);
    float* beta = malloc(sizeof(float) * nv);
    float* araw = malloc(sizeof(float) * nv);
    float* gate = malloc(sizeof(float) * nv);
    float* craw = malloc(sizeof(float) * conv_dim);
    float* cout = malloc(sizeof(float) * conv_dim);
    float* q = malloc(sizeof(float) * key_dim);
    float* k = malloc(sizeof(float) * key_dim);
    float* qe = malloc(sizeof(float) * hk * nv);
    float* ke = malloc(sizeof(float) * hk * nv);
    float* o = malloc(sizeof(float) * value_dim);
    float* res = malloc(sizeof(float) * value_dim);
    float* hq = malloc(sizeof(float) * hv);
    float* hsk = malloc(sizeof(float) * hv);
    float* hd = malloc(sizeof(float) * hv);
    float* normed = malloc(sizeof(float) * hv);
    /* steps 1-3: projections, beta, alpha (ssm.rs:184-199) */
    gemv_rows(qkv, wqkv, input, conv_dim, n_embd);
    gemv_rows(z, wqkv_gate, input, value_dim, n_embd);
    gemv_rows(braw, beta_w, input, nv, n_embd);
    for (int64_t i = 0; i < nv; ++i) beta[i] = sigmoid_r(braw[i]);
    gemv_rows(araw, alpha, input, nv, n_embd);
    for (int64_t i = 0; i < nv; ++i) gate[i] = softplus_r(araw[i] + dt_bias[i]) * a[i];
    /* step 4: depthwise conv1d + state shift (math.rs:165-190), SiLU */
    for (int64_t c = 0; c < conv_dim; ++c) {
        float sum = 0.0f;
        for (int64_t kk = 0; kk < d_conv - 1; ++kk) sum += conv_state[kk * conv_dim + c] * conv1d[c * d_conv + kk];
        sum += qkv[c] * conv1d[c * d_conv + (d_conv - 1)];
        craw[c] = sum;
    }
    if (d_conv - 1 > 1) memmove(conv_state, conv_state + conv_dim, sizeof(float) * (size_t)((d_conv - 2) * conv_dim));
    if (d_conv - 1 > 0) memcpy(conv_state + (d_conv - 2) * conv_dim, qkv, sizeof(float) * (size_t)conv_dim);
    for (int64_t c = 0; c < conv_dim; ++c) cout[c] = silu_r(craw[c]);
    /* steps 5-7: split, L2 norm per k head, repeat to v heads */
    memcpy(q, cout, sizeof(float) * key_dim);
    memcpy(k, cout + key_dim, sizeof(float) * key_dim);
    const float* v = cout + 2 * key_dim;
    for (int64_t h = 0; h < nk; ++h) {
        l2_norm_r(q + h * hk, hk, eps);
        l2_norm_r(k + h * hk, hk, eps);
    }
    const int64_t rep = nv / nk;
    for (int64_t h = 0; h < nv; ++h) {
        const int64_t src = h / rep;
        memcpy(qe + h * hk, q + src * hk, sizeof(float) * hk);
        memcpy(ke + h * hk, k + src * hk, sizeof(float) * hk);
    }
    /* step 8: gated delta rule per v head (ssm.rs:242-284) */
    const float scale = 1.0f / sqrtf((float)hk);
    for (int64_t h = 0; h < nv; ++h) {
        const float* qh = qe + h * hk;
        const float* kh = ke + h * hk;
        const float* vh = v + h * hv;
        float* S = ssm_state + h * hv * hk;
        for (int64_t i = 0; i < hk; ++i) hq[i] = qh[i] * scale;
        const float decay = expf(gate[h]);
        for (int64_t i = 0; i < hv * hk; ++i) S[i] *= decay;
        gemv_rows(hsk, S, kh, hv, hk);
        for (int64_t i = 0; i < hv; ++i) hd[i] = (vh[i] - hsk[i]) * beta[h];
        for (int64_t i = 0; i < hv; ++i)
            for (int64_t j = 0; j < hk; ++j) S[i * hk + j] += hd[i] * kh[j];
        gemv_rows(o + h * hv, S, hq, hv, hk);
    }
    /* step 9: gated RMSNorm per v head (math.rs:53-63), times silu(z) */
    for (int64_t h = 0; h < nv; ++h) {
        const float* oh = o + h * hv;
        float ss = 0.0f;
        for (int64_t i = 0; i < hv; ++i) ss += oh[i] * oh[i];
        const float inv = 1.0f / sqrtf((ss / (float)hv) + eps);
        for (int64_t i = 0; i < hv; ++i) normed[i] = oh[i] * inv * norm_w[i];
        for (int64_t i = 0; i < hv; ++i) res[h * hv + i] = normed[i] * silu_r(z[h * hv + i]);
    }
    /* step 10: output projection */
    gemv_rows(out, w_out, res, n_embd, value_dim);
    free(qkv); free(z); free(braw); free(beta); free(araw); free(gate); free(craw); free(cout); free(q); free(k);
    free(qe); free(ke); free(o); free(res); free(hq); free(hsk); free(hd); free(normed);
    return 0;
}
