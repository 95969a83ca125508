/*
 * ah_oracle_dedup.c — CPU restatement of agent_harness's DedupCount weight
 * codec (src/models/dedup/), the step before load-time quantisation.
 *
 * TEST INFRASTRUCTURE ONLY, like ah_oracle.c: loaded by tests/ and bench.py's
 * CPU-baseline leg as the checker or the timed CPU baseline, never by the
 * product.
 *
 * Restated, element by element, with the reference's fallbacks
 * (`.get(i).copied().unwrap_or(0)`) spelled out:
 *   compress              dedup/compressor.rs:8-160 (scalar tail path)
 *   decompress_all        dedup/decompressor.rs:7-27
 *   decompress_all_global dedup/decompressor.rs:29-85
 *   GlobalTable::new      dedup/global_lookup.rs:7-59
 *   build_chunk_remap     dedup/global_lookup.rs:62-86
 *   decompress_with_remap dedup/global_lookup.rs:89-118
 * The reference's hash maps become arrays and linear searches with the same
 * first-match / last-insert rules.  The reference has no tests of this codec:
 * parity is pinned by these restatements, by the compress -> decompress round
 * trip and by hand-computed cases (tests/test_dedup_cpu.py).
 *
 * Compiled with -ffp-contract=off (the Rust code never fuses a*b+c).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define OR_API __attribute__((visibility("default")))

/* 10f32.powi(n): square-and-multiply; every partial product is exact for
 * n <= 10 (5^10 < 2^24), so any multiplication order gives the same value. */
static float pow10f_i(int n) {
    float r = 1.0f;
    for (int i = 0; i < n; ++i) r *= 10.0f;
    return r;
}

static uint32_t pow10u(int n) {
    uint32_t r = 1;
    for (int i = 0; i < n; ++i) r *= 10u;
    return r;
}

/* Rust `f as u16` / `f as u32`: saturating, NaN -> 0. */
static uint16_t sat_u16(float f) {
    if (!(f > 0.0f)) return 0;
    if (f >= 65535.0f) return 65535;
    return (uint16_t)f;
}
static uint32_t sat_u32(float f) {
    if (!(f > 0.0f)) return 0;
    if (f >= 4294967295.0f) return 4294967295u;
    return (uint32_t)f;
}

static int cmp_u16(const void* a, const void* b) {
    const uint16_t x = *(const uint16_t*)a, y = *(const uint16_t*)b;
    return (x > y) - (x < y);
}

/* DedupCountTensor::compress (compressor.rs:8-160), the scalar tail path of
 * step 4 (:121-135).  Outputs: prefixes / prefix_counts (n_prefix entries, in
 * first-appearance order), unique tail values / counts (n_tail, ascending),
 * tail_digits, avg_precision_lost and the sandbag (prefix_idx, tail_idx,
 * sign_bits[(n+7)/8]).  Capacity 65536 prefixes and tails.  Returns 0, or -1
 * on allocation failure. */
OR_API int or_dedup_compress(const float* w, int64_t n, int prefix_digits, int truncate_rounds,
                             uint16_t* prefixes, uint32_t* prefix_counts, int64_t* n_prefix,
                             uint16_t* tail_values, uint32_t* tail_counts, int64_t* n_tail,
                             int64_t* tail_digits, float* avg_precision_lost,
                             uint16_t* prefix_idx, uint16_t* tail_idx, uint8_t* sign_bits) {
    const int initial_tail_digits = 7 - prefix_digits;             /* TOTAL_DIGITS = 7 (tensor.rs:16) */
    const float prefix_scale = pow10f_i(prefix_digits);
    const float tail_scale = pow10f_i(7);
    int32_t* pmap = malloc(sizeof(int32_t) * 65536);
    uint32_t* tails = malloc(sizeof(uint32_t) * (size_t)(n > 0 ? n : 1));
    int64_t* goff = malloc(sizeof(int64_t) * 65537);
    int64_t* gmem = malloc(sizeof(int64_t) * (size_t)(n > 0 ? n : 1));
    uint8_t* round_ups = calloc((size_t)65536 * (truncate_rounds > 0 ? truncate_rounds : 1), 1);
    uint32_t* tcount = calloc(65536, sizeof(uint32_t));
    if (!pmap || !tails || !goff || !gmem || !round_ups || !tcount) {
        free(pmap); free(tails); free(goff); free(gmem); free(round_ups); free(tcount);
        return -1;
    }
    for (int i = 0; i < 65536; ++i) pmap[i] = -1;
    memset(sign_bits, 0, (size_t)((n + 7) / 8));
    int64_t np = 0;
    /* step 1: group by prefix (:22-45) */
    for (int64_t i = 0; i < n; ++i) {
        const float aw = fabsf(w[i]);
        const uint16_t pi = sat_u16(floorf(aw * prefix_scale));
        const float pv = (float)pi / prefix_scale;
        const float tv = aw - pv;
        const uint32_t ti = sat_u32(roundf(tv * tail_scale));
        if (pmap[pi] < 0) {
            pmap[pi] = (int32_t)np;
            prefixes[np] = pi;
            prefix_counts[np] = 0;
            ++np;
        }
        const int32_t g = pmap[pi];
        prefix_idx[i] = (uint16_t)g;
        if (w[i] < 0.0f) sign_bits[i / 8] |= (uint8_t)(1u << (i % 8));
        prefix_counts[g] += 1;
        tails[i] = ti;
    }
    /* group membership in element order (group_tails) */
    goff[0] = 0;
    for (int64_t g = 0; g < np; ++g) goff[g + 1] = goff[g] + prefix_counts[g];
    {
        int64_t* fill = malloc(sizeof(int64_t) * (size_t)(np > 0 ? np : 1));
        if (!fill) { free(pmap); free(tails); free(goff); free(gmem); free(round_ups); free(tcount); return -1; }
        for (int64_t g = 0; g < np; ++g) fill[g] = goff[g];
        for (int64_t i = 0; i < n; ++i) gmem[fill[prefix_idx[i]]++] = i;
        free(fill);
    }
    /* step 2: truncation with averaging (:47-79) */
    float loss_sum = 0.0f;
    int64_t loss_count = 0;
    int cur = initial_tail_digits;
    for (int r = 0; r < truncate_rounds; ++r) {
        const float cur_div = pow10f_i(prefix_digits + cur);
        const float next_div = pow10f_i(prefix_digits + cur - 1);
        for (int64_t g = 0; g < np; ++g) {
            const int64_t len = goff[g + 1] - goff[g];
            uint64_t sum_last = 0;
            for (int64_t k = goff[g]; k < goff[g + 1]; ++k) sum_last += tails[gmem[k]] % 10u;
            const float avg = (float)sum_last / (float)len;
            const int ru = avg > 5.0f;
            round_ups[(size_t)g * truncate_rounds + r] = (uint8_t)ru;
            for (int64_t k = goff[g]; k < goff[g + 1]; ++k) {
                uint32_t* t = &tails[gmem[k]];
                const float old_val = (float)*t / cur_div;
                *t = ru ? *t / 10u + 1u : *t / 10u;
                const float new_val = (float)*t / next_div;
                loss_sum += fabsf(old_val - new_val);
                loss_count += 1;
            }
        }
        cur -= 1;
    }
    *avg_precision_lost = loss_sum / (float)(loss_count > 0 ? loss_count : 1);  /* count.max(1) */
    /* step 3: unique tails (as u16) with counts, ascending (:82-100) */
    for (int64_t g = 0; g < np; ++g)
        for (int64_t k = goff[g]; k < goff[g + 1]; ++k) tcount[(uint16_t)tails[gmem[k]]] += 1;
    int64_t nt = 0;
    for (int v = 0; v < 65536; ++v)
        if (tcount[v]) {
            tail_values[nt] = (uint16_t)v;
            tail_counts[nt] = tcount[v];
            ++nt;
        }
    /* step 4, scalar path (:121-135): recompute each element's truncated tail */
    for (int64_t i = 0; i < n; ++i) {
        const float aw = fabsf(w[i]);
        const uint16_t pi = sat_u16(floorf(aw * prefix_scale));
        const float pv = (float)pi / prefix_scale;
        uint32_t ti = sat_u32(roundf((aw - pv) * tail_scale));
        const int64_t g = prefix_idx[i];
        for (int r = 0; r < truncate_rounds; ++r)
            ti = round_ups[(size_t)g * truncate_rounds + r] ? ti / 10u + 1u : ti / 10u;
        const uint16_t tv = (uint16_t)ti;
        const uint16_t* hit = bsearch(&tv, tail_values, (size_t)nt, sizeof(uint16_t), cmp_u16);
        tail_idx[i] = hit ? (uint16_t)(hit - tail_values) : 0;
    }
    *n_prefix = np;
    *n_tail = nt;
    *tail_digits = cur;
    free(pmap); free(tails); free(goff); free(gmem); free(round_ups); free(tcount);
    return 0;
}

/* DedupCountTensor::decompress_all (decompressor.rs:7-27).  count is the
 * tensor's count; the sandbag arrays may be shorter (missing entries read 0). */
OR_API void or_dedup_decompress_all(const uint16_t* prefixes, int64_t n_prefix, const uint16_t* tail_values,
                                    int64_t n_tail, int64_t count, int prefix_digits, int tail_digits, float avg_pl,
                                    const uint16_t* prefix_idx, int64_t n_pidx, const uint16_t* tail_idx,
                                    int64_t n_tidx, const uint8_t* sign_bits, int64_t n_sign, float* out) {
    const float prefix_scale = pow10f_i(prefix_digits);
    const float divisor = pow10f_i(prefix_digits + tail_digits);
    for (int64_t i = 0; i < count; ++i) {
        const int64_t p = i < n_pidx ? prefix_idx[i] : 0;
        const int64_t t = i < n_tidx ? tail_idx[i] : 0;
        const uint16_t prefix_int = p < n_prefix ? prefixes[p] : 0;
        const float prefix = (float)prefix_int / prefix_scale;
        const uint16_t tail = t < n_tail ? tail_values[t] : 0;
        float value = prefix + (float)tail / divisor;
        value += avg_pl;
        const int sign = ((i / 8 < n_sign ? sign_bits[i / 8] : 0) >> (i % 8)) & 1;
        out[i] = sign ? -value : value;
    }
}

/* First global prefix index gi with (global_prefixes[gi] * gt_scale).round()
 * as u32 == norm, or -1 (`iter().position`). */
static int64_t find_global_prefix(const float* gprefixes, int64_t n_gp, float gt_scale, uint32_t norm) {
    for (int64_t gi = 0; gi < n_gp; ++gi)
        if (sat_u32(roundf(gprefixes[gi] * gt_scale)) == norm) return gi;
    return -1;
}

static uint32_t norm_prefix(uint16_t pv, int scale_diff) {
    return scale_diff > 0 ? (uint32_t)pv * pow10u(scale_diff) : (uint32_t)pv;
}

/* DedupCountTensor::decompress_all_global (decompressor.rs:29-85).  The global
 * table: g_prefixes[n_gp], and tails_for_prefix as CSR (g_tail_off[n_gp + 1],
 * g_tails).  Returns 0, or -1 where the reference would panic (an empty
 * global table, or an index past a tails_for_prefix row). */
OR_API int or_dedup_decompress_all_global(const uint16_t* prefixes, int64_t n_prefix, const uint16_t* tail_values,
                                          int64_t n_tail, int64_t count, int prefix_digits, int tail_digits,
                                          float avg_pl, const uint16_t* prefix_idx, int64_t n_pidx,
                                          const uint16_t* tail_idx, int64_t n_tidx, const uint8_t* sign_bits,
                                          int64_t n_sign, int g_prefix_digits, const float* g_prefixes, int64_t n_gp,
                                          const uint32_t* g_tail_off, const uint32_t* g_tails, float* out) {
    const float tail_divisor = pow10f_i(g_prefix_digits + tail_digits);
    const float gt_scale = pow10f_i(g_prefix_digits);
    const int scale_diff = g_prefix_digits - prefix_digits;
    /* prefix_lookup: pv -> gi, first insert wins (:37-48) */
    int32_t* plook = malloc(sizeof(int32_t) * 65536);
    int64_t* tlook = malloc(sizeof(int64_t) * (size_t)(n_prefix > 0 ? n_prefix : 1) * (size_t)(n_tail > 0 ? n_tail : 1));
    if (!plook || !tlook) { free(plook); free(tlook); return -1; }
    for (int i = 0; i < 65536; ++i) plook[i] = -1;
    for (int64_t k = 0; k < n_prefix; ++k) {
        const uint16_t pv = prefixes[k];
        if (plook[pv] < 0) {
            const int64_t gi = find_global_prefix(g_prefixes, n_gp, gt_scale, norm_prefix(pv, scale_diff));
            if (gi >= 0) plook[pv] = (int32_t)gi;
        }
    }
    /* tail_lookup: (cp_idx, ct_idx) -> gi over the value -> last index map (:50-61) */
    for (int64_t cp = 0; cp < n_prefix; ++cp) {
        const int64_t gp = plook[prefixes[cp]] >= 0 ? plook[prefixes[cp]] : 0;
        if (gp >= n_gp) { free(plook); free(tlook); return -1; }
        for (int64_t ct = 0; ct < n_tail; ++ct) {
            int64_t hit = -1;
            for (uint32_t gi = g_tail_off[gp]; gi < g_tail_off[gp + 1]; ++gi)
                if (g_tails[gi] == (uint32_t)tail_values[ct]) hit = gi - g_tail_off[gp];  /* last insert wins */
            tlook[cp * n_tail + ct] = hit;
        }
    }
    const float* gp_f = g_prefixes;
    for (int64_t i = 0; i < count; ++i) {
        const int64_t p = i < n_pidx ? prefix_idx[i] : 0;
        const int64_t t = i < n_tidx ? tail_idx[i] : 0;
        const uint16_t pv = p < n_prefix ? prefixes[p] : 0;
        const int64_t gp = plook[pv] >= 0 ? plook[pv] : 0;
        const int64_t gt = (p < n_prefix && t < n_tail && tlook[p * n_tail + t] >= 0) ? tlook[p * n_tail + t] : 0;
        if (gp >= n_gp || g_tail_off[gp] + (uint64_t)gt >= g_tail_off[gp + 1]) { free(plook); free(tlook); return -1; }
        const float prefix = gp_f[gp];
        const uint32_t tail = g_tails[g_tail_off[gp] + gt];
        float value = prefix + (float)tail / tail_divisor;
        value += avg_pl;
        const int sign = ((i / 8 < n_sign ? sign_bits[i / 8] : 0) >> (i % 8)) & 1;
        out[i] = sign ? -value : value;
    }
    free(plook);
    free(tlook);
    return 0;
}

/* GlobalTable::new (global_lookup.rs:7-59) over `n_chunks` tensors given as
 * concatenated prefix / tail lists with per-chunk counts.  Outputs: the
 * prefix_digits of chunk 0, g_prefixes (ascending integer prefixes / scale),
 * and tails_for_prefix as CSR in first-appearance order.  Capacities:
 * g_prefixes 65536, g_tails `tails_cap`.  Returns n_gp, or -1 when tails_cap
 * is too small. */
OR_API int64_t or_dedup_global_table_new(int n_chunks, const int* prefix_digits, const uint16_t* prefixes,
                                         const int64_t* n_prefix, const uint16_t* tail_values, const int64_t* n_tail,
                                         float* g_prefixes, uint32_t* g_tail_off, uint32_t* g_tails,
                                         int64_t tails_cap) {
    if (n_chunks <= 0) { g_tail_off[0] = 0; return 0; }
    const float prefix_scale = pow10f_i(prefix_digits[0]);
    uint8_t* seen = calloc(65536, 1);
    uint16_t* uniq = malloc(sizeof(uint16_t) * 65536);
    if (!seen || !uniq) { free(seen); free(uniq); return -1; }
    int64_t nu = 0;
    int64_t po = 0;
    for (int c = 0; c < n_chunks; ++c) {
        for (int64_t k = 0; k < n_prefix[c]; ++k)
            if (!seen[prefixes[po + k]]) { seen[prefixes[po + k]] = 1; uniq[nu++] = prefixes[po + k]; }
        po += n_prefix[c];
    }
    qsort(uniq, (size_t)nu, sizeof(uint16_t), cmp_u16);
    for (int64_t k = 0; k < nu; ++k) g_prefixes[k] = (float)uniq[k] / prefix_scale;
    /* rows are built in global-prefix order by scanning the chunks once per row;
     * within a row the order is that of the reference's appends (:40-52) */
    int64_t nt = 0;
    g_tail_off[0] = 0;
    for (int64_t gi = 0; gi < nu; ++gi) {
        const int64_t row0 = nt;
        int64_t pofs = 0, tofs = 0;
        for (int c = 0; c < n_chunks; ++c) {
            for (int64_t k = 0; k < n_prefix[c]; ++k) {
                if (prefixes[pofs + k] != uniq[gi]) continue;
                for (int64_t u = 0; u < n_tail[c]; ++u) {
                    const uint32_t tv = tail_values[tofs + u];
                    int found = 0;
                    for (int64_t q = row0; q < nt; ++q)
                        if (g_tails[q] == tv) { found = 1; break; }
                    if (!found) {
                        if (nt >= tails_cap) { free(seen); free(uniq); return -1; }
                        g_tails[nt++] = tv;
                    }
                }
            }
            pofs += n_prefix[c];
            tofs += n_tail[c];
        }
        g_tail_off[gi + 1] = (uint32_t)nt;
    }
    free(seen);
    free(uniq);
    return nu;
}

/* GlobalTable::build_chunk_remap (global_lookup.rs:62-86): for every unique
 * tail of the chunk, its position in the first matching global row. */
OR_API void or_dedup_build_chunk_remap(const uint16_t* prefixes, int64_t n_prefix, const uint16_t* tail_values,
                                       int64_t n_tail, int prefix_digits, int g_prefix_digits,
                                       const float* g_prefixes, int64_t n_gp, const uint32_t* g_tail_off,
                                       const uint32_t* g_tails, uint16_t* remap) {
    const float gt_scale = pow10f_i(g_prefix_digits);
    const int scale_diff = g_prefix_digits - prefix_digits;
    for (int64_t u = 0; u < n_tail; ++u) {
        uint16_t matched = 0;
        for (int64_t k = 0; k < n_prefix; ++k) {
            const int64_t gp = find_global_prefix(g_prefixes, n_gp, gt_scale, norm_prefix(prefixes[k], scale_diff));
            if (gp < 0) continue;
            int64_t pos = -1;
            for (uint32_t q = g_tail_off[gp]; q < g_tail_off[gp + 1]; ++q)
                if (g_tails[q] == (uint32_t)tail_values[u]) { pos = q - g_tail_off[gp]; break; }
            if (pos >= 0) { matched = (uint16_t)pos; break; }
        }
        remap[u] = matched;
    }
}

/* GlobalTable::decompress_with_remap, remap given (global_lookup.rs:89-113).
 * Loops over the sandbag's count.  Returns 0, or -1 where the reference would
 * panic (sandbag arrays shorter than count, a prefix index past the tensor's
 * prefixes, an empty global table). */
OR_API int or_dedup_decompress_with_remap(const uint16_t* prefixes, int64_t n_prefix, int prefix_digits,
                                          int tail_digits, float avg_pl, const uint16_t* prefix_idx, int64_t n_pidx,
                                          const uint16_t* tail_idx, int64_t n_tidx, const uint8_t* sign_bits,
                                          int64_t n_sign, int64_t sandbag_count, int g_prefix_digits,
                                          const float* g_prefixes, int64_t n_gp, const uint32_t* g_tail_off,
                                          const uint32_t* g_tails, const uint16_t* remap, int64_t n_remap,
                                          float* out) {
    const float divisor = pow10f_i(g_prefix_digits + tail_digits);
    const float gt_scale = pow10f_i(g_prefix_digits);
    const int scale_diff = g_prefix_digits - prefix_digits;
    if (sandbag_count > n_pidx || sandbag_count > n_tidx || (sandbag_count + 7) / 8 > n_sign) return -1;
    for (int64_t i = 0; i < sandbag_count; ++i) {
        const int64_t p = prefix_idx[i];
        const int64_t t = tail_idx[i];
        if (p >= n_prefix || n_gp <= 0) return -1;
        const int64_t gi = find_global_prefix(g_prefixes, n_gp, gt_scale, norm_prefix(prefixes[p], scale_diff));
        const int64_t gp = gi >= 0 ? gi : 0;
        const int64_t mapped = t < n_remap ? remap[t] : 0;
        const uint32_t row = g_tail_off[gp + 1] - g_tail_off[gp];
        const uint32_t tail = mapped < row ? g_tails[g_tail_off[gp] + mapped] : 0;
        float value = g_prefixes[gp] + (float)tail / divisor;
        value += avg_pl;
        const int sign = (sign_bits[i / 8] >> (i % 8)) & 1;
        out[i] = sign ? -value : value;
    }
    return 0;
}
