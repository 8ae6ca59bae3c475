/*
 * ctarq_oracle.c -- CPU oracle for the C-TARQ linear path (TEST INFRASTRUCTURE).
 *
 * Restates saccade-core's CPU implementation (Rust) in C.  Parity status:
 * UNPINNED -- the reference cannot be built here and ships no golden vectors;
 * see ctarq_oracle.h.  Used only by tests/, __graft_entry__.smoke() and the
 * CPU-baseline leg of bench.py, never by the shipped library.
 *
 * Build with -ffp-contract=off and without -ffast-math: Rust never fuses a*b+c
 * into an FMA, and several steps below (dequantisation error, dW products,
 * bypass dot products) round the product before the add.
 */
#include "ctarq_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* ------------------------------------------------------------------ f16 */

uint16_t oracle_f32_to_f16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t exp = (x >> 23) & 0xFFu;
    uint32_t man = x & 0x7FFFFFu;
    if (exp == 0xFFu) {
        if (man == 0) return (uint16_t)(sign | 0x7C00u);
        return (uint16_t)(sign | 0x7E00u | (man >> 13));
    }
    int32_t e = (int32_t)exp - 127 + 15;
    if (e >= 0x1F) return (uint16_t)(sign | 0x7C00u);
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
    uint32_t rem = man & 0x1FFFu;
    uint32_t out = sign | ((uint32_t)e << 10) | hm;
    if (rem > 0x1000u || (rem == 0x1000u && (hm & 1u))) out++;
    return (uint16_t)out;
}

float oracle_f16_to_f32(uint16_t h) {
    uint32_t sign = ((uint32_t)h & 0x8000u) << 16;
    uint32_t exp = ((uint32_t)h >> 10) & 0x1Fu;
    uint32_t man = (uint32_t)h & 0x3FFu;
    uint32_t bits;
    if (exp == 0) {
        if (man == 0) {
            bits = sign;
        } else {
            float v = (float)man * 5.9604644775390625e-08f; /* man * 2^-24, exact */
            memcpy(&bits, &v, 4);
            bits |= sign;
        }
    } else if (exp == 0x1F) {
        bits = sign | 0x7F800000u | (man << 13);
    } else {
        bits = sign | ((exp - 15u + 127u) << 23) | (man << 13);
    }
    float out;
    memcpy(&out, &bits, 4);
    return out;
}

void oracle_f32_to_f16_array(const float* src, uint16_t* dst, int64_t n) {
    for (int64_t i = 0; i < n; i++) dst[i] = oracle_f32_to_f16(src[i]);
}

void oracle_bf16_to_f16_array(const uint16_t* src, uint16_t* dst, int64_t n) {
    for (int64_t i = 0; i < n; i++) {
        uint32_t bits = (uint32_t)src[i] << 16;
        float f;
        memcpy(&f, &bits, 4);
        dst[i] = oracle_f32_to_f16(f);
    }
}

/* Rust `f32 as i32`: truncation, saturating, NaN -> 0. */
static int32_t sat_i32(float f) {
    if (f != f) return 0;
    if (f >= 2147483648.0f) return INT32_MAX;
    if (f <= -2147483648.0f) return INT32_MIN;
    return (int32_t)f;
}

/* Rust `f32 as usize`: truncation, saturating at 0 and SIZE_MAX, NaN -> 0. */
static uint64_t sat_usize(float f) {
    if (f != f || f <= 0.0f) return 0;
    if (f >= 18446744073709551616.0f) return UINT64_MAX;
    return (uint64_t)f;
}

/* ------------------------------------------------------------------ heuristics.rs */

/* heuristics.rs:3-14: sequential f32 sums of x and x*x, then E[x^2] - mean^2. */
float oracle_variance_heuristic(const uint16_t* x_f16, int64_t k) {
    float hidden_dim = (float)k;
    float sum = 0.0f, sum_sq = 0.0f;
    for (int64_t i = 0; i < k; i++) {
        float v = oracle_f16_to_f32(x_f16[i]);
        sum += v;
        sum_sq += v * v;
    }
    float mean = sum / hidden_dim;
    return (sum_sq / hidden_dim) - (mean * mean);
}

/* ------------------------------------------------------------------ compress.rs */

static float row_scale(const float* row, int64_t k) {
    /* compress.rs:41-51 (and :149-154): strict '>' running max of |w|, scale = max/7 or 1. */
    float max_abs = 0.0f;
    for (int64_t c = 0; c < k; c++) {
        float a = fabsf(row[c]);
        if (a > max_abs) max_abs = a;
    }
    return max_abs > 0.0f ? max_abs / 7.0f : 1.0f;
}

static int cmp_f32(const void* a, const void* b) {
    float x = *(const float*)a, y = *(const float*)b;
    return (x > y) - (x < y);
}

/* compress.rs:137-176 */
float oracle_percentile_threshold(const float* w, int64_t n_rows, int64_t k, float target_fill_pct) {
    int64_t cap = n_rows * k;
    float* errs = (float*)malloc((size_t)(cap > 0 ? cap : 1) * sizeof(float));
    int64_t n = 0;
    for (int64_t r = 0; r < n_rows; r++) {
        const float* row = w + r * k;
        float scale = row_scale(row, k);
        for (int64_t c = 0; c < k; c++) {
            float val = row[c];
            /* (val / scale).round().max(-8.0).min(7.0) as i32 -- f32::max/min ignore NaN */
            float qf = roundf(val / scale);
            if (!(qf >= -8.0f)) qf = -8.0f;
            if (!(qf <= 7.0f)) qf = 7.0f;
            int32_t q = sat_i32(qf);
            float deq = (float)q * scale;
            float err = fabsf(val - deq);
            if (err > 1e-10f) errs[n++] = err;
        }
    }
    if (n == 0) {
        free(errs);
        return 0.001f;
    }
    qsort(errs, (size_t)n, sizeof(float), cmp_f32);
    float frac = 1.0f - target_fill_pct;
    float prod = frac * (float)n;
    uint64_t idx = sat_usize(prod);
    if (idx > (uint64_t)(n - 1)) idx = (uint64_t)(n - 1);
    float out = errs[idx];
    free(errs);
    return out;
}

/* compress.rs:6-129 */
int oracle_compress(const float* w, int64_t n_rows, int64_t k, float delta_threshold,
                    uint32_t* packed, uint16_t* scale_f16, uint32_t* row_ptrs,
                    uint32_t* col_indices, uint8_t* values, int64_t* nnz_out,
                    uint16_t* delta_scale_f16_out) {
    if (k % 8 != 0) return -1;
    int64_t kw = k / 8;
    float* err_m = (float*)calloc((size_t)(n_rows * k > 0 ? n_rows * k : 1), sizeof(float));
    float max_err = 0.0f;
    for (int64_t r = 0; r < n_rows; r++) {
        const float* row = w + r * k;
        float scale = row_scale(row, k);
        scale_f16[r] = oracle_f32_to_f16(scale);
        for (int64_t p = 0; p < kw; p++) {
            uint32_t word = 0;
            for (int idx = 0; idx < 8; idx++) {
                int64_t c = p * 8 + idx;
                float val = row[c];
                int32_t q = sat_i32(roundf(val / scale));
                if (q < -8) q = -8;
                if (q > 7) q = 7;
                word |= (uint32_t)(q + 8) << (idx * 4);
                float deq = (float)q * scale;
                float err = val - deq;
                if (fabsf(err) > delta_threshold) {
                    err_m[r * k + c] = err;
                    if (fabsf(err) > max_err) max_err = fabsf(err);
                }
            }
            packed[r * kw + p] = word;
        }
    }
    float ds = max_err > 0.0f ? max_err / 127.0f : 1.0f;
    uint32_t cur = 0;
    for (int64_t r = 0; r < n_rows; r++) {
        row_ptrs[r] = cur;
        for (int64_t c = 0; c < k; c++) {
            float e = err_m[r * k + c];
            if (e != 0.0f) {
                col_indices[cur] = (uint32_t)c;
                int32_t qe = sat_i32(roundf(e / ds));
                if (qe < -128) qe = -128;
                if (qe > 127) qe = 127;
                values[cur] = (uint8_t)(int8_t)qe;
                cur++;
            }
        }
    }
    row_ptrs[n_rows] = cur;
    *nnz_out = cur;
    *delta_scale_f16_out = oracle_f32_to_f16(ds);
    free(err_m);
    return 0;
}

/* ------------------------------------------------------------------ calibration.rs */

/* Stable merge sort on floats with partial_cmp-style comparison (NaN compares Equal). */
static void msort(float* a, float* tmp, int64_t n) {
    if (n < 2) return;
    int64_t h = n / 2;
    msort(a, tmp, h);
    msort(a + h, tmp, n - h);
    int64_t i = 0, j = h, o = 0;
    while (i < h && j < n) {
        /* take right only if right < left (keeps stability; NaN -> Equal -> take left) */
        if (a[j] < a[i]) tmp[o++] = a[j++];
        else tmp[o++] = a[i++];
    }
    while (i < h) tmp[o++] = a[i++];
    while (j < n) tmp[o++] = a[j++];
    memcpy(a, tmp, (size_t)n * sizeof(float));
}

/* calibration.rs:10-47 */
int oracle_calibrate(const float* acts, int64_t n, int64_t k, float pct_t4, float pct_t8,
                     float* t4_out, float* t8_out) {
    if (n <= 0) return -1;
    float* var = (float*)malloc((size_t)n * sizeof(float));
    float* tmp = (float*)malloc((size_t)n * sizeof(float));
    for (int64_t t = 0; t < n; t++) {
        float sum = 0.0f, sum_sq = 0.0f;
        for (int64_t i = 0; i < k; i++) {
            float v = acts[t * k + i];
            sum += v;
            sum_sq += v * v;
        }
        float mean = sum / (float)k;
        var[t] = (sum_sq / (float)k) - (mean * mean);
    }
    msort(var, tmp, n);
    uint64_t i4 = sat_usize(roundf((float)n * pct_t4));
    uint64_t i8 = sat_usize(roundf((float)n * pct_t8));
    if (i4 > (uint64_t)(n - 1)) i4 = (uint64_t)(n - 1);
    if (i8 > (uint64_t)(n - 1)) i8 = (uint64_t)(n - 1);
    *t4_out = var[i4];
    *t8_out = var[i8];
    free(var);
    free(tmp);
    return 0;
}

/* ------------------------------------------------------------------ config.rs */

/* config.rs:157-215 build_csc */
int oracle_build_csc(const uint32_t* row_ptrs, const uint32_t* col_indices, const uint8_t* values,
                     int64_t nnz, uint16_t delta_scale_f16, int64_t n_rows, int64_t k,
                     uint32_t* col_ptrs, uint32_t* csc_rows, float* csc_vals) {
    float scale = oracle_f16_to_f32(delta_scale_f16);
    memset(col_ptrs, 0, (size_t)(k + 1) * sizeof(uint32_t));
    for (int64_t i = 0; i < nnz; i++) {
        if ((int64_t)col_indices[i] >= k) return -1;
        col_ptrs[col_indices[i] + 1] += 1;
    }
    for (int64_t j = 1; j <= k; j++) col_ptrs[j] += col_ptrs[j - 1];
    uint32_t* wpos = (uint32_t*)malloc((size_t)(k > 0 ? k : 1) * sizeof(uint32_t));
    memcpy(wpos, col_ptrs, (size_t)k * sizeof(uint32_t));
    for (int64_t r = 0; r < n_rows; r++) {
        for (uint32_t idx = row_ptrs[r]; idx < row_ptrs[r + 1]; idx++) {
            uint32_t c = col_indices[idx];
            uint32_t pos = wpos[c];
            csc_rows[pos] = (uint32_t)r;
            csc_vals[pos] = (float)(int8_t)values[idx] * scale;
            wpos[c] += 1;
        }
    }
    free(wpos);
    return 0;
}

/* config.rs:112-142 */
void oracle_dequant_dense(const uint32_t* packed, const uint16_t* scale_f16, int64_t n_rows, int64_t k,
                          const uint32_t* col_ptrs, const uint32_t* csc_rows, const float* csc_vals,
                          float* w_out) {
    int64_t kw = k / 8;
    for (int64_t r = 0; r < n_rows; r++) {
        float scale = oracle_f16_to_f32(scale_f16[r]);
        for (int64_t p = 0; p < kw; p++) {
            uint32_t word = packed[r * kw + p];
            for (int idx = 0; idx < 8; idx++) {
                int32_t q = (int32_t)((word >> (idx * 4)) & 0xFu) - 8;
                w_out[r * k + p * 8 + idx] = (float)q * scale;
            }
        }
    }
    if (col_ptrs) {
        for (int64_t c = 0; c < k; c++)
            for (uint32_t idx = col_ptrs[c]; idx < col_ptrs[c + 1]; idx++)
                w_out[(int64_t)csc_rows[idx] * k + c] += csc_vals[idx];
    }
}

/* ------------------------------------------------------------------ op.rs */

/* op.rs:69-72 */
int oracle_route_bits(float score, float t4, float t8) {
    int q8 = (score >= t4) && (score < t8);
    int fp16 = score >= t8;
    return q8 | (fp16 << 1);
}

/* op.rs:10-185 cpu_fwd */
void oracle_forward(const uint32_t* packed, const uint16_t* scale_f16, int64_t n_rows, int64_t k,
                    const uint32_t* col_ptrs, const uint32_t* csc_rows, const float* csc_vals,
                    float t4, float t8, const uint16_t* x_f16, int64_t m,
                    uint16_t* y_f16, uint8_t* routed_out, float* acc_out, const uint8_t* force_route,
                    int bypass, const float* dense_w, int n_threads) {
#ifdef _OPENMP
    int nt = n_threads > 0 ? n_threads : omp_get_max_threads();
#else
    (void)n_threads;
#endif
    if (bypass) {
        /* op.rs:30-58: dense f32 (base + dW) dot products, one accumulator, parallel over tokens. */
#ifdef _OPENMP
#pragma omp parallel for num_threads(nt) schedule(static)
#endif
        for (int64_t t = 0; t < m; t++) {
            const uint16_t* xt = x_f16 + t * k;
            for (int64_t r = 0; r < n_rows; r++) {
                const float* wr = dense_w + r * k;
                float acc = 0.0f;
                for (int64_t c = 0; c < k; c++) acc += oracle_f16_to_f32(xt[c]) * wr[c];
                if (acc_out) acc_out[t * n_rows + r] = acc;
                y_f16[t * n_rows + r] = oracle_f32_to_f16(acc);
            }
            if (routed_out) routed_out[t] = 0;
        }
        return;
    }

    /* op.rs:64-73 router over all tokens */
    uint8_t* route = (uint8_t*)malloc((size_t)(m > 0 ? m : 1));
    for (int64_t t = 0; t < m; t++) {
        float score = oracle_variance_heuristic(x_f16 + t * k, k);
        route[t] = oracle_route_bits(score, t4, t8) != 0;
        if (force_route && force_route[t] <= 1) route[t] = force_route[t];
    }

    int64_t kw = k / 8;
    float* tok = (float*)malloc((size_t)(k > 0 ? k : 1) * sizeof(float));
    float* acc = (float*)malloc((size_t)(n_rows > 0 ? n_rows : 1) * sizeof(float));
    for (int64_t t = 0; t < m; t++) {
        for (int64_t i = 0; i < k; i++) tok[i] = oracle_f16_to_f32(x_f16[t * k + i]);

        /* Phase 1 (op.rs:112-150): four accumulators, row-parallel like rayon */
#ifdef _OPENMP
#pragma omp parallel for num_threads(nt) schedule(static)
#endif
        for (int64_t r = 0; r < n_rows; r++) {
            float a0 = 0.0f, a1 = 0.0f, a2 = 0.0f, a3 = 0.0f;
            const uint32_t* wr = packed + r * kw;
            for (int64_t p = 0; p < kw; p++) {
                uint32_t w = wr[p];
                const float* xb = tok + p * 8;
                float n0 = (float)(w & 0xFu) - 8.0f;
                float n1 = (float)((w >> 4) & 0xFu) - 8.0f;
                float n2 = (float)((w >> 8) & 0xFu) - 8.0f;
                float n3 = (float)((w >> 12) & 0xFu) - 8.0f;
                float n4 = (float)((w >> 16) & 0xFu) - 8.0f;
                float n5 = (float)((w >> 20) & 0xFu) - 8.0f;
                float n6 = (float)((w >> 24) & 0xFu) - 8.0f;
                float n7 = (float)(w >> 28) - 8.0f;
                a0 += xb[0] * n0;
                a1 += xb[1] * n1;
                a2 += xb[2] * n2;
                a3 += xb[3] * n3;
                a0 += xb[4] * n4;
                a1 += xb[5] * n5;
                a2 += xb[6] * n6;
                a3 += xb[7] * n7;
            }
            acc[r] = (a0 + a1 + a2 + a3) * oracle_f16_to_f32(scale_f16[r]);
        }

        /* Phase 2 (op.rs:152-170): sequential CSC correction for routed tokens */
        if (route[t] && col_ptrs) {
            for (int64_t c = 0; c < k; c++) {
                uint32_t s = col_ptrs[c], e = col_ptrs[c + 1];
                if (s == e) continue;
                float activation = tok[c];
                for (uint32_t idx = s; idx < e; idx++) acc[csc_rows[idx]] += activation * csc_vals[idx];
            }
        }

        /* Phase 3 (op.rs:172-178) */
        for (int64_t r = 0; r < n_rows; r++) {
            if (acc_out) acc_out[t * n_rows + r] = acc[r];
            y_f16[t * n_rows + r] = oracle_f32_to_f16(acc[r]);
        }
        if (routed_out) routed_out[t] = route[t];
    }
    free(tok);
    free(acc);
    free(route);
}
