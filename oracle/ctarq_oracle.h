/*
 * ctarq_oracle.h -- CPU oracle for the C-TARQ linear path (TEST INFRASTRUCTURE).
 *
 * This is a plain-C restatement of saccade-core's CPU implementation of the
 * C-TARQ linear operator.  Tests compare the CUDA library against it; it is never
 * the thing that ships: only tests/, __graft_entry__.smoke() and the CPU-baseline
 * leg of bench.py may load it.
 *
 * Parity status: UNPINNED.  The reference is Rust-only, its Candle substrate
 * is an empty submodule, and no Rust toolchain exists on this machine, so the
 * reference cannot be built or run; it also ships no tests, golden vectors or
 * fixtures for this path.  The restatement is instead cross-checked against an
 * independent numpy restatement (tests/test_oracle.py) and hand-worked
 * known-answer cases derived from the Rust source.
 *
 * Every function names the reference file:line it restates.  Floating-point
 * semantics follow Rust: no FMA contraction (build with -ffp-contract=off),
 * no fast-math, f32::round = half away from zero (roundf), `as i32` saturates
 * with NaN -> 0, f16 conversion is IEEE round-to-nearest-even (half 2.7.1).
 */
#ifndef CTARQ_ORACLE_H
#define CTARQ_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* IEEE binary16 <-> binary32, round-to-nearest-even (half 2.7.1 from_f32/to_f32). */
uint16_t oracle_f32_to_f16(float f);
float oracle_f16_to_f32(uint16_t h);
void oracle_f32_to_f16_array(const float* src, uint16_t* dst, int64_t n);
void oracle_bf16_to_f16_array(const uint16_t* src, uint16_t* dst, int64_t n);

/* heuristics.rs:3-14 variance_heuristic over one f16 token of length k. */
float oracle_variance_heuristic(const uint16_t* x_f16, int64_t k);

/* compress.rs:137-176 compute_percentile_threshold.  w is f32 [n_rows, k]. */
float oracle_percentile_threshold(const float* w, int64_t n_rows, int64_t k, float target_fill_pct);

/* compress.rs:6-129 compress_tensor_to_saccade.
 * Outputs: packed [n_rows, k/8] u32, scale_f16 [n_rows], row_ptrs [n_rows+1],
 * col_indices/values sized by the caller to at least n_rows*k (upper bound),
 * *nnz_out, *delta_scale_f16_out.  Returns 0 on success, -1 if k % 8 != 0. */
int oracle_compress(const float* w, int64_t n_rows, int64_t k, float delta_threshold,
                    uint32_t* packed, uint16_t* scale_f16, uint32_t* row_ptrs,
                    uint32_t* col_indices, uint8_t* values, int64_t* nnz_out,
                    uint16_t* delta_scale_f16_out);

/* calibration.rs:10-47 ProfileRunner::calibrate on f32 activations [n, k]. Returns -1 if n == 0. */
int oracle_calibrate(const float* acts, int64_t n, int64_t k, float pct_t4, float pct_t8,
                     float* t4_out, float* t8_out);

/* config.rs:157-215 build_csc: CSR (u32 row ptrs, u32 cols, u8 i8-bits, f16 scale) ->
 * CSC with f32 pre-scaled values.  col_ptrs [k+1], row_idx [nnz], vals [nnz].
 * Returns -1 on a column index >= k. */
int oracle_build_csc(const uint32_t* row_ptrs, const uint32_t* col_indices, const uint8_t* values,
                     int64_t nnz, uint16_t delta_scale_f16, int64_t n_rows, int64_t k,
                     uint32_t* col_ptrs, uint32_t* csc_rows, float* csc_vals);

/* config.rs:112-142 dense f32 (base + dW) weight used by the bypass path. */
void oracle_dequant_dense(const uint32_t* packed, const uint16_t* scale_f16, int64_t n_rows, int64_t k,
                          const uint32_t* col_ptrs, const uint32_t* csc_rows, const float* csc_vals,
                          float* w_out);

/* op.rs:64-73 router decision for one score: returns bit0 = use_delta_q8, bit1 = use_delta_fp16. */
int oracle_route_bits(float score, float t4, float t8);

/* op.rs:10-185 cpu_fwd.  x_f16 [m, k]; y_f16 [m, n_rows].
 * csc arrays may be NULL when the layer has no dW (nnz == 0).
 * routed_out (nullable, [m]) receives 1 for tokens whose dW correction ran.
 * acc_out (nullable, [m, n_rows]) receives the f32 accumulator before the f16 cast.
 * force_route (nullable, [m]): entries 0/1 override the router decision (test use only).
 * bypass != 0 follows op.rs:30-58 with dense_w (required then).
 * n_threads <= 0 uses the OpenMP default (row-parallel Phase 1, like rayon). */
void oracle_forward(const uint32_t* packed, const uint16_t* scale_f16, int64_t n_rows, int64_t k,
                    const uint32_t* col_ptrs, const uint32_t* csc_rows, const float* csc_vals,
                    float t4, float t8, const uint16_t* x_f16, int64_t m,
                    uint16_t* y_f16, uint8_t* routed_out, float* acc_out, const uint8_t* force_route,
                    int bypass, const float* dense_w, int n_threads);

#ifdef __cplusplus
}
#endif
#endif
