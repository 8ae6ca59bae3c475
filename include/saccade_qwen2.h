/*
 * saccade_qwen2.h -- C ABI of the Qwen2 decoder glue that surrounds the C-TARQ linears
 * (libsaccade_ctarq.so).  Each entry point is one step of saccade-runner's model, run on the GPU:
 *
 *   sc_qwen2_embed         <- Embedding::forward            saccade-runner/src/model.rs:512
 *   sc_qwen2_add_rmsnorm   <- residual add + RmsNorm::forward  model.rs:92-98, 295-304
 *   sc_qwen2_rope_append   <- RotaryEmbedding::apply + the KV-cache concat  model.rs:111-154, 225-236
 *   sc_qwen2_attention     <- scores, softmax, attn . v (GQA)  model.rs:238-257
 *   sc_qwen2_silu_mul      <- Mlp::forward's silu(gate) * up    model.rs:295-299
 *   sc_qwen2_add_rmsnorm_route, sc_qwen2_silu_mul_route
 *                          <- the two above with the next linears' router (op.rs:64-73,
 *                             heuristics.rs:3-14) in their epilogue, consumed by
 *                             sc_forward_group_routed
 *   sc_qwen2_f16_to_f32    <- ProjectionLayer::forward's to_dtype back to f32  model.rs:61
 *
 * The linears themselves are sc_forward / sc_forward_group calls (saccade_ctarq.h).  Everything is
 * f32 except the inputs of the linears, which these kernels write as f16 (the projection layer's
 * to_dtype(F16), model.rs:58-60).  Calls are asynchronous on `stream` and allocate nothing.
 */
#ifndef SACCADE_QWEN2_H
#define SACCADE_QWEN2_H

#include <stddef.h>
#include <stdint.h>

#include "saccade_ctarq.h"

#ifdef __cplusplus
extern "C" {
#endif

/* out[t] = f32(table[ids[t]]) for an f16 embedding table [vocab, hidden]; an id outside the table
 * records SC_EDEVICE in *status (nullable device word) and reads row 0. */
SC_API sc_status sc_qwen2_embed(const int64_t* ids, int64_t tokens, const uint16_t* table, int64_t vocab,
                                int64_t hidden, float* out, uint32_t* status, void* stream);

/* resid [tokens, hidden] += delta (nullable); out = resid / sqrt(mean(resid^2) + eps) * w, written as
 * f16 (SC_F16: the input of the next linears) or f32 (SC_F32: the final norm before lm_head).  The
 * mean is a fixed-order f32 sum (256 strided partial sums, then those in order).  hidden <= 16384
 * (the row is staged in shared memory); SC_EINVAL otherwise. */
SC_API sc_status sc_qwen2_add_rmsnorm(float* resid, const float* delta, const float* weight, int64_t tokens,
                                      int64_t hidden, float eps, void* out, int out_dtype, void* stream);

/* q [tokens, num_heads, head_dim] rotated in place; k rotated and, with v, written at cache slot
 * slot[t], position pos[t] of k_cache / v_cache [slots, num_kv_heads, max_pos, head_dim]. */
SC_API sc_status sc_qwen2_rope_append(float* q, const float* k, const float* v, const float* cos_table,
                                      const float* sin_table, const int32_t* slot, const int32_t* pos, int64_t tokens,
                                      int num_heads, int num_kv_heads, int head_dim, int max_pos, float* k_cache,
                                      float* v_cache, void* stream);

/* Scratch bytes sc_qwen2_attention needs for `tokens` queries. */
SC_API size_t sc_qwen2_attention_scratch(int64_t tokens, int num_heads, int num_kv_heads, int head_dim, int max_pos);

/* Causal GQA attention: token t attends the keys 0..pos[t] of its cache slot; out_f16 [tokens,
 * num_heads * head_dim].  max_query_pos bounds every pos[t] (it sizes the key blocks launched).
 * Limits (SC_EINVAL otherwise): head_dim 32, 64 or 128; at most 8 query heads per KV head and 128
 * query heads; max_query_pos < 8192.  Keys go in blocks of 256: per block the scores (per-lane
 * partial dot products over head_dim, then a 32-lane xor butterfly), its max, exp evaluated in f64
 * and rounded to f32, the lane-strided sum, p . v over the keys in order; blocks are combined in
 * order, so the result is a fixed function of the inputs. */
SC_API sc_status sc_qwen2_attention(const float* q, const float* k_cache, const float* v_cache, const int32_t* slot,
                                    const int32_t* pos, int64_t tokens, int num_heads, int num_kv_heads, int head_dim,
                                    int max_pos, int max_query_pos, float* scratch, size_t scratch_bytes,
                                    uint16_t* out_f16, void* stream);

/* out_f16[i] = f16(silu(f32(gate[i])) * f32(up[i])), silu(g) = g / (1 + exp(-g)). */
SC_API sc_status sc_qwen2_silu_mul(const uint16_t* gate, const uint16_t* up, int64_t n, uint16_t* out_f16,
                                   void* stream);

/* out[i] = f32(x[i]) for f16 x. */
/* The router of the linears that read the output, fused into the kernel that writes it.  Each
 * kernel is one CTA per token: it writes the token's f16 row exactly as the plain kernel does
 * (same bits), keeps it in shared memory, and routes the token for every layer of `group`
 * (heuristics.rs:3-14, op.rs:64-73: f64 sums decide when the thresholds lie outside the f32 error
 * band, else the reference's f32 chains are replayed), writing mask[l][t] (0/1); the last CTA to
 * finish writes the ascending routed list routed_idx[l][0..n) and n_routed[l][0] of each layer.
 * These are the routing sc_forward_group would compute on the same row, and sc_forward_group_routed
 * takes them instead of routing again.  `counter` is one uint32 in device memory that is zero
 * before the call (the kernel leaves it zero).  The group's layers must read the whole row:
 * in_features == hidden (norm) or width (silu); set_bypass_c_tarq routes every token.
 * add_rmsnorm_route: resid += delta (nullable), out_f16 = f16 RMSNorm as sc_qwen2_add_rmsnorm
 * (hidden <= 16384).  silu_mul_route: out_f16 [tokens, width] = f16(silu(gate) * up) as
 * sc_qwen2_silu_mul (width a multiple of 8, width <= 65536).  No reference counterpart: the
 * reference routes inside each projection (op.rs:64-73). */
SC_API sc_status sc_qwen2_add_rmsnorm_route(float* resid, const float* delta, const float* weight, int64_t tokens,
                                            int64_t hidden, float eps, uint16_t* out_f16, const sc_group* group,
                                            uint8_t* const* mask, int32_t* const* routed_idx,
                                            int32_t* const* n_routed, uint32_t* counter, void* stream);
SC_API sc_status sc_qwen2_silu_mul_route(const uint16_t* gate, const uint16_t* up, int64_t tokens, int64_t width,
                                         uint16_t* out_f16, const sc_group* group, uint8_t* const* mask,
                                         int32_t* const* routed_idx, int32_t* const* n_routed, uint32_t* counter,
                                         void* stream);

SC_API sc_status sc_qwen2_f16_to_f32(const uint16_t* x, int64_t n, float* out, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* SACCADE_QWEN2_H */
