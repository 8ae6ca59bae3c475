/*
 * saccade_ctarq.h -- C ABI of the B200 (sm_100a) C-TARQ linear library.
 *
 * The C-TARQ linear computes, per token of an f16 activation matrix X [M, K],
 *     Y = f16( (sum_k x_k * (q_rk - 8)) * s_r  +  [routed] * sum_{(r,c) in dW} x_c * dW_rc )
 * over a packed 4-bit base (8 nibbles per u32 along K, one f16 scale per output
 * row) and an int8 coordinate-sparse correction dW (CSR, one global f16 scale)
 * that is applied only to tokens whose activation variance crosses the router
 * thresholds.  The entry points mirror saccade-core's operator:
 *
 *   sc_layer_create   <-  SaccadeLinearOp::new     saccade-core/src/config.rs:76-150
 *   sc_forward        <-  CustomOp1::cpu_fwd       saccade-core/src/op.rs:10-185
 *   sc_op_name        <-  CustomOp1::name          saccade-core/src/op.rs:6-8
 *   sc_set_bypass_c_tarq / sc_is_c_tarq_bypassed
 *                     <-  set_bypass_c_tarq / is_c_tarq_bypassed  saccade-core/src/config.rs:4-12
 *   sc_variance_heuristic <- variance_heuristic    saccade-core/src/heuristics.rs:3-14
 *   sc_percentile_threshold <- compute_percentile_threshold  saccade-core/src/compress.rs:137-176
 *   sc_compress       <-  compress_tensor_to_saccade  saccade-core/src/compress.rs:6-129
 *   sc_calibrate      <-  ProfileRunner::calibrate    saccade-core/src/calibration.rs:10-47
 *
 * Conventions
 *   - Every call returns an sc_status; the message of the last failure on the
 *     calling host thread is available from sc_last_error().
 *   - Tensors are dense row-major, contiguous, at offset 0 (op.rs:19-24 assumes the
 *     same).  Pointers are device pointers unless a parameter says "host".
 *   - Forward calls are asynchronous on the given cudaStream_t (passed as void*),
 *     perform no host synchronisation and allocate nothing when given a workspace.
 *   - Device-side waits are bounded; a wait that runs out records SC_ETIMEOUT in
 *     the layer's device status word (read with sc_layer_check) instead of hanging.
 */
#ifndef SACCADE_CTARQ_H
#define SACCADE_CTARQ_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SC_ABI_VERSION 2
#define SC_GROUP_MAX 4      /* layers per sc_group */

#if defined(__GNUC__)
#define SC_API __attribute__((visibility("default")))
#else
#define SC_API
#endif

typedef enum sc_status {
    SC_OK = 0,
    SC_EINVAL = 1,        /* bad argument (K % 8 != 0, null pointer, size mismatch, bad dtype) */
    SC_ENONCONTIG = 2,    /* pointer not aligned as the layout requires */
    SC_ECUDA = 3,         /* a CUDA runtime call failed */
    SC_ETIMEOUT = 4,      /* a bounded device wait ran out */
    SC_EDEVICE = 5,       /* the device recorded a bad index (e.g. a dW column >= K) */
    SC_ENOMEM = 6,        /* workspace too small / allocation failed */
    SC_EUNSUPPORTED = 7   /* combination not supported by this build */
} sc_status;

typedef enum sc_dtype { SC_F16 = 0, SC_BF16 = 1, SC_F32 = 2 } sc_dtype;

/* Arithmetic of Phase 1 (the 4-bit base product). */
typedef enum sc_mode {
    SC_MODE_FAST = 0,   /* tensor cores, f32 accumulation in hardware order (default) */
    SC_MODE_EXACT = 1,  /* CUDA cores in op.rs's exact 4-accumulator f32 order: bit-identical Y */
    SC_MODE_FAST_TC = 2, /* as SC_MODE_FAST (same tolerance); decode of <= 8 tokens dequantises the
                          * weights into tensor memory and runs tcgen05 MMAs instead of mma.sync */
    SC_MODE_FAST_TC8 = 3 /* as SC_MODE_FAST_TC; one-token decode runs fp8 (e4m3) tcgen05 MMAs on an
                          * exact 8-column e4m3 split of x (elements below 2^-34 of their slice's
                          * maximum keep an error under that bound; inf/nan inputs give nan rows) */
} sc_mode;

typedef enum sc_shard { SC_SHARD_NONE = 0, SC_SHARD_COLUMNS = 1, SC_SHARD_ROWS = 2 } sc_shard;

typedef struct sc_layer sc_layer;

/* Reference-format buffers (compress.rs:113-127 keys) plus router thresholds.
 * The library copies and repacks them; the caller keeps ownership. */
typedef struct sc_layer_desc {
    int64_t out_features;               /* N */
    int64_t in_features;                /* K, multiple of 8 */
    const uint32_t* packed_base;        /* saccade_packed_base  u32 [N, K/8] */
    const uint16_t* scale_base;         /* saccade_scale_base   f16 bits [N] */
    const uint32_t* delta_row_ptrs;     /* saccade_delta_row_ptrs u32 [N+1], NULL when nnz == 0 */
    const uint32_t* delta_col_indices;  /* saccade_delta_col_indices u32 [nnz] */
    const uint8_t* delta_values;        /* saccade_delta_values u8 (i8 bits) [nnz] */
    int64_t delta_nnz;
    uint16_t delta_scale;               /* saccade_delta_scale f16 bits */
    float t4, t8;                       /* router thresholds (config.rs:19-24) */
    int device;                         /* CUDA device ordinal */
    int buffers_on_device;              /* 1: the buffer pointers above are device pointers on `device` */
    int mode;                           /* sc_mode */
    /* Tensor-parallel slice of the unsharded matrix described above.
     * COLUMNS: this layer keeps output rows [N*i/n, N*(i+1)/n) rounded to multiples of 16.
     * ROWS:    this layer keeps input columns [K*i/n, K*(i+1)/n) rounded to multiples of 64;
     *          sc_forward_partial then takes the full [M, K] input (the router needs whole
     *          tokens) and writes f32 partial sums for an all-reduce; sc_forward_split takes
     *          only the slice [M, K_slice] (see below).
     * shard_begin < shard_end overrides index/count with an explicit range: output rows
     * [begin, end) for COLUMNS (multiples of 16, or end = N), input columns for ROWS
     * (multiples of 64, or end = K), e.g. whole attention heads of a tensor-parallel rank. */
    int shard_kind;                     /* sc_shard */
    int shard_index, shard_count;
    int64_t shard_begin, shard_end;     /* ABI 2 */
} sc_layer_desc;

typedef struct sc_layer_info {
    int64_t out_features, in_features;  /* of this (possibly sharded) layer */
    int64_t row_begin, col_begin;       /* offset of the shard in the unsharded matrix */
    int64_t full_out_features, full_in_features;
    int64_t delta_nnz;
    int64_t device_bytes;               /* bytes of weights held on the device */
    float t4, t8;
    int mode, device;
} sc_layer_info;

SC_API int sc_abi_version(void);
SC_API const char* sc_op_name(void);                       /* "fused_c_tarq_saccade_linear" */
SC_API size_t sc_last_error(char* buf, size_t len);         /* copies the calling thread's last message */

SC_API sc_status sc_layer_create(const sc_layer_desc* desc, sc_layer** out);
SC_API void sc_layer_destroy(sc_layer* layer);
SC_API sc_status sc_layer_get_info(const sc_layer* layer, sc_layer_info* info);
SC_API sc_status sc_layer_set_thresholds(sc_layer* layer, float t4, float t8);
SC_API sc_status sc_layer_set_mode(sc_layer* layer, int mode);
/* Reads and clears the layer's device status word (synchronises the stream). */
SC_API sc_status sc_layer_check(sc_layer* layer, void* stream);

/* Global bypass switch: every layer then computes the dense base+dW product for all
 * tokens (op.rs:30-58).  mask_out then reports 1 for every token. */
SC_API void sc_set_bypass_c_tarq(int on);
SC_API int sc_is_c_tarq_bypassed(void);

/* Test hook for the bounded device waits; no counterpart in the reference.  While on, every
 * router-fused decode launch of SC_MODE_FAST (one to eight tokens; the mma.sync engines, which
 * hold no tensor memory) leaves the first weight stage of its first CTA unissued, so the base-product warps' wait on that stage runs out after its bound (2 s):
 * the kernel records SC_ETIMEOUT in the layer's status word (read by sc_layer_check) and returns
 * without writing that CTA's outputs.  Nothing faults and the context stays usable.  Leave it
 * off (0) outside tests. */
SC_API void sc_test_drop_weight_copy(int on);

/* Workspace bytes sc_forward_ws needs for m tokens on this layer. */
SC_API size_t sc_workspace_size(const sc_layer* layer, int64_t m);

/* Y[m, N] = C-TARQ(X[m, K]).  x_dtype F16 or BF16 (BF16 is rounded to f16 first, as the
 * caller's to_dtype(F16) does at saccade-runner/src/model.rs:58-61).  y_dtype F16, BF16 or F32;
 * for BF16/F32 the f16 result is widened/rounded afterwards (model.rs:61).  bias (nullable,
 * f32 [N]) is added after the f16 rounding: y = cast(f32(f16(acc)) + b).
 * mask_out (nullable, u8 [m]), routed_idx_out (nullable, i32 [m], ascending token order) and
 * n_routed_out (nullable, i32 [1]) are device outputs of the router.
 * sc_forward uses a per-device default workspace that it allocates on first use and grows
 * when a larger m arrives (both synchronise the device); it is meant for one stream at a time.
 * sc_forward_ws takes a caller workspace of sc_workspace_size() bytes (256-byte aligned).  Its
 * first 64 KiB hold completion counters at fixed offsets: zero-fill them before the first use;
 * every call returns them to zero, so one workspace serves any sequence of layers and token
 * counts.  Calls sharing a workspace must not overlap on the GPU.  After SC_ETIMEOUT, zero the
 * counter region again before reusing the workspace. */
SC_API sc_status sc_forward(const sc_layer* layer, const void* x, int x_dtype, int64_t m,
                     void* y, int y_dtype, const float* bias,
                     uint8_t* mask_out, int32_t* routed_idx_out, int32_t* n_routed_out, void* stream);
SC_API sc_status sc_forward_ws(const sc_layer* layer, const void* x, int x_dtype, int64_t m,
                        void* y, int y_dtype, const float* bias,
                        uint8_t* mask_out, int32_t* routed_idx_out, int32_t* n_routed_out,
                        void* workspace, size_t workspace_bytes, void* stream);

/* Groups: layers that read the same input -- the q, k and v projections of an attention block,
 * or the gate and up projections of an MLP -- computed by one launch.  No counterpart in the
 * reference, which applies each projection separately (saccade-runner/src/model.rs:217-219 and
 * 296-297).  Masks and routed lists are those of sc_forward on each layer; outputs too, bit for
 * bit in SC_MODE_EXACT, and within the fast-mode tolerance otherwise (the group splits the columns
 * for its combined grid, so f32 partial sums are added in another order; still deterministic).  A group holds 1..SC_GROUP_MAX layers on one device with the same in_features and input
 * columns (no ROWS shards); it references the layers, which must outlive it.  sc_forward_group
 * takes arrays of `count` outputs (y) and optional per-layer arrays (bias, mask_out,
 * routed_idx_out, n_routed_out; NULL for none); the workspace is as for sc_forward_ws, sized for
 * the largest sc_workspace_size of the group's layers.  Layers whose decode cannot share one
 * launch (different split or engine, more than 8 tokens) run one after another on the stream. */
typedef struct sc_group sc_group;
SC_API sc_status sc_group_create(sc_layer* const* layers, int count, sc_group** out);
/* Workspace bytes sc_forward_group needs for m tokens: the largest sc_workspace_size of its layers,
 * or more when the group's layers share one launch of the 9..64-token path.  A smaller workspace
 * (at least every layer's own size) makes the group run its layers one after another. */
SC_API size_t sc_group_workspace_size(const sc_group* group, int64_t m);
SC_API void sc_group_destroy(sc_group* group);
SC_API sc_status sc_forward_group(const sc_group* group, const void* x, int x_dtype, int64_t m,
                                  void* const* y, int y_dtype, const float* const* bias,
                                  uint8_t* const* mask_out, int32_t* const* routed_idx_out,
                                  int32_t* const* n_routed_out, void* workspace, size_t workspace_bytes,
                                  void* stream);

/* sc_forward_group with the routing already computed for x (by sc_qwen2_add_rmsnorm_route or
 * sc_qwen2_silu_mul_route, which wrote x): mask, routed_idx and n_routed are INPUTS, one array
 * per layer as those kernels wrote them.  Only where the group runs the 9..64-token launch for m
 * tokens with this workspace (sc_group_takes_routing == 1; a group of one layer counts); x is f16,
 * 16-byte aligned, [m, in_features].  Outputs equal sc_forward_group's on the same x, bit for bit.
 * No reference counterpart (the reference routes inside each projection, op.rs:64-73). */
SC_API int sc_group_takes_routing(const sc_group* group, int64_t m, size_t workspace_bytes);
SC_API sc_status sc_forward_group_routed(const sc_group* group, const uint16_t* x, int64_t m, void* const* y,
                                         int y_dtype, const float* const* bias, const uint8_t* const* mask,
                                         const int32_t* const* routed_idx, const int32_t* const* n_routed,
                                         void* workspace, size_t workspace_bytes, void* stream);

/* sc_forward_static has no counterpart in the reference.  It is sc_forward without any
 * allocation: its scratch is a file-scope __device__ array of SC_STATIC_SCRATCH_BYTES inside
 * this library, one per device, placed when the library's device code is loaded.  It serves
 * callers that cannot allocate device memory or hand in a workspace on their hot path: a
 * custom-op shim whose signature carries no workspace (candle's CustomOp1::cuda_fwd), or a
 * process whose device memory a framework's caching allocator has already reserved, where an
 * extra cudaMalloc fails or fragments the pool.  It calls no cudaMalloc/cudaFree.
 *  - Limit: calls whose sc_workspace_size(layer, m) exceeds SC_STATIC_SCRATCH_BYTES (8 MiB;
 *    enough for m <= 64 on 7B- and 70B-class decoder shapes) are rejected with SC_EINVAL;
 *    use sc_forward_ws for those.  ROWS shards are rejected as by sc_forward.
 *  - Each call first zero-fills the array's 64 KiB counter region on the stream.
 *  - One array per device is shared by every call on that device: calls that overlap on the
 *    GPU (several streams or host threads) race and corrupt each other's results.
 *  - sc_layer_create looks the array up on its device (cudaGetSymbolAddress, which may load
 *    the module), so sc_forward_static itself loads nothing; the address is kept for the life
 *    of the process, so a cudaDeviceReset invalidates it (create the layers again after one). */
#define SC_STATIC_SCRATCH_BYTES (8u * 1024u * 1024u)
SC_API sc_status sc_forward_static(const sc_layer* layer, const void* x, int x_dtype, int64_t m,
                            void* y, int y_dtype, const float* bias,
                            uint8_t* mask_out, int32_t* routed_idx_out, int32_t* n_routed_out, void* stream);

/* Tensor-parallel pieces.  For a ROWS-sharded layer, sc_forward_partial takes the full
 * [m, full_K] input, routes on it, and writes this shard's f32 contribution [m, N] (base times
 * row scale plus the shard's dW columns for routed tokens).  After an all-reduce (sum) of the
 * partials across shards, sc_finalize rounds to f16 and applies the bias like sc_forward. */
SC_API sc_status sc_forward_partial(const sc_layer* layer, const void* x, int x_dtype, int64_t m,
                             float* y_partial, uint8_t* mask_out, int32_t* routed_idx_out,
                             int32_t* n_routed_out, void* workspace, size_t workspace_bytes, void* stream);
SC_API sc_status sc_finalize(const float* acc, int64_t m, int64_t n, void* y, int y_dtype, const float* bias,
                      void* stream);

/* Tensor parallelism without the whole token on every rank (no counterpart in the reference,
 * which runs on one CPU; the exchange has the op's own semantics, op.rs:30-185).  A ROWS shard's
 * sc_forward_split takes only its input slice x [m, K_slice] and writes one f32 exchange buffer
 * of sc_split_exchange_floats(layer, m) floats:
 *     [ y_base m*N | y_delta m*N | stats m*3 ]
 * y_base = (slice of x . (q - 8)) * s for every token, y_delta = the slice's dW for every token,
 * stats = per token sum x, sum x^2, sum |x| over the slice.  The caller sums the buffers of all
 * ranks (one all-reduce, e.g. NCCL sum), then sc_finalize_split routes each token on the summed
 * sums (heuristics.rs:3-14, op.rs:64-73) and writes y = f16(y_base + [routed] y_delta) (+ bias,
 * cast as sc_forward).  The decision equals the reference's f32 one wherever the f64 score lies
 * outside the f32 summation's error bound of both thresholds; tokens inside it (which the
 * unsharded call replays in the exact f32 order, impossible without the whole token) take the
 * f64 decision and are counted in *undecided_out (device u32, incremented; nullable).
 * workspace: sc_workspace_size(layer, m) bytes or NULL (the device's default workspace). */
SC_API size_t sc_split_exchange_floats(const sc_layer* layer, int64_t m);
SC_API sc_status sc_forward_split(const sc_layer* layer, const void* x, int x_dtype, int64_t m, float* exchange,
                                  void* workspace, size_t workspace_bytes, void* stream);
SC_API sc_status sc_finalize_split(const sc_layer* layer, const float* exchange, int64_t m, int ranks, void* y,
                                   int y_dtype, const float* bias, uint8_t* mask_out, uint32_t* undecided_out,
                                   void* stream);

/* Kernels launched by this library so far in this process (a host-side count of launch calls:
 * a captured CUDA graph counts its kernels once, at capture).  No counterpart in the reference. */
SC_API uint64_t sc_launch_count(void);

/* Router only: per-token variance (exact f32 order of heuristics.rs:3-14) and the routing
 * decision of op.rs:64-73, for m tokens of length k. scores (nullable) f32 [m]. */
SC_API sc_status sc_variance_heuristic(const void* x, int x_dtype, int64_t m, int64_t k, float* scores,
                                void* stream);

/* Format producer on the GPU.  w: f32 [n, k] device.  Synchronous (results land on the host). */
SC_API sc_status sc_percentile_threshold(const float* w, int64_t n, int64_t k, float target_fill_pct,
                                  float* threshold_out_host, void* stream);
/* Pass col_indices == NULL to learn nnz first (written to *nnz_out); then call again with
 * col_indices/values of capacity >= nnz.  Outputs are device buffers; delta_scale lands on the host. */
SC_API sc_status sc_compress(const float* w, int64_t n, int64_t k, float delta_threshold,
                      uint32_t* packed_base, uint16_t* scale_base, uint32_t* delta_row_ptrs,
                      uint32_t* delta_col_indices, uint8_t* delta_values, int64_t capacity,
                      int64_t* nnz_out_host, uint16_t* delta_scale_out_host, void* stream);
/* acts: [n, k] device, F32 or F16 (f16 is widened exactly, as compile.rs:152-153 feeds it). */
SC_API sc_status sc_calibrate(const void* acts, int acts_dtype, int64_t n, int64_t k, float pct_t4, float pct_t8,
                       float* t4_out_host, float* t8_out_host, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* SACCADE_CTARQ_H */
