// sc_internal.h -- host-side structures shared by the library's translation units.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <string>

#include "saccade_ctarq.h"

namespace sc {

// Device status word codes (written with atomicCAS so the first error wins).
enum : uint32_t { DEV_OK = 0, DEV_TIMEOUT = 1, DEV_BAD_INDEX = 2 };

// Device layout of one C-TARQ layer (immutable after sc_layer_create).
//
//  wq      u32 [Np/128][KB][2][128][4]   4-bit base in 128-row x 64-column blocks (4 KB):
//                                       chunk c of row r holds columns 64kb+32c .. +31 as
//                                       four words of 8 columns; nibble p of a word holds
//                                       column offset (p&3)*2 + (p>>2) (see dequant_word).
//                                       Padding rows/columns hold nibble 8 (q = 0).
//  scale   f32 [Np]                     f16 row scale widened (config.rs:96-101); 0 on padding.
//  rowptr  u32 [N+1], col u16 [nnz+8], val i8 [nnz+16]
//                                       dW in CSR, columns ascending within a row (compress.rs:89-105).
struct Layer {
    int device = 0;
    int sms = 148;               // multiprocessors of `device`
    int mode = SC_MODE_FAST;
    int64_t N = 0, K = 0;        // this shard's extent
    int64_t Np = 0, Kp = 0;      // padded to 128 rows / 64 columns
    int64_t KB = 0;              // Kp / 64
    int64_t row_begin = 0, col_begin = 0, fullN = 0, fullK = 0;
    int shard_kind = SC_SHARD_NONE;
    int64_t nnz = 0;
    float ds = 1.0f;             // dW scale widened from f16
    float t4 = 0.0f, t8 = 0.0f;
    uint32_t* wq = nullptr;
    float* scale = nullptr;
    uint32_t* rowptr = nullptr;
    uint16_t* col = nullptr;
    int8_t* val = nullptr;
    uint32_t* status = nullptr;  // device status word
    int64_t device_bytes = 0;
    // dW regrouped for the router-fused decode kernel: one block per (128-row tile, column
    // split) holding u16 row offsets [129] (padded to 272 B), u16 local columns and i8 values
    // (each padded to 16 B), so a CTA fetches exactly its entries with one bulk copy.
    int ks_fused = 0;            // column splits (= cluster size) of the fused kernel; 0: not usable
    uint8_t* dwblk = nullptr;
    uint32_t* dwoff = nullptr;   // byte offset of block (rt * ks_fused + split); [RT*ks_fused + 1]
    int dw_global = 0;           // 1: some block exceeds the kernel's shared-memory copy, so every
                                 // CTA reads its block from global memory
    // dW over the row scale, per (128-row tile, 64-column block), for the prefill GEMM: routed
    // tokens' tiles fold it into the dequantised weights ((q - 8) + dW/s, see sc_gemm.cu).
    uint8_t* fold = nullptr;     // lists, each [9 u16 offsets per 16-row tile | pad to 32 B | u32 entries]
    uint32_t* foldoff = nullptr; // byte offset of list (rt * KB + kb); [RT*KB + 1]; null: no fold
    int fold_cap = 0;            // shared-memory slot of one list: 4096 or 8192 bytes
    // dW per (128-row tile, 64-column block) for the 9..64-token GEMM: u16 row offsets [129] (padded
    // to 272 B), then u16 entries (column in the block | i8 value << 6), ascending columns per row.
    uint8_t* dseg = nullptr;
    uint32_t* dsegoff = nullptr; // byte offset of segment (rt * KB + kb); [RT*KB + 1]; null: no dW
    int dseg_max = 0;            // largest segment, bytes (16-byte multiple)
};

// Shared-memory budget of one dW block in the fused decode kernel.
constexpr int64_t kDwBlockMax = 16 * 1024;
#ifndef SC_FUSED_MAX_CLUSTER
#define SC_FUSED_MAX_CLUSTER 16
#endif
#ifndef SC_FUSED_SMALL_PCT
#define SC_FUSED_SMALL_PCT 100  // a launch is small (one CTA per SM) up to this % of the one-CTA-per-SM rings
#endif
#ifndef SC_FUSED_INT8
#define SC_FUSED_INT8 1  // one-token decode in SC_MODE_FAST runs the s8 integer variant
#endif
constexpr int kMaxFusedCluster = SC_FUSED_MAX_CLUSTER;  // CTAs of one row tile (cluster size)

int fused_ksplit(const Layer& L);
int choose_ksplit(int64_t rt, int64_t kb);  // splits of a one-wave launch of rt row tiles x kb column blocks
bool use_fused_ks(const Layer& L, int64_t m, int ks);
bool use_fused(const Layer& L, int64_t m);  // the router-fused decode kernel serves this call

// Completion-counter region at the start of every workspace (see plan_workspace).
constexpr size_t kCounterBytes = 64 * 1024;
constexpr int64_t kMaxRowTiles = (kCounterBytes - 256) / 4;   // 128-row tiles per layer

// Per-call workspace carve-up (offsets in bytes from the workspace base).
struct WsLayout {
    int64_t Mp = 0;              // tokens padded to 8
    size_t xk = 0, mask = 0, scores = 0, ridx = 0, nrouted = 0, counter = 0;
    size_t partial = 0, rtcount = 0;
    size_t xkp = 0, perm = 0;    // prefill GEMM: x in routed-first order and that order
    int gemm_ks = 0;             // prefill GEMM column splits (0: the GEMM does not serve the call)
    size_t xconv = 0;            // 9..64-token GEMM: f16 copy of bf16 (or unaligned) tokens
    int mid_ks = 0;              // its column splits (0: it does not serve the call)
    size_t xt = 0;               // ROWS shards: the slice transposed for sc_forward_split
    size_t total = 0;
    int ksplit = 1;
    int chunk_tokens = 0;        // tokens per decode launch
};

WsLayout plan_workspace(const Layer& L, int64_t m);

void set_error(const std::string& msg);
sc_status cuda_fail(cudaError_t e, const char* what);

// Launch with programmatic stream serialization (PDL): the kernel may start while the
// previous kernel on the stream finishes; it must call griddepcontrol.wait before touching
// anything that kernel writes or reads.
// Dynamic shared memory of the router kernels (the token row, f16): K <= 65536.
constexpr int kRouterMaxRowBytes = 128 * 1024;

// Kernels this library has launched (host-side count of launch calls, sc_launch_count).
extern std::atomic<uint64_t> g_launches;

template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                       Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    g_launches.fetch_add(1, std::memory_order_relaxed);
    return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

// Kernel launchers (each returns the launch error, if any).
cudaError_t launch_repack(const uint32_t* packed, int64_t ref_words_per_row, int64_t row0, int64_t word0,
                          const Layer& L, cudaStream_t s);
cudaError_t launch_scales(const uint16_t* scale_f16, int64_t row0, const Layer& L, cudaStream_t s);

struct RouterArgs {
    const void* x;
    int x_dtype;
    int64_t x_row_stride;   // elements between consecutive tokens of x
    int64_t x_col0;         // first column of x used (0)
    int64_t M, K, Mp, KB;
    float t4, t8;
    int route_all;          // bypass: every token takes dW
    uint16_t* xk;           // [KB][Mp][64] f16 bits (swizzled)
    uint8_t* mask;
    float* scores;
    int32_t* ridx;
    int32_t* nrouted;
    int32_t* perm;          // nullable: routed-first token order for the GEMM
    uint32_t* counter;
    uint32_t* status;
};
cudaError_t launch_router(const RouterArgs& a, cudaStream_t s);

struct DecodeArgs {
    const Layer* L;
    const uint16_t* xk;
    int64_t Mp;             // token stride of xk
    int64_t tok0, ntok;     // token range of this launch
    const uint8_t* mask;
    const int32_t* ridx;
    const int32_t* nrouted;
    int route_all;
    int64_t dcol_begin, dcol_end;   // dW columns applied (shard range, relative to L)
    void* y;                // [M, N] rows tok0..tok0+ntok; or f32 partial when partial_out
    int y_dtype;
    const float* bias;
    int partial_out;        // 1: write f32 accumulators (no f16 rounding)
    float* ws_partial;
    uint32_t* ws_rtcount;
    int ksplit;
};
cudaError_t launch_decode_tc(const DecodeArgs& a, cudaStream_t s);

// Many tokens (prefill): tcgen05 GEMM over 128-token tiles of the router's staged x, taken in
// routed-first order (perm) so that routed tokens share tiles.
struct GemmArgs {
    const Layer* L;
    const uint16_t* xk;     // staged x (xk_index layout) in token order, Mp token rows
    uint16_t* xkp;          // the same in perm order (written by launch_gemm's gather)
    const int32_t* perm;    // staged position -> token: routed at [0, R), the others from round_up(R, 8)
    const int32_t* nrouted; // routed tokens R (device)
    int64_t Mp, M;          // xk token rows, tokens
    int64_t Mpp;            // xkp / perm positions (Mp + 16)
    int route_all;
    int ks;                 // column splits (>= 1)
    float* partial;         // split partials [tiles][ks][128 tokens][128 rows] (ks > 1)
    uint32_t* tcount;       // per-tile split counters (ks > 1), zero between calls
    void* y;                // [M, N]; f32 partial when partial_out
    int y_dtype;
    const float* bias;
    int partial_out;
    int skip_gather;        // xkp and perm already hold this x (a previous layer of the same group)
};
cudaError_t launch_gemm(const GemmArgs& a, cudaStream_t s);
int64_t gemm_tile_tokens();
int gemm_ksplit(const Layer& L, int64_t m);  // column splits of the prefill GEMM for m tokens
cudaError_t build_fold_lists(Layer& L, const uint32_t* srp, const uint16_t* scol, const int8_t* sval,
                             const float* scale);
cudaError_t build_dw_segments(Layer& L, const uint32_t* srp, const uint16_t* scol, const int8_t* sval);
#ifndef SC_GEMM_MIN_TOKENS
#define SC_GEMM_MIN_TOKENS 9  // calls of at least this many tokens (not decoded fused) run the GEMM
#endif
constexpr int64_t kGemmMinTokens = SC_GEMM_MIN_TOKENS;
cudaError_t launch_decode_exact(const DecodeArgs& a, int bypass, cudaStream_t s);

// Decode with the router fused in (<= 8 tokens): one launch reads x directly.
struct FusedArgs {
    const Layer* L;
    const void* x;
    int x_dtype;
    int64_t x_stride;       // elements per token row of x (the router's length)
    int64_t x_col0;         // first column of this layer's slice within a row
    int64_t m;
    int route_all;
    void* y;
    int y_dtype;
    const float* bias;
    int partial_out;
    uint8_t* mask_out;
    int32_t* ridx_out;
    int32_t* nrouted_out;
    float* ws_partial;
    uint32_t* ws_rtcount;
    int ksplit;
    const uint8_t* dwblk;   // dW blocks built for this ksplit (null: the kernel reads the CSR)
    const uint32_t* dwoff;
    int dw_global;          // 1: the blocks are read from global memory (too large to copy)
};
// One launch for n (<= SC_GROUP_MAX) layers that read the same x, all with the same ksplit and mode.
cudaError_t launch_decode_fused(const FusedArgs* f, int n, cudaStream_t s);
// How many thread-block clusters of `ks` CTAs of the router-fused decode kernel can be resident
// at once on the current device (cached per device).
int fused_max_active_clusters(int ks);
int fused_max_kb(int64_t m);  // largest column range (64-column blocks) one fused CTA holds for m tokens
int64_t fused_prefetch_bytes();  // weight bytes the fused kernel prefetches with one CTA on every SM

// 9..16 tokens (batched decode): k_mid_route (routing, skipped when the caller routed already),
// then k_ctarq_mid, a tcgen05 f16 GEMM with the tokens as the MMA's N side and dW of the routed
// tokens from the staged token tiles (sc_mid.cu).  One call serves 1..SC_GROUP_MAX layers reading
// the same x.
#ifndef SC_MID_MIN_TOKENS
#define SC_MID_MIN_TOKENS 9   // calls of at least this many tokens (and at most 64) run it
#endif
#ifndef SC_MID_MAX_TOKENS
#define SC_MID_MAX_TOKENS 64  // ... up to this many
#endif
#ifndef SC_MID_FOLD_MIN_TOKENS
#define SC_MID_FOLD_MIN_TOKENS 17  // from this many tokens routed tokens' dW is folded into a second A
#endif
constexpr int64_t kMidMinTokens = SC_MID_MIN_TOKENS;
constexpr int64_t kMidMaxTokens = SC_MID_MAX_TOKENS;
constexpr int64_t kMidFoldMinTokens = SC_MID_FOLD_MIN_TOKENS;
struct MidArgs {
    int n;                                  // layers (same K and input columns)
    const Layer* layer[SC_GROUP_MAX];
    const void* x;
    int x_dtype;
    int64_t x_stride, x_col0, m;
    int route_all;
    int ks;                                 // column splits (mid_ksplit)
    int routed_in;                          // 1: mask / ridx / nrouted already hold the routing
    uint32_t* counter;                      // the router's completion counter (zero between calls)
    uint16_t* xconv;                        // [m][x_stride] f16: bf16 (or unaligned) tokens for the TMA loads
    uint8_t* mask[SC_GROUP_MAX];
    int32_t* ridx[SC_GROUP_MAX];
    int32_t* nrouted[SC_GROUP_MAX];
    void* y[SC_GROUP_MAX];
    int y_dtype;
    const float* bias[SC_GROUP_MAX];
    int partial_out;
    float* partial;                         // [sum RT][ks][m][128] f32 (ks > 1)
    uint32_t* rtcount;                      // [sum RT] counters (zero between calls)
};
int mid_ksplit(int64_t rt_total, int64_t kb, int sms, int64_t m);
// The layers of a group (at most SC_GROUP_MAX into `out`; returns how many) and whether
// set_bypass_c_tarq is on: what a router outside the library's own launches needs (sc_model.cu).
int group_layers(const sc_group* g, const Layer** out);
int bypass_on();
bool use_mid(const Layer& L, int64_t m);
cudaError_t launch_mid(const MidArgs& a, cudaStream_t s);

// Test hook: the next router-fused decode launches leave CTA 0's first weight stage unissued.
void set_drop_weight_copy(int on);

// Exchange step of a ROWS shard that holds only its input slice (sc_split.cu).
cudaError_t launch_split_extras(const Layer& L, const void* x, int x_dtype, int64_t m, float* y_delta, float* stats,
                                uint16_t* xt, cudaStream_t s);
cudaError_t launch_split_finalize(const Layer& L, const float* exch, int64_t m, int ranks, int route_all, void* y,
                                  int y_dtype, const float* bias, uint8_t* mask_out, uint32_t* undecided,
                                  cudaStream_t s);
cudaError_t launch_finalize(const float* acc, int64_t m, int64_t n, void* y, int y_dtype, const float* bias,
                            cudaStream_t s);

}  // namespace sc
