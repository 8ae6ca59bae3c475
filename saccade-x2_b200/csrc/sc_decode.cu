// sc_decode.cu -- C-TARQ kernels for a few tokens per call (decode, M <= 8) and the exact mode.
//
// The fast kernels stream the 4-bit base through a shared-memory ring filled by one producer
// lane with non-multicast bulk copies (cp.async.bulk + mbarrier complete_tx, L2 evict-first on
// weights).  A CTA owns one 128-row tile and a contiguous range of 64-column blocks (split-K
// across CTAs when a layer has few rows).  Under programmatic dependent launch the producer
// requests its first weight stages before griddepcontrol.wait, so they overlap the previous
// kernel's tail; activations are read only after the wait.
//
//   k_ctarq_fused_mma / k_ctarq_fused_tc (below): the router folded in, one launch per call or
//                group of calls; the production decode path.
//   k_ctarq_mma  (<= 8 tokens, a layer too wide for the fused kernel's x copy, after k_router):
//                eight MMA warps, one 16-row tile each.  Per 64 columns a lane reads 16 bytes of
//                packed nibbles, converts each word into an mma.m16n8k16 A fragment of exact
//                integers q-8 in registers (dequant_word) and multiplies it with the activations,
//                f32 accumulation.  dW warps: one output row per lane; they walk the row's CSR dW
//                entries in the CTA's column range for the routed tokens (op.rs:152-170).
//                Epilogue: y = f16(acc * s + dW) (+ bias after the rounding); with split-K the
//                last CTA of a row tile sums the partials in split order (deterministic).
// More tokens go to the prefill GEMM (sc_gemm.cu).
//
// k_decode_exact: SC_MODE_EXACT.  One thread per row pair replays op.rs exactly: four f32
// accumulators fed in the reference's order with single-rounding f16 x f16 -> f32 FMAs
// (the products are exact), ((a0+a1)+a2)+a3 then * scale, then the dW entries in ascending
// column order with separate multiply and add.  Y is bit-identical to cpu_fwd.  Each
// accumulator is a K/4-long dependent chain: a verification path, not a fast one.
#include <atomic>

#include "sc_device.cuh"
#include "sc_internal.h"

namespace sc {

constexpr int kMaxChunkTokens = 32;

struct TCParams {
    const uint32_t* wq;
    const float* scale;
    const uint32_t* rowptr;
    const uint16_t* col;
    const int8_t* val;
    float ds;
    int64_t nnz;
    const uint16_t* xk;
    int64_t Mp;
    int64_t tok0;
    int ntok;
    const uint8_t* mask;
    int route_all;
    int64_t N, K, KB;
    void* y;
    int y_dtype;
    const float* bias;
    int partial_out;
    float* ws_partial;
    uint32_t* ws_rtcount;
    int ksplit;
    uint32_t* status;
};


// ---------------------------------------------------------------- shared pieces

// Producer lane: weights (4 KB per 64-column block, contiguous per row tile) and the real
// token groups of the activations (1 KB per block and group) into ring stage `slot`.
// Weights of the first `kStages` stages are requested before the dependency wait.
template <int SKB, int S, int G, int WBYTES, int STAGEBYTES>
__device__ __forceinline__ int producer_run(const TCParams& p, unsigned char* smem, uint64_t* full, uint64_t* empty,
                                            int64_t rt, int64_t kb_begin, int64_t kb_end, int greal, int* abort) {
    const int nst = static_cast<int>((kb_end - kb_begin + SKB - 1) / SKB);
    const int Gp = static_cast<int>(p.Mp >> 3);
    const uint64_t pol = policy_evict_first();
    int issued = 0;
    const int pre = nst < S ? nst : S;
    for (int it = 0; it < pre; ++it, ++issued) {
        const int64_t kb0 = kb_begin + static_cast<int64_t>(it) * SKB;
        const int n = static_cast<int>(imin64(SKB, kb_end - kb0));
        mbar_arrive_expect_tx(&full[it], static_cast<uint32_t>(n * 4096));
        bulk_g2s_stream(smem + it * STAGEBYTES, p.wq + (rt * p.KB + kb0) * 1024, static_cast<uint32_t>(n * 4096),
                        &full[it], pol);
    }
    pdl_wait();
    for (int it = 0; it < nst; ++it) {
        const int slot = it % S;
        const int64_t kb0 = kb_begin + static_cast<int64_t>(it) * SKB;
        const int n = static_cast<int>(imin64(SKB, kb_end - kb0));
        unsigned char* st = smem + slot * STAGEBYTES;
        if (it >= S) {
            if (!mbar_wait(&empty[slot], ((it / S) - 1) & 1, p.status)) {
                *abort = 1;
                break;
            }
            mbar_arrive_expect_tx(&full[slot], static_cast<uint32_t>(n * 4096));
            bulk_g2s_stream(st, p.wq + (rt * p.KB + kb0) * 1024, static_cast<uint32_t>(n * 4096), &full[slot], pol);
            ++issued;
        }
        mbar_arrive_expect_tx(&full[slot], static_cast<uint32_t>(n * greal * 1024));
        for (int j = 0; j < n; ++j)
            bulk_g2s(st + WBYTES + j * G * 1024, p.xk + ((kb0 + j) * Gp + (p.tok0 >> 3)) * 512,
                     static_cast<uint32_t>(greal * 1024), &full[slot]);
    }
    return issued;
}

// dW warps: lane `rl` of a 128-row tile accumulates x * (i8 * scale) over the row's CSR entries
// inside [kb_begin*64, kb_end*64) for every routed token of the chunk, in column order.
template <int NT, int LD>
__device__ __forceinline__ void delta_rows(const TCParams& p, float* corrbuf, int rl, int64_t rt, int64_t kb_begin,
                                           int64_t kb_end) {
    const int64_t row = rt * 128 + rl;
    uint32_t routed = 0;
    for (int tt = 0; tt < p.ntok; ++tt)
        if (p.route_all || p.mask[p.tok0 + tt]) routed |= 1u << tt;
    if (routed == 0 || row >= p.N || p.nnz == 0) return;
    const int64_t lo = p.rowptr[row], hi = p.rowptr[row + 1];
    const int64_t e0 = lower_bound_u16(p.col, lo, hi, kb_begin * 64);
    const int64_t e1 = lower_bound_u16(p.col, e0, hi, kb_end * 64);
    float corr[NT];
#pragma unroll
    for (int tt = 0; tt < NT; ++tt) corr[tt] = 0.0f;
    for (int64_t e = e0; e < e1; e += 8) {
        const int cnt = static_cast<int>(imin64(8, e1 - e));
        int64_t cc[8];
        float vv[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            cc[u] = u < cnt ? static_cast<int64_t>(p.col[e + u]) : 0;
            vv[u] = u < cnt ? __fmul_rn(static_cast<float>(p.val[e + u]), p.ds) : 0.0f;
        }
#pragma unroll
        for (int tt = 0; tt < NT; ++tt) {
            if ((routed >> tt) & 1u) {
                const int t = static_cast<int>(p.tok0 + tt);
                float xv[8];
#pragma unroll
                for (int u = 0; u < 8; ++u)
                    xv[u] = u < cnt ? h2f(p.xk[xk_index(cc[u], t, static_cast<int>(p.Mp))]) : 0.0f;
#pragma unroll
                for (int u = 0; u < 8; ++u)
                    if (u < cnt) corr[tt] = __fadd_rn(corr[tt], __fmul_rn(xv[u], vv[u]));
            }
        }
    }
#pragma unroll
    for (int tt = 0; tt < NT; ++tt) corrbuf[rl * LD + tt] = corr[tt];
}

// Epilogue over a [128 x NT] tile of f32 accumulators held in shared memory.  Single-split:
// y = acc*s + dW.  Split-K: partials to the workspace, the last CTA of the row tile sums them
// in split order.  Returns after the stores.
template <int NT, int LD, int NTHREADS>
__device__ __forceinline__ void epilogue_tile(const TCParams& p, const float* accbuf, const float* corrbuf, int64_t rt,
                                              int split, int* s_last) {
    const int tid = threadIdx.x;
    const int cnt = 128 * p.ntok;
    if (p.ksplit == 1) {
        for (int i = tid; i < cnt; i += NTHREADS) {
            const int rl = i & 127, tt = i >> 7;
            const int64_t row = rt * 128 + rl;
            if (row >= p.N) continue;
            const float v = __fadd_rn(__fmul_rn(accbuf[rl * LD + tt], p.scale[row]), corrbuf[rl * LD + tt]);
            const int64_t oi = (p.tok0 + tt) * p.N + row;
            if (p.partial_out) reinterpret_cast<float*>(p.y)[oi] = v;
            else store_output(p.y, p.y_dtype, oi, v, p.bias, row);
        }
        return;
    }
    float* part = p.ws_partial + (rt * p.ksplit) * 128 * kMaxChunkTokens;
    for (int i = tid; i < cnt; i += NTHREADS) {
        const int rl = i & 127, tt = i >> 7;
        const int64_t row = rt * 128 + rl;
        const float v = row < p.N ? __fadd_rn(__fmul_rn(accbuf[rl * LD + tt], p.scale[row]), corrbuf[rl * LD + tt])
                                  : 0.0f;
        part[(split * 128 + rl) * kMaxChunkTokens + tt] = v;
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) {
        const unsigned ticket = atomicAdd(&p.ws_rtcount[rt], 1u);
        *s_last = (ticket == static_cast<unsigned>(p.ksplit - 1)) ? 1 : 0;
    }
    __syncthreads();
    if (!*s_last) return;
    __threadfence();
    for (int i = tid; i < cnt; i += NTHREADS) {
        const int rl = i & 127, tt = i >> 7;
        const int64_t row = rt * 128 + rl;
        if (row >= p.N) continue;
        float v = 0.0f;
        for (int sp = 0; sp < p.ksplit; ++sp) v = __fadd_rn(v, __ldcg(&part[(sp * 128 + rl) * kMaxChunkTokens + tt]));
        const int64_t oi = (p.tok0 + tt) * p.N + row;
        if (p.partial_out) reinterpret_cast<float*>(p.y)[oi] = v;
        else store_output(p.y, p.y_dtype, oi, v, p.bias, row);
    }
    if (tid == 0) p.ws_rtcount[rt] = 0u;
}

// ---------------------------------------------------------------- k_ctarq_mma (<= 8 tokens)

struct MmaCfg {
    static constexpr int kMmaWarps = 8;              // one 16-row tile each
    static constexpr int kProducerWarp = 8;
    static constexpr int kDeltaWarp0 = 9;
    static constexpr int kThreads = 13 * 32;
    static constexpr int NT = 8;
    static constexpr int G = 1;
    static constexpr int SKB = 8;                    // 64-column blocks per stage (32 KB of weights)
    static constexpr int S = 4;
    static constexpr int kWBytes = SKB * 4096;
    static constexpr int kXBytes = SKB * G * 1024;
    static constexpr int kStageBytes = kWBytes + kXBytes;
    static constexpr int kLd = NT + 1;
    static constexpr int kAccOff = S * kStageBytes;
    static constexpr int kCorrOff = kAccOff + 128 * kLd * 4;
    static constexpr int kBarOff = kCorrOff + 128 * kLd * 4;
    static constexpr int kTotal = kBarOff + 2 * S * 8 + 16;
    static_assert(kTotal <= 227 * 1024, "shared memory");
};

__global__ void __launch_bounds__(MmaCfg::kThreads, 1) k_ctarq_mma(TCParams p) {
    using C = MmaCfg;
    constexpr int SKB = C::SKB, S = C::S;
    extern __shared__ __align__(1024) unsigned char smem[];
    float* accbuf = reinterpret_cast<float*>(smem + C::kAccOff);
    float* corrbuf = reinterpret_cast<float*>(smem + C::kCorrOff);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::kBarOff);
    uint64_t* empty = full + S;
    __shared__ int s_last;
    __shared__ int s_abort;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int64_t rt = blockIdx.x / p.ksplit;
    const int split = static_cast<int>(blockIdx.x - rt * p.ksplit);
    const int64_t kb_begin = (p.KB * split) / p.ksplit;
    const int64_t kb_end = (p.KB * (split + 1)) / p.ksplit;
    const int nst = static_cast<int>((kb_end - kb_begin + SKB - 1) / SKB);

    pdl_launch_dependents();
    for (int i = tid; i < 2 * 128 * C::kLd; i += C::kThreads) accbuf[i] = 0.0f;  // acc and dW tiles
    if (tid == 0) {
        for (int i = 0; i < S; ++i) {
            mbar_init(&full[i], 2);
            mbar_init(&empty[i], C::kMmaWarps);
        }
        fence_mbar_init();
        s_abort = 0;
    }
    __syncthreads();

    int issued = 0;
    if (warp == C::kProducerWarp) {
        if (lane == 0)
            issued = producer_run<SKB, S, C::G, C::kWBytes, C::kStageBytes>(p, smem, full, empty, rt, kb_begin, kb_end,
                                                                           1, &s_abort);
    } else if (warp < C::kMmaWarps) {
        float acc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
        const int g = lane >> 2, c = lane & 3;
        const bool has_tok = g < p.ntok;
        // B fragment of step s: x[token g][k0 + 4c .. +3] (the permuted K of the A fragment)
        const int xoff = g * 16 + (c & 1) * 8 + (c >> 1) * 128;
        for (int it = 0; it < nst; ++it) {
            const int slot = it % S;
            if (!mbar_wait(&full[slot], (it / S) & 1, p.status)) {
                s_abort = 1;
                break;
            }
            const int64_t kb0 = kb_begin + static_cast<int64_t>(it) * SKB;
            const int n = static_cast<int>(imin64(SKB, kb_end - kb0));
            const unsigned char* st = smem + slot * C::kStageBytes;
#pragma unroll
            for (int j = 0; j < SKB; ++j) {
                if (j < n) {
                    const uint4 wv = *reinterpret_cast<const uint4*>(st + j * 4096 + warp * 512 + lane * 16);
                    const unsigned char* xb = st + C::kWBytes + j * 1024 + xoff;
                    const uint32_t words[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
                    for (int s = 0; s < 4; ++s) {
                        uint2 b = make_uint2(0u, 0u);
                        if (has_tok) b = *reinterpret_cast<const uint2*>(xb + s * 256);
                        uint32_t a[4];
                        dequant_word(words[s], a);
                        mma_16816(acc[s & 1], a, b.x, b.y);
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[slot]);
        }
        // fragment -> tile: rows g, g+8 of this warp's tile; tokens 2c, 2c+1
        const int r0 = warp * 16 + g;
        accbuf[r0 * C::kLd + 2 * c] = acc[0][0] + acc[1][0];
        accbuf[r0 * C::kLd + 2 * c + 1] = acc[0][1] + acc[1][1];
        accbuf[(r0 + 8) * C::kLd + 2 * c] = acc[0][2] + acc[1][2];
        accbuf[(r0 + 8) * C::kLd + 2 * c + 1] = acc[0][3] + acc[1][3];
    } else {
        pdl_wait();
        delta_rows<C::NT, C::kLd>(p, corrbuf, (warp - C::kDeltaWarp0) * 32 + lane, rt, kb_begin, kb_end);
    }
    __syncwarp();
    __syncthreads();
    if (s_abort) {
        if (warp == C::kProducerWarp && lane == 0)
            for (int it = issued > S ? issued - S : 0; it < issued; ++it)
                mbar_wait(&full[it % S], (it / S) & 1, nullptr, kDrainNs);
        return;
    }
    pdl_wait();
    epilogue_tile<C::NT, C::kLd, C::kThreads>(p, accbuf, corrbuf, rt, split, &s_last);
}

// ---------------------------------------------------------------- router-fused decode (<= 8 tokens)

// Decode kernels with the router folded in.  The ksplit CTAs that share a 128-row tile form a
// thread-block cluster; each takes a column slice.  Four auxiliary warps stage the slice of
// every token into shared memory (bf16 rounded to f16) while summing x, x^2 and |x| in f32;
// each CTA pushes its sums to every CTA of the cluster (st.async into the receiver's shared
// memory, completing on its mbarrier), so every CTA adds the whole-token sums in rank order --
// identical in every cluster -- and takes the reference's routing decision (route_token, with
// the band widened by the bound on the f32 summation error).  dW comes from a per-CTA block
// prepared at load time and fetched with one bulk copy; auxiliary thread r owns row r of the
// tile: it adds that row's dW, scales, and pushes the row to the cluster CTA that owns it, which
// adds the splits in rank order and writes y.  CTA 0 publishes the mask and the routed-token
// list.  The ring carries weights only, so the producer never waits on the previous kernel;
// about 108 KB of shared memory lets two CTAs (of this call and the next) share an SM.  x is
// staged for ntp = ntok rounded up to a power of two tokens, as [8-column chunk][ntp][8 f16].
//
// Two base-product engines share that frame: k_ctarq_fused_tc dequantises the weights into
// tensor memory and runs tcgen05 MMAs (M=128, N=16, K=16) on the staged x; k_ctarq_fused_mma
// runs mma.sync on the same data.
struct FusedParams {
    TCParams t;
    const void* x;
    int x_dtype;
    int64_t x_stride;   // elements between tokens of x
    int64_t x_col0;     // column of x where this layer's slice starts (rows shards)
    int64_t Kfull;      // values per token used by the router
    float t4, t8;
    uint8_t* mask_out;
    int32_t* ridx_out;
    int32_t* nrouted_out;
    const uint8_t* dwblk;   // blocked dW (null: read the CSR)
    const uint32_t* dwoff;
    int dw_global;          // 1: each CTA reads its block from global memory (no shared-memory copy)
    int ntp;                // staged token rows: 1, 2, 4 or 8
    int full_row;           // one token whose whole row fits the staging region: one bulk copy of
                            // it, and the one-token kernels route on their own sums (no exchange)
    RouteConsts rc;         // of Kfull
    double gT;              // bound factor of this kernel's own f32 sums (gamma of their depth, doubled)
    int drop_copy;          // test hook (sc_test_drop_weight_copy): CTA 0 never issues its first weight
                            // stage, so the base-product warps' bounded wait on it runs out
};

// Up to kGroupMax layers reading the same x in one launch: layer i owns the CTAs
// [cta_start[i], cta_start[i+1]) (whole clusters, all layers with the same ksplit).
constexpr int kGroupMax = SC_GROUP_MAX;
struct FusedGroup {
    int n;
    int cta_start[kGroupMax + 1];
    FusedParams p[kGroupMax];
};

// This CTA's layer; its parameters copied to shared memory by one thread (static indices only,
// so the parameter block stays in the constant bank).
__device__ __forceinline__ int fused_group_layer(const FusedGroup& g, int* bid) {
    int gi = 0, start = 0;
#pragma unroll
    for (int i = 1; i < kGroupMax; ++i)
        if (i < g.n && static_cast<int>(blockIdx.x) >= g.cta_start[i]) {
            gi = i;
            start = g.cta_start[i];
        }
    *bid = static_cast<int>(blockIdx.x) - start;
    return gi;
}
__device__ __forceinline__ void fused_copy_params(const FusedGroup& g, int gi, FusedParams& dst) {
#pragma unroll
    for (int i = 0; i < kGroupMax; ++i)
        if (i == gi) dst = g.p[i];
}

// Shared-memory regions after the weight ring, common to both engines.
struct FusedRegions {
    static constexpr int NT = 8;
    static constexpr int kAuxThreads = 128;
    static constexpr int kXsBytes = 32 * 1024;   // staged x: 32768 / (128 * ntp) column blocks
    static constexpr int kPad = 128;             // MMA operand rows past the last staged chunk read here
    // fp8 and integer engines (one token): f16 x in [0, 8 KB), its e4m3 split (512 B per 64-column
    // block) or its base-256 digit columns (384 B per block) in [8 KB, 32 KB) of the same region
    static constexpr int kXb8 = 8 * 1024;
    static constexpr int kMaxKbF8 = (kXsBytes - kXb8) / 512;
    static constexpr int kMaxKbI8 = (kXsBytes - kXb8) / 384;
    static_assert(kMaxKbI8 * 128 <= kXb8, "the f16 slice of the integer engine fits below its digits");
    static constexpr int kXs = 0;
    static constexpr int kDw = kXsBytes + kPad;
    static constexpr int kStats = kDw + static_cast<int>(kDwBlockMax);             // [ranks][8 tokens][3] f64
    static constexpr int kRed = kStats + kMaxFusedCluster * NT * 3 * 8;            // [ks][rows of rank][8] f32
    static constexpr int kBytes = kRed + (128 + kMaxFusedCluster) * NT * 4;
    static constexpr int kBars = 5;                                                // x_ready dw_ready stats red xrow
};

// Scale and flags of the e4m3 split of this CTA's slice of x (one token).
struct F8Split {
    float wmax[4];   // per auxiliary warp: max |x|
    int exp;         // x = 2^exp * sum_c 2^(-4c) X_c
    int nonfinite;   // the slice holds an inf or nan: the fp8 engine writes nan for the tile
};

struct FusedCtx {
    const FusedParams* fp;
    unsigned char* xs;
    const unsigned char* dws;
    double* rstats;
    float* rbuf;
    uint64_t* x_ready;   // 4 arrivals (auxiliary warps): x staged
    uint64_t* dw_ready;  // bulk copy of the dW block
    uint64_t* stats_bar; // cluster sums received
    uint64_t* red_bar;   // split partials of owned rows received
    uint64_t* xrow_bar;  // bulk copy of the whole token (full_row)
    unsigned char* xrow; // the staged whole token (full_row); xs is this CTA's slice of it
    int* s_abort;
    unsigned* s_mask;
    double (*s_red)[FusedRegions::NT][4];
    struct F8Split* split8;  // e4m3 x split (fp8 engine) or null
    unsigned char* xb8;      // e4m3 x columns: [32-column step][2 halves][8 columns][16 B]
    int64_t rt, kb_begin, kb_end;
    int bid;  // CTA index within this layer's part of the grid
    int split, ks, nkb, ntok, cs, rb, nr;
    bool use_blk;   // dW in the blocked layout
    bool blk_copy;  // ... bulk-copied to shared memory (else read in place from global memory)
    bool local;  // route on this CTA's own sums of the staged whole token (one-token kernels)
};

// one_token: the kernel handles one token (its auxiliary path can route locally on a full row).
__device__ __forceinline__ FusedCtx fused_ctx(const FusedParams& fp, int bid, unsigned char* regions, uint64_t* bars,
                                              int* s_abort, unsigned* s_mask, double (*s_red)[FusedRegions::NT][4],
                                              bool one_token) {
    using R = FusedRegions;
    const TCParams& p = fp.t;
    FusedCtx c;
    c.fp = &fp;
    c.xs = regions + R::kXs;
    c.dws = regions + R::kDw;
    c.rstats = reinterpret_cast<double*>(regions + R::kStats);
    c.rbuf = reinterpret_cast<float*>(regions + R::kRed);
    c.x_ready = bars;
    c.dw_ready = bars + 1;
    c.stats_bar = bars + 2;
    c.red_bar = bars + 3;
    c.xrow_bar = bars + 4;
    c.xrow = regions + R::kXs;
    c.local = false;
    c.s_abort = s_abort;
    c.s_mask = s_mask;
    c.s_red = s_red;
    c.ks = p.ksplit;
    c.ntok = p.ntok;
    c.bid = bid;
    c.rt = bid / c.ks;
    c.split = static_cast<int>(bid - c.rt * c.ks);   // = cluster rank
    c.kb_begin = (p.KB * c.split) / c.ks;
    c.kb_end = (p.KB * (c.split + 1)) / c.ks;
    c.nkb = static_cast<int>(c.kb_end - c.kb_begin);
    c.cs = fp.ntp * 16;
    c.rb = (128 * c.split) / c.ks;
    c.nr = (128 * (c.split + 1)) / c.ks - c.rb;
    c.use_blk = fp.dwblk != nullptr && p.nnz > 0;
    c.blk_copy = c.use_blk && !fp.dw_global;
    c.local = one_token && fp.full_row;
    if (c.local) c.xs = c.xrow + (fp.x_col0 + c.kb_begin * 64) * 2;
    c.split8 = nullptr;
    c.xb8 = regions + R::kXs + R::kXb8;
    return c;
}

// One thread: the common mbarriers and the byte counts expected from the cluster (TK: token
// capacity of the kernel, the f32 values pushed per row).
template <int TK>
__device__ __forceinline__ void fused_init_bars(const FusedCtx& c) {
    mbar_init(c.x_ready, 4);
    mbar_init(c.dw_ready, 1);
    mbar_init(c.stats_bar, 1);
    mbar_init(c.red_bar, 1);
    mbar_init(c.xrow_bar, 1);
    fence_mbar_init();
    if (c.ks > 1) {
        if (!c.local) mbar_arrive_expect_tx(c.stats_bar, static_cast<uint32_t>(c.ks * c.ntok * 24));
        mbar_arrive_expect_tx(c.red_bar, static_cast<uint32_t>(c.ks * c.nr * TK * 4));
    }
}

// Producer lane: the CTA's dW block first (the auxiliary warps wait on it; the weights are
// consumed progressively), then the weights through the ring (stages of SKB 4 KB blocks).
// Returns the number of stages issued.
template <int SKB, int S>
__device__ __forceinline__ int fused_produce(const FusedCtx& c, unsigned char* ring, uint64_t* full, uint64_t* empty) {
    const TCParams& p = c.fp->t;
    constexpr int kStage = SKB * 4096;
    const int nst = (c.nkb + SKB - 1) / SKB;
    const uint64_t pol = policy_evict_first();
    const int pre = nst < S ? nst : S;
    int issued = 0;
    if (c.blk_copy) {
        const uint32_t o0 = c.fp->dwoff[c.bid], o1 = c.fp->dwoff[c.bid + 1];
        mbar_arrive_expect_tx(c.dw_ready, o1 - o0);
        bulk_g2s(const_cast<unsigned char*>(c.dws), c.fp->dwblk + o0, o1 - o0, c.dw_ready);
    }
    for (int it = 0; it < pre; ++it, ++issued) {
        const int64_t kb0 = c.kb_begin + static_cast<int64_t>(it) * SKB;
        const int n = static_cast<int>(imin64(SKB, c.kb_end - kb0));
        if (it == 0 && c.bid == 0 && c.fp->drop_copy) continue;  // nothing ever completes this stage
        mbar_arrive_expect_tx(&full[it], static_cast<uint32_t>(n * 4096));
        bulk_g2s_stream(ring + it * kStage, p.wq + (c.rt * p.KB + kb0) * 1024, static_cast<uint32_t>(n * 4096),
                        &full[it], pol);
    }
    for (int it = pre; it < nst; ++it, ++issued) {
        const int slot = it % S;
        const int64_t kb0 = c.kb_begin + static_cast<int64_t>(it) * SKB;
        const int n = static_cast<int>(imin64(SKB, c.kb_end - kb0));
        if (!mbar_wait(&empty[slot], ((it / S) - 1) & 1, p.status)) {
            *c.s_abort = 1;
            break;
        }
        mbar_arrive_expect_tx(&full[slot], static_cast<uint32_t>(n * 4096));
        bulk_g2s_stream(ring + slot * kStage, p.wq + (c.rt * p.KB + kb0) * 1024, static_cast<uint32_t>(n * 4096),
                        &full[slot], pol);
    }
    return issued;
}

__device__ __forceinline__ uint4 load_x8(const void* x, int x_dtype, bool vec, int64_t base) {
    if (vec) return __ldg(reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(x) + base));
    uint16_t h[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) h[e] = x_f16_bits(x, x_dtype, base + e);
    return *reinterpret_cast<const uint4*>(h);
}

// fp8 engine, auxiliary threads after staging one token: split the staged slice of x into 8
// e4m3 columns with x = 2^e * sum_c 2^(-4c) X_c.  e puts the slice's max |x| in [128, 256); each
// column takes the e4m3 rounding of the residual scaled by 16^c and leaves an exact f32 residual,
// so every element of magnitude >= max * 2^-34 is represented exactly (an f16 needs at most 3
// columns once it is an e4m3 normal, and each column lifts a smaller one by 2^4); smaller ones
// keep an error below 2^-34 of the slice maximum.  Columns are written as the MMA's K-major B
// operand: [32-column step][2 halves of 16][8 columns][16 bytes].
__device__ __forceinline__ void fused_split8(const FusedCtx& c, int at) {
    const int wi = at >> 5, lane = at & 31;
    const int nin = c.nkb * 8;
    F8Split& sp = *c.split8;
    float amax = 0.0f;
    bool bad = false;
    for (int ci = at; ci < nin; ci += FusedRegions::kAuxThreads) {
        const uint4 hv = *reinterpret_cast<const uint4*>(c.xs + ci * c.cs);
        const uint32_t w[4] = {hv.x, hv.y, hv.z, hv.w};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const float lo = h2f(lo16(w[q])), hi = h2f(hi16(w[q]));
            bad |= !isfinite(lo) || !isfinite(hi);
            amax = fmaxf(amax, fmaxf(fabsf(lo), fabsf(hi)));
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    bad = __any_sync(0xffffffffu, bad);
    if (lane == 0) {
        sp.wmax[wi] = amax;
        if (bad) sp.nonfinite = 1;
    }
    asm volatile("bar.sync 1, 128;" ::: "memory");
    const float m = fmaxf(fmaxf(sp.wmax[0], sp.wmax[1]), fmaxf(sp.wmax[2], sp.wmax[3]));
    int e = 0;
    if (m > 0.0f) {
        frexpf(m, &e);  // m in [2^(e-1), 2^e)
        e -= 8;         // m * 2^-e in [128, 256)
    }
    if (at == 0) sp.exp = e;
    const float down = ldexpf(1.0f, -e);  // exact power of two (e in [-32, 8] for finite f16 input)
    for (int ci = at; ci < nin; ci += FusedRegions::kAuxThreads) {
        const uint4 hv = *reinterpret_cast<const uint4*>(c.xs + ci * c.cs);
        const uint32_t w[4] = {hv.x, hv.y, hv.z, hv.w};
        float t[8];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            t[2 * q] = h2f(lo16(w[q])) * down;
            t[2 * q + 1] = h2f(hi16(w[q])) * down;
        }
        unsigned char* b = c.xb8 + (ci >> 2) * 256 + ((ci >> 1) & 1) * 128 + (ci & 1) * 8;
#pragma unroll 1
        for (int col = 0; col < 8; ++col) {
            uint32_t part[4];
            bool rest = false;
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                part[q] = cvt_e4m3x2_f32(t[2 * q], t[2 * q + 1]);
                const uint32_t back = cvt_f16x2_e4m3x2(part[q]);
                t[2 * q] = (t[2 * q] - h2f(lo16(back))) * 16.0f;          // exact residual, scaled exactly
                t[2 * q + 1] = (t[2 * q + 1] - h2f(hi16(back))) * 16.0f;
                rest |= t[2 * q] != 0.0f || t[2 * q + 1] != 0.0f;
            }
            *reinterpret_cast<uint2*>(b + col * 16) = make_uint2(part[0] | (part[1] << 16), part[2] | (part[3] << 16));
            if (!rest) {
                for (int z = col + 1; z < 8; ++z) *reinterpret_cast<uint2*>(b + z * 16) = make_uint2(0u, 0u);
                break;
            }
        }
    }
}

// Auxiliary warps (four consecutive warps; thread `at` = 32 * (warp % 4) + lane owns row `at`
// of the tile): stage x, route, publish the mask, and accumulate this row's dW into corr.
// TK: tokens the kernel handles (8; 1 for the one-token engines, whose code is then that much
// shorter on this latency-bound path).
template <int TK>
__device__ __forceinline__ void fused_aux_front(const FusedCtx& c, int at, float (&corr)[TK], float& row_scale) {
    using R = FusedRegions;
    constexpr int NT = TK;
    const FusedParams& fp = *c.fp;
    const TCParams& p = fp.t;
    const int wi = at >> 5, lane = at & 31;
    const int ntok = c.ntok, ks = c.ks;
#pragma unroll
    for (int t = 0; t < NT; ++t) corr[t] = 0.0f;
    // this row's scale: a weight, so it is read before waiting on the previous kernel
    row_scale = c.rt * 128 + at < p.N ? __ldg(p.scale + c.rt * 128 + at) : 0.0f;
    pdl_wait();
    const int64_t slice0 = fp.x_col0 + c.kb_begin * 64;             // first staged column of x
    const int64_t slice1 = fp.x_col0 + imin64(c.kb_end * 64, p.K);  // end of its real columns
    const bool vec = fp.x_dtype == SC_F16 && ((reinterpret_cast<uintptr_t>(fp.x) | (fp.x_stride * 2)) & 15) == 0 &&
                     (fp.x_col0 & 7) == 0;
    const int nin = c.nkb * 8;  // staged 8-column chunks
    float a1[NT], a2[NT], a3[NT];
#pragma unroll
    for (int t = 0; t < NT; ++t) a1[t] = a2[t] = a3[t] = 0.0f;
    bool local = false;
    if constexpr (TK == 1) local = c.local;
    if (local) {
        // the whole token in one bulk copy (its start and length are 16-byte multiples), the
        // slice's padding past the token zeroed, the sums taken from shared memory
        const uint32_t bytes = static_cast<uint32_t>(fp.Kfull * 2);
        if (at == 0) {
            mbar_arrive_expect_tx(c.xrow_bar, bytes);
            bulk_g2s(c.xrow, static_cast<const unsigned char*>(fp.x) + p.tok0 * fp.x_stride * 2, bytes, c.xrow_bar);
        }
        if (!mbar_wait(c.xrow_bar, 0, p.status)) *c.s_abort = 1;
        for (int64_t ci = at; ci < fp.Kfull / 8; ci += R::kAuxThreads)
            sum_x8(*reinterpret_cast<const uint4*>(c.xrow + ci * 16), a1[0], a2[0], a3[0]);
        // the slice's columns past the layer's K (padding blocks) must read as zeros
        asm volatile("bar.sync 1, 128;" ::: "memory");
        const int64_t pad1 = (fp.x_col0 + c.kb_end * 64) * 2;
        for (int64_t o = (fp.x_col0 + p.K) * 2 + static_cast<int64_t>(at) * 16; o < pad1; o += R::kAuxThreads * 16)
            *reinterpret_cast<uint4*>(c.xrow + o) = make_uint4(0u, 0u, 0u, 0u);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(c.x_ready);
    } else {
        // pass 1: stage the slice (ntp token rows; rows >= ntok and columns >= K are zero)
        for (int ci = at; ci < nin; ci += R::kAuxThreads) {
            const int64_t colx = slice0 + static_cast<int64_t>(ci) * 8;
            const bool inb = colx < slice1;
            unsigned char* dst = c.xs + ci * c.cs;
#pragma unroll
            for (int g4 = 0; g4 < NT; g4 += 4) {
                if (g4 < fp.ntp) {
                    uint4 v[4];
#pragma unroll
                    for (int u = 0; u < 4; ++u) {
                        v[u] = make_uint4(0u, 0u, 0u, 0u);
                        if (g4 + u < NT && g4 + u < ntok && inb)
                            v[u] = load_x8(fp.x, fp.x_dtype, vec, (p.tok0 + g4 + u) * fp.x_stride + colx);
                    }
#pragma unroll
                    for (int u = 0; u < 4; ++u) {
                        if (g4 + u < NT) {
                            sum_x8(v[u], a1[g4 + u], a2[g4 + u], a3[g4 + u]);
                            if (g4 + u < fp.ntp) *reinterpret_cast<uint4*>(dst + (g4 + u) * 16) = v[u];
                        }
                    }
                }
            }
        }
        if (c.split8) fused_split8(c, at);
        fence_proxy_async_smem();  // the tensor cores read the staged x through the async proxy
        __syncwarp();
        if (lane == 0) mbar_arrive(c.x_ready);
        // pass 2 (rows shards): this CTA's share of the columns outside the layer's slice
        const int64_t nch = fp.Kfull / 8;
        const int64_t in0 = fp.x_col0 / 8, in1 = (fp.x_col0 + p.K) / 8;
        const int64_t nout = nch - (in1 - in0);
        const int64_t o0 = (nout * c.split) / ks, o1 = (nout * (c.split + 1)) / ks;
        for (int64_t j = o0 + at; j < o1; j += R::kAuxThreads) {
            const int64_t ch = j < in0 ? j : j + (in1 - in0);
#pragma unroll
            for (int g4 = 0; g4 < NT; g4 += 4) {
                if (g4 < ntok) {
                    uint4 v[4];
#pragma unroll
                    for (int u = 0; u < 4; ++u) {
                        v[u] = make_uint4(0u, 0u, 0u, 0u);
                        if (g4 + u < NT && g4 + u < ntok)
                            v[u] = load_x8(fp.x, fp.x_dtype, vec, (p.tok0 + g4 + u) * fp.x_stride + ch * 8);
                    }
#pragma unroll
                    for (int u = 0; u < 4; ++u)
                        if (g4 + u < NT) sum_x8(v[u], a1[g4 + u], a2[g4 + u], a3[g4 + u]);
                }
            }
        }
    }
    // warp sums in f32 (five more levels of the summation tree, inside gT), then f64
#pragma unroll
    for (int t = 0; t < NT; ++t) {
        if (t < ntok) {
            float d1 = a1[t], d2 = a2[t], d3 = a3[t];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                d1 += __shfl_down_sync(0xffffffffu, d1, o);
                d2 += __shfl_down_sync(0xffffffffu, d2, o);
                d3 += __shfl_down_sync(0xffffffffu, d3, o);
            }
            if (lane == 0) {
                c.s_red[0][t][wi] = d1;
                c.s_red[1][t][wi] = d2;
                c.s_red[2][t][wi] = d3;
            }
        }
    }
    asm volatile("bar.sync 1, 128;" ::: "memory");
    if (local) {
        if (at == 0) {
            const double S1 = ((c.s_red[0][0][0] + c.s_red[0][0][1]) + c.s_red[0][0][2]) + c.s_red[0][0][3];
            const double S2 = ((c.s_red[1][0][0] + c.s_red[1][0][1]) + c.s_red[1][0][2]) + c.s_red[1][0][3];
            const double SA = ((c.s_red[2][0][0] + c.s_red[2][0][1]) + c.s_red[2][0][2]) + c.s_red[2][0][3];
            const void* xrow = static_cast<const unsigned char*>(fp.x) + p.tok0 * fp.x_stride * 2;
            const bool r = p.route_all ? true
                                       : route_token(S1, S2, SA, fp.Kfull, fp.rc, fp.t4, fp.t8, xrow, fp.x_dtype,
                                                     nullptr, fp.gT * SA, fp.gT * S2);
            *c.s_mask = r ? 1u : 0u;
        }
    } else if (ks > 1) {
        cluster_wait();  // every mbarrier of the cluster is initialised
        if (wi == 0 && lane < ks) {
            // lane r sends this CTA's sums to rank r, into slot [split]
            const uint32_t dst = dsmem_addr(c.rstats + c.split * NT * 3, static_cast<uint32_t>(lane));
            const uint32_t bar = dsmem_addr(c.stats_bar, static_cast<uint32_t>(lane));
            for (int t = 0; t < ntok; ++t)
                for (int q = 0; q < 3; ++q)
                    st_async_f64(dst + (t * 3 + q) * 8,
                                 ((c.s_red[q][t][0] + c.s_red[q][t][1]) + c.s_red[q][t][2]) + c.s_red[q][t][3], bar);
        }
    } else if (at == 0) {
        for (int t = 0; t < ntok; ++t)
            for (int q = 0; q < 3; ++q)
                c.rstats[t * 3 + q] = ((c.s_red[q][t][0] + c.s_red[q][t][1]) + c.s_red[q][t][2]) + c.s_red[q][t][3];
    }
    if (at == 0 && !local) {
        const bool ok = ks == 1 || mbar_wait(c.stats_bar, 0, p.status);
        unsigned m = 0u;
        for (int t = 0; t < ntok && ok; ++t) {
            double S1 = 0.0, S2 = 0.0, SA = 0.0;
            for (int r = 0; r < ks; ++r) {
                S1 += c.rstats[(r * NT + t) * 3 + 0];
                S2 += c.rstats[(r * NT + t) * 3 + 1];
                SA += c.rstats[(r * NT + t) * 3 + 2];
            }
            const void* xrow = static_cast<const unsigned char*>(fp.x) + (p.tok0 + t) * fp.x_stride * 2;
            const bool r = p.route_all ? true
                                       : route_token(S1, S2, SA, fp.Kfull, fp.rc, fp.t4, fp.t8, xrow, fp.x_dtype, nullptr,
                                                     fp.gT * SA, fp.gT * S2);
            if (r) m |= 1u << t;
        }
        if (!ok) *c.s_abort = 1;
        *c.s_mask = m;
    }
    asm volatile("bar.sync 1, 128;" ::: "memory");
    const unsigned mask = *c.s_mask;
    if (c.bid == 0 && wi == 0) {
        for (int t = lane; t < ntok; t += 32) {
            const int r = (mask >> t) & 1u;
            if (fp.mask_out) fp.mask_out[p.tok0 + t] = static_cast<uint8_t>(r);
            if (fp.ridx_out && r) fp.ridx_out[__popc(mask & ((1u << t) - 1u))] = static_cast<int32_t>(p.tok0 + t);
        }
        if (lane == 0 && fp.nrouted_out) *fp.nrouted_out = __popc(mask);
    }
    // dW of this thread's row for the routed tokens, x from the staged copy, column order
    const int64_t row = c.rt * 128 + at;
    if (mask == 0u || row >= p.N || p.nnz == 0) return;
    auto add_entry = [&](int64_t cl, int8_t q) {
        const float v = __fmul_rn(static_cast<float>(q), p.ds);
        const unsigned char* xp = c.xs + ((cl >> 3) * fp.ntp) * 16 + (cl & 7) * 2;
#pragma unroll
        for (int t = 0; t < NT; ++t)
            if ((mask >> t) & 1u)
                corr[t] = __fadd_rn(corr[t], __fmul_rn(h2f(*reinterpret_cast<const uint16_t*>(xp + t * 16)), v));
    };
    if (c.blk_copy) {
        if (!mbar_wait(c.dw_ready, 0, p.status)) {
            *c.s_abort = 1;
            return;
        }
        const uint16_t* roff = reinterpret_cast<const uint16_t*>(c.dws);
        const int n = roff[128];
        const uint16_t* bcol = reinterpret_cast<const uint16_t*>(c.dws + 272);
        const int8_t* bval = reinterpret_cast<const int8_t*>(c.dws + 272 + ((n * 2 + 15) / 16) * 16);
        for (int e = roff[at]; e < roff[at + 1]; ++e) add_entry(bcol[e], bval[e]);
    } else if (c.use_blk) {
        // the same block read in place (same order), pulled into L2 in one bulk prefetch now that
        // a token is routed; B entries loaded before they are added
        constexpr int B = 8;
        const uint32_t o0 = fp.dwoff[c.bid];
        const unsigned char* blk = fp.dwblk + o0;
        if (at == 0) bulk_prefetch_l2(blk, fp.dwoff[c.bid + 1] - o0);
        const uint16_t* roff = reinterpret_cast<const uint16_t*>(blk);
        const int n = roff[128];
        const uint16_t* bcol = reinterpret_cast<const uint16_t*>(blk + 272);
        const int8_t* bval = reinterpret_cast<const int8_t*>(blk + 272 + ((n * 2 + 15) / 16) * 16);
        const int e1 = roff[at + 1];
        for (int e = roff[at]; e < e1; e += B) {
            const int cnt = e1 - e < B ? e1 - e : B;
            int cc[B], vv[B];
#pragma unroll
            for (int u = 0; u < B; ++u) {
                cc[u] = u < cnt ? static_cast<int>(__ldg(bcol + e + u)) : 0;
                vv[u] = u < cnt ? static_cast<int>(__ldg(bval + e + u)) : 0;
            }
#pragma unroll
            for (int u = 0; u < B; ++u)
                if (u < cnt) add_entry(cc[u], static_cast<int8_t>(vv[u]));
        }
    } else {
        const int64_t lo = p.rowptr[row], hi = p.rowptr[row + 1];
        const int64_t e0 = (ks == 1) ? lo : lower_bound_u16(p.col, lo, hi, c.kb_begin * 64);
        const int64_t e1 = (ks == 1) ? hi : lower_bound_u16(p.col, e0, hi, c.kb_end * 64);
        for (int64_t e = e0; e < e1; e += 8) {
            const int cnt = static_cast<int>(imin64(8, e1 - e));
            int64_t cc[8];
            int8_t vv[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                cc[u] = u < cnt ? static_cast<int64_t>(p.col[e + u]) - c.kb_begin * 64 : 0;
                vv[u] = u < cnt ? p.val[e + u] : 0;
            }
#pragma unroll
            for (int u = 0; u < 8; ++u)
                if (u < cnt) add_entry(cc[u], vv[u]);
        }
    }
}

// Auxiliary thread `at` with this split's row contribution v: with one split, write y; else
// push the row to the cluster CTA that owns it and, for owned rows, add the splits in rank
// order and write y.
template <int TK>
__device__ __forceinline__ void fused_aux_finish(const FusedCtx& c, int at, const float (&v)[TK]) {
    constexpr int NT = TK;
    const TCParams& p = c.fp->t;
    const int ks = c.ks;
    pdl_wait();
    auto store_row = [&](int64_t r, const float* w) {
        for (int t = 0; t < c.ntok; ++t) {
            const int64_t oi = (p.tok0 + t) * p.N + r;
            if (p.partial_out) reinterpret_cast<float*>(p.y)[oi] = w[t];
            else store_output(p.y, p.y_dtype, oi, w[t], p.bias, r);
        }
    };
    const int64_t row = c.rt * 128 + at;
    if (ks == 1) {
        if (!*c.s_abort && row < p.N) store_row(row, v);
        return;
    }
    {
        if (c.local) cluster_wait();  // every mbarrier of the cluster is initialised
        // rank o owns rows [128 o / ks, 128 (o+1) / ks)
        const int o = (at * ks + ks - 1) / 128;
        const int orb = (128 * o) / ks, onr = (128 * (o + 1)) / ks - orb;
        const uint32_t dst = dsmem_addr(c.rbuf + (c.split * onr + (at - orb)) * NT, static_cast<uint32_t>(o));
        const uint32_t bar = dsmem_addr(c.red_bar, static_cast<uint32_t>(o));
        if constexpr (NT == 1) {
            st_async_f32(dst, v[0], bar);
        } else {
            static_assert(NT == 8, "rows are pushed as one f32 or two float4");
            st_async_v4_f32(dst, v[0], v[1], v[2], v[3], bar);
            st_async_v4_f32(dst + 16, v[4], v[5], v[6], v[7], bar);
        }
    }
    if (at < c.nr) {
        const bool ok = mbar_wait(c.red_bar, 0, p.status);
        const int64_t r = c.rt * 128 + c.rb + at;
        if (ok && !*c.s_abort && r < p.N) {
            float w[NT];
#pragma unroll
            for (int t = 0; t < NT; ++t) w[t] = 0.0f;
            for (int sp = 0; sp < ks; ++sp) {
#pragma unroll
                for (int t = 0; t < NT; ++t) w[t] = __fadd_rn(w[t], c.rbuf[(sp * c.nr + at) * NT + t]);
            }
            store_row(r, w);
        }
    }
}

// ---- engine 1: tcgen05 (weights dequantised into tensor memory)
// The fp8 variant (F8, one token): weights (q - 8, exact in e4m3) go to tensor memory as e4m3 and
// x as an exact split into 8 e4m3 columns with power-of-two scales (fused_split8), so each MMA
// (kind::f8f6f4, K = 32) covers twice the columns of the f16 one and the A tiles are half the bytes.
template <bool F8>
struct FusedTcCfg {
    static constexpr int kDqWarps = 8;               // two per TMEM sub-partition, one 16-row tile each
    static constexpr int kProducerWarp = 8;
    static constexpr int kMmaWarp = 9;
    static constexpr int kAuxWarp0 = 10;
    static constexpr int kThreads = 14 * 32;
    // One ring stage is one hand-off between the dequantising warps and the MMA thread: every
    // hand-off costs a few hundred cycles of latency, so it carries 3 blocks.
    static constexpr int SKB = 3;
    static constexpr int S = 4;
    static constexpr int kStageBytes = SKB * 4096;
    static constexpr int kColsPerBlock = F8 ? 16 : 32;        // TMEM columns of one 64-column block of A
    static constexpr int kAB = F8 ? 4 : 2;                    // TMEM A buffers, one stage each
    static constexpr uint32_t kTmemCols = 256;                // D in [0, 16), A buffers from column 32
    static constexpr int kRegions = S * kStageBytes;
    static constexpr int kBarOff = kRegions + FusedRegions::kBytes;
    static constexpr int kNumBars = 2 * S + 2 * kAB + 1 + FusedRegions::kBars;
    static constexpr int kTmemSlotOff = kBarOff + kNumBars * 8;
    static constexpr int kTotal = kTmemSlotOff + 16;
    static_assert(32 + kAB * SKB * kColsPerBlock <= static_cast<int>(kTmemCols), "tensor memory");
    static_assert(2 * (kTotal + 2048 + 1024) <= 228 * 1024, "two CTAs per SM (with static and reserved smem)");
};

template <bool F8>
__global__ void __launch_bounds__(FusedTcCfg<F8>::kThreads, 2) k_ctarq_fused_tc(FusedGroup g) {
    using C = FusedTcCfg<F8>;
    constexpr int SKB = C::SKB, S = C::S, AB = C::kAB, NT = FusedRegions::NT, CPB = C::kColsPerBlock, TK = NT;
    pdl_launch_dependents();
    __shared__ FusedParams fp;
    int bid;
    const int gi = fused_group_layer(g, &bid);
    if (threadIdx.x == 0) fused_copy_params(g, gi, fp);
    __syncthreads();
    const TCParams& p = fp.t;
    extern __shared__ __align__(1024) unsigned char smem[];
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::kBarOff);
    uint64_t* empty = full + S;
    uint64_t* a_full = empty + S;
    uint64_t* a_empty = a_full + AB;
    uint64_t* done = a_empty + AB;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::kTmemSlotOff);
    __shared__ int s_abort;
    __shared__ unsigned s_mask;
    __shared__ double s_red[3][NT][4];
    __shared__ F8Split s_split;
    FusedCtx c = fused_ctx(fp, bid, smem + C::kRegions, done + 1, &s_abort, &s_mask, s_red, false);
    if (F8) c.split8 = &s_split;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

    if (tid == 0) {
        for (int i = 0; i < S; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], C::kDqWarps);
        }
        for (int i = 0; i < AB; ++i) {
            mbar_init(&a_full[i], C::kDqWarps);
            mbar_init(&a_empty[i], 1);
        }
        mbar_init(done, 1);
        fused_init_bars<TK>(c);
        s_abort = 0;
        s_mask = 0u;
        s_split.nonfinite = 0;
    }
    if (warp == C::kMmaWarp) {
        tmem_alloc(tmem_slot, C::kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    if (c.ks > 1) cluster_arrive_relaxed();  // this CTA's mbarriers are initialised (released above)

    int issued = 0;
    float corr[NT];
    float row_scale = 0.0f;
    const int at = 32 * (warp & 3) + lane;  // auxiliary threads: tile row, in this warp's TMEM lanes
    if (warp == C::kProducerWarp) {
        if (lane == 0) issued = fused_produce<SKB, S>(c, smem, full, empty);
    } else if (warp == C::kMmaWarp) {
        // the whole warp runs the loop (uniform); one elected lane issues
        constexpr uint32_t idesc = idesc_f16_f32(128, 16);  // e4m3 operands share the type code 0 of f16
        bool ok = __all_sync(0xffffffffu, mbar_wait(c.x_ready, 0, p.status));
        const int nst = (c.nkb + SKB - 1) / SKB;
        // B descriptors: f16 x staged as [chunk][ntp][16 B] (one K = 16 step = 2 chunks); e4m3 x as
        // [32-column step][2 halves][8 columns][16 B] (one K = 32 step = 256 B); rows 8..15 of the
        // N = 16 operand alias rows 0..7 (SBO = 0) and are not read back
        const uint64_t bd0 = F8 ? desc_kmajor(c.xb8, 128, 0) : desc_kmajor(c.xs, c.cs, 0);
        const uint64_t step = F8 ? 16u : static_cast<uint64_t>(fp.ntp) * 2u;  // per K step, in 16-byte units
        constexpr int kSteps = F8 ? 2 : 4;                                    // K steps per 64-column block
        for (int u = 0; u < nst && ok; ++u) {
            const int b = u % AB;
            ok = __all_sync(0xffffffffu, mbar_wait(&a_full[b], (u / AB) & 1, p.status));
            if (!ok) break;
            tc_fence_after();
            const int n = c.nkb - u * SKB < SKB ? c.nkb - u * SKB : SKB;
            const uint32_t a0 = tmem + 32 + b * SKB * CPB;
            const uint64_t bu = bd0 + static_cast<uint64_t>(u * SKB * kSteps) * step;
            if (elect_one()) {
                for (int k = 0; k < n; ++k) {
#pragma unroll
                    for (int i = 0; i < kSteps; ++i) {
                        const uint64_t bdesc = bu + static_cast<uint64_t>(k * kSteps + i) * step;
                        if (F8) tc_mma_ts_f8(tmem, a0 + k * CPB + i * 8, bdesc, idesc, (u | k | i) ? 1u : 0u);
                        else tc_mma_ts(tmem, a0 + k * CPB + i * 8, bdesc, idesc, (u | k | i) ? 1u : 0u);
                    }
                }
                tc_commit(&a_empty[b]);
            }
            __syncwarp();
        }
        if (!ok && lane == 0) s_abort = 1;
        if (elect_one()) tc_commit(done);  // also after an abort, so that the TMEM can be released
        __syncwarp();
    } else if (warp < C::kDqWarps) {
        const int sp = warp & 3, q = warp >> 2;
        const int tile = 2 * sp + q;
        const uint32_t lane_addr = static_cast<uint32_t>(32 * sp + 16 * q) << 16;
        const int nst = (c.nkb + SKB - 1) / SKB;
        for (int u = 0; u < nst; ++u) {
            const int slot = u % S, b = u % AB;
            if (!mbar_wait(&full[slot], (u / S) & 1, p.status)) {
                s_abort = 1;
                break;
            }
            // the stage goes to registers and its ring slot back to the producer at once, so
            // the ring keeps every stage in flight while this unit waits for a TMEM buffer
            const int n = c.nkb - u * SKB < SKB ? c.nkb - u * SKB : SKB;
            uint4 wv[SKB];
#pragma unroll
            for (int k = 0; k < SKB; ++k)
                if (k < n)
                    wv[k] = *reinterpret_cast<const uint4*>(smem + slot * C::kStageBytes + k * 4096 + tile * 512 + lane * 16);
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[slot]);
            if (u >= AB && !mbar_wait(&a_empty[b], ((u / AB) - 1) & 1, p.status)) {
                s_abort = 1;
                break;
            }
            tc_fence_after();
#pragma unroll
            for (int k = 0; k < SKB; ++k) {
                if (k < n) {
                    const uint32_t words[4] = {wv[k].x, wv[k].y, wv[k].z, wv[k].w};
                    const uint32_t col = tmem + lane_addr + 32 + (b * SKB + k) * CPB;
                    if (F8) {
                        // K = 32 step t covers the 16-column steps 2t, 2t+1: TMEM column 4 * (s % 2) + c
#pragma unroll
                        for (int t = 0; t < 2; ++t) {
                            uint32_t g0, g80, g1, g81;
                            dequant_word_e4m3(words[2 * t], g0, g80);
                            dequant_word_e4m3(words[2 * t + 1], g1, g81);
                            tc_st_16x128b_x2(col + t * 8, g0, g80, g1, g81);
                        }
                    } else {
#pragma unroll
                        for (int st = 0; st < 4; ++st) {
                            uint32_t h[4];
                            dequant_word(words[st], h);
                            tc_st_16x256b(col + st * 8, h[0], h[2], h[1], h[3]);
                        }
                    }
                }
            }
            tc_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&a_full[b]);
        }
    } else {
        fused_aux_front<TK>(c, at, corr, row_scale);
    }
    __syncwarp();
    if (warp < C::kAuxWarp0 && c.ks > 1) cluster_wait();
    // auxiliary threads: this split's contribution to row `at` (acc * row scale + dW; 0 past N)
    float v[NT];
    if (warp >= C::kAuxWarp0) {
        const int64_t row = c.rt * 128 + at;
        const float sc = row_scale;
        uint32_t d[8];
        const bool ok = mbar_wait(done, 0, p.status);
        tc_fence_after();
        tc_ld8(tmem + (static_cast<uint32_t>(32 * (warp & 3)) << 16), d);
        tc_wait_ld();
        if (!ok) s_abort = 1;
        if (F8) {
            // acc = 2^e * sum_c 2^(-4c) D_c (token 0), summed in f64 and rounded once
            double a = 0.0;
#pragma unroll
            for (int col = 0; col < 8; ++col) a += ldexp(static_cast<double>(__uint_as_float(d[col])), s_split.exp - 4 * col);
            const float acc = s_split.nonfinite ? __int_as_float(0x7fc00000) : static_cast<float>(a);
            v[0] = row < p.N ? __fadd_rn(__fmul_rn(acc, sc), corr[0]) : 0.0f;
#pragma unroll
            for (int t = 1; t < NT; ++t) v[t] = 0.0f;
        } else {
#pragma unroll
            for (int t = 0; t < NT; ++t)
                v[t] = row < p.N ? __fadd_rn(__fmul_rn(__uint_as_float(d[t]), sc), corr[t]) : 0.0f;
        }
    }
    __syncwarp();  // single-lane roles rejoin their warp before the warp-wide TMEM release below
    tc_fence_before();
    __syncthreads();
    if (warp == C::kMmaWarp) {
        if (s_abort) mbar_wait(done, 0, nullptr, kDrainNs);
        tc_fence_after();
        tmem_dealloc(tmem, C::kTmemCols);
    }
    if (s_abort && warp == C::kProducerWarp && lane == 0) {
        for (int it = issued > S ? issued - S : 0; it < issued; ++it)
            mbar_wait(&full[it % S], (it / S) & 1, nullptr, kDrainNs);
        if (c.blk_copy) mbar_wait(c.dw_ready, 0, nullptr, kDrainNs);
    }
    if (warp >= C::kAuxWarp0) fused_aux_finish<TK>(c, at, v);
}

// ---- engine 2: mma.sync on the same frame
#ifndef SC_FUSED_MMA_SKB
#define SC_FUSED_MMA_SKB 4  // 4 KB blocks per ring stage of the mma.sync engines
#endif
#ifndef SC_FUSED_MMA_STAGES
#define SC_FUSED_MMA_STAGES 3
#endif
struct FusedMmaCfg {
    static constexpr int kMmaWarps = 8;
    static constexpr int kProducerWarp = 8;
    static constexpr int kAuxWarp0 = 9;
    static constexpr int kThreads = 13 * 32;
    static constexpr int SKB = SC_FUSED_MMA_SKB;
    static constexpr int S = SC_FUSED_MMA_STAGES;
    static constexpr int kStageBytes = SKB * 4096;
    static constexpr int kLd = FusedRegions::NT + 1;
    static constexpr int kAccOff = S * kStageBytes;
    static constexpr int kRegions = kAccOff + 128 * kLd * 4;
    static constexpr int kBarOff = kRegions + FusedRegions::kBytes;
    static constexpr int kTotal = kBarOff + (2 * S + FusedRegions::kBars) * 8;
    static_assert(2 * (kTotal + 2048 + 1024) <= 228 * 1024, "two CTAs per SM (with static and reserved smem)");
};

// I8 (one token): the integer variant.  The weights become s8 bytes 16 (q - 8) (dequant_word_s8,
// 3 instructions a word instead of 9) and x becomes six signed base-256 digit columns of the
// integer x * 2^24 (f16_digits), so m16n8k32 s8 MMAs (two per 64-column block instead of four
// f16 ones) accumulate the products exactly in s32; the row is recombined in f64 and rounded once
// to f32.  A CTA whose slice of x holds an inf or nan runs the f16 loop instead, so the
// non-finite results are those of the f16 engine.
template <bool I8>
__global__ void __launch_bounds__(FusedMmaCfg::kThreads, 2) k_ctarq_fused_mma(FusedGroup g) {
    using C = FusedMmaCfg;
    constexpr int SKB = C::SKB, S = C::S, NT = FusedRegions::NT, TK = I8 ? 1 : NT;
    pdl_launch_dependents();
    __shared__ FusedParams fp;
    int bid;
    const int gi = fused_group_layer(g, &bid);
    if (threadIdx.x == 0) fused_copy_params(g, gi, fp);
    __syncthreads();
    const TCParams& p = fp.t;
    extern __shared__ __align__(1024) unsigned char smem[];
    float* accbuf = reinterpret_cast<float*>(smem + C::kAccOff);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::kBarOff);
    uint64_t* empty = full + S;
    __shared__ int s_abort;
    __shared__ int s_f16;  // this CTA accumulates in f32 (always without I8; with I8 for a non-finite slice)
    __shared__ unsigned s_mask;
    __shared__ double s_red[3][NT][4];
    const FusedCtx c = fused_ctx(fp, bid, smem + C::kRegions, empty + S, &s_abort, &s_mask, s_red, TK == 1);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int nst = (c.nkb + SKB - 1) / SKB;

    if (tid == 0) {
        for (int i = 0; i < S; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], C::kMmaWarps);
        }
        fused_init_bars<TK>(c);
        s_abort = 0;
        s_f16 = I8 ? 0 : 1;
        s_mask = 0u;
    }
    for (int i = tid; i < 128 * C::kLd; i += C::kThreads) accbuf[i] = 0.0f;
    __syncthreads();
    if (c.ks > 1) cluster_arrive_relaxed();

    int issued = 0;
    float corr[TK];
    float row_scale = 0.0f;
    const int at = 32 * (warp & 3) + lane;
    if (warp == C::kProducerWarp) {
        if (lane == 0) issued = fused_produce<SKB, S>(c, smem, full, empty);
    } else if (warp < C::kMmaWarps) {
        const int g = lane >> 2, cq = lane & 3;
        const int r0 = warp * 16 + g;
        if (!mbar_wait(c.x_ready, 0, p.status)) s_abort = 1;
        if constexpr (I8) {
            // digit columns of the slice: block kb, lane (g, c) with g < 6 holds at byte
            // kb * 384 + (4 g + c) * 16 the four B words {b0, b1} x 2 MMAs of digit g; word s of a
            // lane packs the digits of columns 16 s + 4c + {0, 2, 1, 3} (the order of the weight
            // bytes of dequant_word_s8)
            bool bad = false;
            for (int q = tid; q < c.nkb * 16; q += 32 * C::kMmaWarps) {
                const int kb = q >> 4, sg = (q >> 2) & 3, cc = q & 3;
                const uint2 u = *reinterpret_cast<const uint2*>(c.xs + (kb * 8 + 2 * sg + (cc >> 1)) * 16 + (cc & 1) * 8);
                const uint32_t u0 = u.x, u1 = u.y;  // columns 4c, 4c+1 and 4c+2, 4c+3 of the step
                uint32_t lo[4], hi[4];
                f16_digits(u0 & 0xFFFFu, lo[0], hi[0], bad);
                f16_digits(u1 & 0xFFFFu, lo[1], hi[1], bad);
                f16_digits(u0 >> 16, lo[2], hi[2], bad);
                f16_digits(u1 >> 16, lo[3], hi[3], bad);
                // byte transpose: word of digit d = byte d of the four elements
                const uint32_t t0 = __byte_perm(lo[0], lo[1], 0x5140), t1 = __byte_perm(lo[0], lo[1], 0x7362);
                const uint32_t t2 = __byte_perm(lo[2], lo[3], 0x5140), t3 = __byte_perm(lo[2], lo[3], 0x7362);
                const uint32_t h0 = __byte_perm(hi[0], hi[1], 0x5140), h1 = __byte_perm(hi[2], hi[3], 0x5140);
                uint32_t* dst = reinterpret_cast<uint32_t*>(c.xb8 + kb * 384 + cc * 16 + sg * 4);
                dst[0] = __byte_perm(t0, t2, 0x5410);
                dst[16] = __byte_perm(t0, t2, 0x7632);
                dst[32] = __byte_perm(t1, t3, 0x5410);
                dst[48] = __byte_perm(t1, t3, 0x7632);
                dst[64] = __byte_perm(h0, h1, 0x5410);
                dst[80] = __byte_perm(h0, h1, 0x7632);
            }
            if (__any_sync(0xffffffffu, bad) && lane == 0) s_f16 = 1;
            asm volatile("bar.sync 2, 256;" ::: "memory");  // the eight MMA warps
        }
        if (!I8 || s_f16) {
            float acc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
            const bool has_tok = g < c.ntok;
            const int xoff = (cq >> 1) * c.cs + g * 16 + (cq & 1) * 8;
            for (int it = 0; it < nst && !s_abort; ++it) {
                const int slot = it % S;
                if (!mbar_wait(&full[slot], (it / S) & 1, p.status)) {
                    s_abort = 1;
                    break;
                }
                const int n = static_cast<int>(imin64(SKB, c.kb_end - (c.kb_begin + static_cast<int64_t>(it) * SKB)));
                const unsigned char* st = smem + slot * C::kStageBytes;
                const unsigned char* xk0 = c.xs + (it * SKB) * 8 * c.cs + xoff;
#pragma unroll
                for (int j = 0; j < SKB; ++j) {
                    if (j < n) {
                        const uint4 wv = *reinterpret_cast<const uint4*>(st + j * 4096 + warp * 512 + lane * 16);
                        const uint32_t words[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
                        for (int s = 0; s < 4; ++s) {
                            uint2 b = make_uint2(0u, 0u);
                            if (has_tok) b = *reinterpret_cast<const uint2*>(xk0 + j * 8 * c.cs + 2 * s * c.cs);
                            uint32_t a[4];
                            dequant_word(words[s], a);
                            mma_16816(acc[s & 1], a, b.x, b.y);
                        }
                    }
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&empty[slot]);
            }
            accbuf[r0 * C::kLd + 2 * cq] = acc[0][0] + acc[1][0];
            accbuf[r0 * C::kLd + 2 * cq + 1] = acc[0][1] + acc[1][1];
            accbuf[(r0 + 8) * C::kLd + 2 * cq] = acc[0][2] + acc[1][2];
            accbuf[(r0 + 8) * C::kLd + 2 * cq + 1] = acc[0][3] + acc[1][3];
        } else {
            int acc[2][4] = {{0, 0, 0, 0}, {0, 0, 0, 0}};
            for (int it = 0; it < nst && !s_abort; ++it) {
                const int slot = it % S;
                if (!mbar_wait(&full[slot], (it / S) & 1, p.status)) {
                    s_abort = 1;
                    break;
                }
                const int n = static_cast<int>(imin64(SKB, c.kb_end - (c.kb_begin + static_cast<int64_t>(it) * SKB)));
                const unsigned char* st = smem + slot * C::kStageBytes;
                const unsigned char* dg = c.xb8 + (it * SKB) * 384 + lane * 16;
#pragma unroll
                for (int j = 0; j < SKB; ++j) {
                    if (j < n) {
                        const uint4 wv = *reinterpret_cast<const uint4*>(st + j * 4096 + warp * 512 + lane * 16);
                        uint4 dv = make_uint4(0u, 0u, 0u, 0u);  // digit columns 6 and 7 are zero
                        if (lane < 24) dv = *reinterpret_cast<const uint4*>(dg + j * 384);
                        uint32_t a[4];
                        dequant_word_s8(wv.x, a[0], a[1]);
                        dequant_word_s8(wv.y, a[2], a[3]);
                        mma_16832_s8(acc[0], a, dv.x, dv.y);
                        dequant_word_s8(wv.z, a[0], a[1]);
                        dequant_word_s8(wv.w, a[2], a[3]);
                        mma_16832_s8(acc[1], a, dv.z, dv.w);
                    }
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&empty[slot]);
            }
            // row r0 (and r0 + 8), digit columns 2c and 2c + 1 (6 and 7 are zero)
            int* ai = reinterpret_cast<int*>(accbuf);
            if (cq < 3) {
                ai[r0 * C::kLd + 2 * cq] = acc[0][0] + acc[1][0];
                ai[r0 * C::kLd + 2 * cq + 1] = acc[0][1] + acc[1][1];
                ai[(r0 + 8) * C::kLd + 2 * cq] = acc[0][2] + acc[1][2];
                ai[(r0 + 8) * C::kLd + 2 * cq + 1] = acc[0][3] + acc[1][3];
            }
        }
    } else {
        fused_aux_front<TK>(c, at, corr, row_scale);
    }
    __syncwarp();
    if (warp < C::kAuxWarp0 && c.ks > 1) cluster_wait();
    __syncthreads();
    if (s_abort && warp == C::kProducerWarp && lane == 0) {
        for (int it = issued > S ? issued - S : 0; it < issued; ++it)
            mbar_wait(&full[it % S], (it / S) & 1, nullptr, kDrainNs);
        if (c.blk_copy) mbar_wait(c.dw_ready, 0, nullptr, kDrainNs);
    }
    if (warp < C::kAuxWarp0) return;
    const int64_t row = c.rt * 128 + at;
    const float sc = row_scale;
    float v[TK];
    if (I8 && !s_f16) {
        // sum_k 16 (q_k - 8) X_k = sum_d 256^d S_d with X = x * 2^24: recombined in f64 (exact while
        // below 2^53, one rounding beyond), scaled by 2^-28 exactly, rounded once to f32
        const int* ai = reinterpret_cast<const int*>(accbuf) + at * C::kLd;
        double sum = static_cast<double>(ai[5]);
#pragma unroll
        for (int d = 4; d >= 0; --d) sum = sum * 256.0 + static_cast<double>(ai[d]);
        const float a0 = static_cast<float>(sum * 0x1p-28);
        v[0] = row < p.N ? __fadd_rn(__fmul_rn(a0, sc), corr[0]) : 0.0f;
    } else {
#pragma unroll
        for (int t = 0; t < TK; ++t)
            v[t] = row < p.N ? __fadd_rn(__fmul_rn(accbuf[at * C::kLd + t], sc), corr[t]) : 0.0f;
    }
    fused_aux_finish<TK>(c, at, v);
}

// ---------------------------------------------------------------- launchers

template <typename Kern>
static cudaError_t set_smem_once(Kern kernel, int bytes, std::atomic<uint64_t>& flags) {
    int dev = 0;
    cudaGetDevice(&dev);
    const uint64_t bit = 1ull << (dev & 63);
    if (flags.load() & bit) return cudaSuccess;
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e == cudaSuccess) flags.fetch_or(bit);
    return e;
}

cudaError_t launch_decode_tc(const DecodeArgs& a, cudaStream_t s) {
    const Layer& L = *a.L;
    TCParams p;
    p.wq = L.wq;
    p.scale = L.scale;
    p.rowptr = L.rowptr;
    p.col = L.col;
    p.val = L.val;
    p.ds = L.ds;
    p.nnz = L.nnz;
    p.xk = a.xk;
    p.Mp = a.Mp;
    p.tok0 = a.tok0;
    p.ntok = static_cast<int>(a.ntok);
    p.mask = a.mask;
    p.route_all = a.route_all;
    p.N = L.N;
    p.K = L.K;
    p.KB = L.KB;
    p.y = a.y;
    p.y_dtype = a.y_dtype;
    p.bias = a.bias;
    p.partial_out = a.partial_out;
    p.ws_partial = a.ws_partial;
    p.ws_rtcount = a.ws_rtcount;
    p.ksplit = a.ksplit;
    p.status = L.status;
    const dim3 grid(static_cast<unsigned>((L.Np / 128) * p.ksplit));
    if (a.ntok <= 8) {
        static std::atomic<uint64_t> f{0};
        cudaError_t e = set_smem_once(k_ctarq_mma, MmaCfg::kTotal, f);
        if (e != cudaSuccess) return e;
        return launch_pdl(k_ctarq_mma, grid, dim3(MmaCfg::kThreads), MmaCfg::kTotal, s, p);
    }
    return cudaErrorInvalidValue;
}

// ---------------------------------------------------------------- exact (reference-order) kernel

constexpr int kExactTok = 2;  // tokens per pass over the weights

struct ExactParams {
    const uint32_t* wq;
    const float* scale;
    const uint32_t* rowptr;
    const uint16_t* col;
    const int8_t* val;
    float ds;
    int64_t nnz;
    const uint16_t* xk;
    int64_t Mp;
    int64_t tok0;
    int ntok;
    const uint8_t* mask;
    int route_all;
    int bypass;
    int64_t N, K, KB;
    void* y;
    int y_dtype;
    const float* bias;
    int partial_out;
};

__device__ __forceinline__ uint16_t half_sel(uint32_t h2, int e) { return e ? hi16(h2) : lo16(h2); }

// q-8 (f16 bits) of element e (0..7) of the reference word `grp` for row g (r = 0) or g+8
// (r = 1), from the dequantised words of the four lanes c = 0..3 of the kstep holding it.
__device__ __forceinline__ uint16_t wq_elem(const uint32_t (&hq)[4][4], int half, int e, int r) {
    const int c = 2 * half + (e >> 2);
    const int j4 = e & 3;
    return half_sel(hq[c][(j4 < 2 ? 0 : 2) + r], j4 & 1);
}

__global__ void __launch_bounds__(128) k_decode_exact(ExactParams p) {
    pdl_launch_dependents();
    pdl_wait();
    const int64_t gtid = blockIdx.x * 128ll + threadIdx.x;
    const int64_t rt = gtid >> 6;                  // 64 row pairs per 128-row tile
    const int tile = static_cast<int>((gtid >> 3) & 7), g = static_cast<int>(gtid & 7);
    const int64_t rows[2] = {rt * 128 + tile * 16 + g, rt * 128 + tile * 16 + g + 8};
    if (rt >= p.N / 128 + ((p.N % 128) ? 1 : 0)) return;
    const int64_t kw = p.K / 8;
    const int Mp = static_cast<int>(p.Mp);
    float s_r[2], lo[2], hi[2];
    int64_t lo_e[2], hi_e[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        const bool in = rows[r] < p.N;
        s_r[r] = in ? p.scale[rows[r]] : 0.0f;
        lo_e[r] = (in && p.nnz > 0) ? p.rowptr[rows[r]] : 0;
        hi_e[r] = (in && p.nnz > 0) ? p.rowptr[rows[r] + 1] : 0;
        lo[r] = hi[r] = 0.0f;
    }
    (void)lo;
    (void)hi;
    for (int tb = 0; tb < p.ntok; tb += kExactTok) {
        const int nt = min(kExactTok, p.ntok - tb);
        float a[2][4][kExactTok];
        float accb[2][kExactTok];
#pragma unroll
        for (int r = 0; r < 2; ++r)
#pragma unroll
            for (int t = 0; t < kExactTok; ++t) {
                accb[r][t] = 0.0f;
#pragma unroll
                for (int j = 0; j < 4; ++j) a[r][j][t] = 0.0f;
            }
        int64_t bp[2] = {lo_e[0], lo_e[1]};
        for (int64_t kb = 0; kb < p.KB; ++kb) {
            // lanes 4g..4g+3 of this tile: 16 words, [c][s]
            const uint4* src = reinterpret_cast<const uint4*>(p.wq + (rt * p.KB + kb) * 1024 + tile * 128 + g * 16);
            uint32_t w[4][4];
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                const uint4 v = __ldg(src + c);
                w[c][0] = v.x;
                w[c][1] = v.y;
                w[c][2] = v.z;
                w[c][3] = v.w;
            }
#pragma unroll
            for (int s = 0; s < 4; ++s) {
                const int64_t grp0 = kb * 8 + 2 * s;  // reference words grp0 (cols 16s..16s+7) and grp0+1
                if (grp0 >= kw) break;
                uint32_t hq[4][4];
#pragma unroll
                for (int c = 0; c < 4; ++c) dequant_word(w[c][s], hq[c]);
#pragma unroll
                for (int half = 0; half < 2; ++half) {
                    const int64_t grp = grp0 + half;
                    if (grp >= kw) break;
#pragma unroll
                    for (int t = 0; t < kExactTok; ++t) {
                        if (t >= nt) break;
                        const int tok = static_cast<int>(p.tok0 + tb + t);
                        uint16_t xv[8];
                        *reinterpret_cast<uint4*>(xv) = *reinterpret_cast<const uint4*>(p.xk + xk_index(grp * 8, tok, Mp));
                        if (!p.bypass) {
#pragma unroll
                            for (int r = 0; r < 2; ++r)
#pragma unroll
                                for (int j = 0; j < 4; ++j) {
                                    float v = a[r][j][t];
                                    v = fma_f16_f32(xv[j], wq_elem(hq, half, j, r), v);
                                    v = fma_f16_f32(xv[j + 4], wq_elem(hq, half, j + 4, r), v);
                                    a[r][j][t] = v;
                                }
                        } else {
#pragma unroll
                            for (int r = 0; r < 2; ++r) {
                                int64_t e = bp[r];
#pragma unroll
                                for (int i = 0; i < 8; ++i) {
                                    const int64_t colg = grp * 8 + i;
                                    float wv = __fmul_rn(h2f(wq_elem(hq, half, i, r)), s_r[r]);
                                    while (e < hi_e[r] && static_cast<int64_t>(p.col[e]) < colg) ++e;
                                    if (e < hi_e[r] && static_cast<int64_t>(p.col[e]) == colg)
                                        wv = __fadd_rn(wv, __fmul_rn(static_cast<float>(p.val[e]), p.ds));
                                    accb[r][t] = __fadd_rn(accb[r][t], __fmul_rn(h2f(xv[i]), wv));
                                }
                            }
                        }
                    }
                    if (p.bypass) {
#pragma unroll
                        for (int r = 0; r < 2; ++r)
                            while (bp[r] < hi_e[r] && static_cast<int64_t>(p.col[bp[r]]) < (grp + 1) * 8) ++bp[r];
                    }
                }
            }
        }
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            if (rows[r] >= p.N) continue;
            for (int t = 0; t < nt; ++t) {
                const int64_t tok = p.tok0 + tb + t;
                float acc;
                if (p.bypass) {
                    acc = accb[r][t];
                } else {
                    acc = __fmul_rn(__fadd_rn(__fadd_rn(__fadd_rn(a[r][0][t], a[r][1][t]), a[r][2][t]), a[r][3][t]),
                                    s_r[r]);
                    if (p.route_all || p.mask[tok]) {
                        for (int64_t e = lo_e[r]; e < hi_e[r]; ++e) {
                            const float dv = __fmul_rn(static_cast<float>(p.val[e]), p.ds);
                            const float xv = h2f(p.xk[xk_index(p.col[e], static_cast<int>(tok), Mp)]);
                            acc = __fadd_rn(acc, __fmul_rn(xv, dv));
                        }
                    }
                }
                const int64_t oi = tok * p.N + rows[r];
                if (p.partial_out) reinterpret_cast<float*>(p.y)[oi] = acc;
                else store_output(p.y, p.y_dtype, oi, acc, p.bias, rows[r]);
            }
        }
    }
}

// Test hook behind sc_test_drop_weight_copy (0: off).
static std::atomic<int> g_drop_copy{0};
void set_drop_weight_copy(int on) { g_drop_copy.store(on ? 1 : 0); }

static void fill_fused_params(const FusedArgs& f, FusedParams& fp) {
    const Layer& L = *f.L;
    TCParams& p = fp.t;
    p.wq = L.wq;
    p.scale = L.scale;
    p.rowptr = L.rowptr;
    p.col = L.col;
    p.val = L.val;
    p.ds = L.ds;
    p.nnz = L.nnz;
    p.xk = nullptr;
    p.Mp = 0;
    p.tok0 = 0;
    p.ntok = static_cast<int>(f.m);
    p.mask = nullptr;
    p.route_all = f.route_all;
    p.N = L.N;
    p.K = L.K;
    p.KB = L.KB;
    p.y = f.y;
    p.y_dtype = f.y_dtype;
    p.bias = f.bias;
    p.partial_out = f.partial_out;
    p.ws_partial = f.ws_partial;
    p.ws_rtcount = f.ws_rtcount;
    p.ksplit = f.ksplit;
    p.status = L.status;
    fp.x = f.x;
    fp.x_dtype = f.x_dtype;
    fp.x_stride = f.x_stride;
    fp.x_col0 = f.x_col0;
    fp.Kfull = f.x_stride;
    fp.t4 = L.t4;
    fp.t8 = L.t8;
    fp.mask_out = f.mask_out;
    fp.ridx_out = f.ridx_out;
    fp.nrouted_out = f.nrouted_out;
    fp.dwblk = f.dwblk;
    fp.dwoff = f.dwoff;
    fp.dw_global = f.dw_global;
    fp.ntp = f.m <= 1 ? 1 : f.m <= 2 ? 2 : f.m <= 4 ? 4 : 8;
    fp.rc = route_consts(fp.Kfull);
    fp.drop_copy = g_drop_copy.load();
    // each auxiliary thread adds at most T values sequentially in f32 (both passes), then five
    // shuffle levels add partial sums; the bound uses the depth, doubled for safety
    const int64_t ks = p.ksplit;
    const int64_t kbmax = (L.KB + ks - 1) / ks;
    const int64_t nout = fp.Kfull / 8 - L.K / 8;
    const int64_t omax = (nout + ks - 1) / ks;
    constexpr int64_t A = FusedRegions::kAuxThreads;
    int64_t T = 8 * ((kbmax * 8 + A - 1) / A + (omax + A - 1) / A) + 5;
    // one f16 token whose whole row (and the slice padding past it) fits below the fp8/integer
    // engines' second region, 16-byte aligned: one bulk copy, each thread sums its chunks of it
    const int64_t row_end = std::max<int64_t>(fp.Kfull, fp.x_col0 + L.KB * 64) * 2;
    fp.full_row = f.m == 1 && fp.x_dtype == SC_F16 && (reinterpret_cast<uintptr_t>(fp.x) & 15) == 0 &&
                  (fp.Kfull * 2) % 16 == 0 && row_end <= FusedRegions::kXb8;
    if (fp.full_row) T = 8 * ((fp.Kfull / 8 + A - 1) / A) + 5;
    const double u = 5.9604644775390625e-08;
    fp.gT = 2.0 * static_cast<double>(T) * u / (1.0 - static_cast<double>(T) * u);
}

cudaError_t launch_decode_fused(const FusedArgs* f, int n, cudaStream_t s) {
    if (n < 1 || n > kGroupMax) return cudaErrorInvalidValue;
    FusedGroup g = {};
    g.n = n;
    int ctas = 0;
    for (int i = 0; i < n; ++i) {
        if (f[i].ksplit != f[0].ksplit || f[i].L->mode != f[0].L->mode) return cudaErrorInvalidValue;
        fill_fused_params(f[i], g.p[i]);
        g.cta_start[i] = ctas;
        ctas += static_cast<int>((f[i].L->Np / 128) * f[i].ksplit);
    }
    for (int i = n; i <= kGroupMax; ++i) g.cta_start[i] = ctas;
    const int ksplit = f[0].ksplit;
    const bool tc = f[0].L->mode == SC_MODE_FAST_TC || f[0].L->mode == SC_MODE_FAST_TC8;
    // one token in SC_MODE_FAST_TC8: the fp8 variant when the e4m3 split of x fits
    bool f8 = f[0].L->mode == SC_MODE_FAST_TC8 && f[0].m == 1;
    for (int i = 0; i < n && f8; ++i) f8 = (f[i].L->KB + ksplit - 1) / ksplit <= FusedRegions::kMaxKbF8;
    // one token in SC_MODE_FAST: the integer variant when the digit columns of x fit
    bool i8 = SC_FUSED_INT8 && f[0].L->mode == SC_MODE_FAST && f[0].m == 1;
    for (int i = 0; i < n && i8; ++i) i8 = (f[i].L->KB + ksplit - 1) / ksplit <= FusedRegions::kMaxKbI8;
    const int which = f8 ? 2 : tc ? 1 : i8 ? 3 : 0;
    if (tc || f8)  // the test hook only reaches the mma.sync engines, which hold no tensor memory
        for (int i = 0; i < n; ++i) g.p[i].drop_copy = 0;
    auto kern = f8 ? k_ctarq_fused_tc<true> : tc ? k_ctarq_fused_tc<false> : i8 ? k_ctarq_fused_mma<true> : k_ctarq_fused_mma<false>;
    const int threads = f8 ? FusedTcCfg<true>::kThreads : tc ? FusedTcCfg<false>::kThreads : FusedMmaCfg::kThreads;
    const int smem = f8 ? FusedTcCfg<true>::kTotal : tc ? FusedTcCfg<false>::kTotal : FusedMmaCfg::kTotal;
    static std::atomic<uint64_t> flags[4] = {{0}, {0}, {0}, {0}};
    int dev = 0;
    cudaGetDevice(&dev);
    const uint64_t bit = 1ull << (dev & 63);
    if (!(flags[which].load() & bit)) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e == cudaSuccess) e = cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
        if (e == cudaSuccess)  // two CTAs per SM need the largest shared-memory carveout
            e = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
        if (e != cudaSuccess) return e;
        flags[which].fetch_or(bit);
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(ctas));
    cfg.blockDim = dim3(threads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = static_cast<unsigned>(ksplit);
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = ksplit > 1 ? 2 : 1;
    g_launches.fetch_add(1, std::memory_order_relaxed);
    return cudaLaunchKernelEx(&cfg, kern, g);
}

int fused_max_active_clusters(int ks) {
    static std::atomic<int> cache[64][kMaxFusedCluster + 1];  // 0: not queried yet
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64 || ks < 1 || ks > kMaxFusedCluster) return 0;
    const int have = cache[dev][ks].load();
    if (have > 0) return have;
    // the three engines take the same grid shape and near-identical shared memory; the mma.sync
    // engine (the largest footprint) stands for all of them
    auto kern = k_ctarq_fused_mma<false>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, FusedMmaCfg::kTotal) != cudaSuccess ||
        cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) != cudaSuccess ||
        cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, 100) != cudaSuccess)
        return 0;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(ks * 64));
    cfg.blockDim = dim3(FusedMmaCfg::kThreads);
    cfg.dynamicSmemBytes = FusedMmaCfg::kTotal;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = static_cast<unsigned>(ks);
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess || n <= 0) {
        cudaGetLastError();
        return 0;
    }
    cache[dev][ks].store(n);
    return n;
}

int fused_max_kb(int64_t m) {
    const int ntp = m <= 1 ? 1 : m <= 2 ? 2 : m <= 4 ? 4 : 8;
    return FusedRegions::kXsBytes / (128 * ntp);
}

int64_t fused_prefetch_bytes() {
    static std::atomic<int> sms[64];  // 0: not queried yet
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return 0;
    int n = sms[dev].load();
    if (n == 0) {
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) {
            cudaGetLastError();
            return 0;
        }
        sms[dev].store(n);
    }
    return static_cast<int64_t>(n) * FusedMmaCfg::S * FusedMmaCfg::kStageBytes;
}

cudaError_t launch_decode_exact(const DecodeArgs& a, int bypass, cudaStream_t s) {
    const Layer& L = *a.L;
    ExactParams p;
    p.wq = L.wq;
    p.scale = L.scale;
    p.rowptr = L.rowptr;
    p.col = L.col;
    p.val = L.val;
    p.ds = L.ds;
    p.nnz = L.nnz;
    p.xk = a.xk;
    p.Mp = a.Mp;
    p.tok0 = a.tok0;
    p.ntok = static_cast<int>(a.ntok);
    p.mask = a.mask;
    p.route_all = a.route_all;
    p.bypass = bypass;
    p.N = L.N;
    p.K = L.K;
    p.KB = L.KB;
    p.y = a.y;
    p.y_dtype = a.y_dtype;
    p.bias = a.bias;
    p.partial_out = a.partial_out;
    const int64_t threads = (L.Np / 128) * 64;  // one per row pair
    return launch_pdl(k_decode_exact, dim3(static_cast<unsigned>((threads + 127) / 128)), dim3(128), 0, s, p);
}

// ---------------------------------------------------------------- finalize

__global__ void k_finalize(const float* __restrict__ acc, int64_t total, int64_t n, void* y, int y_dtype,
                           const float* bias) {
    pdl_launch_dependents();
    pdl_wait();
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x)
        store_output(y, y_dtype, i, acc[i], bias, i % n);
}

cudaError_t launch_finalize(const float* acc, int64_t m, int64_t n, void* y, int y_dtype, const float* bias,
                            cudaStream_t s) {
    const int64_t total = m * n;
    if (total == 0) return cudaSuccess;
    int64_t blocks = (total + 255) / 256;
    if (blocks > 148 * 16) blocks = 148 * 16;
    return launch_pdl(k_finalize, dim3(static_cast<unsigned>(blocks)), dim3(256), 0, s, acc, total, n, y, y_dtype,
                      bias);
}

}  // namespace sc
