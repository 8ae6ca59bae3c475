// sc_gemm.cu -- C-TARQ linear for many tokens (prefill): a tcgen05 GEMM over 128-token tiles.
//
// One CTA computes one or two 128-row x 128-token tiles of Y (two share every x block, when the
// grid of pairs still fills the GPU) over a range of K (op.rs:99-178 for those rows and tokens).  The router (sc_router.cu) has decided every token, staged x as K-major
// core matrices (xk_index) and listed the tokens routed first (perm); k_gather_tokens copies
// the staged x into that order, so the routed tokens fill whole tiles.  For one 64-column
// block the 8-token groups of a tile are 1 KB each and contiguous, so a tile's activations
// arrive with one bulk copy per block and are the MMA's B operand as they lie (LBO 128 B
// between 8-column chunks, SBO 1 KB between token groups).
//
// Roles (18 warps, one CTA per SM):
//   producer lane   weights (4 KB per block and row tile, contiguous per row tile), the tile's x
//                   blocks and, for a tile of routed tokens, the blocks' dW lists, through a ring
//                   of S stages; the first stages' weights are requested before the dependency wait;
//   16 dequantising warps, one 16-row tile each, in two sets of 8: one set per row tile, or with
//                   one row tile alternate blocks (the next block is read while the current one's
//                   stores drain): W4U words -> f16 (q - 8) with dequant_word; in a
//                   tile of routed tokens the row's dW is folded in as (q - 8) + dW/s (s the row
//                   scale), one f16 per weight; then into tensor memory with tcgen05.st.16x256b;
//   MMA warp        one elected lane issues tcgen05.mma.kind::f16 M=128 N=128 K=16 (A from tensor
//                   memory, B from shared memory, f32 D in tensor memory), 4 per block and row tile,
//                   both row tiles on the same B (x) block: half the x traffic per MMA;
//   epilogue        the dequantising warps read D (tcgen05.ld, 32 rows x 8 tokens) and write
//                   y = f16(acc * s [+ dW]) (+ bias after rounding) for the tile's tokens.  A tile
//                   holding both routed and other tokens (at most one per row tile), or a layer
//                   without fold lists, adds the routed tokens' dW here from the CSR entries in
//                   column order (op.rs:152-170).  With column splits each CTA writes its f32
//                   partial and the last one of the tile adds them in split order.
//
// Numerics (fast mode): the products are f16 x f16 -> f32 on the tensor cores; folding dW/s into
// the weight rounds it to f16 next to an integer of magnitude <= 8 (2^-8 absolute), so a routed
// row's dW carries a relative error of up to ~2^-8 of its own, far below the fast-mode tolerance
// on y.
#include <cuda_fp16.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstring>
#include <vector>

#include "sc_device.cuh"
#include "sc_internal.h"

namespace sc {

// Bytes of one block's dW list slot in a ring stage: 4 KB (~10 % dW on average) in every
// variant, 8 KB (~23 %) in a one-row-tile variant for layers whose lists need it.
constexpr int kFoldCap = 4096;
constexpr int kFoldCapWide = 8192;

struct GemmParams {
    const uint32_t* wq;
    const float* scale;
    const uint32_t* rowptr;
    const uint16_t* col;
    const int8_t* val;
    float ds;
    int64_t nnz;
    const uint8_t* fold;
    const uint32_t* foldoff;
    const uint16_t* xk;     // staged x in token order (read when perm is the identity)
    const uint16_t* xkp;
    const int32_t* perm;
    const int32_t* nrouted;
    int64_t Mp, M, Mpp;     // xk token rows, tokens, xkp positions
    int route_all;
    int64_t N, KB, RT, T;   // rows, column blocks, row tiles, token tiles (one more than ceil(M/128))
    int rpc;                // row tiles per CTA: 2 when the grid still fills the GPU, else 1
    int64_t RTP;            // CTAs per token tile and split: ceil(RT / rpc)
    int ks;
    float* partial;
    uint32_t* tcount;
    void* y;
    int y_dtype;
    const float* bias;
    int partial_out;
    uint32_t* status;
};

// RPC: 128-row tiles per CTA (1, or 2 sharing every x block); FC: bytes of a dW list slot.  The
// ring, the tensor memory and every index are compile-time for each.
template <int RPC, int FC = kFoldCap>
struct GemmCfg {
    static constexpr int NT = 128;                   // tokens per tile (MMA N)
    static constexpr int kRowTiles = RPC;
    static constexpr int kDqWarps = 16;              // two sets of 8 (16-row tiles): per row tile, or alternate blocks
    static constexpr int kProducerWarp = 16;
    static constexpr int kMmaWarp = 17;
    static constexpr int kThreads = 18 * 32;
    static constexpr int G = NT / 8;                 // 8-token groups of a tile
    static constexpr int SKB = 2;                    // 64-column blocks per ring stage
    static constexpr int S = RPC == 1 ? 4 : 3;       // ring stages
    // A stage holds [row tile][block] 4 KB weights, the blocks' x (16 KB each), then [row tile]
    // [block] dW lists: 48 KB with one row tile, 64 KB with two (56 KB with one and 8 KB slots).
    static constexpr int kFold = FC;
    static constexpr int kWBytes = RPC * SKB * 4096;
    static constexpr int kXBytes = SKB * G * 1024;
    static constexpr int kFBytes = RPC * SKB * kFold;
    static constexpr int kStageBytes = kWBytes + kXBytes + kFBytes;
    static constexpr int kAB = 4;                    // TMEM A buffers per row tile, one block (32 columns) each
    static constexpr uint32_t kTmemCols = RPC == 1 ? 256 : 512;  // D of row tile t at t*128, A after the D's
    static constexpr int kBarOff = S * kStageBytes;
    static constexpr int kNumBars = 2 * S + 2 * kAB + 1;
    static constexpr int kTmemSlotOff = kBarOff + kNumBars * 8;
    static constexpr int kTotal = kTmemSlotOff + 16;
    static_assert(RPC == 1 || RPC == 2, "row tiles per CTA");
    static_assert(FC % 16 == 0 && (kStageBytes % 1024) == 0, "list slots keep the x tiles 1 KB aligned");
    static_assert(RPC * NT + RPC * kAB * 32 <= static_cast<int>(kTmemCols), "tensor memory");
    static_assert(kTotal <= 227 * 1024, "shared memory");
};


// Token tile tt of a row tile, from the routed count R (read after the dependency wait): tiles
// [0, ceil(R/128)) hold the routed positions [0, R), the next ones the others from
// round_up(R, 8); the last tile of the launch may be empty.  identity: perm is the identity
// (nothing or everything routed) and x is read in token order.
struct GemmTile {
    int64_t R, pos0;
    int ntile;
    bool routed, fold, identity;
};
__device__ __forceinline__ GemmTile gemm_tile(const GemmParams& p, int64_t tt) {
    constexpr int NT = GemmCfg<1>::NT;
    GemmTile g;
    g.R = p.route_all ? p.M : static_cast<int64_t>(*p.nrouted);
    const int64_t TR = (g.R + NT - 1) / NT, RB = (g.R + 7) & ~static_cast<int64_t>(7);
    g.identity = g.R == 0 || g.R == p.M;
    g.routed = tt < TR;
    if (g.routed) {
        g.pos0 = tt * NT;
        g.ntile = static_cast<int>(imin64(NT, g.R - g.pos0));
    } else {
        g.pos0 = RB + (tt - TR) * NT;
        const int64_t left = RB + (p.M - g.R) - g.pos0;
        g.ntile = static_cast<int>(left <= 0 ? 0 : imin64(NT, left));
    }
    g.fold = g.routed && p.foldoff != nullptr;
    return g;
}

template <int RPC, int FC>
__global__ void __launch_bounds__(GemmCfg<RPC, FC>::kThreads, 1) k_ctarq_gemm(GemmParams p) {
    using C = GemmCfg<RPC, FC>;
    constexpr int SKB = C::SKB, AB = C::kAB, NT = C::NT, G = C::G, S = C::S;
    extern __shared__ __align__(1024) unsigned char smem[];
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::kBarOff);
    uint64_t* empty = full + C::S;
    uint64_t* a_full = empty + C::S;
    uint64_t* a_empty = a_full + AB;
    uint64_t* done = a_empty + AB;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::kTmemSlotOff);
    __shared__ int s_abort;
    __shared__ int s_last;
    __shared__ int s_empty;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    // token-tile-major order: the last token tile (empty unless the routed and the other tokens
    // both leave a partial tile) comes last in the grid
    const int64_t tile_id = blockIdx.x / p.ks;
    const int sp = static_cast<int>(blockIdx.x - tile_id * p.ks);
    const int64_t tt = tile_id / p.RTP;
    const int64_t rt0 = (tile_id - tt * p.RTP) * RPC;          // first row tile of the CTA
    const int nrt = static_cast<int>(imin64(RPC, p.RT - rt0));     // row tiles present
    constexpr int kStage = C::kStageBytes;
    constexpr int kW = C::kWBytes;                                 // offset of x in a stage
    constexpr int kF = C::kWBytes + C::kXBytes;                    // offset of the dW lists
    if (tt == p.T - 1) {
        // the only tile that can be empty: look before setting anything up
        pdl_wait();
        if (gemm_tile(p, tt).ntile == 0) return;
    }
    const int kb_begin = static_cast<int>((p.KB * sp) / p.ks);
    const int kb_end = static_cast<int>((p.KB * (sp + 1)) / p.ks);
    const int nkb = kb_end - kb_begin;

    pdl_launch_dependents();
    // token groups past the real tokens are never copied: they read as zero in every stage
    for (int i = tid; i < S * (C::kXBytes / 16); i += C::kThreads) {
        const int st = i / (C::kXBytes / 16), off = i - st * (C::kXBytes / 16);
        reinterpret_cast<uint4*>(smem + st * kStage + kW)[off] = make_uint4(0, 0, 0, 0);
    }
    fence_proxy_async_smem();
    if (tid == 0) {
        for (int i = 0; i < S; ++i) {
            mbar_init(&full[i], 2);
            mbar_init(&empty[i], 1);
        }
        for (int i = 0; i < AB; ++i) {
            mbar_init(&a_full[i], 8 * nrt);  // every present row tile's set writes its block
            mbar_init(&a_empty[i], 1);
        }
        mbar_init(done, 1);
        fence_mbar_init();
        s_abort = 0;
        s_empty = 0;
    }
    if (warp == C::kMmaWarp) {
        tmem_alloc(tmem_slot, C::kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    int issued = 0;
    const int nst = (nkb + SKB - 1) / SKB;
    const int pre = nst < S ? nst : S;
    if (warp == C::kProducerWarp) {
        if (lane == 0) {
            const uint64_t pol = policy_evict_first();
            for (int it = 0; it < pre; ++it, ++issued) {
                const int kb0 = kb_begin + it * SKB;
                const int n = kb_end - kb0 < SKB ? kb_end - kb0 : SKB;
                mbar_arrive_expect_tx(&full[it], static_cast<uint32_t>(nrt * n * 4096));
                for (int r = 0; r < nrt; ++r)
                    bulk_g2s_stream(smem + it * kStage + r * SKB * 4096, p.wq + ((rt0 + r) * p.KB + kb0) * 1024,
                                    static_cast<uint32_t>(n * 4096), &full[it], pol);
            }
            pdl_wait();
            const GemmTile g = gemm_tile(p, tt);
            const int64_t pos0 = g.pos0;
            const int greal = (g.ntile + 7) >> 3;
            const bool fold = g.fold;
            const uint16_t* xsrc = g.identity ? p.xk : p.xkp;
            const int64_t Gp = (g.identity ? p.Mp : p.Mpp) >> 3;
            if (g.ntile == 0) {
                // no tokens: complete the prefetched stages' phases (their weights still land)
                s_empty = 1;
                for (int it = 0; it < pre; ++it) mbar_arrive_expect_tx(&full[it], 0u);
            }
            for (int it = 0; it < nst && g.ntile > 0; ++it) {
                const int slot = it % S, kb0 = kb_begin + it * SKB;
                const int n = kb_end - kb0 < SKB ? kb_end - kb0 : SKB;
                unsigned char* st = smem + slot * kStage;
                if (it >= S) {
                    if (!mbar_wait(&empty[slot], ((it / S) - 1) & 1, p.status)) {
                        s_abort = 1;
                        break;
                    }
                    mbar_arrive_expect_tx(&full[slot], static_cast<uint32_t>(nrt * n * 4096));
                    for (int r = 0; r < nrt; ++r)
                        bulk_g2s_stream(st + r * SKB * 4096, p.wq + ((rt0 + r) * p.KB + kb0) * 1024,
                                        static_cast<uint32_t>(n * 4096), &full[slot], pol);
                    ++issued;
                }
                uint32_t fbytes = 0;
                if (fold)
                    for (int r = 0; r < nrt; ++r)
                        fbytes += p.foldoff[(rt0 + r) * p.KB + kb0 + n] - p.foldoff[(rt0 + r) * p.KB + kb0];
                mbar_arrive_expect_tx(&full[slot], static_cast<uint32_t>(n * greal * 1024) + fbytes);
                for (int j = 0; j < n; ++j) {
                    bulk_g2s(st + kW + j * G * 1024, xsrc + ((kb0 + j) * Gp + (pos0 >> 3)) * 512,
                             static_cast<uint32_t>(greal * 1024), &full[slot]);
                    if (fold) {
                        for (int r = 0; r < nrt; ++r) {
                            const int64_t li = (rt0 + r) * p.KB + kb0 + j;
                            const uint32_t o0 = p.foldoff[li], o1 = p.foldoff[li + 1];
                            bulk_g2s(st + kF + (r * SKB + j) * C::kFold, p.fold + o0, o1 - o0,
                                     &full[slot]);
                        }
                    }
                }
            }
        }
    } else if (warp == C::kMmaWarp) {
        // warp-uniform loop, one elected lane issues (the same lane every time, so its commits
        // track all of its MMAs)
        const uint32_t idesc = idesc_f16_f32(128, NT);
        pdl_wait();
        bool ok = true;
        const int nmma = gemm_tile(p, tt).ntile > 0 ? nkb : 0;
        for (int j = 0; j < nmma && ok; ++j) {
            const int s = j / SKB, kbl = j - s * SKB, slot = s % S, b = j % AB;
            if (kbl == 0) ok = mbar_wait(&full[slot], (s / S) & 1, p.status);
            if (ok) ok = mbar_wait(&a_full[b], (j / AB) & 1, p.status);
            ok = __all_sync(0xffffffffu, ok);  // the elected lane below needs the whole warp
            if (!ok) break;
            tc_fence_after();
            const unsigned char* xs = smem + slot * kStage + kW + kbl * G * 1024;
            if (elect_one()) {
                // every row tile against the same x block: D of tile r in columns [r*128, r*128+128)
                for (int r = 0; r < nrt; ++r) {
#pragma unroll
                    for (int i = 0; i < 4; ++i)
                        tc_mma_ts(tmem + r * NT, tmem + C::kRowTiles * NT + (r * AB + b) * 32 + i * 8,
                                  desc_kmajor(xs + 2 * i * 128, 128, 1024), idesc, (j | i) ? 1u : 0u);
                }
                tc_commit(&a_empty[b]);
                if (kbl == SKB - 1 || j == nkb - 1) tc_commit(&empty[slot]);
            }
            __syncwarp();
        }
        if (!ok) s_abort = 1;
        if (elect_one()) tc_commit(done);  // also after an abort, so that the TMEM can be released
        __syncwarp();
    } else {
        // two row tiles: set s takes row tile s, every block; one row tile: the sets take
        // alternate blocks of it (two independent store pipelines)
        const int sq = warp & 3, q = (warp >> 2) & 1, set = warp >> 3;
        const int tile = 2 * sq + q;
        const uint32_t lane_addr = static_cast<uint32_t>(32 * sq + 16 * q) << 16;
        const int r = nrt == 1 ? 0 : set;          // row tile of this warp
        const int jstep = nrt == 1 ? 2 : 1;
        const int64_t rt = rt0 + r;
        pdl_wait();
        const GemmTile g = gemm_tile(p, tt);
        const int64_t pos0 = g.pos0, R = g.R;
        const int ntile = g.ntile;
        const bool fold = g.fold;
        const int64_t Mx = g.identity ? p.Mp : p.Mpp;  // token rows of the x copy read
        const uint16_t* xsrc = g.identity ? p.xk : p.xkp;
        // Software-pipelined: the next block of this set is read and dequantised while the
        // current block's tensor-memory stores drain.
        auto load_block = [&](int jj, uint32_t (&hh)[4][4]) -> bool {
            const int s = jj / SKB, kbl = jj - s * SKB, slot = s % S;
            if (!mbar_wait(&full[slot], (s / S) & 1, p.status)) return false;
            const unsigned char* stg = smem + slot * kStage;
            const uint4 wv =
                *reinterpret_cast<const uint4*>(stg + (r * SKB + kbl) * 4096 + tile * 512 + lane * 16);
            const uint32_t words[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
            for (int st = 0; st < 4; ++st) dequant_word(words[st], hh[st]);
            if (fold) {
                // this lane's entries of the block (register slot, half, f16 dW/s)
                const unsigned char* lst = stg + kF + (r * SKB + kbl) * C::kFold;
                const uint16_t* offs = reinterpret_cast<const uint16_t*>(lst) + tile * 33 + lane;
                const uint32_t* ent = reinterpret_cast<const uint32_t*>(lst + kFoldHdr);
                const int e1 = offs[1];
                for (int e = offs[0]; e < e1; ++e) {
                    const uint32_t w = ent[e];
                    fold_add(hh, static_cast<int>((w >> 5) & 15u), static_cast<int>((w >> 9) & 1u),
                             static_cast<uint16_t>(w >> 16));
                }
            }
            return true;
        };
        uint32_t h[4][4];
        int j = nrt == 1 ? set : 0;
        bool have = ntile > 0 && j < nkb;
        if (have && !load_block(j, h)) {
            s_abort = 1;
            have = false;
        }
        while (have) {
            const int b = j % AB;
            if (j >= AB && !mbar_wait(&a_empty[b], ((j / AB) - 1) & 1, p.status)) {
                s_abort = 1;
                break;
            }
            tc_fence_after();
#pragma unroll
            for (int st = 0; st < 4; ++st)
                tc_st_16x256b(tmem + lane_addr + C::kRowTiles * NT + (r * AB + b) * 32 + st * 8, h[st][0], h[st][2],
                              h[st][1], h[st][3]);
            const int jn = j + jstep;
            uint32_t hn[4][4];
            bool next = jn < nkb;
            if (next && !load_block(jn, hn)) {
                s_abort = 1;
                next = false;
            }
            tc_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&a_full[b]);
            if (!next) break;
#pragma unroll
            for (int st = 0; st < 4; ++st)
#pragma unroll
                for (int r = 0; r < 4; ++r) h[st][r] = hn[st][r];
            j = jn;
        }
        // epilogue: rows 32 sq + lane of row tile r; tokens [64 q, +64) with two row tiles, else
        // [32 (2 set + q), +32)
        if (ntile > 0 && mbar_wait(done, 0, p.status) && !s_abort) {
            tc_fence_after();
            const int64_t row = rt * 128 + 32 * sq + lane;
            const bool live = row < p.N;
            const float sc = live ? p.scale[row] : 0.0f;
            // dW entries of this row inside the CTA's columns, for routed tokens not folded
            int64_t e0 = 0, e1 = 0;
            if (!fold && live && p.nnz > 0 && g.routed) {
                const int64_t lo = p.rowptr[row], hi = p.rowptr[row + 1];
                e0 = p.ks == 1 ? lo : lower_bound_u16(p.col, lo, hi, static_cast<int64_t>(kb_begin) * 64);
                e1 = p.ks == 1 ? hi : lower_bound_u16(p.col, e0, hi, static_cast<int64_t>(kb_end) * 64);
            }
            const uint32_t lane_rows = static_cast<uint32_t>(32 * sq) << 16;
            float* part = p.partial + ((tile_id * p.ks + sp) * NT) * 256;
            const int nch = nrt == 1 ? 4 : 8, cq = nrt == 1 ? 2 * set + q : q;
#pragma unroll 1
            for (int cb = nch * cq; cb < nch * cq + nch; ++cb) {
                const int t0 = cb * 8;
                if (t0 >= ntile) break;
                uint32_t d[8];
                tc_ld8(tmem + lane_rows + r * NT + t0, d);
                tc_wait_ld();
                float corr[8];
#pragma unroll
                for (int u = 0; u < 8; ++u) corr[u] = 0.0f;
                const int nr = g.routed ? static_cast<int>(imin64(8, ntile - t0)) : 0;  // routed, unfolded
                if (e1 > e0 && nr > 0) {
                    for (int64_t e = e0; e < e1; ++e) {
                        const int64_t cl = p.col[e];
                        const float v = __fmul_rn(static_cast<float>(p.val[e]), p.ds);
                        const uint16_t* xg = xsrc + xk_index(cl, static_cast<int>(pos0 + t0), static_cast<int>(Mx));
#pragma unroll
                        for (int u = 0; u < 8; ++u)
                            if (u < nr) corr[u] = __fadd_rn(corr[u], __fmul_rn(h2f(xg[u * 8]), v));
                    }
                }
#pragma unroll
                for (int u = 0; u < 8; ++u) {
                    if (t0 + u < ntile) {
                        const float v = __fadd_rn(__fmul_rn(__uint_as_float(d[u]), sc), corr[u]);
                        if (p.ks > 1) {
                            part[(t0 + u) * 256 + r * 128 + 32 * sq + lane] = v;
                        } else if (live) {
                            const int64_t oi = static_cast<int64_t>(p.perm[pos0 + t0 + u]) * p.N + row;
                            if (p.partial_out) reinterpret_cast<float*>(p.y)[oi] = v;
                            else store_output(p.y, p.y_dtype, oi, v, p.bias, row);
                        }
                    }
                }
            }
            if (p.ks > 1) __threadfence();  // the partials, before this CTA's split is counted
        } else if (ntile > 0) {
            s_abort = 1;
        }
        (void)R;
        tc_fence_before();
    }
    __syncwarp();  // single-lane roles rejoin their warp before the warp-wide TMEM release below
    __syncthreads();
    if (warp == C::kMmaWarp) {
        // every tcgen05 operation of this CTA has completed (done observed, loads waited)
        if (s_abort) mbar_wait(done, 0, nullptr, kDrainNs);
        tc_fence_after();
        tmem_dealloc(tmem, C::kTmemCols);
    }
    if (s_abort || s_empty) {
        if (warp == C::kProducerWarp && lane == 0)
            for (int it = issued > S ? issued - S : 0; it < issued; ++it)
                mbar_wait(&full[it % S], (it / S) & 1, nullptr, kDrainNs);
        return;
    }
    if (p.ks > 1) {
        const GemmTile g = gemm_tile(p, tt);
        const int64_t pos0 = g.pos0;
        const int ntile = g.ntile;
        // the last split of the tile to finish adds the partials in split order
        if (tid == 0) s_last = atomicAdd(&p.tcount[tile_id], 1u) == static_cast<unsigned>(p.ks - 1);
        __syncthreads();
        if (!s_last) return;
        __threadfence();
        const float* base = p.partial + (tile_id * p.ks * NT) * 256;
        const int rows = 128 * nrt;  // this CTA's rows (its row tiles only)
        for (int i = tid; i < ntile * rows; i += C::kThreads) {
            const int t = i / rows, rl = i - t * rows;
            const int64_t r = rt0 * 128 + rl;
            if (r >= p.N) continue;
            float v = 0.0f;
            for (int k = 0; k < p.ks; ++k) v = __fadd_rn(v, __ldcg(base + (k * NT + t) * 256 + rl));
            const int64_t oi = static_cast<int64_t>(p.perm[pos0 + t]) * p.N + r;
            if (p.partial_out) reinterpret_cast<float*>(p.y)[oi] = v;
            else store_output(p.y, p.y_dtype, oi, v, p.bias, r);
        }
        if (tid == 0) p.tcount[tile_id] = 0u;
    }
}

// xkp[position p] = xk[token perm[p]] for every 16-byte chunk, positions laid out as the GEMM
// tiles read them (routed [0, R), the others from round_up(R, 8)); other positions are zeroed.
// One thread per destination chunk, in destination order (coalesced stores).
__global__ void k_gather_tokens(const uint16_t* __restrict__ xk, uint16_t* __restrict__ xkp,
                                const int32_t* __restrict__ perm, const int32_t* __restrict__ nrouted, int route_all,
                                int64_t M, int64_t Mp, int64_t Mpp, int64_t KB) {
    pdl_launch_dependents();
    pdl_wait();
    const int64_t R = route_all ? M : *nrouted;
    if (R == 0 || R == M) return;  // perm is the identity: the GEMM reads xk itself
    const int64_t RB = (R + 7) & ~static_cast<int64_t>(7);
    const int64_t total = KB * Mpp * 8;  // chunks
    const int64_t Gpp = Mpp >> 3;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        // i = ((kb * Mpp/8 + p/8) * 8 + chunk) * 8 + p%8
        const int64_t pi = i & 7, ch = (i >> 3) & 7, rest = i >> 6;
        const int64_t kb = rest / Gpp, pg = rest - kb * Gpp;
        const int64_t pos = pg * 8 + pi;
        uint4 v = make_uint4(0u, 0u, 0u, 0u);
        if (pos < R || (pos >= RB && pos < RB + (M - R))) {
            const int t = perm[pos];
            v = *reinterpret_cast<const uint4*>(xk + xk_index(kb * 64 + ch * 8, t, static_cast<int>(Mp)));
        }
        *reinterpret_cast<uint4*>(xkp + i * 8) = v;
    }
}

int64_t gemm_tile_tokens() { return GemmCfg<1>::NT; }

// Row tiles per CTA: two (sharing every x block, half the x traffic per MMA) while the grid of
// pairs still fills every SM once, else one (more CTAs, a deeper ring).  Layers whose dW lists
// need the 8 KB slots take one (two row tiles would not fit the shared memory).
static int gemm_rows_per_cta(const Layer& L, int64_t m) {
    if (L.fold != nullptr && L.fold_cap > kFoldCap) return 1;
    const int64_t pairs = (L.Np / 128 + 1) / 2 * ((m + GemmCfg<1>::NT - 1) / GemmCfg<1>::NT);
    return pairs >= L.sms ? 2 : 1;
}

int gemm_ksplit(const Layer& L, int64_t m) {
    // column splits while the tiles alone leave SMs idle, each split keeping >= 8 blocks (the
    // launch's extra token tile is usually empty and is not counted)
    const int rpc = gemm_rows_per_cta(L, m);
    const int64_t tiles = (L.Np / 128 + rpc - 1) / rpc * ((m + GemmCfg<1>::NT - 1) / GemmCfg<1>::NT);
    int64_t ks = std::max<int64_t>(1, static_cast<int64_t>(L.sms) / std::max<int64_t>(1, tiles));
    ks = std::min<int64_t>(ks, std::min<int64_t>(16, std::max<int64_t>(1, L.KB / 8)));
    return static_cast<int>(ks);
}

cudaError_t launch_gemm(const GemmArgs& a, cudaStream_t s) {
    const Layer& L = *a.L;
    GemmParams p;
    p.wq = L.wq;
    p.scale = L.scale;
    p.rowptr = L.rowptr;
    p.col = L.col;
    p.val = L.val;
    p.ds = L.ds;
    p.nnz = L.nnz;
    p.fold = L.fold;
    p.foldoff = L.foldoff;
    p.xk = a.xk;
    p.xkp = a.xkp;
    p.perm = a.perm;
    p.nrouted = a.nrouted;
    p.Mp = a.Mp;
    p.M = a.M;
    p.Mpp = a.Mpp;
    p.route_all = a.route_all;
    p.N = L.N;
    p.KB = L.KB;
    p.RT = L.Np / 128;
    p.rpc = gemm_rows_per_cta(L, a.M);
    p.RTP = (p.RT + p.rpc - 1) / p.rpc;
    p.T = (a.M + GemmCfg<1>::NT - 1) / GemmCfg<1>::NT + 1;
    p.ks = a.ks;
    p.partial = a.partial;
    p.tcount = a.tcount;
    p.y = a.y;
    p.y_dtype = a.y_dtype;
    p.bias = a.bias;
    p.partial_out = a.partial_out;
    p.status = L.status;
    const int64_t chunks = L.KB * a.Mpp * 8;
    const int64_t gblocks = std::min<int64_t>((chunks + 255) / 256, static_cast<int64_t>(L.sms) * 16);
    cudaError_t e = cudaSuccess;
    if (!a.skip_gather) {
        e = launch_pdl(k_gather_tokens, dim3(static_cast<unsigned>(gblocks)), dim3(256), 0, s, a.xk, a.xkp, a.perm,
                       a.nrouted, a.route_all, a.M, a.Mp, a.Mpp, L.KB);
        if (e != cudaSuccess) return e;
    }
    static std::atomic<uint64_t> flags[3] = {{0}, {0}, {0}};
    int dev = 0;
    cudaGetDevice(&dev);
    const uint64_t bit = 1ull << (dev & 63);
    const int var = p.rpc == 2 ? 1 : (L.fold != nullptr && L.fold_cap > kFoldCap) ? 2 : 0;
    auto kern = var == 1 ? k_ctarq_gemm<2, kFoldCap> : var == 2 ? k_ctarq_gemm<1, kFoldCapWide> : k_ctarq_gemm<1, kFoldCap>;
    const int smem = var == 1 ? GemmCfg<2>::kTotal : var == 2 ? GemmCfg<1, kFoldCapWide>::kTotal : GemmCfg<1>::kTotal;
    if (!(flags[var].load() & bit)) {
        e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return e;
        flags[var].fetch_or(bit);
    }
    return launch_pdl(kern, dim3(static_cast<unsigned>(p.RTP * p.T * p.ks)), dim3(GemmCfg<1>::kThreads), smem, s, p);
}

// Fold lists from the host CSR (columns ascending per row) and the f32 row scales: for every
// (row tile, block), a header of u16 entry offsets [16-row tile][lane 0..32] (kFoldHdr bytes;
// entry o[t][l] .. o[t][l+1] belong to lane l of tile t), then one u32 per entry, grouped by
// (tile, lane): bits 0-4 the lane (4 g + c) holding the weight in the dequantised fragment, 5-8
// the register slot (step * 4 + register), 9 the half, 16-31 the f16 of dW/s.  The slot size
// (L.fold_cap) is the smaller of 4 KB and 8 KB that holds every list.  Left empty (no fold: the
// GEMM adds dW in its epilogue) when a list exceeds 8 KB or a value is not representable.
cudaError_t build_fold_lists(Layer& L, const uint32_t* srp, const uint16_t* scol, const int8_t* sval,
                             const float* scale) {
    L.fold = nullptr;
    L.foldoff = nullptr;
    L.fold_cap = 0;
    if (L.nnz == 0) return cudaSuccess;
    size_t max_bytes = 0;
    const int64_t RT = L.Np / 128, KB = L.KB;
    std::vector<uint32_t> off(RT * KB + 1, 0);
    std::vector<uint8_t> blob;
    std::vector<std::vector<uint32_t>> per(KB * 8 * 32);  // [kb][tile16][lane] entries of one row tile
    for (int64_t rt = 0; rt < RT; ++rt) {
        for (auto& v : per) v.clear();
        for (int r = 0; r < 128; ++r) {
            const int64_t row = rt * 128 + r;
            if (row >= L.N) break;
            for (uint32_t q = srp[row]; q < srp[row + 1]; ++q) {
                const double dw = static_cast<double>(static_cast<float>(sval[q]) * L.ds);
                if (dw == 0.0) continue;
                const double sc = static_cast<double>(scale[row]);
                if (!(sc > 0.0)) return cudaSuccess;
                const __half hv = __float2half_rn(static_cast<float>(dw / sc));
                if (!std::isfinite(__half2float(hv))) return cudaSuccess;
                const int cl = scol[q] % 64, kb = scol[q] / 64;
                const int rl = r % 16, g = rl & 7, upper = rl >> 3;
                const int stp = cl >> 4, cc = cl & 15, c = cc >> 2, k = cc & 3;
                const uint32_t lane = static_cast<uint32_t>(g * 4 + c);
                const uint32_t slot = static_cast<uint32_t>(stp * 4 + upper + (k >= 2 ? 2 : 0));
                const uint32_t half = static_cast<uint32_t>(k & 1);
                per[(kb * 8 + r / 16) * 32 + lane].push_back(lane | (slot << 5) | (half << 9) |
                                                             (static_cast<uint32_t>(__half_as_ushort(hv)) << 16));
            }
        }
        for (int64_t kb = 0; kb < KB; ++kb) {
            size_t n = 0;
            for (int t = 0; t < 8 * 32; ++t) n += per[kb * 256 + t].size();
            const size_t bytes = ((kFoldHdr + 4 * n) + 15) / 16 * 16;
            if (bytes > static_cast<size_t>(kFoldCapWide)) return cudaSuccess;
            max_bytes = std::max(max_bytes, bytes);
            const size_t at = blob.size();
            blob.resize(at + bytes, 0);
            uint16_t hdr[kFoldHdr / 2] = {};
            uint32_t acc = 0;
            for (int t = 0; t < 8; ++t) {
                for (int l = 0; l < 32; ++l) {
                    const auto& v = per[kb * 256 + t * 32 + l];
                    hdr[t * 33 + l] = static_cast<uint16_t>(acc);
                    std::memcpy(&blob[at + kFoldHdr + 4 * acc], v.data(), 4 * v.size());
                    acc += static_cast<uint32_t>(v.size());
                }
                hdr[t * 33 + 32] = static_cast<uint16_t>(acc);
            }
            std::memcpy(&blob[at], hdr, sizeof(hdr));
            off[rt * KB + kb + 1] = static_cast<uint32_t>(blob.size());
        }
    }
    uint8_t* dblob = nullptr;
    uint32_t* doff = nullptr;
    cudaError_t e = cudaMalloc(&dblob, blob.size());
    if (e == cudaSuccess) e = cudaMalloc(&doff, off.size() * 4);
    if (e == cudaSuccess) e = cudaMemcpy(dblob, blob.data(), blob.size(), cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMemcpy(doff, off.data(), off.size() * 4, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) {
        cudaFree(dblob);
        cudaFree(doff);
        return e;
    }
    L.fold = dblob;
    L.foldoff = doff;
    L.fold_cap = max_bytes <= static_cast<size_t>(kFoldCap) ? kFoldCap : kFoldCapWide;
    L.device_bytes += static_cast<int64_t>(blob.size() + off.size() * 4);
    return cudaSuccess;
}

}  // namespace sc
