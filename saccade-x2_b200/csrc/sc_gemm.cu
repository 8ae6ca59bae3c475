// sc_gemm.cu -- C-TARQ linear for many tokens (prefill): a tcgen05 GEMM over 128-token tiles.
//
// One CTA computes a 128-row x 128-token tile of Y over the whole K (op.rs:99-178 for those
// rows and tokens).  The router (sc_router.cu) has decided every token and staged x as K-major
// core matrices (xk_index): for one 64-column block the 8-token groups of a tile are 1 KB each
// and contiguous, so a tile's activations arrive with one bulk copy per block and are the MMA's
// B operand as they lie (LBO 128 B between 8-column chunks, SBO 1 KB between token groups).
//
// Roles (10 warps, one CTA per SM):
//   producer lane   weights (4 KB per block, contiguous per row tile) and the tile's x blocks
//                   through a ring of S stages; the first stages' weights are requested before
//                   the dependency wait (they do not depend on the previous kernel);
//   8 dequantising  warps, one 16-row tile each: W4U words -> f16 (q - 8) with dequant_word, into
//                   tensor memory with tcgen05.st.16x256b (A operand, natural K order);
//   MMA warp        one elected lane issues tcgen05.mma.kind::f16 M=128 N=128 K=16 (A from tensor
//                   memory, B from shared memory, f32 D in tensor memory), 4 per block, and
//                   commits the A buffer and ring stage it consumed;
//   epilogue        the dequantising warps read D (tcgen05.ld, 32 lanes x 8 tokens), add the
//                   row's dW for routed tokens (CSR entries in column order, x from the staged
//                   copy, op.rs:152-170) and write y = f16(acc * s + dW) (+ bias after rounding).
//
// The MMA runs at N = 128 (64 cycles per instruction, 4x the tokens of the 32-token decode
// kernel per instruction), and each weight block is fetched once per 128 tokens.
#include <atomic>

#include "sc_device.cuh"
#include "sc_internal.h"

namespace sc {

struct GemmParams {
    const uint32_t* wq;
    const float* scale;
    const uint32_t* rowptr;
    const uint16_t* col;
    const int8_t* val;
    float ds;
    int64_t nnz;
    const uint16_t* xk;
    int64_t Mp, M;
    const uint8_t* mask;
    int route_all;
    int64_t N, KB, RT, T;   // rows, column blocks, row tiles, token tiles
    void* y;
    int y_dtype;
    const float* bias;
    int partial_out;
    uint32_t* status;
};

struct GemmCfg {
    static constexpr int NT = 128;                   // tokens per tile (MMA N)
    static constexpr int kDqWarps = 8;               // two per TMEM sub-partition, one 16-row tile each
    static constexpr int kProducerWarp = 8;
    static constexpr int kMmaWarp = 9;
    static constexpr int kThreads = 10 * 32;
    static constexpr int G = NT / 8;                 // 8-token groups of a tile
    static constexpr int SKB = 2;                    // 64-column blocks per ring stage
    static constexpr int S = 4;
    static constexpr int kWBytes = SKB * 4096;
    static constexpr int kXBytes = SKB * G * 1024;
    static constexpr int kStageBytes = kWBytes + kXBytes;
    static constexpr int kAB = 4;                    // TMEM A buffers, one block (32 columns) each
    static constexpr uint32_t kTmemCols = 256;       // D in [0, 128), A buffers in [128, 256)
    static constexpr int kBarOff = S * kStageBytes;
    static constexpr int kNumBars = 2 * S + 2 * kAB + 1;
    static constexpr int kTmemSlotOff = kBarOff + kNumBars * 8;
    static constexpr int kTotal = kTmemSlotOff + 16;
    static_assert(NT + kAB * 32 <= static_cast<int>(kTmemCols), "tensor memory");
    static_assert(kTotal <= 227 * 1024, "shared memory");
};

__global__ void __launch_bounds__(GemmCfg::kThreads, 1) k_ctarq_gemm(GemmParams p) {
    using C = GemmCfg;
    constexpr int SKB = C::SKB, S = C::S, AB = C::kAB, NT = C::NT, G = C::G;
    extern __shared__ __align__(1024) unsigned char smem[];
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::kBarOff);
    uint64_t* empty = full + S;
    uint64_t* a_full = empty + S;
    uint64_t* a_empty = a_full + AB;
    uint64_t* done = a_empty + AB;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::kTmemSlotOff);
    __shared__ int s_abort;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int64_t rt = blockIdx.x / p.T;
    const int64_t tok0 = (blockIdx.x - rt * p.T) * NT;
    const int ntile = static_cast<int>(imin64(NT, p.M - tok0));
    const int greal = (ntile + 7) >> 3;
    const int nkb = static_cast<int>(p.KB);

    pdl_launch_dependents();
    // token groups past the real tokens are never copied: they read as zero in every stage
    for (int i = tid; i < S * (C::kXBytes / 16); i += C::kThreads) {
        const int st = i / (C::kXBytes / 16), off = i - st * (C::kXBytes / 16);
        reinterpret_cast<uint4*>(smem + st * C::kStageBytes + C::kWBytes)[off] = make_uint4(0, 0, 0, 0);
    }
    fence_proxy_async_smem();
    if (tid == 0) {
        for (int i = 0; i < S; ++i) {
            mbar_init(&full[i], 2);
            mbar_init(&empty[i], 1);
        }
        for (int i = 0; i < AB; ++i) {
            mbar_init(&a_full[i], C::kDqWarps);
            mbar_init(&a_empty[i], 1);
        }
        mbar_init(done, 1);
        fence_mbar_init();
        s_abort = 0;
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
    if (warp == C::kProducerWarp) {
        if (lane == 0) {
            const uint64_t pol = policy_evict_first();
            const int64_t Gp = p.Mp >> 3;
            const int pre = nst < S ? nst : S;
            for (int it = 0; it < pre; ++it, ++issued) {
                const int kb0 = it * SKB;
                const int n = nkb - kb0 < SKB ? nkb - kb0 : SKB;
                mbar_arrive_expect_tx(&full[it], static_cast<uint32_t>(n * 4096));
                bulk_g2s_stream(smem + it * C::kStageBytes, p.wq + (rt * p.KB + kb0) * 1024,
                                static_cast<uint32_t>(n * 4096), &full[it], pol);
            }
            pdl_wait();
            for (int it = 0; it < nst; ++it) {
                const int slot = it % S, kb0 = it * SKB;
                const int n = nkb - kb0 < SKB ? nkb - kb0 : SKB;
                unsigned char* st = smem + slot * C::kStageBytes;
                if (it >= S) {
                    if (!mbar_wait(&empty[slot], ((it / S) - 1) & 1, p.status)) {
                        s_abort = 1;
                        break;
                    }
                    mbar_arrive_expect_tx(&full[slot], static_cast<uint32_t>(n * 4096));
                    bulk_g2s_stream(st, p.wq + (rt * p.KB + kb0) * 1024, static_cast<uint32_t>(n * 4096), &full[slot],
                                    pol);
                    ++issued;
                }
                mbar_arrive_expect_tx(&full[slot], static_cast<uint32_t>(n * greal * 1024));
                for (int j = 0; j < n; ++j)
                    bulk_g2s(st + C::kWBytes + j * G * 1024, p.xk + ((kb0 + j) * Gp + (tok0 >> 3)) * 512,
                             static_cast<uint32_t>(greal * 1024), &full[slot]);
            }
        }
    } else if (warp == C::kMmaWarp) {
        // warp-uniform loop, one elected lane issues (the same lane every time, so its commits
        // track all of its MMAs)
        const uint32_t idesc = idesc_f16_f32(128, NT);
        bool ok = true;
        for (int j = 0; j < nkb && ok; ++j) {
            const int s = j / SKB, kbl = j - s * SKB, slot = s % S, b = j % AB;
            if (kbl == 0) ok = mbar_wait(&full[slot], (s / S) & 1, p.status);
            if (ok) ok = mbar_wait(&a_full[b], (j / AB) & 1, p.status);
            ok = __all_sync(0xffffffffu, ok);  // the elected lane below needs the whole warp
            if (!ok) break;
            tc_fence_after();
            const unsigned char* xs = smem + slot * C::kStageBytes + C::kWBytes + kbl * G * 1024;
            if (elect_one()) {
#pragma unroll
                for (int i = 0; i < 4; ++i)
                    tc_mma_ts(tmem, tmem + NT + b * 32 + i * 8, desc_kmajor(xs + 2 * i * 128, 128, 1024), idesc,
                              (j | i) ? 1u : 0u);
                tc_commit(&a_empty[b]);
                if (kbl == SKB - 1 || j == nkb - 1) tc_commit(&empty[slot]);
            }
            __syncwarp();
        }
        if (!ok) s_abort = 1;
        if (elect_one()) tc_commit(done);  // also after an abort, so that the TMEM can be released
        __syncwarp();
    } else {
        const int sp = warp & 3, q = warp >> 2;
        const int tile = 2 * sp + q;
        const uint32_t lane_addr = static_cast<uint32_t>(32 * sp + 16 * q) << 16;
        for (int j = 0; j < nkb; ++j) {
            const int s = j / SKB, kbl = j - s * SKB, slot = s % S, b = j % AB;
            bool ok = true;
            if (kbl == 0 && !mbar_wait(&full[slot], (s / S) & 1, p.status)) ok = false;
            if (ok && j >= AB && !mbar_wait(&a_empty[b], ((j / AB) - 1) & 1, p.status)) ok = false;
            if (!ok) {
                s_abort = 1;
                break;
            }
            tc_fence_after();
            const uint4 wv =
                *reinterpret_cast<const uint4*>(smem + slot * C::kStageBytes + kbl * 4096 + tile * 512 + lane * 16);
            const uint32_t words[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
            for (int st = 0; st < 4; ++st) {
                uint32_t h[4];
                dequant_word(words[st], h);
                tc_st_16x256b(tmem + lane_addr + NT + b * 32 + st * 8, h[0], h[2], h[1], h[3]);
            }
            tc_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&a_full[b]);
        }
        // epilogue: warp q of sub-partition sp owns rows 32 sp + lane and tokens [64 q, 64 q + 64)
        if (mbar_wait(done, 0, p.status) && !s_abort) {
            tc_fence_after();
            pdl_wait();  // y and the routing mask belong to this call's predecessors' stream order
            const int64_t row = rt * 128 + 32 * sp + lane;
            const bool live = row < p.N;
            const float sc = live ? p.scale[row] : 0.0f;
            const int64_t e0 = (live && p.nnz > 0) ? p.rowptr[row] : 0, e1 = (live && p.nnz > 0) ? p.rowptr[row + 1] : 0;
            const uint32_t lane_rows = static_cast<uint32_t>(32 * sp) << 16;
#pragma unroll 1
            for (int cb = 8 * q; cb < 8 * q + 8; ++cb) {
                const int t0 = cb * 8;
                if (t0 >= ntile) break;
                uint32_t d[8];
                tc_ld8(tmem + lane_rows + t0, d);
                tc_wait_ld();
                unsigned rm = 0;
#pragma unroll
                for (int u = 0; u < 8; ++u)
                    if (t0 + u < ntile && (p.route_all || p.mask[tok0 + t0 + u])) rm |= 1u << u;
                float corr[8];
#pragma unroll
                for (int u = 0; u < 8; ++u) corr[u] = 0.0f;
                if (rm) {
                    for (int64_t e = e0; e < e1; ++e) {
                        const int64_t cl = p.col[e];
                        const float v = __fmul_rn(static_cast<float>(p.val[e]), p.ds);
                        const uint16_t* xg = p.xk + xk_index(cl, static_cast<int>(tok0 + t0), static_cast<int>(p.Mp));
#pragma unroll
                        for (int u = 0; u < 8; ++u)
                            if ((rm >> u) & 1u) corr[u] = __fadd_rn(corr[u], __fmul_rn(h2f(xg[u * 8]), v));
                    }
                }
                if (live) {
#pragma unroll
                    for (int u = 0; u < 8; ++u) {
                        if (t0 + u < ntile) {
                            const float v = __fadd_rn(__fmul_rn(__uint_as_float(d[u]), sc), corr[u]);
                            const int64_t oi = (tok0 + t0 + u) * p.N + row;
                            if (p.partial_out) reinterpret_cast<float*>(p.y)[oi] = v;
                            else store_output(p.y, p.y_dtype, oi, v, p.bias, row);
                        }
                    }
                }
            }
        } else {
            s_abort = 1;
        }
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
    if (s_abort && warp == C::kProducerWarp && lane == 0)
        for (int it = issued > S ? issued - S : 0; it < issued; ++it)
            mbar_wait(&full[it % S], (it / S) & 1, nullptr, kDrainNs);
}

int64_t gemm_tile_tokens() { return GemmCfg::NT; }

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
    p.xk = a.xk;
    p.Mp = a.Mp;
    p.M = a.M;
    p.mask = a.mask;
    p.route_all = a.route_all;
    p.N = L.N;
    p.KB = L.KB;
    p.RT = L.Np / 128;
    p.T = (a.M + GemmCfg::NT - 1) / GemmCfg::NT;
    p.y = a.y;
    p.y_dtype = a.y_dtype;
    p.bias = a.bias;
    p.partial_out = a.partial_out;
    p.status = L.status;
    static std::atomic<uint64_t> flags{0};
    int dev = 0;
    cudaGetDevice(&dev);
    const uint64_t bit = 1ull << (dev & 63);
    if (!(flags.load() & bit)) {
        cudaError_t e = cudaFuncSetAttribute(k_ctarq_gemm, cudaFuncAttributeMaxDynamicSharedMemorySize, GemmCfg::kTotal);
        if (e != cudaSuccess) return e;
        flags.fetch_or(bit);
    }
    return launch_pdl(k_ctarq_gemm, dim3(static_cast<unsigned>(p.RT * p.T)), dim3(GemmCfg::kThreads), GemmCfg::kTotal,
                      s, p);
}

}  // namespace sc
