// sc_decode.cu -- C-TARQ decode kernels (few tokens per call).
//
// k_decode_tc: the fast path.  One CTA owns 128 output rows (eight 16-row tiles) and a
// contiguous range of 64-column blocks (split-K across CTAs when there are few rows).
//   warp 8 (producer)   : one lane streams the weight tiles and the staged activations
//                         into an 8-stage shared-memory ring with non-multicast bulk copies
//                         (cp.async.bulk + mbarrier complete_tx); weights carry an L2
//                         evict-first hint since each byte is read exactly once.
//   warps 0-7 (MMA)     : one 16-row tile each; per 64-column block a lane reads 16 bytes
//                         (four packed words), turns each word into an A fragment of exact
//                         f16 integers q-8 (sc_device.cuh: dequant_word) and issues
//                         m16n8k16 MMAs against the activations, f32 accumulation in registers.
//                         The row scale is applied once at the end, as op.rs:148 does.
//   warps 9-12 (dW)     : one output row per lane; while the MMA warps stream, they walk the
//                         row's CSR dW entries inside this CTA's column range and accumulate
//                         x * (i8 * scale) for the routed tokens (op.rs:152-170).
// Epilogue: y = f16(acc * s + dW) (+ bias), or for split-K the last CTA of a row tile sums
// the per-split partials in split order (deterministic) and stores.
//
// k_decode_exact: SC_MODE_EXACT.  One thread per row pair of a tile replays op.rs exactly:
// four f32 accumulators fed in the reference's order with single-rounding
// f16 x f16 -> f32 FMAs (the products are exact), ((a0+a1)+a2)+a3 then * scale, then the
// dW entries in ascending column order with separate multiply and add.  Y is
// bit-identical to the reference's cpu_fwd.  Each accumulator is a K/4-long dependent
// chain, so this path is latency-bound; it exists for verification.
#include <atomic>

#include "sc_device.cuh"
#include "sc_internal.h"

namespace sc {

constexpr int kMmaWarps = 8;
constexpr int kDeltaWarps = 4;
constexpr int kProducerWarp = kMmaWarps;
constexpr int kThreadsTC = (kMmaWarps + 1 + kDeltaWarps) * 32;  // 416
constexpr int kSKB = 2;      // 64-column blocks per stage
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
    int64_t N, K, KB, NT16;
    void* y;
    int y_dtype;
    const float* bias;
    int partial_out;
    float* ws_partial;
    uint32_t* ws_rtcount;
    int ksplit;
    uint32_t* status;
};

template <int NG>
struct TCSmem {
    // 8 stages (80 KB) for one token group and 6 (72 KB) for two keep two CTAs per SM;
    // four groups take 8 stages (128 KB) and one CTA per SM.
    static constexpr int kStages = NG == 2 ? 6 : 8;
    static constexpr int kWBytes = kMmaWarps * kSKB * 512;    // weights per stage
    static constexpr int kXBytes = kSKB * NG * 1024;          // activations per stage
    static constexpr int kStageBytes = kWBytes + kXBytes;
    static constexpr int kTok = NG * 8;
    static constexpr int kLd = kTok + 1;                      // padded row of acc/corr tiles
    static constexpr int kRingBytes = kStages * kStageBytes;
    static constexpr int kAccOff = kRingBytes;
    static constexpr int kCorrOff = kAccOff + 128 * kLd * 4;
    static constexpr int kBarOff = kCorrOff + 128 * kLd * 4;
    static constexpr int kTotal = kBarOff + 2 * kStages * 8 + 16;
};

__device__ __forceinline__ int64_t lower_bound_u16(const uint16_t* col, int64_t lo, int64_t hi, int64_t key) {
    while (lo < hi) {
        const int64_t mid = (lo + hi) >> 1;
        if (static_cast<int64_t>(col[mid]) < key) lo = mid + 1;
        else hi = mid;
    }
    return lo;
}

template <int NG>
__global__ void __launch_bounds__(kThreadsTC, NG <= 2 ? 2 : 1) k_decode_tc(TCParams p) {
    using S = TCSmem<NG>;
    constexpr int kStages = S::kStages;
    extern __shared__ __align__(128) unsigned char smem[];
    float* accbuf = reinterpret_cast<float*>(smem + S::kAccOff);
    float* corrbuf = reinterpret_cast<float*>(smem + S::kCorrOff);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + S::kBarOff);
    uint64_t* empty = full + kStages;
    __shared__ int s_last;
    __shared__ int s_abort;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int64_t rt = blockIdx.x / p.ksplit;
    const int split = static_cast<int>(blockIdx.x - rt * p.ksplit);
    const int64_t kb_begin = (p.KB * split) / p.ksplit;
    const int64_t kb_end = (p.KB * (split + 1)) / p.ksplit;
    const int nst = static_cast<int>((kb_end - kb_begin + kSKB - 1) / kSKB);
    const int64_t tile0 = rt * kMmaWarps;
    const int ntiles = static_cast<int>(imin64(kMmaWarps, p.NT16 - tile0));

    if (tid == 0) {
        for (int i = 0; i < kStages; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], kMmaWarps);
        }
        fence_mbar_init();
        s_abort = 0;
    }
    for (int i = tid; i < 128 * S::kLd; i += kThreadsTC) corrbuf[i] = 0.0f;
    __syncthreads();

    int issued = 0;  // producer lane 0: stages whose copies were issued
    if (warp == kProducerWarp) {
        if (lane == 0) {
            const uint64_t pol = policy_evict_first();
            for (int it = 0; it < nst; ++it, ++issued) {
                const int slot = it % kStages;
                if (it >= kStages) {
                    if (!mbar_wait(&empty[slot], ((it / kStages) - 1) & 1, p.status)) {
                        s_abort = 1;
                        break;
                    }
                }
                const int64_t kb0 = kb_begin + static_cast<int64_t>(it) * kSKB;
                const int nkb = static_cast<int>(imin64(kSKB, kb_end - kb0));
                unsigned char* st = smem + slot * S::kStageBytes;
                const uint32_t bytes = static_cast<uint32_t>(ntiles * nkb * 512 + nkb * NG * 1024);
                mbar_arrive_expect_tx(&full[slot], bytes);
                for (int w = 0; w < ntiles; ++w) {
                    const uint32_t* src = p.wq + ((tile0 + w) * p.KB + kb0) * 128;
                    bulk_g2s_stream(st + w * kSKB * 512, src, static_cast<uint32_t>(nkb * 512), &full[slot], pol);
                }
                for (int j = 0; j < nkb; ++j) {
                    const uint16_t* src = p.xk + ((kb0 + j) * p.Mp + p.tok0) * 64;
                    bulk_g2s(st + S::kWBytes + j * NG * 1024, src, NG * 1024, &full[slot]);
                }
            }
        }
    } else if (warp < kMmaWarps) {
        float acc[NG][4];
#pragma unroll
        for (int g = 0; g < NG; ++g)
#pragma unroll
            for (int i = 0; i < 4; ++i) acc[g][i] = 0.0f;
        const bool valid = warp < ntiles;
        const int tl = lane >> 2, c = lane & 3;
        for (int it = 0; it < nst; ++it) {
            const int slot = it % kStages;
            if (!mbar_wait(&full[slot], (it / kStages) & 1, p.status)) {
                s_abort = 1;
                break;
            }
            const int64_t kb0 = kb_begin + static_cast<int64_t>(it) * kSKB;
            const int nkb = static_cast<int>(imin64(kSKB, kb_end - kb0));
            const unsigned char* st = smem + slot * S::kStageBytes;
            if (valid) {
                for (int j = 0; j < nkb; ++j) {
                    const uint4 wv = *reinterpret_cast<const uint4*>(st + warp * kSKB * 512 + j * 512 + lane * 16);
                    const uint32_t words[4] = {wv.x, wv.y, wv.z, wv.w};
                    const uint32_t* xw = reinterpret_cast<const uint32_t*>(st + S::kWBytes + j * NG * 1024);
#pragma unroll
                    for (int s = 0; s < 4; ++s) {
                        uint32_t a[4];
                        dequant_word(words[s], a);
#pragma unroll
                        for (int g = 0; g < NG; ++g) {
                            const uint32_t* xr = xw + g * 256 + tl * 32;
                            const uint32_t b0 = xr[((2 * s) ^ tl) * 4 + c];
                            const uint32_t b1 = xr[((2 * s + 1) ^ tl) * 4 + c];
                            mma_16816(acc[g], a, b0, b1);
                        }
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[slot]);
        }
        if (valid) {
            const int r0 = warp * 16 + tl;
#pragma unroll
            for (int g = 0; g < NG; ++g) {
                const int t0 = g * 8 + 2 * c;
                accbuf[r0 * S::kLd + t0] = acc[g][0];
                accbuf[r0 * S::kLd + t0 + 1] = acc[g][1];
                accbuf[(r0 + 8) * S::kLd + t0] = acc[g][2];
                accbuf[(r0 + 8) * S::kLd + t0 + 1] = acc[g][3];
            }
        }
    } else {
        // dW warps: one output row per lane, entries of this CTA's column range
        const int rl = (warp - kMmaWarps - 1) * 32 + lane;
        const int64_t row = rt * 128 + rl;
        uint32_t routed = 0;
        for (int tt = 0; tt < p.ntok; ++tt)
            if (p.route_all || p.mask[p.tok0 + tt]) routed |= 1u << tt;
        if (routed != 0 && row < p.N && p.nnz > 0) {
            const int64_t lo = p.rowptr[row], hi = p.rowptr[row + 1];
            const int64_t e0 = lower_bound_u16(p.col, lo, hi, kb_begin * 64);
            const int64_t e1 = lower_bound_u16(p.col, e0, hi, kb_end * 64);
            float corr[S::kTok];
#pragma unroll
            for (int tt = 0; tt < S::kTok; ++tt) corr[tt] = 0.0f;
            for (int64_t e = e0; e < e1; ++e) {
                const int64_t cc = p.col[e];
                const float v = __fmul_rn(static_cast<float>(p.val[e]), p.ds);
#pragma unroll
                for (int tt = 0; tt < S::kTok; ++tt) {
                    if (tt < p.ntok && ((routed >> tt) & 1u)) {
                        const int t = static_cast<int>(p.tok0 + tt);
                        const float xv = h2f(p.xk[xk_index(cc, t, static_cast<int>(p.Mp))]);
                        corr[tt] = __fadd_rn(corr[tt], __fmul_rn(xv, v));
                    }
                }
            }
#pragma unroll
            for (int tt = 0; tt < S::kTok; ++tt) corrbuf[rl * S::kLd + tt] = corr[tt];
        }
    }
    __syncthreads();
    if (s_abort) {
        // A wait ran out (already recorded).  Let this CTA's own bulk copies land before its
        // shared memory is released: bounded waits on the last stages that were issued.
        if (warp == kProducerWarp && lane == 0) {
            for (int it = issued > kStages ? issued - kStages : 0; it < issued; ++it)
                mbar_wait(&full[it % kStages], (it / kStages) & 1, nullptr, kDrainNs);
        }
        return;
    }

    // epilogue
    const int cnt = 128 * p.ntok;
    if (p.ksplit == 1) {
        for (int i = tid; i < cnt; i += kThreadsTC) {
            const int rl = i & 127, tt = i >> 7;
            const int64_t row = rt * 128 + rl;
            if (row >= p.N) continue;
            const float v = __fadd_rn(__fmul_rn(accbuf[rl * S::kLd + tt], p.scale[row]), corrbuf[rl * S::kLd + tt]);
            const int64_t oi = (p.tok0 + tt) * p.N + row;
            if (p.partial_out) reinterpret_cast<float*>(p.y)[oi] = v;
            else store_output(p.y, p.y_dtype, oi, v, p.bias, row);
        }
        return;
    }
    float* part = p.ws_partial + (rt * p.ksplit) * 128 * kMaxChunkTokens;
    for (int i = tid; i < cnt; i += kThreadsTC) {
        const int rl = i & 127, tt = i >> 7;
        const int64_t row = rt * 128 + rl;
        const float v = row < p.N ? __fadd_rn(__fmul_rn(accbuf[rl * S::kLd + tt], p.scale[row]),
                                              corrbuf[rl * S::kLd + tt])
                                  : 0.0f;
        part[(split * 128 + rl) * kMaxChunkTokens + tt] = v;
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) {
        const unsigned ticket = atomicAdd(&p.ws_rtcount[rt], 1u);
        s_last = (ticket == static_cast<unsigned>(p.ksplit - 1)) ? 1 : 0;
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    for (int i = tid; i < cnt; i += kThreadsTC) {
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

template <int NG>
static cudaError_t launch_tc_ng(const TCParams& p, int64_t RT, cudaStream_t s) {
    const int smem = TCSmem<NG>::kTotal;
    // The shared-memory opt-in is per device; remember it per ordinal.
    static std::atomic<uint64_t> attr_set{0};
    int dev = 0;
    cudaGetDevice(&dev);
    const uint64_t bit = 1ull << (dev & 63);
    if (!(attr_set.load() & bit)) {
        cudaError_t e = cudaFuncSetAttribute(k_decode_tc<NG>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return e;
        attr_set.fetch_or(bit);
    }
    k_decode_tc<NG><<<static_cast<unsigned>(RT * p.ksplit), kThreadsTC, smem, s>>>(p);
    return cudaGetLastError();
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
    p.NT16 = L.Np / 16;
    p.y = a.y;
    p.y_dtype = a.y_dtype;
    p.bias = a.bias;
    p.partial_out = a.partial_out;
    p.ws_partial = a.ws_partial;
    p.ws_rtcount = a.ws_rtcount;
    p.ksplit = a.ksplit;
    p.status = L.status;
    const int64_t RT = (L.Np + 127) / 128;
    const int ng = static_cast<int>((a.ntok + 7) / 8);
    switch (ng) {
        case 1: return launch_tc_ng<1>(p, RT, s);
        case 2: return launch_tc_ng<2>(p, RT, s);
        case 3:
        case 4: return launch_tc_ng<4>(p, RT, s);
        default: return cudaErrorInvalidValue;
    }
}

// ---------------------------------------------------------------------------------------
// Exact (reference-order) kernel

constexpr int kExactThreads = 128;  // 16 tiles of 16 rows (8 row pairs each) per CTA
constexpr int kExactTok = 4;        // tokens per pass over the weights

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
    int64_t N, K, KB, NT16;
    void* y;
    int y_dtype;
    const float* bias;
    int partial_out;
};

__device__ __forceinline__ uint16_t half_sel(uint32_t h2, int e) { return e ? hi16(h2) : lo16(h2); }

// Weight (q-8 as f16 bits) of row (g or g+8 by rh) at column offset i (0..15) of a kstep,
// given the 4 lanes' dequantised registers hq[c][0..3].
__device__ __forceinline__ uint16_t wq_at(const uint32_t (&hq)[4][4], int rh, int i) {
    const int hi8 = i >> 3, ii = i & 7;
    const int c = ii >> 1, e = ii & 1;
    return half_sel(hq[c][(hi8 ? 2 : 0) + rh], e);
}

__global__ void __launch_bounds__(kExactThreads) k_decode_exact(ExactParams p) {
    const int64_t gtid = blockIdx.x * (int64_t)kExactThreads + threadIdx.x;
    const int64_t tile = gtid >> 3;
    const int gid = static_cast<int>(gtid & 7);
    if (tile >= p.NT16) return;
    const int64_t rowA = tile * 16 + gid, rowB = rowA + 8;
    const int64_t kw = p.K / 8;  // valid 8-column groups
    const int Mp = static_cast<int>(p.Mp);

    for (int tb = 0; tb < p.ntok; tb += kExactTok) {
        const int nt = min(kExactTok, p.ntok - tb);
        float a[2][4][kExactTok];
        float accb[2][kExactTok];  // bypass: one accumulator per row (op.rs:39-48)
#pragma unroll
        for (int r = 0; r < 2; ++r)
#pragma unroll
            for (int t = 0; t < kExactTok; ++t) {
                accb[r][t] = 0.0f;
#pragma unroll
                for (int j = 0; j < 4; ++j) a[r][j][t] = 0.0f;
            }
        // bypass merges the dW entries into the dense weight while walking the columns
        int64_t bp[2] = {0, 0}, bpe[2] = {0, 0};
        float sc[2] = {0.0f, 0.0f};
        if (p.bypass) {
            const int64_t rows[2] = {rowA, rowB};
#pragma unroll
            for (int r = 0; r < 2; ++r) {
                if (rows[r] < p.N) {
                    sc[r] = p.scale[rows[r]];
                    if (p.nnz > 0) {
                        bp[r] = p.rowptr[rows[r]];
                        bpe[r] = p.rowptr[rows[r] + 1];
                    }
                }
            }
        }
        for (int64_t kb = 0; kb < p.KB; ++kb) {
            const uint4* src = reinterpret_cast<const uint4*>(p.wq + ((tile * p.KB + kb) * 32 + gid * 4) * 4);
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
                const int64_t k0 = kb * 64 + 16 * s;
                const int64_t grp0 = k0 >> 3;  // groups grp0 (cols k0..k0+7) and grp0+1
                if (grp0 >= kw) break;
                const bool second = (grp0 + 1) < kw;
                uint32_t hq[4][4];
#pragma unroll
                for (int c = 0; c < 4; ++c) dequant_word(w[c][s], hq[c]);
                if (p.bypass) {
#pragma unroll
                    for (int r = 0; r < 2; ++r)
                        while (bp[r] < bpe[r] && static_cast<int64_t>(p.col[bp[r]]) < k0) ++bp[r];
                }
#pragma unroll
                for (int t = 0; t < kExactTok; ++t) {
                    if (t >= nt) break;
                    const int tok = static_cast<int>(p.tok0 + tb + t);
                    uint16_t xv[16];
                    const uint16_t* xr = p.xk + (kb * Mp + tok) * 64;
                    *reinterpret_cast<uint4*>(&xv[0]) = *reinterpret_cast<const uint4*>(xr + (((2 * s) ^ (tok & 7)) * 8));
                    *reinterpret_cast<uint4*>(&xv[8]) =
                        *reinterpret_cast<const uint4*>(xr + (((2 * s + 1) ^ (tok & 7)) * 8));
                    if (!p.bypass) {
#pragma unroll
                        for (int r = 0; r < 2; ++r) {
#pragma unroll
                            for (int j = 0; j < 4; ++j) {
                                float v = a[r][j][t];
                                v = fma_f16_f32(xv[j], wq_at(hq, r, j), v);
                                v = fma_f16_f32(xv[j + 4], wq_at(hq, r, j + 4), v);
                                if (second) {
                                    v = fma_f16_f32(xv[j + 8], wq_at(hq, r, j + 8), v);
                                    v = fma_f16_f32(xv[j + 12], wq_at(hq, r, j + 12), v);
                                }
                                a[r][j][t] = v;
                            }
                        }
                    } else {
                        const int lim = second ? 16 : 8;
#pragma unroll
                        for (int r = 0; r < 2; ++r) {
                            int64_t e = bp[r];  // first dW entry of this row at or after column k0
                            for (int i = 0; i < lim; ++i) {
                                const int64_t colg = k0 + i;
                                float wv = __fmul_rn(h2f(wq_at(hq, r, i)), sc[r]);
                                while (e < bpe[r] && static_cast<int64_t>(p.col[e]) < colg) ++e;
                                if (e < bpe[r] && static_cast<int64_t>(p.col[e]) == colg)
                                    wv = __fadd_rn(wv, __fmul_rn(static_cast<float>(p.val[e]), p.ds));
                                accb[r][t] = __fadd_rn(accb[r][t], __fmul_rn(h2f(xv[i]), wv));
                            }
                        }
                    }
                }
            }
        }
        const int64_t rows[2] = {rowA, rowB};
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            if (rows[r] >= p.N) continue;
            const float s_r = p.scale[rows[r]];
            const int64_t lo = p.nnz > 0 ? p.rowptr[rows[r]] : 0, hi = p.nnz > 0 ? p.rowptr[rows[r] + 1] : 0;
            for (int t = 0; t < nt; ++t) {
                const int64_t tok = p.tok0 + tb + t;
                float acc;
                if (p.bypass) {
                    acc = accb[r][t];
                } else {
                    acc = __fmul_rn(__fadd_rn(__fadd_rn(__fadd_rn(a[r][0][t], a[r][1][t]), a[r][2][t]), a[r][3][t]),
                                    s_r);
                    if (p.route_all || p.mask[tok]) {
                        for (int64_t e = lo; e < hi; ++e) {
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
    p.NT16 = L.Np / 16;
    p.y = a.y;
    p.y_dtype = a.y_dtype;
    p.bias = a.bias;
    p.partial_out = a.partial_out;
    const int64_t threads = p.NT16 * 8;
    const int64_t blocks = (threads + kExactThreads - 1) / kExactThreads;
    k_decode_exact<<<static_cast<unsigned>(blocks), kExactThreads, 0, s>>>(p);
    return cudaGetLastError();
}

// ---------------------------------------------------------------------------------------

__global__ void k_finalize(const float* __restrict__ acc, int64_t total, int64_t n, void* y, int y_dtype,
                           const float* bias) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x)
        store_output(y, y_dtype, i, acc[i], bias, i % n);
}

cudaError_t launch_finalize(const float* acc, int64_t m, int64_t n, void* y, int y_dtype, const float* bias,
                            cudaStream_t s) {
    const int64_t total = m * n;
    if (total == 0) return cudaSuccess;
    int64_t blocks = (total + 255) / 256;
    if (blocks > 148 * 16) blocks = 148 * 16;
    k_finalize<<<static_cast<unsigned>(blocks), 256, 0, s>>>(acc, total, n, y, y_dtype, bias);
    return cudaGetLastError();
}

}  // namespace sc
