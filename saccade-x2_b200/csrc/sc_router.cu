// sc_router.cu -- per-token variance router (heuristics.rs:3-14, op.rs:64-73).
//
// One CTA per token.  The CTA widens the token to f16 (bf16 inputs are rounded to f16,
// as the caller's to_dtype(F16) does at model.rs:58-61), stores it into the staged
// activation layout xk used by the GEMV, and reduces sum(x), sum(x^2) and sum(|x|) in
// f64 with warp shuffles.
//
// The reference decides on an f32 variance summed sequentially over k.  The f64 sums
// are (to ~1e-16) the exact sums, and the standard bound on sequential f32 summation
// (|fl(sum) - sum| <= gamma_{k-1} * sum|terms|, gamma_n = n*u/(1-n*u), u = 2^-24)
// bounds how far the reference's f32 score can lie from the f64 one.  When both
// thresholds are farther than that bound the decision is the reference's; otherwise
// the CTA replays the reference's sequential f32 chains for that token in parallel
// (replay_score, sc_device.cuh), and only a threshold within about an ulp of the score
// sends one thread through the whole chain.  The mask therefore equals the reference's
// mask for every token.
//
// The last CTA to finish (completion counter in the workspace) compacts the mask into
// the ascending routed-token list and resets the counter for the next call.
//
// The staged layout xk is the tcgen05 K-major core-matrix layout of sc_device.cuh:
// xk_index, with tokens padded to a multiple of 16 (the MMA N granularity).
#include <atomic>

#include "sc_device.cuh"
#include "sc_internal.h"

namespace sc {

struct RouterKernelArgs {
    const void* x;
    int x_dtype;
    int vec_ok;             // x rows 16-byte aligned: load 8 elements at a time
    int64_t row_stride;
    int64_t Kfull;          // elements per token used for the score
    int64_t col0;           // first column staged into xk (multiple of 64)
    int64_t K;              // columns staged into xk
    int64_t M, Mp, KB;
    float t4, t8;
    int route_all;
    uint16_t* xk;
    uint8_t* mask;
    float* scores;
    int32_t* ridx;
    int32_t* nrouted;
    int32_t* perm;          // nullable: staged order, routed tokens (ascending) then the others
    uint32_t* counter;
    uint32_t* status;
};

template <int kThreads>
__global__ void __launch_bounds__(kThreads) k_router(RouterKernelArgs a) {
    constexpr int kWarps = kThreads / 32;
    __shared__ double red[3][kWarps];
    __shared__ int s_last;
    __shared__ int s_wsum[kWarps];
    __shared__ int s_open;
    __shared__ ReplayShared s_replay;
    extern __shared__ __align__(16) uint16_t s_row[];  // the token as f16 bits [Kfull]
    const int64_t t = blockIdx.x;
    const int tid = threadIdx.x;
    const int lane = tid & 31, warp = tid >> 5;
    // Programmatic dependent launch: let the GEMV start streaming its weights now, but touch
    // x, xk and the routing outputs only once the previous kernel on the stream is complete.
    pdl_launch_dependents();
    pdl_wait();

    if (t >= a.M) {
        // padding tokens (up to a multiple of 16): zero rows in xk
        for (int64_t ch = tid; ch < a.KB * 8; ch += kThreads)
            *reinterpret_cast<uint4*>(&a.xk[xk_index(ch * 8, static_cast<int>(t), static_cast<int>(a.Mp))]) =
                make_uint4(0, 0, 0, 0);
    } else {
        double s1 = 0.0, s2 = 0.0, sa = 0.0;
        const int64_t row_off = t * a.row_stride;
        const int64_t nch = a.Kfull / 8;
        const int64_t ch_lo = a.col0 / 8, ch_hi = (a.col0 + a.K) / 8;
        for (int64_t ch = tid; ch < nch; ch += kThreads) {
            uint16_t h[8];
            if (a.x_dtype == SC_BF16) {
                const __nv_bfloat16* xs = reinterpret_cast<const __nv_bfloat16*>(a.x) + row_off + ch * 8;
                __nv_bfloat16 b[8];
                if (a.vec_ok) {
                    *reinterpret_cast<uint4*>(b) = __ldg(reinterpret_cast<const uint4*>(xs));
                } else {
#pragma unroll
                    for (int j = 0; j < 8; ++j) b[j] = xs[j];
                }
#pragma unroll
                for (int j = 0; j < 8; ++j) h[j] = f32_to_f16_bits(__bfloat162float(b[j]));
            } else {
                const uint16_t* xs = reinterpret_cast<const uint16_t*>(a.x) + row_off + ch * 8;
                if (a.vec_ok) {
                    *reinterpret_cast<uint4*>(h) = __ldg(reinterpret_cast<const uint4*>(xs));
                } else {
#pragma unroll
                    for (int j = 0; j < 8; ++j) h[j] = xs[j];
                }
            }
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const double v = static_cast<double>(h2f(h[j]));
                s1 += v;
                s2 += v * v;
                sa += fabs(v);
            }
            *reinterpret_cast<uint4*>(&s_row[ch * 8]) = *reinterpret_cast<const uint4*>(h);
            if (ch >= ch_lo && ch < ch_hi)
                *reinterpret_cast<uint4*>(&a.xk[xk_index((ch - ch_lo) * 8, static_cast<int>(t), static_cast<int>(a.Mp))]) =
                    *reinterpret_cast<const uint4*>(h);
        }
        // zero the padding columns of the staged slice
        for (int64_t lc = (a.K / 8) + tid; lc < a.KB * 8; lc += kThreads)
            *reinterpret_cast<uint4*>(&a.xk[xk_index(lc * 8, static_cast<int>(t), static_cast<int>(a.Mp))]) =
                make_uint4(0, 0, 0, 0);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            s1 += __shfl_down_sync(0xffffffffu, s1, o);
            s2 += __shfl_down_sync(0xffffffffu, s2, o);
            sa += __shfl_down_sync(0xffffffffu, sa, o);
        }
        if (lane == 0) {
            red[0][warp] = s1;
            red[1][warp] = s2;
            red[2][warp] = sa;
        }
        __syncthreads();
        if (tid == 0) {
            double S1 = 0.0, S2 = 0.0, SA = 0.0;
            for (int w = 0; w < kWarps; ++w) {
                S1 += red[0][w];
                S2 += red[1][w];
                SA += red[2][w];
            }
            double var = 0.0;
            const int d = a.route_all ? 1 : route_band(S1, S2, SA, route_consts(a.Kfull), a.t4, a.t8, 0.0, 0.0, &var);
            s_open = d < 0 ? 1 : 0;
            if (d >= 0) {
                a.mask[t] = static_cast<uint8_t>(d);
                if (a.scores) a.scores[t] = static_cast<float>(var);
            }
        }
        __syncthreads();
        if (s_open) {
            // the f64 score is inside the f32 error band: the CTA replays the reference's chains
            replay_score<kThreads>(s_row, a.Kfull, s_replay);
            if (tid == 0) {
                const bool rl = route_rule_f32(s_replay.lo, a.t4, a.t8), rh = route_rule_f32(s_replay.hi, a.t4, a.t8);
                float score = s_replay.lo;
                bool routed = rl;
                if (rl != rh || !(s_replay.lo == s_replay.lo)) {  // a threshold within an ulp, or inf / nan
                    score = exact_variance_row(s_row, a.Kfull);
                    routed = route_rule_f32(score, a.t4, a.t8);
                }
                a.mask[t] = routed ? 1 : 0;
                if (a.scores) a.scores[t] = score;
            }
        }
    }

    // completion count; the last CTA compacts the mask
    if (tid == 0) {
        __threadfence();
        const unsigned ticket = atomicAdd(a.counter, 1u);
        s_last = (ticket == gridDim.x - 1) ? 1 : 0;
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    int base = 0;
    for (int64_t t0 = 0; t0 < a.M; t0 += kThreads) {
        const int64_t tt = t0 + tid;
        const int v = (tt < a.M) ? (reinterpret_cast<volatile uint8_t*>(a.mask)[tt] != 0) : 0;
        const unsigned bal = __ballot_sync(0xffffffffu, v);
        if (lane == 0) s_wsum[warp] = __popc(bal);
        __syncthreads();
        int pre = 0, tot = 0;
        for (int w = 0; w < kWarps; ++w) {
            if (w < warp) pre += s_wsum[w];
            tot += s_wsum[w];
        }
        pre += __popc(bal & ((1u << lane) - 1u));
        if (v) a.ridx[base + pre] = static_cast<int32_t>(tt);
        base += tot;
        __syncthreads();
    }
    if (a.perm) {
        // the GEMM's token order: perm[0, R) = the routed tokens, then from round_up(R, 8) (a
        // whole 8-token group) the others
        for (int64_t i = tid; i < base; i += kThreads) a.perm[i] = a.ridx[i];
        int ub = (base + 7) & ~7;
        for (int64_t t0 = 0; t0 < a.M; t0 += kThreads) {
            const int64_t tt = t0 + tid;
            const int v = (tt < a.M) ? (reinterpret_cast<volatile uint8_t*>(a.mask)[tt] == 0) : 0;
            const unsigned bal = __ballot_sync(0xffffffffu, v);
            if (lane == 0) s_wsum[warp] = __popc(bal);
            __syncthreads();
            int pre = 0, tot = 0;
            for (int w = 0; w < kWarps; ++w) {
                if (w < warp) pre += s_wsum[w];
                tot += s_wsum[w];
            }
            pre += __popc(bal & ((1u << lane) - 1u));
            if (v) a.perm[ub + pre] = static_cast<int32_t>(tt);
            ub += tot;
            __syncthreads();
        }
    }
    if (tid == 0) {
        *a.nrouted = base;
        *a.counter = 0u;
    }
}

cudaError_t launch_router(const RouterArgs& r, cudaStream_t s) {
    RouterKernelArgs a;
    a.x = r.x;
    a.x_dtype = r.x_dtype;
    a.row_stride = r.x_row_stride;
    a.vec_ok = ((reinterpret_cast<uintptr_t>(r.x) & 15u) == 0 && (r.x_row_stride % 8) == 0) ? 1 : 0;
    a.Kfull = r.x_row_stride;
    a.col0 = r.x_col0;
    a.K = r.K;
    a.M = r.M;
    a.Mp = r.Mp;
    a.KB = r.KB;
    a.t4 = r.t4;
    a.t8 = r.t8;
    a.route_all = r.route_all;
    a.xk = r.xk;
    a.mask = r.mask;
    a.scores = r.scores;
    a.ridx = r.ridx;
    a.nrouted = r.nrouted;
    a.perm = r.perm;
    a.counter = r.counter;
    a.status = r.status;
    // dynamic shared memory: the token row (f16), for the replay of tokens inside the error band
    const size_t row_bytes = static_cast<size_t>((a.Kfull * 2 + 15) / 16 * 16);
    static std::atomic<uint64_t> flags{0};
    int dev = 0;
    cudaGetDevice(&dev);
    const uint64_t bit = 1ull << (dev & 63);
    if (!(flags.load() & bit)) {
        const cudaError_t e =
            cudaFuncSetAttribute(k_router<256>, cudaFuncAttributeMaxDynamicSharedMemorySize, kRouterMaxRowBytes);
        if (e != cudaSuccess) return e;
        flags.fetch_or(bit);
    }
    if (row_bytes > static_cast<size_t>(kRouterMaxRowBytes)) return cudaErrorInvalidValue;
    return launch_pdl(k_router<256>, dim3(static_cast<unsigned>(r.Mp)), dim3(256), row_bytes, s, a);
}

}  // namespace sc
