// sc_split.cu -- the exchange step of a row-sharded (tensor-parallel) C-TARQ layer.
//
// A layer whose input columns are split over ranks (o and down of a Qwen2 block) routes on the
// whole token, which no single rank holds.  Each rank therefore computes, from its own slice only:
//   y_base  = (sum over the slice of x * (q - 8)) * s                 (every token, f32)
//   y_delta = sum over the slice's dW entries of x * dW               (every token, f32)
//   stats   = sum x, sum x^2, sum |x| over the slice                  (every token, f64 rounded to f32)
// laid out as one f32 buffer [y_base m*n | y_delta m*n | stats m*3], summed over the ranks by one
// all-reduce; the finalize step then takes the routing decision on the summed sums
// (heuristics.rs:3-14, op.rs:64-73) with the band of the reference's sequential f32 summation,
// widened by the f32 rounding of the partial sums and of their sum over `ranks` values, and
// writes y = f16(y_base + [routed] y_delta) (+ bias after the rounding).  A token whose score lies
// inside the band cannot be replayed in the reference's f32 order (its slices are on other
// ranks): it takes the f64 decision and is counted in `undecided`.
#include "sc_device.cuh"
#include "sc_internal.h"

namespace sc {

// The slice transposed, xt[c][t] (f16 bits; tokens padded with zeros to a multiple of 16), so that one
// dW entry reads the values of 16 tokens with two 16-byte loads.
__global__ void __launch_bounds__(256) k_split_transpose(const void* __restrict__ x, int x_dtype, int64_t m, int64_t K,
                                                         int64_t Tp, uint16_t* __restrict__ xt) {
    pdl_launch_dependents();
    pdl_wait();
    __shared__ uint16_t tile[32][33];
    const int64_t c0 = static_cast<int64_t>(blockIdx.x) * 32, t0 = static_cast<int64_t>(blockIdx.y) * 32;
    const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;  // 32 x 8
    for (int r = ty; r < 32; r += 8) {
        const int64_t t = t0 + r, c = c0 + tx;
        tile[r][tx] = (t < m && c < K) ? x_f16_bits(x, x_dtype, t * K + c) : 0;
    }
    __syncthreads();
    for (int r = ty; r < 32; r += 8) {
        const int64_t c = c0 + r, t = t0 + tx;
        if (c < K && t < Tp) xt[c * Tp + t] = tile[tx][r];
    }
}

// y_delta[t][r] for 8 rows (one warp each) and 16 tokens per CTA.  A row's dW entries are spread over
// its warp's lanes (lane l takes entries l, l + 32, ...: coalesced column and value loads, and rows
// whose counts differ widely -- a percentile threshold keeps the largest errors, which gather in
// the rows with large scales -- cost their own length / 32, not the longest row's length); each lane
// reads the 16 tokens' values of an entry's column from xt with two 16-byte loads, and the lanes'
// sums meet in a fixed xor butterfly (deterministic).
constexpr int kDeltaRowsPerCta = 8;
__global__ void __launch_bounds__(32 * kDeltaRowsPerCta) k_split_delta(const uint16_t* __restrict__ xt, int64_t Tp,
                                                                       int64_t m, const uint32_t* __restrict__ rowptr,
                                                                       const uint16_t* __restrict__ col,
                                                                       const int8_t* __restrict__ val, float ds,
                                                                       int64_t N, float* __restrict__ y_delta) {
    pdl_launch_dependents();
    pdl_wait();
    const int lane = threadIdx.x & 31;
    const int64_t row = static_cast<int64_t>(blockIdx.x) * kDeltaRowsPerCta + (threadIdx.x >> 5);
    const int64_t t0 = static_cast<int64_t>(blockIdx.y) * 16;
    if (row >= N) return;  // the whole warp
    float acc[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) acc[j] = 0.0f;
    const int64_t e1 = rowptr[row + 1];
    for (int64_t e = rowptr[row] + lane; e < e1; e += 32) {
        const int64_t c = col[e];
        const float v = __fmul_rn(static_cast<float>(val[e]), ds);
        const uint4* p = reinterpret_cast<const uint4*>(xt + c * Tp + t0);
        const uint4 a = __ldg(p), b = __ldg(p + 1);
        const uint32_t w[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            acc[2 * j] = __fadd_rn(acc[2 * j], __fmul_rn(h2f(static_cast<uint16_t>(w[j] & 0xFFFFu)), v));
            acc[2 * j + 1] = __fadd_rn(acc[2 * j + 1], __fmul_rn(h2f(static_cast<uint16_t>(w[j] >> 16)), v));
        }
    }
#pragma unroll
    for (int j = 0; j < 16; ++j)
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) acc[j] = __fadd_rn(acc[j], __shfl_xor_sync(0xffffffffu, acc[j], o));
    float out = acc[0];
#pragma unroll
    for (int j = 1; j < 16; ++j)
        if (lane == j) out = acc[j];
    if (lane < 16 && t0 + lane < m) y_delta[(t0 + lane) * N + row] = out;
}

// The slice's router sums of each token (one CTA per token), in f64.
__global__ void __launch_bounds__(256) k_split_stats(const void* __restrict__ x, int x_dtype, int64_t K,
                                                     float* __restrict__ stats) {
    pdl_launch_dependents();
    pdl_wait();
    __shared__ double red[3][8];
    const int64_t t = blockIdx.x;
    double s1 = 0.0, s2 = 0.0, sa = 0.0;
    for (int64_t i = threadIdx.x; i < K; i += 256) {
        const double v = static_cast<double>(h2f(x_f16_bits(x, x_dtype, t * K + i)));
        s1 += v;
        s2 += v * v;
        sa += fabs(v);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        s1 += __shfl_down_sync(0xffffffffu, s1, o);
        s2 += __shfl_down_sync(0xffffffffu, s2, o);
        sa += __shfl_down_sync(0xffffffffu, sa, o);
    }
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (lane == 0) {
        red[0][warp] = s1;
        red[1][warp] = s2;
        red[2][warp] = sa;
    }
    __syncthreads();
    if (threadIdx.x < 3) {
        double s = 0.0;
        for (int w = 0; w < 8; ++w) s += red[threadIdx.x][w];
        stats[t * 3 + threadIdx.x] = static_cast<float>(s);
    }
}

// y = f16(y_base + [routed] y_delta) (+ bias after the rounding), the decision from the summed sums.
__global__ void __launch_bounds__(256) k_split_finalize(const float* __restrict__ exch, int64_t m, int64_t n,
                                                        int64_t full_k, int ranks, float t4, float t8, int route_all,
                                                        void* y, int y_dtype, const float* __restrict__ bias,
                                                        uint8_t* mask_out, uint32_t* undecided) {
    pdl_launch_dependents();
    pdl_wait();
    __shared__ int s_r;
    const int64_t t = blockIdx.x;
    const float* y_base = exch;
    const float* y_delta = exch + m * n;
    const float* stats = exch + 2 * m * n;
    if (threadIdx.x == 0) {
        const double S1 = stats[t * 3], S2 = stats[t * 3 + 1], SA = stats[t * 3 + 2];
        // each rank's f64 sum rounded to f32 (u), then `ranks` f32 values summed in any order
        // ((ranks - 1) u): |S - exact| <= (ranks + 1) u sum|terms| (to first order; 2x slack)
        const double w = 2.0 * (ranks + 1) * 5.9604644775390625e-08;
        double var;
        const int d = route_all ? 1 : route_band(S1, S2, SA, route_consts(full_k), t4, t8, w * SA, w * S2, &var);
        if (d < 0 && undecided) atomicAdd(undecided, 1u);
        const bool r = d < 0 ? route_rule_f64(var, t4, t8) : d == 1;
        s_r = r ? 1 : 0;
        if (mask_out) mask_out[t] = r ? 1 : 0;
    }
    __syncthreads();
    const bool r = s_r != 0;
    for (int64_t i = threadIdx.x; i < n; i += 256) {
        float v = y_base[t * n + i];
        if (r) v = __fadd_rn(v, y_delta[t * n + i]);
        store_output(y, y_dtype, t * n + i, v, bias, i);
    }
}

cudaError_t launch_split_extras(const Layer& L, const void* x, int x_dtype, int64_t m, float* y_delta, float* stats,
                                uint16_t* xt, cudaStream_t s) {
    cudaError_t e = cudaSuccess;
    if (L.nnz > 0) {
        const int64_t Tp = (m + 15) / 16 * 16;
        e = launch_pdl(k_split_transpose, dim3(static_cast<unsigned>((L.K + 31) / 32), static_cast<unsigned>((Tp + 31) / 32)),
                       dim3(256), 0, s, x, x_dtype, m, L.K, Tp, xt);
        if (e == cudaSuccess) {
            const dim3 grid(static_cast<unsigned>((L.N + kDeltaRowsPerCta - 1) / kDeltaRowsPerCta),
                            static_cast<unsigned>(Tp / 16));
            e = launch_pdl(k_split_delta, grid, dim3(32 * kDeltaRowsPerCta), 0, s, static_cast<const uint16_t*>(xt), Tp,
                           m, L.rowptr,
                           L.col, L.val, L.ds, L.N, y_delta);
        }
    } else {
        e = cudaMemsetAsync(y_delta, 0, static_cast<size_t>(m * L.N * 4), s);
    }
    if (e == cudaSuccess)
        e = launch_pdl(k_split_stats, dim3(static_cast<unsigned>(m)), dim3(256), 0, s, x, x_dtype, L.K, stats);
    return e;
}

cudaError_t launch_split_finalize(const Layer& L, const float* exch, int64_t m, int ranks, int route_all, void* y,
                                  int y_dtype, const float* bias, uint8_t* mask_out, uint32_t* undecided,
                                  cudaStream_t s) {
    return launch_pdl(k_split_finalize, dim3(static_cast<unsigned>(m)), dim3(256), 0, s, exch, m, L.N, L.fullK, ranks,
                      L.t4, L.t8, route_all, y, y_dtype, bias, mask_out, undecided);
}

}  // namespace sc
