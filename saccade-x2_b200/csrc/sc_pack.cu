// sc_pack.cu -- the C-TARQ format producer on the GPU.
//
//   sc_percentile_threshold  compress.rs:137-176   k-th smallest reconstruction error by a
//                                                   4-pass, 8-bit radix select over the f32 bits
//   sc_compress              compress.rs:6-129     4-bit pack, f16 row scale, strict '>'
//                                                   threshold, global dW scale, i8 CSR in
//                                                   ascending column order
//   sc_calibrate             calibration.rs:10-47  per-token variance, order statistics
//   sc_variance_heuristic    heuristics.rs:3-14    per-token variance
//
// Every value is produced with the same IEEE f32 operations the reference performs
// (correctly rounded divide, round-half-away-from-zero, no contraction), so the outputs
// are bit-identical to compress_tensor_to_saccade and friends.  These are load-time
// tools; they synchronise the stream to return scalars to the host.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <string>
#include <vector>

#include "sc_device.cuh"
#include "sc_internal.h"

namespace sc {

// Rust `f32 as i32` after round(): saturating, NaN -> 0; then clamp to [lo, hi].
__device__ __forceinline__ int round_clamp(float v, int lo, int hi) {
    const float r = roundf(v);
    int q;
    if (r != r) q = 0;
    else if (r >= 2147483648.0f) q = 2147483647;
    else if (r <= -2147483648.0f) q = -2147483647 - 1;
    else q = static_cast<int>(r);
    return q < lo ? lo : (q > hi ? hi : q);
}

// compress.rs:41-51: scale = max|w| / 7 (1.0 for an all-zero row).  One CTA per row.
__global__ void k_row_scale(const float* __restrict__ w, int64_t n, int64_t k, float* __restrict__ scale) {
    __shared__ float red[32];
    const int64_t r = blockIdx.x;
    float m = 0.0f;
    for (int64_t c = threadIdx.x; c < k; c += blockDim.x) {
        const float a = fabsf(w[r * k + c]);
        if (a > m) m = a;
    }
    for (int o = 16; o > 0; o >>= 1) {
        const float v = __shfl_down_sync(0xffffffffu, m, o);
        if (v > m) m = v;
    }
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
    __syncthreads();
    if (threadIdx.x == 0) {
        float mm = 0.0f;
        for (int i = 0; i < static_cast<int>(blockDim.x >> 5); ++i)
            if (red[i] > mm) mm = red[i];
        scale[r] = mm > 0.0f ? __fdiv_rn(mm, 7.0f) : 1.0f;
    }
}

__device__ __forceinline__ float recon_error(float val, float s, int* q_out) {
    const int q = round_clamp(__fdiv_rn(val, s), -8, 7);
    if (q_out) *q_out = q;
    return __fsub_rn(val, __fmul_rn(static_cast<float>(q), s));
}

// One radix-select pass over |err| > 1e-10 (compress.rs:156-164): histogram of bits
// [shift, shift+8) among keys whose higher bits equal `prefix` under `pmask`.
__global__ void k_err_hist(const float* __restrict__ w, const float* __restrict__ scale, int64_t n, int64_t k,
                           uint32_t prefix, uint32_t pmask, int shift, unsigned long long* __restrict__ hist) {
    __shared__ unsigned int h[256];
    for (int i = threadIdx.x; i < 256; i += blockDim.x) h[i] = 0;
    __syncthreads();
    const int64_t total = n * k;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = i / k;
        const float e = fabsf(recon_error(w[i], scale[r], nullptr));
        if (e > 1e-10f) {
            const uint32_t key = __float_as_uint(e);
            if ((key & pmask) == prefix) atomicAdd(&h[(key >> shift) & 255u], 1u);
        }
    }
    __syncthreads();
    for (int i = threadIdx.x; i < 256; i += blockDim.x)
        if (h[i]) atomicAdd(&hist[i], static_cast<unsigned long long>(h[i]));
}

// compress.rs:54-83 packing plus per-row count of kept errors and their global max.
__global__ void k_pack_count(const float* __restrict__ w, const float* __restrict__ scale, int64_t n, int64_t k,
                             float thr, uint32_t* __restrict__ packed, uint16_t* __restrict__ scale_f16,
                             uint32_t* __restrict__ counts, unsigned int* __restrict__ max_bits) {
    __shared__ unsigned int s_cnt;
    __shared__ float s_max[32];
    const int64_t r = blockIdx.x;
    if (threadIdx.x == 0) s_cnt = 0;
    __syncthreads();
    const float s = scale[r];
    const int64_t kw = k / 8;
    unsigned int cnt = 0;
    float mx = 0.0f;
    for (int64_t p = threadIdx.x; p < kw; p += blockDim.x) {
        uint32_t word = 0;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const float val = w[r * k + p * 8 + j];
            int q;
            const float err = recon_error(val, s, &q);
            word |= static_cast<uint32_t>(q + 8) << (4 * j);
            const float ae = fabsf(err);
            if (ae > thr) {
                if (err != 0.0f) ++cnt;  // compress.rs:94 skips exact zeros when building the CSR
                if (ae > mx) mx = ae;
            }
        }
        packed[r * kw + p] = word;
    }
    for (int o = 16; o > 0; o >>= 1) {
        cnt += __shfl_down_sync(0xffffffffu, cnt, o);
        const float v = __shfl_down_sync(0xffffffffu, mx, o);
        if (v > mx) mx = v;
    }
    if ((threadIdx.x & 31) == 0) {
        atomicAdd(&s_cnt, cnt);
        s_max[threadIdx.x >> 5] = mx;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        float m = 0.0f;
        for (int i = 0; i < static_cast<int>(blockDim.x >> 5); ++i)
            if (s_max[i] > m) m = s_max[i];
        counts[r] = s_cnt;
        if (m > 0.0f) atomicMax(max_bits, __float_as_uint(m));
        scale_f16[r] = f32_to_f16_bits(s);
    }
}

// Exclusive scan of counts[n] into row_ptrs[n+1] by one CTA.
__global__ void k_scan_rows(const uint32_t* __restrict__ counts, int64_t n, uint32_t* __restrict__ row_ptrs) {
    __shared__ uint32_t s_part[1024];
    __shared__ uint32_t s_carry;
    if (threadIdx.x == 0) s_carry = 0;
    __syncthreads();
    for (int64_t base = 0; base < n; base += 1024) {
        const int64_t i = base + threadIdx.x;
        const uint32_t v = i < n ? counts[i] : 0u;
        s_part[threadIdx.x] = v;
        __syncthreads();
        for (int off = 1; off < 1024; off <<= 1) {
            const uint32_t t = threadIdx.x >= static_cast<unsigned>(off) ? s_part[threadIdx.x - off] : 0u;
            __syncthreads();
            s_part[threadIdx.x] += t;
            __syncthreads();
        }
        if (i < n) row_ptrs[i] = s_carry + s_part[threadIdx.x] - v;
        __syncthreads();
        if (threadIdx.x == 1023) s_carry += s_part[1023];
        __syncthreads();
    }
    if (threadIdx.x == 0) row_ptrs[n] = s_carry;
}

// compress.rs:89-105: one warp per row walks the columns in order; ballot ranks keep the
// CSR ascending.  ds = max_err / 127 (compress.rs:87).
__global__ void k_fill_csr(const float* __restrict__ w, const float* __restrict__ scale, int64_t n, int64_t k,
                           float thr, float ds, const uint32_t* __restrict__ row_ptrs, uint32_t* __restrict__ cols,
                           uint8_t* __restrict__ vals) {
    const int64_t r = blockIdx.x * (int64_t)(blockDim.x >> 5) + (threadIdx.x >> 5);
    if (r >= n) return;
    const int lane = threadIdx.x & 31;
    const float s = scale[r];
    uint32_t pos = row_ptrs[r];
    for (int64_t c0 = 0; c0 < k; c0 += 32) {
        const int64_t c = c0 + lane;
        float err = 0.0f;
        bool keep = false;
        if (c < k) {
            err = recon_error(w[r * k + c], s, nullptr);
            keep = fabsf(err) > thr && err != 0.0f;
        }
        const unsigned bal = __ballot_sync(0xffffffffu, keep);
        if (keep) {
            const uint32_t at = pos + __popc(bal & ((1u << lane) - 1u));
            cols[at] = static_cast<uint32_t>(c);
            vals[at] = static_cast<uint8_t>(static_cast<int8_t>(round_clamp(__fdiv_rn(err, ds), -128, 127)));
        }
        pos += __popc(bal);
    }
}

// heuristics.rs:3-14 / calibration.rs:36-45, one thread per token, sequential f32 sums.
__global__ void k_variance_exact(const void* __restrict__ x, int dtype, int64_t m, int64_t k,
                                 float* __restrict__ out) {
    const int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (t >= m) return;
    float sum = 0.0f, sq = 0.0f;
    for (int64_t i = 0; i < k; ++i) {
        float v;
        if (dtype == SC_F32) v = reinterpret_cast<const float*>(x)[t * k + i];
        else if (dtype == SC_BF16)
            v = __half2float(__float2half_rn(__bfloat162float(reinterpret_cast<const __nv_bfloat16*>(x)[t * k + i])));
        else v = __half2float(reinterpret_cast<const __half*>(x)[t * k + i]);
        sum = __fadd_rn(sum, v);
        sq = __fadd_rn(sq, __fmul_rn(v, v));
    }
    const float hd = static_cast<float>(k);
    const float mean = __fdiv_rn(sum, hd);
    out[t] = __fsub_rn(__fdiv_rn(sq, hd), __fmul_rn(mean, mean));
}

// Histogram pass over float keys mapped to an order-preserving u32 (negatives flipped).
__device__ __forceinline__ uint32_t order_key(float f) {
    const uint32_t b = __float_as_uint(f);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

__global__ void k_key_hist(const float* __restrict__ v, int64_t n, uint32_t prefix, uint32_t pmask, int shift,
                           unsigned long long* __restrict__ hist) {
    __shared__ unsigned int h[256];
    for (int i = threadIdx.x; i < 256; i += blockDim.x) h[i] = 0;
    __syncthreads();
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const uint32_t key = order_key(v[i]);
        if ((key & pmask) == prefix) atomicAdd(&h[(key >> shift) & 255u], 1u);
    }
    __syncthreads();
    for (int i = threadIdx.x; i < 256; i += blockDim.x)
        if (h[i]) atomicAdd(&hist[i], static_cast<unsigned long long>(h[i]));
}

struct DevBuf {
    void* p = nullptr;
    ~DevBuf() { cudaFree(p); }
};

// Radix select driver: find the key of rank `rank` (0-based) among the keys a histogram
// pass counts.  `pass(prefix, pmask, shift, hist)` launches one histogram pass.
template <typename PassFn>
static sc_status radix_select(PassFn pass, uint64_t rank, unsigned long long* d_hist, cudaStream_t s,
                              uint32_t* key_out) {
    uint32_t prefix = 0, pmask = 0;
    for (int shift = 24; shift >= 0; shift -= 8) {
        cudaError_t e = cudaMemsetAsync(d_hist, 0, 256 * sizeof(unsigned long long), s);
        if (e == cudaSuccess) e = pass(prefix, pmask, shift, d_hist);
        unsigned long long h[256];
        if (e == cudaSuccess) e = cudaMemcpyAsync(h, d_hist, sizeof(h), cudaMemcpyDeviceToHost, s);
        if (e == cudaSuccess) e = cudaStreamSynchronize(s);
        if (e != cudaSuccess) return cuda_fail(e, "radix select");
        uint64_t acc = 0;
        int b = 0;
        for (; b < 256; ++b) {
            if (acc + h[b] > rank) break;
            acc += h[b];
        }
        if (b == 256) {
            set_error("radix select: rank beyond population");
            return SC_EINVAL;
        }
        rank -= acc;
        prefix |= static_cast<uint32_t>(b) << shift;
        pmask |= 0xFFu << shift;
    }
    *key_out = prefix;
    return SC_OK;
}

static int grid_for(int64_t total) {
    int64_t b = (total + 255) / 256;
    return static_cast<int>(std::min<int64_t>(std::max<int64_t>(b, 1), 148 * 8));
}

// Rust `f32 as usize`: truncation, saturating at 0, NaN -> 0.
static uint64_t f32_to_usize(float f) {
    if (!(f > 0.0f)) return 0;
    if (f >= 18446744073709551616.0f) return UINT64_MAX;
    return static_cast<uint64_t>(f);
}

}  // namespace sc

using namespace sc;

extern "C" {

sc_status sc_variance_heuristic(const void* x, int x_dtype, int64_t m, int64_t k, float* scores, void* stream) {
    if (!x || !scores || m < 0 || k <= 0 || (x_dtype != SC_F16 && x_dtype != SC_BF16 && x_dtype != SC_F32)) {
        set_error("sc_variance_heuristic: bad argument");
        return SC_EINVAL;
    }
    if (m == 0) return SC_OK;
    k_variance_exact<<<static_cast<unsigned>((m + 127) / 128), 128, 0, static_cast<cudaStream_t>(stream)>>>(
        x, x_dtype, m, k, scores);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? SC_OK : cuda_fail(e, "sc_variance_heuristic");
}

sc_status sc_percentile_threshold(const float* w, int64_t n, int64_t k, float target_fill_pct, float* thr_out,
                                  void* stream) {
    if (!w || !thr_out || n <= 0 || k <= 0) {
        set_error("sc_percentile_threshold: bad argument");
        return SC_EINVAL;
    }
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    DevBuf scale, hist;
    cudaError_t e = cudaMalloc(&scale.p, n * 4);
    if (e == cudaSuccess) e = cudaMalloc(&hist.p, 256 * sizeof(unsigned long long));
    if (e != cudaSuccess) return cuda_fail(e, "sc_percentile_threshold: cudaMalloc");
    float* d_scale = static_cast<float*>(scale.p);
    unsigned long long* d_hist = static_cast<unsigned long long*>(hist.p);
    k_row_scale<<<static_cast<unsigned>(n), 256, 0, s>>>(w, n, k, d_scale);
    // population: number of errors > 1e-10 (one pass with an empty prefix mask)
    e = cudaMemsetAsync(d_hist, 0, 256 * sizeof(unsigned long long), s);
    if (e != cudaSuccess) return cuda_fail(e, "sc_percentile_threshold");
    k_err_hist<<<grid_for(n * k), 256, 0, s>>>(w, d_scale, n, k, 0u, 0u, 24, d_hist);
    unsigned long long h[256];
    e = cudaMemcpyAsync(h, d_hist, sizeof(h), cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return cuda_fail(e, "sc_percentile_threshold");
    uint64_t pop = 0;
    for (int i = 0; i < 256; ++i) pop += h[i];
    if (pop == 0) {
        *thr_out = 0.001f;  // compress.rs:167-169
        return SC_OK;
    }
    const float prod = (1.0f - target_fill_pct) * static_cast<float>(pop);
    uint64_t idx = f32_to_usize(prod);
    if (idx > pop - 1) idx = pop - 1;
    uint32_t key = 0;
    sc_status st = radix_select(
        [&](uint32_t prefix, uint32_t pmask, int shift, unsigned long long* hh) {
            k_err_hist<<<grid_for(n * k), 256, 0, s>>>(w, d_scale, n, k, prefix, pmask, shift, hh);
            return cudaGetLastError();
        },
        idx, d_hist, s, &key);
    if (st != SC_OK) return st;
    float thr;
    std::memcpy(&thr, &key, 4);
    *thr_out = thr;
    return SC_OK;
}

sc_status sc_compress(const float* w, int64_t n, int64_t k, float thr, uint32_t* packed, uint16_t* scale_f16,
                      uint32_t* row_ptrs, uint32_t* cols, uint8_t* vals, int64_t capacity, int64_t* nnz_out,
                      uint16_t* ds_out, void* stream) {
    if (!w || n <= 0 || k <= 0 || !packed || !scale_f16 || !row_ptrs || !nnz_out) {
        set_error("sc_compress: bad argument");
        return SC_EINVAL;
    }
    if (k % 8 != 0) {
        set_error("in_features must be a multiple of 8");
        return SC_EINVAL;
    }
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    DevBuf scale, counts, maxb;
    cudaError_t e = cudaMalloc(&scale.p, n * 4);
    if (e == cudaSuccess) e = cudaMalloc(&counts.p, n * 4);
    if (e == cudaSuccess) e = cudaMalloc(&maxb.p, 16);
    if (e == cudaSuccess) e = cudaMemsetAsync(maxb.p, 0, 16, s);
    if (e != cudaSuccess) return cuda_fail(e, "sc_compress: setup");
    float* d_scale = static_cast<float*>(scale.p);
    k_row_scale<<<static_cast<unsigned>(n), 256, 0, s>>>(w, n, k, d_scale);
    k_pack_count<<<static_cast<unsigned>(n), 128, 0, s>>>(w, d_scale, n, k, thr, packed, scale_f16,
                                                          static_cast<uint32_t*>(counts.p),
                                                          static_cast<unsigned int*>(maxb.p));
    k_scan_rows<<<1, 1024, 0, s>>>(static_cast<uint32_t*>(counts.p), n, row_ptrs);
    uint32_t nnz = 0, mbits = 0;
    e = cudaGetLastError();
    if (e == cudaSuccess) e = cudaMemcpyAsync(&nnz, row_ptrs + n, 4, cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaMemcpyAsync(&mbits, maxb.p, 4, cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return cuda_fail(e, "sc_compress: pack");
    *nnz_out = nnz;
    float mx;
    std::memcpy(&mx, &mbits, 4);
    const float ds = mx > 0.0f ? mx / 127.0f : 1.0f;  // compress.rs:87
    if (ds_out) {
        __half hd = __float2half_rn(ds);
        std::memcpy(ds_out, &hd, 2);
    }
    if (!cols) return SC_OK;
    if (!vals || capacity < static_cast<int64_t>(nnz)) {
        set_error("sc_compress: CSR capacity " + std::to_string(capacity) + " < nnz " + std::to_string(nnz));
        return SC_ENOMEM;
    }
    if (nnz > 0) {
        k_fill_csr<<<static_cast<unsigned>((n + 7) / 8), 256, 0, s>>>(w, d_scale, n, k, thr, ds, row_ptrs, cols, vals);
        e = cudaGetLastError();
        if (e == cudaSuccess) e = cudaStreamSynchronize(s);
        if (e != cudaSuccess) return cuda_fail(e, "sc_compress: fill");
    }
    return SC_OK;
}

sc_status sc_calibrate(const void* acts, int dtype, int64_t n, int64_t k, float pct_t4, float pct_t8, float* t4_out,
                       float* t8_out, void* stream) {
    if (!acts || n <= 0 || k <= 0 || !t4_out || !t8_out || (dtype != SC_F32 && dtype != SC_F16)) {
        set_error("sc_calibrate: bad argument (needs at least one token)");
        return SC_EINVAL;
    }
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    DevBuf var, hist;
    cudaError_t e = cudaMalloc(&var.p, n * 4);
    if (e == cudaSuccess) e = cudaMalloc(&hist.p, 256 * sizeof(unsigned long long));
    if (e != cudaSuccess) return cuda_fail(e, "sc_calibrate: cudaMalloc");
    float* d_var = static_cast<float*>(var.p);
    k_variance_exact<<<static_cast<unsigned>((n + 127) / 128), 128, 0, s>>>(acts, dtype, n, k, d_var);
    const float pcts[2] = {pct_t4, pct_t8};
    float outs[2];
    for (int j = 0; j < 2; ++j) {
        // calibration.rs:41-42: idx = min(round(n * pct) as usize, n - 1)
        const float prod = static_cast<float>(n) * pcts[j];
        const float rr = std::round(prod);  // half away from zero, like f32::round
        uint64_t idx = f32_to_usize(rr);
        if (idx > static_cast<uint64_t>(n - 1)) idx = static_cast<uint64_t>(n - 1);
        uint32_t key = 0;
        sc_status st = radix_select(
            [&](uint32_t prefix, uint32_t pmask, int shift, unsigned long long* hh) {
                k_key_hist<<<grid_for(n), 256, 0, s>>>(d_var, n, prefix, pmask, shift, hh);
                return cudaGetLastError();
            },
            idx, static_cast<unsigned long long*>(hist.p), s, &key);
        if (st != SC_OK) return st;
        const uint32_t b = (key & 0x80000000u) ? (key & 0x7FFFFFFFu) : ~key;
        std::memcpy(&outs[j], &b, 4);
    }
    *t4_out = outs[0];
    *t8_out = outs[1];
    return SC_OK;
}

}  // extern "C"
