// sc_model.cu -- the Qwen2 decoder glue around the C-TARQ linears (saccade-runner/src/model.rs),
// as sm_100a kernels: embedding gather, residual add + RMSNorm, RoPE + KV-cache append, GQA
// attention over the cache, SiLU(gate) * up.  Every tensor is f32 except the inputs of the linears,
// which the kernels write as f16 directly (the projection layer's to_dtype(F16), model.rs:58-61).
//
// The KV cache is f32, like the reference's (model.rs:228-236 concatenates f32 tensors), laid out
// [slot][kv_head][position][head_dim] so that one (slot, kv head) is a contiguous stream.
#include <cuda_fp16.h>

#include <atomic>
#include <string>

#include "saccade_qwen2.h"
#include "sc_device.cuh"
#include "sc_internal.h"

namespace sc {

// exp of an f32 value evaluated in f64 and rounded once to f32: the correctly rounded result but for
// inputs whose f64 value lies within an f64 rounding error of an f32 halfway point, so that a host
// computing exp in f64 and rounding to f32 gets the same f32.
__device__ __forceinline__ float exp_f32(float x) { return static_cast<float>(exp(static_cast<double>(x))); }

// ---------------------------------------------------------------- embedding (model.rs:512)
__global__ void k_embed(const int64_t* __restrict__ ids, const uint16_t* __restrict__ table, int64_t hidden,
                        int64_t vocab, float* __restrict__ out, uint32_t* status) {
    pdl_launch_dependents();
    pdl_wait();
    const int64_t t = blockIdx.x;
    int64_t id = ids[t];
    if (id < 0 || id >= vocab) {
        record_error(status, DEV_BAD_INDEX);
        id = 0;
    }
    const uint16_t* row = table + id * hidden;
    for (int64_t h = threadIdx.x; h < hidden; h += blockDim.x) out[t * hidden + h] = h2f(row[h]);
}

// ---------------------------------------------------------------- residual add + RMSNorm (model.rs:92-98)
// resid += delta (when given); out = f16((resid / sqrt(mean(resid^2) + eps)) * w).  The mean is a
// fixed-order f32 sum: thread t adds elements t, t + 256, ... in order, then thread 0 adds the 256
// partial sums in order.
constexpr int kNormThreads = 256;
constexpr int64_t kNormMaxHidden = 16384;

// One token's row: x += d (when given) in place, the f32 row into xs (shared), the denominator
// sqrt(mean(x^2) + eps) returned to every thread.  Each thread issues its loads 8 at a time and then
// adds in element order.
__device__ __forceinline__ float norm_stage(float* __restrict__ x, const float* __restrict__ d, int64_t hidden, float eps,
                                            float* xs, float* part, float* s_denom) {
    const int tid = threadIdx.x;
    float acc = 0.0f;
    for (int64_t h0 = tid; h0 < hidden; h0 += kNormThreads * 8) {
        float v[8], dv[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int64_t h = h0 + j * kNormThreads;
            v[j] = h < hidden ? x[h] : 0.0f;
            dv[j] = (d && h < hidden) ? d[h] : 0.0f;
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int64_t h = h0 + j * kNormThreads;
            if (h < hidden) {
                float vv = v[j];
                if (d) {
                    vv = __fadd_rn(vv, dv[j]);
                    x[h] = vv;
                }
                xs[h] = vv;
                acc = __fadd_rn(acc, __fmul_rn(vv, vv));
            }
        }
    }
    part[tid] = acc;
    __syncthreads();
    if (tid == 0) {
        float sum = 0.0f;
        for (int i = 0; i < kNormThreads; ++i) sum = __fadd_rn(sum, part[i]);
        const float var = __fdiv_rn(sum, static_cast<float>(hidden));
        *s_denom = __fsqrt_rn(__fadd_rn(var, eps));
    }
    __syncthreads();
    return *s_denom;
}

__global__ void __launch_bounds__(kNormThreads) k_add_rmsnorm(float* __restrict__ resid, const float* __restrict__ delta,
                                                               const float* __restrict__ w, int64_t hidden, float eps,
                                                               void* __restrict__ out, int out_f32) {
    extern __shared__ __align__(16) float s_x[];  // the token's f32 row [hidden]
    __shared__ float part[kNormThreads];
    __shared__ float s_denom;
    pdl_launch_dependents();
    pdl_wait();
    const int64_t t = blockIdx.x;
    const float d = norm_stage(resid + t * hidden, delta ? delta + t * hidden : nullptr, hidden, eps, s_x, part, &s_denom);
#pragma unroll 4
    for (int64_t h = threadIdx.x; h < hidden; h += kNormThreads) {
        const float y = __fmul_rn(__fdiv_rn(s_x[h], d), w[h]);
        if (out_f32) static_cast<float*>(out)[t * hidden + h] = y;
        else static_cast<uint16_t*>(out)[t * hidden + h] = f32_to_f16_bits(y);
    }
}

// The same f16 output, kept in shared memory too, then the token routed for the next linears.
__global__ void __launch_bounds__(kNormThreads) k_add_rmsnorm_route(float* __restrict__ resid,
                                                                     const float* __restrict__ delta,
                                                                     const float* __restrict__ w, int64_t hidden,
                                                                     float eps, uint16_t* __restrict__ out,
                                                                     TokenRoute r) {
    extern __shared__ __align__(16) unsigned char s_dyn[];  // f32 row [hidden], then the f16 row [hidden]
    __shared__ float part[kNormThreads];
    __shared__ float s_denom;
    float* xs = reinterpret_cast<float*>(s_dyn);
    uint16_t* row = reinterpret_cast<uint16_t*>(s_dyn + hidden * 4);
    pdl_launch_dependents();
    pdl_wait();
    const int t = blockIdx.x;
    const float d = norm_stage(resid + t * hidden, delta ? delta + t * hidden : nullptr, hidden, eps, xs, part, &s_denom);
    double s1 = 0.0, s2 = 0.0, sa = 0.0;
#pragma unroll 4
    for (int64_t h = threadIdx.x; h < hidden; h += kNormThreads) {
        const uint16_t hb = f32_to_f16_bits(__fmul_rn(__fdiv_rn(xs[h], d), w[h]));
        out[t * hidden + h] = hb;
        row[h] = hb;
        const double v = static_cast<double>(h2f(hb));
        s1 += v;
        s2 += v * v;
        sa += fabs(v);
    }
    route_row<kNormThreads>(r, t, row, hidden, s1, s2, sa);
}

// ---------------------------------------------------------------- RoPE + KV append (model.rs:111-154, 228-236)
// q [T][nh][hd], k, v [T][nkv][hd] (f32, biases already added).  Token t sits in cache slot
// slot[t] at position pos[t]: q and k are rotated in f32 (x * cos + rotate_half(x) * sin, two
// roundings as the reference's separate multiply and add), k and v are written into the cache.
// Grid (tokens, items / 256): one item per thread, a rotated pair of q (nh x hd/2 items), a rotated
// pair of k written to the cache (nkv x hd/2), or a pair of v copied to the cache (nkv x hd/2).
constexpr int kRopeThreads = 256;
__global__ void __launch_bounds__(kRopeThreads) k_rope_append(float* __restrict__ q, const float* __restrict__ k,
                                                               const float* __restrict__ v,
                                                               const float* __restrict__ cos_t,
                                                               const float* __restrict__ sin_t,
                                                               const int32_t* __restrict__ slot,
                                                               const int32_t* __restrict__ pos, int nh, int nkv,
                                                               int hd, int max_pos, float* __restrict__ kc,
                                                               float* __restrict__ vc) {
    pdl_launch_dependents();
    pdl_wait();
    const int64_t t = blockIdx.x;
    const int half = hd / 2;
    const int nq = nh * half, nk = nkv * half;
    const int i = blockIdx.y * kRopeThreads + threadIdx.x;
    if (i >= nq + 2 * nk) return;
    const int p = pos[t], s = slot[t];
    const float* c = cos_t + static_cast<int64_t>(p) * hd;
    const float* sn = sin_t + static_cast<int64_t>(p) * hd;
    if (i < nq) {
        const int h = i / half, d = i % half;
        float* qh = q + (t * nh + h) * hd;
        const float x1 = qh[d], x2 = qh[d + half];
        // out[d] = x1 * cos[d] + (-x2) * sin[d];  out[d + half] = x2 * cos[d + half] + x1 * sin[d + half]
        qh[d] = __fadd_rn(__fmul_rn(x1, c[d]), __fmul_rn(-x2, sn[d]));
        qh[d + half] = __fadd_rn(__fmul_rn(x2, c[d + half]), __fmul_rn(x1, sn[d + half]));
    } else if (i < nq + nk) {
        const int j = i - nq, h = j / half, d = j % half;
        const float* kh = k + (t * nkv + h) * hd;
        const float x1 = kh[d], x2 = kh[d + half];
        float* dst = kc + ((static_cast<int64_t>(s) * nkv + h) * max_pos + p) * hd;
        dst[d] = __fadd_rn(__fmul_rn(x1, c[d]), __fmul_rn(-x2, sn[d]));
        dst[d + half] = __fadd_rn(__fmul_rn(x2, c[d + half]), __fmul_rn(x1, sn[d + half]));
    } else {
        const int j = i - nq - nk, h = j / half, d = j % half;
        const float* vh = v + (t * nkv + h) * hd;
        float* dst = vc + ((static_cast<int64_t>(s) * nkv + h) * max_pos + p) * hd;
        dst[d] = vh[d];
        dst[d + half] = vh[d + half];
    }
}

// ---------------------------------------------------------------- attention (model.rs:238-257)
// One CTA per (token, kv head, block of keys): the G = nh / nkv query heads of the group against
// keys [kb * kKeys, min(pos + 1, (kb + 1) * kKeys)) of the token's cache slot (causal: keys up to
// its own position).  scores = (q . k) * scale, softmax over all keys, out = attn . v.  A CTA writes
// its block's max, sum of exp and unnormalised output; k_attn_combine rescales and adds the blocks
// in order (one block: the plain softmax).
constexpr int kAttnThreads = 256;
constexpr int kAttnKeys = 256;      // keys per CTA
constexpr int kAttnMaxG = 8;        // query heads per kv head
constexpr int kAttnMaxHd = 128;
constexpr int kAttnChunk = 32;      // keys staged in shared memory at a time (coalesced 16-byte loads)

__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gsrc) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem_dst)), "l"(gsrc) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

__global__ void __launch_bounds__(kAttnThreads) k_attn(const float* __restrict__ q, const float* __restrict__ kc,
                                                       const float* __restrict__ vc, const int32_t* __restrict__ slot,
                                                       const int32_t* __restrict__ pos, int nh, int nkv, int hd,
                                                       int max_pos, float scale, int nblk, float* __restrict__ part_o,
                                                       float* __restrict__ part_ml) {
    pdl_launch_dependents();
    pdl_wait();
    __shared__ float s_q[kAttnMaxG][kAttnMaxHd];
    __shared__ float s_p[kAttnMaxG][kAttnKeys];
    __shared__ float s_m[kAttnMaxG], s_l[kAttnMaxG];
    __shared__ __align__(16) float s_kv[2][kAttnChunk * kAttnMaxHd];  // K or V rows [chunk][hd], two buffers
    const int64_t t = blockIdx.x / (nkv * nblk);
    const int rem = blockIdx.x % (nkv * nblk);
    const int h = rem / nblk, kb = rem % nblk;
    const int G = nh / nkv;
    const int L = pos[t] + 1;
    const int k0 = kb * kAttnKeys, k1 = min(L, k0 + kAttnKeys);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const float* kbase = kc + (static_cast<int64_t>(slot[t]) * nkv + h) * max_pos * hd;
    const float* vbase = vc + (static_cast<int64_t>(slot[t]) * nkv + h) * max_pos * hd;
    for (int i = tid; i < G * hd; i += kAttnThreads) s_q[i / hd][i % hd] = q[(t * nh + h * G + i / hd) * hd + i % hd];
    __syncthreads();
    const int nk = k1 > k0 ? k1 - k0 : 0;
    // issues the asynchronous copy of rows [c0, c0 + cn) of a K or V block into buffer `buf` (16 bytes
    // per thread and copy); the next chunk streams in while the current one is used
    auto issue = [&](const float* base, int c0, int buf) {
        const int cn = min(kAttnChunk, nk - c0);
        const float4* src = reinterpret_cast<const float4*>(base + static_cast<int64_t>(k0 + c0) * hd);
        float4* dst = reinterpret_cast<float4*>(s_kv[buf]);
        for (int i = tid; i < cn * hd / 4; i += kAttnThreads) cp_async16(dst + i, src + i);
        cp_async_commit();
    };
    // waits for chunk c0's copy (buffer c0 / kAttnChunk & 1), issuing chunk c0 + kAttnChunk first
    auto next = [&](const float* base, int c0) {
        if (c0 + kAttnChunk < nk) {
            issue(base, c0 + kAttnChunk, ((c0 / kAttnChunk) + 1) & 1);
            cp_async_wait<1>();
        } else {
            cp_async_wait<0>();
        }
        __syncthreads();
    };
    // scores: one warp per key, lanes over head_dim, a fixed shuffle tree
    if (nk > 0) issue(kbase, 0, 0);
    for (int c0 = 0; c0 < nk; c0 += kAttnChunk) {
        const int cn = min(kAttnChunk, nk - c0);
        next(kbase, c0);
        const float* kvbuf = s_kv[(c0 / kAttnChunk) & 1];
        for (int j = warp; j < cn; j += kAttnThreads / 32) {
            const float* kr = kvbuf + j * hd;
            float kv[kAttnMaxHd / 32];
#pragma unroll
            for (int e = 0; e < kAttnMaxHd / 32; ++e) kv[e] = (lane + 32 * e < hd) ? kr[lane + 32 * e] : 0.0f;
            for (int g = 0; g < G; ++g) {
                float d = 0.0f;
#pragma unroll
                for (int e = 0; e < kAttnMaxHd / 32; ++e)
                    if (lane + 32 * e < hd) d = __fadd_rn(d, __fmul_rn(s_q[g][lane + 32 * e], kv[e]));
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) d = __fadd_rn(d, __shfl_xor_sync(0xffffffffu, d, o));
                if (lane == 0) s_p[g][c0 + j] = __fmul_rn(d, scale);
            }
        }
        __syncthreads();
    }
    // per head: block max, exp, block sum (one warp per head)
    for (int g = warp; g < G; g += kAttnThreads / 32) {
        float m = -INFINITY;
        for (int j = lane; j < nk; j += 32) m = fmaxf(m, s_p[g][j]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        float l = 0.0f;
        for (int j = lane; j < nk; j += 32) {
            const float e = exp_f32(__fsub_rn(s_p[g][j], m));
            s_p[g][j] = e;
            l = __fadd_rn(l, e);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) l = __fadd_rn(l, __shfl_xor_sync(0xffffffffu, l, o));
        if (lane == 0) {
            s_m[g] = m;
            s_l[g] = l;
        }
    }
    __syncthreads();
    // unnormalised output of this block: thread (d, head group) adds its heads' p * v over the keys in
    // order, so each V element is read by kAttnThreads / hd threads instead of once per query head
    const int64_t pbase = (t * nkv + h) * static_cast<int64_t>(nblk) + kb;
    {
        const int ngrp = kAttnThreads / hd;
        const int d = tid % hd, grp = tid / hd;
        float o[kAttnMaxG / 2] = {};
        if (nk > 0) issue(vbase, 0, 0);
        for (int c0 = 0; c0 < nk; c0 += kAttnChunk) {
            const int cn = min(kAttnChunk, nk - c0);
            next(vbase, c0);
            const float* kvbuf = s_kv[(c0 / kAttnChunk) & 1];
            for (int j = 0; j < cn; ++j) {
                const float vv = kvbuf[j * hd + d];
#pragma unroll
                for (int r = 0; r < kAttnMaxG / 2; ++r) {
                    const int g = grp + r * ngrp;
                    if (g < G) o[r] = __fadd_rn(o[r], __fmul_rn(s_p[g][c0 + j], vv));
                }
            }
            __syncthreads();  // this buffer is read before the next chunk but one is copied into it
        }
#pragma unroll
        for (int r = 0; r < kAttnMaxG / 2; ++r) {
            const int g = grp + r * ngrp;
            if (g < G) part_o[(pbase * G + g) * hd + d] = o[r];
        }
    }
    if (tid < G) {
        part_ml[(pbase * G + tid) * 2] = s_m[tid];
        part_ml[(pbase * G + tid) * 2 + 1] = s_l[tid];
    }
}

// Rescales the key blocks of every (token, head) to their common max, adds them in block order and
// writes out = o / l as f16 [T][nh * hd] (the o projection's input).  One CTA per token and 256
// outputs; the factors exp(m_b - m) and the sum l depend on the head only, so the CTA's heads get
// them first, one thread per head.
constexpr int kCombineThreads = 256;
constexpr int kCombineMaxHeads = 8;   // heads one CTA's 256 outputs span (head_dim >= 32)
constexpr int kCombineMaxBlk = 32;
__global__ void __launch_bounds__(kCombineThreads) k_attn_combine(const float* __restrict__ part_o,
                                                                  const float* __restrict__ part_ml,
                                                                  const int32_t* __restrict__ pos, int nh, int nkv,
                                                                  int hd, int nblk, uint16_t* __restrict__ out) {
    pdl_launch_dependents();
    pdl_wait();
    __shared__ float s_f[kCombineMaxHeads][kCombineMaxBlk];
    __shared__ float s_l[kCombineMaxHeads];
    const int64_t t = blockIdx.x;
    const int i0 = blockIdx.y * kCombineThreads;
    const int hq0 = i0 / hd, hq1 = min(nh, (i0 + kCombineThreads - 1) / hd + 1);
    const int G = nh / nkv;
    const int nb = (pos[t] + kAttnKeys) / kAttnKeys;  // blocks holding keys of this token
    // this thread's output of the first blocks, loaded before the factors are known
    constexpr int kPre = 4;
    const int i = i0 + threadIdx.x;
    float pre[kPre];
    const bool mine = i < nh * hd;
    const int hq = mine ? i / hd : 0, d = mine ? i % hd : 0;
    const int64_t pbo = (t * nkv + hq / G) * static_cast<int64_t>(nblk);
#pragma unroll
    for (int b = 0; b < kPre; ++b) pre[b] = (mine && b < nb) ? part_o[((pbo + b) * G + hq % G) * hd + d] : 0.0f;
    if (static_cast<int>(threadIdx.x) < hq1 - hq0) {
        const int hf = hq0 + threadIdx.x;  // the head whose factors this thread computes
        const int gf = hf % G;
        const int64_t pb = (t * nkv + hf / G) * static_cast<int64_t>(nblk);
        float m = -INFINITY;
        for (int b = 0; b < nb; ++b) m = fmaxf(m, part_ml[((pb + b) * G + gf) * 2]);
        float l = 0.0f;
        for (int b = 0; b < nb; ++b) {
            const float f = nb == 1 ? 1.0f : exp_f32(__fsub_rn(part_ml[((pb + b) * G + gf) * 2], m));
            s_f[threadIdx.x][b] = f;
            l = __fadd_rn(l, __fmul_rn(part_ml[((pb + b) * G + gf) * 2 + 1], f));
        }
        s_l[threadIdx.x] = l;
    }
    __syncthreads();
    if (!mine) return;
    const int g = hq % G;
    float o = 0.0f;
#pragma unroll
    for (int b = 0; b < kPre; ++b)
        if (b < nb) o = __fadd_rn(o, __fmul_rn(pre[b], s_f[hq - hq0][b]));
    for (int b = kPre; b < nb; ++b) o = __fadd_rn(o, __fmul_rn(part_o[((pbo + b) * G + g) * hd + d], s_f[hq - hq0][b]));
    out[t * nh * hd + i] = f32_to_f16_bits(__fdiv_rn(o, s_l[hq - hq0]));
}

// ---------------------------------------------------------------- SiLU(gate) * up (model.rs:295-299)
// h = f16(silu(g) * u) with g, u the f16 outputs of gate and up widened (the projection layer's
// to_dtype(F32)) and silu(g) = g / (1 + exp(-g)).
__device__ __forceinline__ uint16_t silu_mul_bits(uint16_t g16, uint16_t u16) {
    const float g = h2f(g16);
    const float sg = __fdiv_rn(g, __fadd_rn(1.0f, exp_f32(-g)));
    return f32_to_f16_bits(__fmul_rn(sg, h2f(u16)));
}

__global__ void k_silu_mul(const uint16_t* __restrict__ gate, const uint16_t* __restrict__ up, int64_t n,
                           uint16_t* __restrict__ out) {
    pdl_launch_dependents();
    pdl_wait();
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x)
        out[i] = silu_mul_bits(gate[i], up[i]);
}

// 8 elements per thread with 16-byte loads and stores (n a multiple of 8, pointers 16-byte aligned).
__global__ void k_silu_mul8(const uint16_t* __restrict__ gate, const uint16_t* __restrict__ up, int64_t n8,
                            uint16_t* __restrict__ out) {
    pdl_launch_dependents();
    pdl_wait();
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n8;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        uint16_t g[8], u[8], h[8];
        *reinterpret_cast<uint4*>(g) = __ldg(reinterpret_cast<const uint4*>(gate) + i);
        *reinterpret_cast<uint4*>(u) = __ldg(reinterpret_cast<const uint4*>(up) + i);
#pragma unroll
        for (int j = 0; j < 8; ++j) h[j] = silu_mul_bits(g[j], u[j]);
        reinterpret_cast<uint4*>(out)[i] = *reinterpret_cast<const uint4*>(h);
    }
}

// One CTA per token: the same output, kept in shared memory too, then the token routed for the
// linears that read it (width a multiple of 8, rows 16-byte aligned).
constexpr int kSiluRouteThreads = 256;
constexpr int64_t kSiluRouteMaxWidth = 65536;
__global__ void __launch_bounds__(kSiluRouteThreads) k_silu_mul_route(const uint16_t* __restrict__ gate,
                                                                       const uint16_t* __restrict__ up, int64_t width,
                                                                       uint16_t* __restrict__ out, TokenRoute r) {
    extern __shared__ __align__(16) uint16_t s_row[];  // the token's f16 row [width]
    pdl_launch_dependents();
    pdl_wait();
    const int t = blockIdx.x;
    const uint4* g4 = reinterpret_cast<const uint4*>(gate + static_cast<int64_t>(t) * width);
    const uint4* u4 = reinterpret_cast<const uint4*>(up + static_cast<int64_t>(t) * width);
    uint4* o4 = reinterpret_cast<uint4*>(out + static_cast<int64_t>(t) * width);
    double s1 = 0.0, s2 = 0.0, sa = 0.0;
#pragma unroll 2
    for (int64_t c = threadIdx.x; c < width / 8; c += kSiluRouteThreads) {
        uint16_t g[8], u[8], h[8];
        *reinterpret_cast<uint4*>(g) = __ldg(g4 + c);
        *reinterpret_cast<uint4*>(u) = __ldg(u4 + c);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            h[j] = silu_mul_bits(g[j], u[j]);
            const double v = static_cast<double>(h2f(h[j]));
            s1 += v;
            s2 += v * v;
            sa += fabs(v);
        }
        o4[c] = *reinterpret_cast<const uint4*>(h);
        reinterpret_cast<uint4*>(s_row)[c] = *reinterpret_cast<const uint4*>(h);
    }
    route_row<kSiluRouteThreads>(r, t, s_row, width, s1, s2, sa);
}

// f16 -> f32 (plus an optional f32 bias per column): the projection layer's to_dtype(F32).
__global__ void k_f16_to_f32(const uint16_t* __restrict__ x, int64_t n, float* __restrict__ out) {
    pdl_launch_dependents();
    pdl_wait();
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x)
        out[i] = h2f(x[i]);
}

static int grid_for(int64_t n, int threads) {
    int64_t b = (n + threads - 1) / threads;
    if (b > 4096) b = 4096;
    return static_cast<int>(b > 0 ? b : 1);
}

// Raises a kernel's dynamic shared-memory limit once per device.
template <typename Kern>
static cudaError_t allow_smem(Kern kern, std::atomic<uint64_t>& flags, int bytes) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    const uint64_t bit = 1ull << (dev & 63);
    if (flags.load() & bit) return cudaSuccess;
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e == cudaSuccess) flags.fetch_or(bit);
    return e;
}

// The routing of `group`'s layers for `tokens` rows of length K into the caller's arrays.
static sc_status make_route(const sc_group* group, int64_t K, int64_t tokens, uint8_t* const* mask,
                            int32_t* const* ridx, int32_t* const* nrouted, uint32_t* counter, TokenRoute* r,
                            const char* who) {
    if (!group || !mask || !ridx || !nrouted || !counter) {
        set_error(std::string(who) + ": null group, routing array or counter");
        return SC_EINVAL;
    }
    const Layer* Ls[SC_GROUP_MAX];
    const int n = group_layers(group, Ls);
    if (n < 1 || tokens > 0x7fffffff) {
        set_error(std::string(who) + ": empty group or too many tokens");
        return SC_EINVAL;
    }
    int cur = -1;
    if (cudaGetDevice(&cur) != cudaSuccess || cur != Ls[0]->device) {
        set_error(std::string(who) + ": the group's layers live on device " + std::to_string(Ls[0]->device) +
                  ", which is not the current device");
        return SC_EINVAL;
    }
    *r = TokenRoute{};
    r->M = static_cast<int>(tokens);
    r->nl = n;
    for (int i = 0; i < n; ++i) {
        const Layer& L = *Ls[i];
        if (L.K != K || L.shard_kind == SC_SHARD_ROWS || !mask[i] || !ridx[i] || !nrouted[i]) {
            set_error(std::string(who) + ": layer " + std::to_string(i) +
                      " does not read whole rows of this length, or its routing arrays are null");
            return SC_EINVAL;
        }
        r->t4[i] = L.t4;
        r->t8[i] = L.t8;
        r->mask[i] = mask[i];
        r->ridx[i] = ridx[i];
        r->nrouted[i] = nrouted[i];
    }
    for (int i = n; i < SC_GROUP_MAX; ++i) {
        r->t4[i] = r->t4[0];
        r->t8[i] = r->t8[0];
        r->mask[i] = r->mask[0];
        r->ridx[i] = r->ridx[0];
        r->nrouted[i] = r->nrouted[0];
    }
    r->route_all = bypass_on();
    r->rc = route_consts(K);
    r->counter = counter;
    return SC_OK;
}

}  // namespace sc

using namespace sc;

extern "C" {

sc_status sc_qwen2_embed(const int64_t* ids, int64_t tokens, const uint16_t* table, int64_t vocab, int64_t hidden,
                         float* out, uint32_t* status, void* stream) {
    if (tokens <= 0) return tokens == 0 ? SC_OK : SC_EINVAL;
    if (!ids || !table || !out || hidden <= 0) return SC_EINVAL;
    const cudaError_t e = launch_pdl(k_embed, dim3(static_cast<unsigned>(tokens)), dim3(256), 0,
                                     static_cast<cudaStream_t>(stream), ids, table, hidden, vocab, out, status);
    return e == cudaSuccess ? SC_OK : cuda_fail(e, "sc_qwen2_embed");
}

sc_status sc_qwen2_add_rmsnorm(float* resid, const float* delta, const float* weight, int64_t tokens, int64_t hidden,
                               float eps, void* out, int out_dtype, void* stream) {
    if (tokens <= 0) return tokens == 0 ? SC_OK : SC_EINVAL;
    if (!resid || !weight || !out || hidden <= 0 || hidden > kNormMaxHidden ||
        (out_dtype != SC_F16 && out_dtype != SC_F32))
        return SC_EINVAL;
    static std::atomic<uint64_t> flags{0};
    cudaError_t e = allow_smem(k_add_rmsnorm, flags, static_cast<int>(kNormMaxHidden * 4));
    if (e == cudaSuccess)
        e = launch_pdl(k_add_rmsnorm, dim3(static_cast<unsigned>(tokens)), dim3(kNormThreads),
                       static_cast<size_t>(hidden * 4), static_cast<cudaStream_t>(stream), resid, delta, weight, hidden,
                       eps, out, out_dtype == SC_F32 ? 1 : 0);
    return e == cudaSuccess ? SC_OK : cuda_fail(e, "sc_qwen2_add_rmsnorm");
}

sc_status sc_qwen2_add_rmsnorm_route(float* resid, const float* delta, const float* weight, int64_t tokens,
                                     int64_t hidden, float eps, uint16_t* out_f16, const sc_group* group,
                                     uint8_t* const* mask, int32_t* const* routed_idx, int32_t* const* n_routed,
                                     uint32_t* counter, void* stream) {
    if (tokens <= 0) return tokens == 0 ? SC_OK : SC_EINVAL;
    if (!resid || !weight || !out_f16 || hidden <= 0 || hidden > kNormMaxHidden || hidden % 8) {
        set_error("sc_qwen2_add_rmsnorm_route: null pointer, or hidden not a multiple of 8 up to 16384");
        return SC_EINVAL;
    }
    TokenRoute r;
    const sc_status st = make_route(group, hidden, tokens, mask, routed_idx, n_routed, counter, &r,
                                    "sc_qwen2_add_rmsnorm_route");
    if (st != SC_OK) return st;
    static std::atomic<uint64_t> flags{0};
    cudaError_t e = allow_smem(k_add_rmsnorm_route, flags, static_cast<int>(kNormMaxHidden * 6));
    if (e == cudaSuccess)
        e = launch_pdl(k_add_rmsnorm_route, dim3(static_cast<unsigned>(tokens)), dim3(kNormThreads),
                       static_cast<size_t>(hidden * 6), static_cast<cudaStream_t>(stream), resid, delta, weight, hidden,
                       eps, out_f16, r);
    return e == cudaSuccess ? SC_OK : cuda_fail(e, "sc_qwen2_add_rmsnorm_route");
}

sc_status sc_qwen2_rope_append(float* q, const float* k, const float* v, const float* cos_table, const float* sin_table,
                               const int32_t* slot, const int32_t* pos, int64_t tokens, int num_heads, int num_kv_heads,
                               int head_dim, int max_pos, float* k_cache, float* v_cache, void* stream) {
    if (tokens <= 0) return tokens == 0 ? SC_OK : SC_EINVAL;
    if (!q || !k || !v || !cos_table || !sin_table || !slot || !pos || !k_cache || !v_cache || head_dim % 2 ||
        num_kv_heads <= 0 || num_heads % num_kv_heads)
        return SC_EINVAL;
    const int items = (num_heads + 2 * num_kv_heads) * (head_dim / 2);
    const cudaError_t e = launch_pdl(k_rope_append,
                                     dim3(static_cast<unsigned>(tokens),
                                          static_cast<unsigned>((items + kRopeThreads - 1) / kRopeThreads)),
                                     dim3(kRopeThreads), 0, static_cast<cudaStream_t>(stream), q, k, v, cos_table,
                                     sin_table, slot, pos, num_heads, num_kv_heads, head_dim, max_pos, k_cache,
                                     v_cache);
    return e == cudaSuccess ? SC_OK : cuda_fail(e, "sc_qwen2_rope_append");
}

size_t sc_qwen2_attention_scratch(int64_t tokens, int num_heads, int num_kv_heads, int head_dim, int max_pos) {
    const int64_t nblk = (max_pos + kAttnKeys - 1) / kAttnKeys;
    const int64_t G = num_kv_heads > 0 ? num_heads / num_kv_heads : 0;
    return static_cast<size_t>(tokens * num_kv_heads * nblk * G * (head_dim + 2) * 4);
}

sc_status sc_qwen2_attention(const float* q, const float* k_cache, const float* v_cache, const int32_t* slot,
                             const int32_t* pos, int64_t tokens, int num_heads, int num_kv_heads, int head_dim,
                             int max_pos, int max_query_pos, float* scratch, size_t scratch_bytes, uint16_t* out_f16,
                             void* stream) {
    if (tokens <= 0) return tokens == 0 ? SC_OK : SC_EINVAL;
    if (!q || !k_cache || !v_cache || !slot || !pos || !scratch || !out_f16 || num_kv_heads <= 0 ||
        num_heads % num_kv_heads || num_heads / num_kv_heads > kAttnMaxG || head_dim > kAttnMaxHd ||
        kAttnThreads % head_dim != 0 || head_dim % 32 != 0 || num_heads > 128 ||
        max_query_pos >= max_pos || (max_query_pos + kAttnKeys) / kAttnKeys > kCombineMaxBlk)
        return SC_EINVAL;
    if (scratch_bytes < sc_qwen2_attention_scratch(tokens, num_heads, num_kv_heads, head_dim, max_pos))
        return SC_ENOMEM;
    // blocks up to the largest query position of this call (every token attends keys <= its own)
    const int nblk_alloc = (max_pos + kAttnKeys - 1) / kAttnKeys;
    const int nblk = (max_query_pos + kAttnKeys) / kAttnKeys;
    (void)nblk_alloc;
    const int G = num_heads / num_kv_heads;
    float* part_o = scratch;
    float* part_ml = scratch + tokens * num_kv_heads * static_cast<int64_t>(nblk) * G * head_dim;
    const float scale = static_cast<float>(1.0 / sqrt(static_cast<double>(head_dim)));
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    cudaError_t e = launch_pdl(k_attn, dim3(static_cast<unsigned>(tokens * num_kv_heads * nblk)), dim3(kAttnThreads), 0, s,
                               q, k_cache, v_cache, slot, pos, num_heads, num_kv_heads, head_dim, max_pos, scale, nblk,
                               part_o, part_ml);
    if (e == cudaSuccess)
        e = launch_pdl(k_attn_combine,
                       dim3(static_cast<unsigned>(tokens),
                            static_cast<unsigned>((num_heads * head_dim + kCombineThreads - 1) / kCombineThreads)),
                       dim3(kCombineThreads), 0, s, part_o, part_ml, pos,
                       num_heads, num_kv_heads, head_dim, nblk, out_f16);
    return e == cudaSuccess ? SC_OK : cuda_fail(e, "sc_qwen2_attention");
}

sc_status sc_qwen2_silu_mul(const uint16_t* gate, const uint16_t* up, int64_t n, uint16_t* out_f16, void* stream) {
    if (n <= 0) return n == 0 ? SC_OK : SC_EINVAL;
    if (!gate || !up || !out_f16) return SC_EINVAL;
    const bool vec = n % 8 == 0 && ((reinterpret_cast<uintptr_t>(gate) | reinterpret_cast<uintptr_t>(up) |
                                     reinterpret_cast<uintptr_t>(out_f16)) & 15u) == 0;
    const cudaError_t e =
        vec ? launch_pdl(k_silu_mul8, dim3(grid_for(n / 8, 256)), dim3(256), 0, static_cast<cudaStream_t>(stream), gate,
                         up, n / 8, out_f16)
            : launch_pdl(k_silu_mul, dim3(grid_for(n, 256)), dim3(256), 0, static_cast<cudaStream_t>(stream), gate, up,
                         n, out_f16);
    return e == cudaSuccess ? SC_OK : cuda_fail(e, "sc_qwen2_silu_mul");
}

sc_status sc_qwen2_silu_mul_route(const uint16_t* gate, const uint16_t* up, int64_t tokens, int64_t width,
                                  uint16_t* out_f16, const sc_group* group, uint8_t* const* mask,
                                  int32_t* const* routed_idx, int32_t* const* n_routed, uint32_t* counter,
                                  void* stream) {
    if (tokens <= 0) return tokens == 0 ? SC_OK : SC_EINVAL;
    if (!gate || !up || !out_f16 || width <= 0 || width % 8 || width > kSiluRouteMaxWidth ||
        ((reinterpret_cast<uintptr_t>(gate) | reinterpret_cast<uintptr_t>(up) | reinterpret_cast<uintptr_t>(out_f16)) &
         15u) != 0) {
        set_error("sc_qwen2_silu_mul_route: null or unaligned pointer, or width not a multiple of 8 up to 65536");
        return SC_EINVAL;
    }
    TokenRoute r;
    const sc_status st = make_route(group, width, tokens, mask, routed_idx, n_routed, counter, &r,
                                    "sc_qwen2_silu_mul_route");
    if (st != SC_OK) return st;
    static std::atomic<uint64_t> flags{0};
    cudaError_t e = allow_smem(k_silu_mul_route, flags, static_cast<int>(kSiluRouteMaxWidth * 2));
    if (e == cudaSuccess)
        e = launch_pdl(k_silu_mul_route, dim3(static_cast<unsigned>(tokens)), dim3(kSiluRouteThreads),
                       static_cast<size_t>(width * 2), static_cast<cudaStream_t>(stream), gate, up, width, out_f16, r);
    return e == cudaSuccess ? SC_OK : cuda_fail(e, "sc_qwen2_silu_mul_route");
}

sc_status sc_qwen2_f16_to_f32(const uint16_t* x, int64_t n, float* out, void* stream) {
    if (n <= 0) return n == 0 ? SC_OK : SC_EINVAL;
    if (!x || !out) return SC_EINVAL;
    const cudaError_t e =
        launch_pdl(k_f16_to_f32, dim3(grid_for(n, 256)), dim3(256), 0, static_cast<cudaStream_t>(stream), x, n, out);
    return e == cudaSuccess ? SC_OK : cuda_fail(e, "sc_qwen2_f16_to_f32");
}

}  // extern "C"
