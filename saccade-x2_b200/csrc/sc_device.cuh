// sc_device.cuh -- device-side helpers shared by the C-TARQ kernels (sm_100a).
//
// PTX wrappers for mbarriers, non-multicast bulk copies and the register-level
// tensor-core MMA, the 4-bit -> f16 nibble conversion of the fragment-tiled
// weight layout, and the bounded waits every spin in this library goes through.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "sc_internal.h"

namespace sc {

// Every spin in this library is bounded in wall time (%globaltimer, nanoseconds): a
// wait that outlives the bound records DEV_TIMEOUT and gives up instead of hanging.
constexpr uint64_t kWaitNs = 2000000000ull;       // 2 s: far beyond any legitimate wait here
constexpr uint64_t kDrainNs = 200000000ull;       // 0.2 s for draining copies after an abort

__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void record_error(uint32_t* status, uint32_t code) {
    if (status) atomicCAS(status, DEV_OK, code);
}

__device__ __forceinline__ int64_t imin64(int64_t a, int64_t b) { return a < b ? a : b; }

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait on an mbarrier phase.  Returns false (and records DEV_TIMEOUT) if the
// phase does not complete within `limit_ns`; callers then skip their remaining work.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, uint32_t* status,
                                          uint64_t limit_ns = kWaitNs) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    for (;;) {
        for (int i = 0; i < 64; ++i)
            if (mbar_try_wait(bar, parity)) return true;
        if (globaltimer_ns() - t0 > limit_ns) break;
    }
    record_error(status, DEV_TIMEOUT);
    return false;
}

// Non-multicast bulk copy global -> this CTA's shared memory, completing on `bar`.
// Both addresses 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* smem_dst, const void* gsrc, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(smem_dst)),
        "l"(gsrc), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// Same, with an L2 evict-first hint for data streamed exactly once (the weights).
__device__ __forceinline__ void bulk_g2s_stream(void* smem_dst, const void* gsrc, uint32_t bytes, uint64_t* bar,
                                                uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], "
        "%4;" ::"r"(smem_u32(smem_dst)),
        "l"(gsrc), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}

__device__ __forceinline__ uint64_t policy_evict_first() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}

// Programmatic dependent launch: wait for the preceding kernel's memory, or let the
// next kernel start its prologue.  Both are no-ops without the launch attribute.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__device__ __forceinline__ uint32_t lop3_and_or(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t d;
    // (a & b) | c
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

// One packed u32 of the fragment-tiled layout -> the four half2 registers of an
// m16n8k16 A fragment, each element the exact integer q - 8.
//   nibble p (bits 4p..4p+3) holds row (p&1 ? g+8 : g), column 2c + ((p>>1)&1)*8 + (p>>2)
//   h[0] = {(g,2c),(g,2c+1)}  h[1] = {(g+8,2c),(g+8,2c+1)}
//   h[2] = {(g,2c+8),(g,2c+9)}  h[3] = {(g+8,2c+8),(g+8,2c+9)}
// OR-ing a nibble into the mantissa of half 1024 gives 1024+n (low nibble of each half)
// or 1024+16n (second nibble); one subtract / one fma maps both to n-8 exactly.
__device__ __forceinline__ void dequant_word(uint32_t w, uint32_t (&h)[4]) {
    const uint32_t kMagic = 0x64006400u;  // half2(1024, 1024)
    const uint32_t t0 = lop3_and_or(w, 0x000F000Fu, kMagic);
    const uint32_t t1 = lop3_and_or(w, 0x00F000F0u, kMagic);
    const uint32_t w8 = w >> 8;
    const uint32_t t2 = lop3_and_or(w8, 0x000F000Fu, kMagic);
    const uint32_t t3 = lop3_and_or(w8, 0x00F000F0u, kMagic);
    const __half2 k1032 = __halves2half2(__ushort_as_half(0x6408), __ushort_as_half(0x6408));  // 1032
    const __half2 k1_16 = __halves2half2(__ushort_as_half(0x2C00), __ushort_as_half(0x2C00));  // 1/16
    const __half2 km72 = __halves2half2(__ushort_as_half(0xD480), __ushort_as_half(0xD480));   // -72
    __half2 r0 = __hsub2(*reinterpret_cast<const __half2*>(&t0), k1032);
    __half2 r1 = __hfma2(*reinterpret_cast<const __half2*>(&t1), k1_16, km72);
    __half2 r2 = __hsub2(*reinterpret_cast<const __half2*>(&t2), k1032);
    __half2 r3 = __hfma2(*reinterpret_cast<const __half2*>(&t3), k1_16, km72);
    h[0] = *reinterpret_cast<uint32_t*>(&r0);
    h[1] = *reinterpret_cast<uint32_t*>(&r1);
    h[2] = *reinterpret_cast<uint32_t*>(&r2);
    h[3] = *reinterpret_cast<uint32_t*>(&r3);
}

// D[16x8] += A[16x16] * B[16x8], f16 inputs, f32 accumulation (register operands).
__device__ __forceinline__ void mma_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// acc + x*w with x, w f16 and one rounding (the product of an f16 value and a small
// integer is exact in f32, so this equals Rust's separate mul-then-add).
__device__ __forceinline__ float fma_f16_f32(uint16_t x, uint16_t w, float acc) {
    asm("fma.rn.f32.f16 %0, %1, %2, %0;" : "+f"(acc) : "h"(x), "h"(w));
    return acc;
}

__device__ __forceinline__ uint16_t lo16(uint32_t v) { return static_cast<uint16_t>(v & 0xFFFFu); }
__device__ __forceinline__ uint16_t hi16(uint32_t v) { return static_cast<uint16_t>(v >> 16); }

__device__ __forceinline__ float h2f(uint16_t h) { return __half2float(__ushort_as_half(h)); }

// Index (in halves) of element (token t, column col) of the staged activation layout
// xk[KB][Mp][64]: within each 64-column block, 16-byte chunks are XOR-swizzled by t%8
// so that the 8 tokens x 4 column pairs of an MMA B fragment hit 32 distinct banks.
__device__ __forceinline__ int64_t xk_index(int64_t col, int t, int Mp) {
    const int64_t kb = col >> 6;
    const int within = static_cast<int>(col & 63);
    const int chunk = (within >> 3) ^ (t & 7);
    return (kb * Mp + t) * 64 + chunk * 8 + (within & 7);
}

__device__ __forceinline__ uint16_t f32_to_f16_bits(float v) { return __half_as_ushort(__float2half_rn(v)); }

// Output cast of the op: f16 rounding first (op.rs:176), then bias in f32 and the
// caller's dtype (model.rs:61 casts the f16 result back).
__device__ __forceinline__ void store_output(void* y, int y_dtype, int64_t idx, float acc, const float* bias,
                                             int64_t row) {
    __half h = __float2half_rn(acc);
    if (bias == nullptr) {
        if (y_dtype == 0) {
            reinterpret_cast<__half*>(y)[idx] = h;
        } else if (y_dtype == 1) {
            reinterpret_cast<__nv_bfloat16*>(y)[idx] = __float2bfloat16_rn(__half2float(h));
        } else {
            reinterpret_cast<float*>(y)[idx] = __half2float(h);
        }
        return;
    }
    float v = __fadd_rn(__half2float(h), bias[row]);
    if (y_dtype == 0) {
        reinterpret_cast<__half*>(y)[idx] = __float2half_rn(v);
    } else if (y_dtype == 1) {
        reinterpret_cast<__nv_bfloat16*>(y)[idx] = __float2bfloat16_rn(v);
    } else {
        reinterpret_cast<float*>(y)[idx] = v;
    }
}

}  // namespace sc
