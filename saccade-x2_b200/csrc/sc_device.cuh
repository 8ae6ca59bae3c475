// sc_device.cuh -- device-side helpers shared by the C-TARQ kernels (sm_100a).
//
// PTX wrappers for mbarriers, non-multicast bulk copies and the tcgen05 tensor-core
// instructions (TMEM alloc/st/ld, MMA with A in tensor memory), the 4-bit -> f16 nibble
// conversion of the device weight layout, and the bounded waits every spin goes through.
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

__device__ __forceinline__ bool mbar_test_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
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
    if (mbar_test_wait(bar, parity)) return true;  // a completed phase: no suspend
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

// ---------------------------------------------------------------- thread-block clusters
// All threads of every CTA of the cluster execute cluster_sync() the same number of times,
// so it needs no bound: it is a barrier, not a spin.
__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
// Shared-memory address of the same object in cluster CTA `rank`.
__device__ __forceinline__ uint32_t dsmem_addr(const void* local, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(local)), "r"(rank));
    return r;
}
__device__ __forceinline__ float ld_dsmem_f32(uint32_t addr) {
    float v;
    asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
    return v;
}
__device__ __forceinline__ double ld_dsmem_f64(uint32_t addr) {
    double v;
    asm volatile("ld.shared::cluster.f64 %0, [%1];" : "=d"(v) : "r"(addr) : "memory");
    return v;
}
// Split cluster barrier: every thread of the cluster arrives once and waits once.
__device__ __forceinline__ void cluster_arrive() { asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory"); }
// Relaxed arrive: enough after mbarrier initialisation, which fence_mbar_init() has released.
__device__ __forceinline__ void cluster_arrive_relaxed() {
    asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory"); }
// Stores into the shared memory of a cluster CTA (addresses from dsmem_addr) that complete
// their bytes on that CTA's mbarrier `rbar`; the receiver waits on its own mbarrier.
__device__ __forceinline__ void st_async_f64(uint32_t raddr, double v, uint32_t rbar) {
    asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.f64 [%0], %1, [%2];" ::"r"(raddr), "d"(v),
                 "r"(rbar)
                 : "memory");
}
__device__ __forceinline__ void st_async_f32(uint32_t raddr, float v, uint32_t rbar) {
    asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.b32 [%0], %1, [%2];" ::"r"(raddr),
                 "r"(__float_as_uint(v)), "r"(rbar)
                 : "memory");
}
__device__ __forceinline__ void st_async_v4_f32(uint32_t raddr, float a, float b, float c, float d, uint32_t rbar) {
    asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.f32 [%0], {%1, %2, %3, %4}, [%5];" ::"r"(
                     raddr),
                 "f"(a), "f"(b), "f"(c), "f"(d), "r"(rbar)
                 : "memory");
}
// Arrive on an mbarrier of cluster CTA `rank`, releasing this thread's prior writes at
// cluster scope.
__device__ __forceinline__ void mbar_arrive_remote(uint64_t* local_bar, uint32_t rank) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(dsmem_addr(local_bar, rank))
                 : "memory");
}
__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
// Bounded wait with cluster-scope acquire (for arrivals from other CTAs of the cluster).
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t parity, uint32_t* status,
                                                  uint64_t limit_ns = kWaitNs) {
    if (mbar_try_wait_cluster(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    for (;;) {
        for (int i = 0; i < 64; ++i)
            if (mbar_try_wait_cluster(bar, parity)) return true;
        if (globaltimer_ns() - t0 > limit_ns) break;
    }
    record_error(status, DEV_TIMEOUT);
    return false;
}

// Non-multicast bulk copy global -> this CTA's shared memory, completing on `bar`.
// Both addresses 16-byte aligned, bytes a multiple of 16.
// [gsrc, gsrc + bytes) into L2 (address 16-byte aligned, bytes a multiple of 16); no completion.
__device__ __forceinline__ void bulk_prefetch_l2(const void* gsrc, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(gsrc), "r"(bytes) : "memory");
}

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

// One packed u32 of the device layout -> four half2 registers holding exact integers q - 8.
// The word belongs to lane (g, c) of a 16-row tile and one 16-column step at k0:
//   nibble p holds row g + (p & 1) * 8, column k0 + 4c + ((p >> 1) & 1) * 2 + (p >> 2), so
//   h[0] = row g    {4c, 4c+1}     h[1] = row g+8  {4c, 4c+1}
//   h[2] = row g    {4c+2, 4c+3}   h[3] = row g+8  {4c+2, 4c+3}
// {h0,h1,h2,h3} is the A fragment of mma.m16n8k16 when the step's K order is permuted so
// that fragment columns {2c, 2c+1 | 2c+8, 2c+9} mean K {4c, 4c+1 | 4c+2, 4c+3}; {h0,h2,h1,h3}
// is the register set of tcgen05.st.16x256b (TMEM lanes g and g+8, columns 2c and 2c+1).
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

// Router sums of 8 f16 values (one 16-byte chunk) in f32, in element order: x, x^2 (one rounding
// through fma) and |x|.
__device__ __forceinline__ void sum_x8(uint4 v, float& a1, float& a2, float& a3) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        const float lo = h2f(lo16(w[q])), hi = h2f(hi16(w[q]));
        a1 += lo;
        a2 = fmaf(lo, lo, a2);
        a3 += fabsf(lo);
        a1 += hi;
        a2 = fmaf(hi, hi, a2);
        a3 += fabsf(hi);
    }
}

// First index in [lo, hi) of an ascending u16 column list whose column is >= key.
__device__ __forceinline__ int64_t lower_bound_u16(const uint16_t* col, int64_t lo, int64_t hi, int64_t key) {
    while (lo < hi) {
        const int64_t mid = (lo + hi) >> 1;
        if (static_cast<int64_t>(col[mid]) < key) lo = mid + 1;
        else hi = mid;
    }
    return lo;
}

// Index (in halves) of element (token t, column col) of the staged activation layout
// xk[KB][Mp/8][8 chunks][8 tokens][8 halves]: for each 64-column block and group of 8
// tokens, 8 "core matrices" of 8 tokens x 8 columns (128 B each), which is the canonical
// K-major, unswizzled operand layout of tcgen05.mma (LBO 128 B between column chunks,
// SBO 1 KB between token groups).
__device__ __forceinline__ int64_t xk_index(int64_t col, int t, int Mp) {
    const int64_t kb = col >> 6;
    const int chunk = static_cast<int>((col & 63) >> 3);
    return ((kb * (Mp >> 3) + (t >> 3)) * 8 + chunk) * 64 + (t & 7) * 8 + (col & 7);
}

// ---------------------------------------------------------------- tcgen05 (5th-gen tensor core)

__device__ __forceinline__ void tmem_alloc(uint32_t* smem_dst, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_dst)),
                 "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tc_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// 32 lanes x 16 consecutive 32-bit columns, one row per thread of the warp.
__device__ __forceinline__ void tc_st16(uint32_t taddr, const uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
        "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
        "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
        : "memory");
}
// 16 lanes x 256 bits: thread (g = lane/4, c = lane%4) writes TMEM lanes base+g (r0, r1 at
// columns 2c, 2c+1) and base+g+8 (r2, r3 at columns 2c, 2c+1).
__device__ __forceinline__ void tc_st_16x256b(uint32_t taddr, uint32_t r0, uint32_t r1, uint32_t r2, uint32_t r3) {
    asm volatile("tcgen05.st.sync.aligned.16x256b.x1.b32 [%0], {%1,%2,%3,%4};" ::"r"(taddr), "r"(r0), "r"(r1),
                 "r"(r2), "r"(r3)
                 : "memory");
}
__device__ __forceinline__ void tc_st8(uint32_t taddr, const uint32_t (&r)[8]) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(taddr), "r"(r[0]),
                 "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
                 : "memory");
}
__device__ __forceinline__ void tc_ld8(uint32_t taddr, uint32_t (&r)[8]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                 : "r"(taddr)
                 : "memory");
}

// D[128 x N] (+)= A[128 x 16] (TMEM, f16) * B[16 x N] (shared memory, f16), f32 accumulation.
__device__ __forceinline__ void tc_mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                          uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// kind::f8f6f4 (e4m3 A from tensor memory, e4m3 B from shared memory, f32 D), K = 32.
__device__ __forceinline__ void tc_mma_ts_f8(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                             uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// 16 lanes x 128 bits, twice along the columns: thread t writes r0 -> (lane t/4, column t%4),
// r1 -> (lane t/4 + 8, column t%4), r2 -> (lane t/4, column 4 + t%4), r3 -> (lane t/4 + 8, column 4 + t%4).
__device__ __forceinline__ void tc_st_16x128b_x2(uint32_t taddr, uint32_t r0, uint32_t r1, uint32_t r2, uint32_t r3) {
    asm volatile("tcgen05.st.sync.aligned.16x128b.x2.b32 [%0], {%1,%2,%3,%4};" ::"r"(taddr), "r"(r0), "r"(r1),
                 "r"(r2), "r"(r3)
                 : "memory");
}

// ---------------------------------------------------------------- e4m3 (fp8) conversions
// Two f16 -> two e4m3 (round to nearest even, saturating); low half -> low byte.
__device__ __forceinline__ uint32_t cvt_e4m3x2_f16x2(uint32_t h2) {
    uint16_t r;
    asm("cvt.rn.satfinite.e4m3x2.f16x2 %0, %1;" : "=h"(r) : "r"(h2));
    return r;
}
// Two f32 -> two e4m3 (nearest even, saturating): lo -> low byte, hi -> high byte.
__device__ __forceinline__ uint32_t cvt_e4m3x2_f32(float lo, float hi) {
    uint16_t r;
    asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
    return r;
}
// Two e4m3 (low byte, high byte) -> two f16 (exact).
__device__ __forceinline__ uint32_t cvt_f16x2_e4m3x2(uint32_t e2) {
    uint32_t r;
    asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(r) : "h"(static_cast<uint16_t>(e2)));
    return r;
}

// One device-layout word as e4m3 weights q - 8 (exact: |q - 8| <= 8): r_g = row g, columns
// 4c..4c+3 of the 16-column step (bytes in column order), r_g8 = row g + 8 (see dequant_word).
__device__ __forceinline__ void dequant_word_e4m3(uint32_t w, uint32_t& r_g, uint32_t& r_g8) {
    uint32_t h[4];
    dequant_word(w, h);  // h0 = row g cols 0,1; h1 = row g+8 cols 0,1; h2 = row g cols 2,3; h3 = row g+8 cols 2,3
    r_g = __byte_perm(cvt_e4m3x2_f16x2(h[0]), cvt_e4m3x2_f16x2(h[2]), 0x5410);
    r_g8 = __byte_perm(cvt_e4m3x2_f16x2(h[1]), cvt_e4m3x2_f16x2(h[3]), 0x5410);
}

// ---- integer engine (one token): exact s8 x s8 -> s32 products
// D[16x8] += A[16x32] * B[32x8], s8 inputs, s32 accumulation (register operands).
__device__ __forceinline__ void mma_16832_s8(int (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// One W4U word as s8 bytes 16 * (q - 8) (the nibble moved to the top of its byte, top bit
// flipped): r_g = row g, nibbles 0, 2, 4, 6 (columns 4c, 4c+2, 4c+1, 4c+3 of the 16-column
// step), r_g8 = row g + 8, nibbles 1, 3, 5, 7 (the same columns).
__device__ __forceinline__ void dequant_word_s8(uint32_t w, uint32_t& r_g, uint32_t& r_g8) {
    r_g = ((w << 4) & 0xF0F0F0F0u) ^ 0x80808080u;
    r_g8 = (w & 0xF0F0F0F0u) ^ 0x80808080u;
}

// An f16 value x as the integer X = x * 2^24 (exact: |X| < 2^40 for every finite f16) in six
// signed base-256 digits, X = sum_i d_i 256^i with d_i in [-128, 127]: the bytes of
// X + 0x808080808080 are d_i + 128, and flipping their top bits gives d_i as s8.  lo holds
// digits 0-3, hi digits 4-5.  Infinities and NaNs set `bad` (their digits are meaningless).
__device__ __forceinline__ void f16_digits(uint32_t h, uint32_t& lo, uint32_t& hi, bool& bad) {
    const uint32_t e = (h >> 10) & 31u, m = h & 1023u;
    bad |= e == 31u;
    const uint64_t mag = static_cast<uint64_t>(e ? (m | 1024u) : m) << (e ? e - 1u : 0u);
    const uint64_t X = (h & 0x8000u) ? 0ull - mag : mag;
    const uint64_t Y = (X + 0x808080808080ull) ^ 0x808080808080ull;
    lo = static_cast<uint32_t>(Y);
    hi = static_cast<uint32_t>(Y >> 32);
}

// Arrive on `bar` once every tcgen05 operation this thread issued so far has completed.
// One lane of a converged warp (the same one every time): issues tcgen05 work in warp-uniform
// loops so that addresses and descriptors stay in uniform registers.
__device__ __forceinline__ bool elect_one() {
    uint32_t pred;
    asm volatile("{\n\t.reg .pred p;\n\telect.sync _|p, 0xffffffff;\n\tselp.u32 %0, 1, 0, p;\n\t}" : "=r"(pred));
    return pred != 0;
}
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}
// Shared-memory matrix descriptor, K-major, no swizzle: core matrices of 8 rows x 16 B,
// `lbo` bytes between the two core matrices along K, `sbo` bytes between 8-row groups.
__device__ __forceinline__ uint64_t desc_kmajor(const void* smem_ptr, uint32_t lbo, uint32_t sbo) {
    uint64_t d = static_cast<uint64_t>((smem_u32(smem_ptr) >> 4) & 0x3FFFu);
    d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
    d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32;
    d |= static_cast<uint64_t>(1) << 46;  // descriptor version for sm_100
    return d;
}
// Instruction descriptor of kind::f16: f16 A and B, f32 D, both K-major, M x N.
__host__ __device__ constexpr uint32_t idesc_f16_f32(int M, int N) {
    return (1u << 4) | (static_cast<uint32_t>(N >> 3) << 17) | (static_cast<uint32_t>(M >> 4) << 24);
}
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
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


// ---------------------------------------------------------------- router decision

// op.rs:69-72: (score >= t4 && score < t8) || score >= t8; both flags select the dW.
__device__ __forceinline__ bool route_rule_f32(float score, float t4, float t8) {
    return (score >= t4 && score < t8) || (score >= t8);
}
__device__ __forceinline__ bool route_rule_f64(double score, float t4, float t8) {
    const double a = t4, b = t8;
    return (score >= a && score < b) || (score >= b);
}

// The token's value i as f16 bits (bf16 inputs are rounded to f16 first, as the caller's
// to_dtype(F16) does at model.rs:58-61).
__device__ __forceinline__ uint16_t x_f16_bits(const void* x, int x_dtype, int64_t i) {
    if (x_dtype == SC_BF16)
        return f32_to_f16_bits(__bfloat162float(reinterpret_cast<const __nv_bfloat16*>(x)[i]));
    return reinterpret_cast<const uint16_t*>(x)[i];
}

// Replays heuristics.rs:3-14 exactly on one token: f16 -> f32, sequential f32 sums, f32 divide.
static __device__ __noinline__ float exact_variance(const void* xrow, int x_dtype, int64_t Kfull) {
    float sum = 0.0f, sq = 0.0f;
    for (int64_t i = 0; i < Kfull; ++i) {
        const float v = h2f(x_f16_bits(xrow, x_dtype, i));
        sum = __fadd_rn(sum, v);
        sq = __fadd_rn(sq, __fmul_rn(v, v));
    }
    const float hd = static_cast<float>(Kfull);
    const float mean = __fdiv_rn(sum, hd);
    return __fsub_rn(__fdiv_rn(sq, hd), __fmul_rn(mean, mean));
}

// Routing decision of one token from (near-)exact f64 sums of x, x^2 and |x| over Kfull
// values.  The reference decides on a sequentially summed f32 variance; the standard bound
// |fl(sum) - sum| <= gamma_{k-1} * sum|terms| (gamma_n = n*u/(1-n*u), u = 2^-24), carried
// through the mean, the square and the subtraction and doubled for safety, says how far that
// f32 score can be from the f64 one.  If both thresholds lie farther away the f64 decision
// is the reference's; otherwise the exact f32 chain is replayed for this token.
//
// S1, S2, SA may themselves carry a summation error: E1x, E2x bound |S1 - sum x| and
// |S2 - sum x^2| (0 for exact sums); they widen the band accordingly.
// Constants of the bound below for a token of n values: inv_n = 1/n and
// gam = gamma_{n-1} = (n-1)u / (1 - (n-1)u).
struct RouteConsts {
    double inv_n, gam;
};
__host__ __device__ inline RouteConsts route_consts(int64_t Kfull) {
    const double n = static_cast<double>(Kfull);
    const double nu = (n - 1.0) * 5.9604644775390625e-08;
    return RouteConsts{1.0 / n, nu / (1.0 - nu)};
}

// The decision from the sums alone: 1 routed, 0 not routed, -1 when a threshold lies inside the
// band (only the exact f32 chain decides then).  *var_out receives the f64 score.
__device__ __forceinline__ int route_band(double S1, double S2, double SA, const RouteConsts& rc, float t4, float t8,
                                          double E1x, double E2x, double* var_out) {
    const double u = 5.9604644775390625e-08;  // 2^-24
    const double inv_n = rc.inv_n;            // products with 1/n differ from quotients by f64 ulps, far inside B
    const double gam = rc.gam;
    const double E1 = gam * (SA + E1x) + E1x, E2 = gam * (S2 + E2x) + E2x;
    const double mean = S1 * inv_n, A = S2 * inv_n;
    const double errMean = (E1 + u * (fabs(S1) + E1)) * inv_n;
    const double errA = (E2 + u * (S2 + E2)) * inv_n;
    const double am = fabs(mean) + errMean;
    const double errSq = errMean * (2.0 * fabs(mean) + errMean) + u * am * am;
    const double var = A - mean * mean;
    double B = errA + errSq + u * (fabs(var) + errA + errSq);
    B = 2.0 * B + 1e-37;
    const double d4 = fabs(var - static_cast<double>(t4));
    const double d8 = fabs(var - static_cast<double>(t8));
    *var_out = var;
    if (isfinite(var) && isfinite(B) && !(d4 <= B) && !(d8 <= B)) return route_rule_f64(var, t4, t8) ? 1 : 0;
    return -1;
}

__device__ __forceinline__ bool route_token(double S1, double S2, double SA, int64_t Kfull, const RouteConsts& rc,
                                            float t4, float t8, const void* xrow, int x_dtype, float* score_out,
                                            double E1x = 0.0, double E2x = 0.0) {
    double var;
    const int d = route_band(S1, S2, SA, rc, t4, t8, E1x, E2x, &var);
    if (d >= 0) {
        if (score_out) *score_out = static_cast<float>(var);
        return d == 1;
    }
    const float score = exact_variance(xrow, x_dtype, Kfull);
    if (score_out) *score_out = score;
    return route_rule_f32(score, t4, t8);
}
__device__ __forceinline__ bool route_token(double S1, double S2, double SA, int64_t Kfull, float t4, float t8,
                                            const void* xrow, int x_dtype, float* score_out, double E1x = 0.0,
                                            double E2x = 0.0) {
    return route_token(S1, S2, SA, Kfull, route_consts(Kfull), t4, t8, xrow, x_dtype, score_out, E1x, E2x);
}

// ---------------------------------------------------------------- dW/s folded into dequantised weights

// Header of one fold list (per 128-row tile and 64-column block): u16 entry offsets
// [8 tiles of 16 rows][33 lanes + end], then u32 entries (see build_fold_lists).
constexpr int kFoldHdr = 528;

// Add f16 value `v` to the half `hi` of 32-bit register h[slot / 4][slot % 4]: one predicated add
// per register (static indices keep the 16 registers out of local memory, and no lane branches, so
// lanes with different slots do not serialise on a divergent switch).
__device__ __forceinline__ void fold_add(uint32_t (&h)[4][4], int slot, int hi, uint16_t v) {
    const uint32_t add = hi ? (static_cast<uint32_t>(v) << 16) : static_cast<uint32_t>(v);
#pragma unroll
    for (int q = 0; q < 16; ++q) {
        const __half2 t = __hadd2(*reinterpret_cast<const __half2*>(&h[q / 4][q % 4]),
                                  *reinterpret_cast<const __half2*>(&add));
        const uint32_t r = *reinterpret_cast<const uint32_t*>(&t);
        h[q / 4][q % 4] = slot == q ? r : h[q / 4][q % 4];
    }
}

// ---------------------------------------------------------------- parallel exact replay
//
// The reference's score of a token whose f64 score lies inside the error band, computed by a whole
// CTA instead of one thread walking K dependent f32 adds (heuristics.rs:3-14).
//
// Sum of squares (terms v_i = x_i^2, exact in f32, all >= 0): while the running f32 sum q stays in
// one binade [2^B, 2^(B+1)) its grid is g = 2^(B-23) and every step adds an integer number of g:
// q_i = q_(i-1) + g * r_i with r_i = v_i / g rounded to nearest, ties to the even result (so a tie's
// r_i depends on the parity of q / g).  The exact prefix sums P_i bound the chain, |q_i - P_i| <=
// gamma_i P_i for non-negative terms, so a step is provably inside binade B when P_(i-1)(1 - gamma)
// >= 2^B and P_i + gamma P_(i-1) < 2^(B+1).  Each thread takes a contiguous chunk, computes its
// offsets by a block scan of the P_i, and summarises its chunk as items in order: runs of such steps
// of one binade (the sum of r_i for either parity of q / g at the run's start) and ranges of the
// other steps (binade crossings, leading zeros), at most kReplayItems per thread (the rest of a
// chunk becomes one range).  One thread then walks the items: a run adds g * R in one exact f32 add
// (the result stays on the grid inside the binade), a range replays its adds one by one.  The result
// equals the sequential chain bit for bit.
//
// Sum (signed terms): its chain stays within e1 = u sum_i |P_i| (1 + 1.01 n u) of the exact sum
// (|e_i| <= |e_(i-1)|(1 + u) + u |P_i|), with the exact prefix sums P_i in units of 2^-24.  The score
// fl(fl(q / n) - fl(m * m)), m = fl(s / n), is monotone in |m|, so [lo, hi] over the chain's possible
// s holds the reference's score; both ends decide the same unless a threshold lies within about an
// ulp of the score.  lo = hi = nan when x holds inf or nan.
constexpr int kReplayItems = 4;
constexpr int kReplayMaxThreads = 256;
struct ReplayShared {
    // items: {0 | end parity after an even start << 1 | after an odd start << 2, B, R even, R odd}
    // or {1, i0, i1, 0}
    int4 flat[kReplayMaxThreads * kReplayItems];  // the items of all threads in order
    double w2[kReplayMaxThreads / 32];
    long long w1[kReplayMaxThreads / 32];
    double wabs[kReplayMaxThreads / 32];
    int wcnt[kReplayMaxThreads / 32];
    int wstart[kReplayMaxThreads / 32], wmerged[kReplayMaxThreads / 32];
    float lo, hi;
};

// The reference's exact sequential f32 score of one row of f16 bits (heuristics.rs:3-14).
static __device__ __noinline__ float exact_variance_row(const uint16_t* row, int64_t K) {
    float sum = 0.0f, sq = 0.0f;
    for (int64_t i = 0; i < K; ++i) {
        const float v = h2f(row[i]);
        sum = __fadd_rn(sum, v);
        sq = __fadd_rn(sq, __fmul_rn(v, v));
    }
    const float hd = static_cast<float>(K);
    const float mean = __fdiv_rn(sum, hd);
    return __fsub_rn(__fdiv_rn(sq, hd), __fmul_rn(mean, mean));
}

// A thread's items, in registers until their place in the flat list is known (static indices only).
struct ReplayItems {
    int4 v[kReplayItems];
    __device__ __forceinline__ void put(int n, int4 x) {
#pragma unroll
        for (int j = 0; j < kReplayItems; ++j)
            if (j == n) v[j] = x;
    }
};

// `row`: the token's K values as f16 bits, in shared memory (read many times).
template <int kThreads>
__device__ void replay_score(const uint16_t* row, int64_t K, ReplayShared& sh) {
    static_assert(kThreads % 32 == 0 && kThreads <= kReplayMaxThreads, "replay threads");
    constexpr int kWarps = kThreads / 32;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int64_t c = (K + kThreads - 1) / kThreads;
    const int64_t i0 = min(K, static_cast<int64_t>(tid) * c), i1 = min(K, i0 + c);
    double l2 = 0.0;
    long long l1 = 0;
    int bad = 0;
    for (int64_t i = i0; i < i1; ++i) {
        const float xf = h2f(row[i]);
        if (!isfinite(xf)) {
            bad = 1;
            continue;
        }
        l2 += static_cast<double>(__fmul_rn(xf, xf));
        l1 += __float2ll_rn(__fmul_rn(xf, 16777216.0f));  // exact: an f16 times 2^24 is an integer < 2^40
    }
    double s2 = l2;
    long long s1 = l1;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const double a2 = __shfl_up_sync(0xffffffffu, s2, o);
        const long long a1 = __shfl_up_sync(0xffffffffu, s1, o);
        if (lane >= o) {
            s2 += a2;
            s1 += a1;
        }
    }
    if (lane == 31) {
        sh.w2[warp] = s2;
        sh.w1[warp] = s1;
    }
    if (__syncthreads_or(bad)) {
        if (tid == 0) sh.lo = sh.hi = __int_as_float(0x7fc00000);
        __syncthreads();
        return;
    }
    double P2 = s2 - l2;
    long long P1 = s1 - l1;
    long long tot1 = 0;
    for (int w = 0; w < kWarps; ++w) {
        if (w < warp) {
            P2 += sh.w2[w];
            P1 += sh.w1[w];
        }
        tot1 += sh.w1[w];
    }
    double absP1 = 0.0;
    ReplayItems its;
    int n_it = 0, kind = -1, curB = 0, par0 = 0, par1 = 1;
    float R0 = 0.0f, R1 = 0.0f;
    int64_t seq0 = 0, seq1 = 0;
    bool tail = false;
    for (int64_t i = i0; i < i1; ++i) {
        const float xf = h2f(row[i]);
        const float v = __fmul_rn(xf, xf);
        const double Pp = P2;
        P2 += static_cast<double>(v);
        P1 += __float2ll_rn(__fmul_rn(xf, 16777216.0f));
        absP1 += fabs(static_cast<double>(P1));
        if (tail) continue;
        bool certain = false;
        int B = 0;
        float sc = 0.0f;
        if (Pp > 0.0) {
            B = static_cast<int>((__double_as_longlong(Pp) >> 52) & 0x7FF) - 1023;
            const double iu = static_cast<double>(i + 1) * 5.9604644775390625e-08;
            const double d = iu * (1.0 + 2.0 * iu) + 1e-9;  // >= gamma = iu / (1 - iu) for iu <= 1/2
            const double base = __longlong_as_double(static_cast<long long>(B + 1023) << 52);
            if (Pp * (1.0 - d) >= base && P2 + d * Pp < 2.0 * base) {
                sc = __fmul_rn(v, __int_as_float((127 + 23 - B) << 23));  // v / g, exact
                certain = true;
            }
        }
        if (certain) {
            if (!(kind == 0 && curB == B)) {
                if (kind == 0) {
                    its.put(n_it++, make_int4((par0 << 1) | (par1 << 2), curB, __float_as_int(R0), __float_as_int(R1)));
                } else if (kind == 1) {
                    its.put(n_it++, make_int4(1, static_cast<int>(seq0), static_cast<int>(seq1), 0));
                }
                if (n_it == kReplayItems - 1) {  // the rest of the chunk as one range
                    tail = true;
                    kind = 1;
                    seq0 = i;
                    continue;
                }
                kind = 0;
                curB = B;
                R0 = R1 = 0.0f;
                par0 = 0;
                par1 = 1;
            }
            const float fl = floorf(sc);
            const bool tie = __fsub_rn(sc, fl) == 0.5f;
            const float rr = rintf(sc);
            const int fli = static_cast<int>(fl);
            const float r0 = tie ? ((((par0 + fli) & 1) == 0) ? fl : __fadd_rn(fl, 1.0f)) : rr;
            const float r1 = tie ? ((((par1 + fli) & 1) == 0) ? fl : __fadd_rn(fl, 1.0f)) : rr;
            R0 = __fadd_rn(R0, r0);  // integers below 2^24: exact
            R1 = __fadd_rn(R1, r1);
            par0 = (par0 + static_cast<int>(r0)) & 1;
            par1 = (par1 + static_cast<int>(r1)) & 1;
        } else {
            if (kind != 1) {
                if (kind == 0) its.put(n_it++, make_int4((par0 << 1) | (par1 << 2), curB, __float_as_int(R0), __float_as_int(R1)));
                if (n_it == kReplayItems - 1) tail = true;
                kind = 1;
                seq0 = i;
            }
            seq1 = i + 1;
        }
    }
    if (kind == 0) {
        its.put(n_it++, make_int4((par0 << 1) | (par1 << 2), curB, __float_as_int(R0), __float_as_int(R1)));
    } else if (kind == 1) {
        its.put(n_it++, make_int4(1, static_cast<int>(seq0), static_cast<int>(tail ? i1 : seq1), 0));
    }
    // the items in chunk order: an exclusive scan of the counts places each thread's items
    int cs = n_it;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int a = __shfl_up_sync(0xffffffffu, cs, o);
        if (lane >= o) cs += a;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) absP1 += __shfl_down_sync(0xffffffffu, absP1, o);
    if (lane == 31) sh.wcnt[warp] = cs;
    if (lane == 0) sh.wabs[warp] = absP1;
    __syncthreads();
    int at = cs - n_it, total = 0;
    for (int w = 0; w < kWarps; ++w) {
        if (w < warp) at += sh.wcnt[w];
        total += sh.wcnt[w];
    }
#pragma unroll
    for (int j = 0; j < kReplayItems; ++j)
        if (j < n_it) sh.flat[at + j] = its.v[j];
    if (lane == 0) sh.wstart[warp] = at;
    __syncthreads();
    // each warp's lane 0 composes consecutive runs of one binade (the parity after a run is a function
    // of the parity before it), in place; thread 0 then walks what remains
    if (lane == 0) {
        const int b0 = sh.wstart[warp], b1 = warp + 1 < kWarps ? sh.wstart[warp + 1] : total;
        int out = b0;
        for (int j = b0; j < b1; ++j) {
            const int4 it = sh.flat[j];
            if (out > b0) {
                int4& pv = sh.flat[out - 1];
                if (it.x != 1 && (pv.x & 1) == 0 && pv.y == it.y) {
                    const int e0 = (pv.x >> 1) & 1, e1 = (pv.x >> 2) & 1;  // parity after pv from an even / odd start
                    const float R0 = __fadd_rn(__int_as_float(pv.z), __int_as_float(e0 ? it.w : it.z));
                    const float R1 = __fadd_rn(__int_as_float(pv.w), __int_as_float(e1 ? it.w : it.z));
                    const int f0 = e0 ? (it.x >> 2) & 1 : (it.x >> 1) & 1;
                    const int f1 = e1 ? (it.x >> 2) & 1 : (it.x >> 1) & 1;
                    pv = make_int4((f0 << 1) | (f1 << 2), pv.y, __float_as_int(R0), __float_as_int(R1));
                    continue;
                }
            }
            sh.flat[out++] = it;
        }
        sh.wmerged[warp] = out;
    }
    __syncthreads();
    if (tid == 0) {
        float q = 0.0f;
        for (int w = 0; w < kWarps; ++w) {
            const int b0 = sh.wstart[w], b1 = sh.wmerged[w];
            for (int j = b0; j < b1; ++j) {
                const int4 it = sh.flat[j];
                if ((it.x & 1) == 0) {
                    const float R = __int_as_float((__float_as_uint(q) & 1u) ? it.w : it.z);
                    q = __fadd_rn(q, __fmul_rn(R, __int_as_float((127 + it.y - 23) << 23)));
                } else {
                    for (int i = it.y; i < it.z; ++i) {
                        const float xf = h2f(row[i]);
                        q = __fadd_rn(q, __fmul_rn(xf, xf));
                    }
                }
            }
        }
        double sabs = 0.0;
        for (int w = 0; w < kWarps; ++w) sabs += sh.wabs[w];
        const double u = 5.9604644775390625e-08, n = static_cast<double>(K);
        const double S1 = static_cast<double>(tot1) * 5.9604644775390625e-08;
        const double e1 = u * (sabs * 5.9604644775390625e-08) * (1.0 + 1.01 * n * u) * (1.0 + 1e-6) + 1e-300;
        const float hd = static_cast<float>(K);
        const float qd = __fdiv_rn(q, hd);
        const float mlo = __fdiv_rn(__double2float_rd(S1 - e1), hd);
        const float mhi = __fdiv_rn(__double2float_ru(S1 + e1), hd);
        const float a = __fmul_rn(mlo, mlo), b = __fmul_rn(mhi, mhi);
        const float mmax = fmaxf(a, b);
        const float mmin = (mlo <= 0.0f && mhi >= 0.0f) ? 0.0f : fminf(a, b);
        sh.lo = __fsub_rn(qd, mmax);
        sh.hi = __fsub_rn(qd, mmin);
    }
    __syncthreads();
}

// ---------------------------------------------------------------- routing one token for a group
//
// The per-token router of 1..SC_GROUP_MAX layers that read the same token (heuristics.rs:3-14,
// op.rs:64-73), run by the CTA that holds the token: every decision the f64 sums settle
// (route_band), the CTA-parallel replay for the others, the mask byte per layer; the last CTA of
// the grid to finish compacts every layer's mask into its ascending routed list and count.
struct TokenRoute {
    int M;                            // tokens of the call (one CTA each)
    int nl;                           // layers routed (0..SC_GROUP_MAX)
    float t4[SC_GROUP_MAX], t8[SC_GROUP_MAX];
    int route_all;                    // bypass: every token routed
    RouteConsts rc;                   // of the token's length
    uint8_t* mask[SC_GROUP_MAX];
    int32_t* ridx[SC_GROUP_MAX];
    int32_t* nrouted[SC_GROUP_MAX];
    uint32_t* counter;                // completion counter, zero between calls (the last CTA resets it)
};

// Token t of the call, its K values as f16 bits in shared memory `row` (written by this CTA before
// the call; the first barrier here publishes them); s1, s2, sa: this thread's f64 partial sums of
// x, x^2, |x| over the values it wrote.  Every thread of the CTA calls it.
template <int kThreads>
__device__ void route_row(const TokenRoute& a, int t, const uint16_t* row, int64_t K, double s1, double s2, double sa) {
    constexpr int kWarps = kThreads / 32;
    __shared__ double red[3][kWarps];
    __shared__ int s_last;
    __shared__ int s_wsum[kWarps];
    __shared__ int s_open;
    __shared__ ReplayShared s_replay;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
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
    double S1 = 0.0, S2 = 0.0, SA = 0.0;
    if (tid == 0) {
        for (int w = 0; w < kWarps; ++w) {
            S1 += red[0][w];
            S2 += red[1][w];
            SA += red[2][w];
        }
        int open = 0;
        for (int l = 0; l < a.nl; ++l) {
            double var;
            const int d = a.route_all ? 1 : route_band(S1, S2, SA, a.rc, a.t4[l], a.t8[l], 0.0, 0.0, &var);
            if (d >= 0) {
                a.mask[l][t] = static_cast<uint8_t>(d);
            } else {
                open = 1;
            }
        }
        s_open = open;
    }
    __syncthreads();
    if (s_open) {
        // some layer's threshold is inside the f32 error band: the CTA replays the reference's chains
        // once for the token, then every open decision is taken on that score
        replay_score<kThreads>(row, K, s_replay);
        if (tid == 0) {
            bool have_exact = false;
            float exact = 0.0f;
            for (int l = 0; l < a.nl; ++l) {
                double var;
                if (route_band(S1, S2, SA, a.rc, a.t4[l], a.t8[l], 0.0, 0.0, &var) >= 0) continue;
                const bool rl = route_rule_f32(s_replay.lo, a.t4[l], a.t8[l]);
                const bool rh = route_rule_f32(s_replay.hi, a.t4[l], a.t8[l]);
                bool routed = rl;
                if (rl != rh || !(s_replay.lo == s_replay.lo)) {
                    if (!have_exact) exact = exact_variance_row(row, K);
                    have_exact = true;
                    routed = route_rule_f32(exact, a.t4[l], a.t8[l]);
                }
                a.mask[l][t] = routed ? 1 : 0;
            }
        }
    }
    // completion count; the last CTA compacts every layer's mask
    if (tid == 0) {
        __threadfence();
        const unsigned ticket = atomicAdd(a.counter, 1u);
        s_last = (ticket == static_cast<unsigned>(a.M) - 1u) ? 1 : 0;
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    for (int l = 0; l < a.nl; ++l) {
        int base = 0;
        for (int t0 = 0; t0 < a.M; t0 += kThreads) {
            const int tt = t0 + tid;
            const int v = (tt < a.M) ? (reinterpret_cast<volatile uint8_t*>(a.mask[l])[tt] != 0) : 0;
            const unsigned bal = __ballot_sync(0xffffffffu, v);
            if (lane == 0) s_wsum[warp] = __popc(bal);
            __syncthreads();
            int pre = 0, tot = 0;
            for (int w = 0; w < kWarps; ++w) {
                if (w < warp) pre += s_wsum[w];
                tot += s_wsum[w];
            }
            pre += __popc(bal & ((1u << lane) - 1u));
            if (v) a.ridx[l][base + pre] = tt;
            base += tot;
            __syncthreads();
        }
        if (tid == 0) *a.nrouted[l] = base;
    }
    if (tid == 0) *a.counter = 0u;
}

}  // namespace sc
