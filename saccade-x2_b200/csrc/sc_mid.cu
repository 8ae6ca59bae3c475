// sc_mid.cu -- C-TARQ for 9..64 tokens per call (batched decode).
//
// k_mid_route (one CTA per token) routes every token exactly like the reference for each layer of
// a group (heuristics.rs:3-14, op.rs:64-73: f64 sums, then the f32 chain replayed for a token near
// a threshold -- route_token), and compacts the routed-token lists; for bf16 (or unaligned) tokens
// it also writes the f16 copy that the GEMM's tensor loads read (the caller's to_dtype(F16),
// model.rs:58-61).  A caller that has routed the tokens already skips it.
//
// k_ctarq_mid is a tcgen05 GEMM with the weights as the MMA's M side and the tokens as its N side
// (N = tokens rounded up to 16): A = 128 rows x 16 columns of exact f16 integers q - 8 in tensor
// memory (dequant_word), B = the f16 tokens in shared memory, D = f32 in tensor memory,
// kind::f16 (M = 128, N <= 64, K = 16).  Roles per CTA (one 128-row tile, one column split):
//   weight producer  the 4-bit base through a deep ring of bulk copies (before the dependency wait);
//   x producer       one TMA box per 64-column block: 64 f16 (128 B) of every token, landing in the
//                    128-byte-swizzled K-major operand layout (rows past the last token and columns
//                    past the last one zero-filled);
//   4 warps          dequantise the weights into tensor memory (A), three stages deep (from 17 tokens
//                    three sets of 4, taking the stages in turn);
//   MMA warp         one elected lane issues 4 MMAs per 64-column block;
//   4 aux warps      one thread per row: the row's dW entries of each staged block (op.rs:152-170,
//                    CSR columns ascending) for the routed tokens, from the staged x; then the
//                    epilogue y = f16(acc * s + dW) (+ bias after the rounding).
// With several column splits each split writes its f32 rows and the last CTA of the row tile adds
// them in split order (deterministic).
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <atomic>
#include <cstring>
#include <mutex>
#include <vector>

#include "sc_device.cuh"
#include "sc_internal.h"

namespace sc {

// ---------------------------------------------------------------- the router (and f16 copy)

struct MidRouteParams {
    const void* x;
    int x_dtype;
    int vec_ok;
    int64_t x_stride;                 // elements per token (the router's length)
    uint16_t* xcopy;                  // nullable: f16 copy of the tokens [M][x_stride]
    TokenRoute r;
};

__device__ __forceinline__ void load_f16x8(const void* x, int x_dtype, bool vec, int64_t base, uint16_t (&h)[8]) {
    if (x_dtype == SC_BF16) {
        const __nv_bfloat16* xs = reinterpret_cast<const __nv_bfloat16*>(x) + base;
        __nv_bfloat16 b[8];
        if (vec) {
            *reinterpret_cast<uint4*>(b) = __ldg(reinterpret_cast<const uint4*>(xs));
        } else {
#pragma unroll
            for (int j = 0; j < 8; ++j) b[j] = xs[j];
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) h[j] = f32_to_f16_bits(__bfloat162float(b[j]));
    } else {
        const uint16_t* xs = reinterpret_cast<const uint16_t*>(x) + base;
        if (vec) {
            *reinterpret_cast<uint4*>(h) = __ldg(reinterpret_cast<const uint4*>(xs));
        } else {
#pragma unroll
            for (int j = 0; j < 8; ++j) h[j] = xs[j];
        }
    }
}

template <int kThreads>
__global__ void __launch_bounds__(kThreads) k_mid_route(MidRouteParams a) {
    extern __shared__ __align__(16) uint16_t s_row[];  // the token as f16 bits [x_stride]
    const int t = blockIdx.x;
    const int tid = threadIdx.x;
    pdl_launch_dependents();
    pdl_wait();
    const int64_t row_off = static_cast<int64_t>(t) * a.x_stride;
    double s1 = 0.0, s2 = 0.0, sa = 0.0;
    for (int64_t ch = tid; ch < a.x_stride / 8; ch += kThreads) {
        uint16_t h[8];
        load_f16x8(a.x, a.x_dtype, a.vec_ok, row_off + ch * 8, h);
        if (a.xcopy) *reinterpret_cast<uint4*>(a.xcopy + row_off + ch * 8) = *reinterpret_cast<const uint4*>(h);
        *reinterpret_cast<uint4*>(&s_row[ch * 8]) = *reinterpret_cast<const uint4*>(h);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const double v = static_cast<double>(h2f(h[j]));
            s1 += v;
            s2 += v * v;
            sa += fabs(v);
        }
    }
    route_row<kThreads>(a.r, t, s_row, a.x_stride, s1, s2, sa);
}

// ---------------------------------------------------------------- the tcgen05 GEMM

struct MidLayer {
    const uint32_t* wq;
    const float* scale;
    const uint32_t* rowptr;
    const uint16_t* col;
    const int8_t* val;
    float ds;
    int64_t nnz;
    int64_t N, KB, RT;
    void* y;
    int y_dtype;
    const float* bias;
    int partial_out;
    float* partial;        // [RT][ks][T][128] f32 (ks > 1)
    uint32_t* rtcount;     // [RT] completion counters (ks > 1), zero between calls
    uint32_t* status;
    const int32_t* ridx;   // routed tokens, ascending
    const int32_t* nrouted;
    const uint8_t* dseg;   // dW segments per (row tile, block) (null: no dW)
    const uint32_t* dsegoff;
    const uint8_t* fold;   // dW/s fold lists per (row tile, block) (the folding variant)
    const uint32_t* foldoff;
    int cta0;              // first CTA of this layer
};

struct alignas(64) MidParams {
    CUtensorMap xmap;      // the f16 tokens: dims {Kfull, M}, box {64, Tp}, 128-byte swizzle
    int nl;
    int ks;                // column splits (every layer of the launch)
    int T, Tp;             // tokens, tokens rounded up to 16 (MMA N)
    int wstages, xstages;  // ring depths
    int route_all;
    int dslot;             // shared-memory slot of one dW segment, or of one fold list in the folding
                           // variant (0: dW read in place from global memory)
    int64_t x_col0;        // first column of the layers' slice within a token
    MidLayer L[SC_GROUP_MAX];
};

struct MidCfg {
    static constexpr int SKB = 2;                // 64-column blocks per ring stage
    static constexpr int AB = 3;                 // tensor-memory A buffers (one stage each)
    static constexpr int kColsPerBlock = 32;     // TMEM columns of one block of f16 A (128 rows x 128 B)
    static constexpr uint32_t kTmemCols = 256;   // D in [0, 64), A buffers from column 64
    static constexpr uint32_t kAcol = 64;
    static constexpr int kMaxTok = 64;
    static constexpr int kMaxW = 8, kMaxX = 6;   // ring depths at most
    static_assert(kAcol + AB * SKB * kColsPerBlock <= kTmemCols, "tensor memory");
    static constexpr int kNumBars = 2 * kMaxW + 2 * kMaxX + 2 * AB + 1;
    static constexpr int kWStage = SKB * 4096;
    __host__ __device__ static int xblock_bytes(int Tp) { return Tp * 128; }
    __host__ __device__ static int xstage_bytes(int Tp) { return SKB * Tp * 128; }
    __host__ __device__ static int corr_bytes(int T) { return 128 * (T + 1) * 4; }
    static constexpr int kMaxSlot = 4096;        // dW segment slot at most (denser dW: read in place)
    // dynamic shared memory: x ring (1024-aligned stages) first, weight ring, dW segment slots (one
    // per block of the x ring), dW sums, barriers
    __host__ __device__ static int total_bytes(int ws, int xs, int T, int Tp, int dslot, bool fold) {
        return 1024 + xs * xstage_bytes(Tp) + ws * kWStage + xs * SKB * dslot + (fold ? 0 : corr_bytes(T)) +
               kNumBars * 8 + 16;
    }
};

// Ring depths for T tokens: the weights 8 stages deep (64 KB in flight per CTA), x 4 stages;
// 6 weight stages when that keeps two CTAs on an SM.
static void mid_stages(int T, int Tp, int dslot, bool fold, int* ws, int* xs) {
    *ws = 8;
    *xs = 4;
    if (!fold && MidCfg::total_bytes(8, 4, T, Tp, dslot, false) > 100 * 1024 &&
        MidCfg::total_bytes(6, 4, T, Tp, dslot, false) <= 100 * 1024)
        *ws = 6;
}

__device__ __forceinline__ void tma_load_2d(void* smem_dst, const CUtensorMap* map, int c0, int c1, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
            "r"(smem_u32(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(smem_u32(bar))
        : "memory");
}

// Shared-memory descriptor of a K-major operand in the 128-byte swizzle layout: rows of 128 B
// (64 f16 of K), 8-row groups 1024 B apart; the K step's start is advanced inside the row.
__device__ __forceinline__ uint64_t desc_kmajor_sw128(const void* smem_ptr) {
    uint64_t d = static_cast<uint64_t>((smem_u32(smem_ptr) >> 4) & 0x3FFFu);
    d |= static_cast<uint64_t>(1) << 16;            // leading byte offset (unused with this swizzle)
    d |= static_cast<uint64_t>(1024 >> 4) << 32;    // stride byte offset: 8 rows x 128 B
    d |= static_cast<uint64_t>(1) << 46;            // descriptor version for sm_100
    d |= static_cast<uint64_t>(2) << 61;            // layout: 128-byte swizzle
    return d;
}

__device__ __forceinline__ void tc_ld16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr)
        : "memory");
}

__device__ __forceinline__ void aux_bar() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

// f16 element (token t, column c) of a staged block: row t is 128 B, its 16-byte chunk j stored at
// chunk position j ^ (t % 8).
__device__ __forceinline__ float staged_x(const unsigned char* blk, int t, int c) {
    return h2f(*reinterpret_cast<const uint16_t*>(blk + t * 128 + ((((c >> 3) ^ t) & 7) << 4) + (c & 7) * 2));
}

// Warps of the two variants: the folding one has three sets of 4 dequantising warps taking stages in
// turn (a set's hand-off latency hides behind the others' work; three A buffers allow three stages in
// flight); roles follow the dequantisers.
template <bool kFold>
struct MidRoles {
    static constexpr int kDq = kFold ? 12 : 4;   // dequantising warps; warp w: TMEM lanes 32 (w % 4)
    static constexpr int kSets = kDq / 4;
    static constexpr int kWProducer = kDq, kXProducer = kDq + 1, kMma = kDq + 2, kAux0 = kDq + 3;
    static constexpr int kThreads = (kDq + 7) * 32;
};

template <bool kFold>
__global__ void __launch_bounds__(MidRoles<kFold>::kThreads, kFold ? 1 : 2)
    k_ctarq_mid(const __grid_constant__ MidParams P) {
    using C = MidCfg;
    using R = MidRoles<kFold>;
    constexpr int SKB = C::SKB, AB = C::AB, CPB = C::kColsPerBlock;
    // folding: D (plain weights) at TMEM column 0, D' (folded) at 64, per block A then A' from 128
    constexpr uint32_t kTmemCols = kFold ? 512u : C::kTmemCols;
    constexpr uint32_t kAcol = kFold ? 128u : C::kAcol;
    constexpr int kBlkCols = kFold ? 2 * CPB : CPB;
    pdl_launch_dependents();
    extern __shared__ unsigned char smem_raw[];
    __shared__ int s_abort;
    __shared__ int s_last;
    __shared__ int s_nr;
    __shared__ int s_fold;  // folding variant: this launch's tokens include routed ones
    __shared__ int s_ridx[C::kMaxTok];
    __shared__ int s_pos[C::kMaxTok];
    constexpr int kMaxDoff = 512;
    __shared__ uint32_t s_doff[kMaxDoff + 1];  // dW segment offsets of this split's blocks

    int li = 0;
#pragma unroll
    for (int i = 1; i < SC_GROUP_MAX; ++i)
        if (i < P.nl && static_cast<int>(blockIdx.x) >= P.L[i].cta0) li = i;
    const MidLayer& L = P.L[li];
    const int bid = static_cast<int>(blockIdx.x) - L.cta0;
    const int ks = P.ks;
    const int64_t rt = bid / ks;
    const int split = bid - static_cast<int>(rt) * ks;
    const int64_t kb_begin = (L.KB * split) / ks, kb_end = (L.KB * (split + 1)) / ks;
    const int nkb = static_cast<int>(kb_end - kb_begin);
    const int nst = (nkb + SKB - 1) / SKB;
    const int T = P.T, Tp = P.Tp, WS = P.wstages, XS = P.xstages;
    const int xbb = C::xblock_bytes(Tp), xsb = C::xstage_bytes(Tp);

    // the 128-byte swizzle wants 1024-byte aligned tiles
    unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    unsigned char* xring = smem;
    unsigned char* wring = smem + XS * xsb;
    unsigned char* dring = wring + WS * C::kWStage;  // [XS][SKB] dW segment slots
    const int dslot = P.dslot;
    float* corr_s = reinterpret_cast<float*>(dring + XS * SKB * dslot);
    uint64_t* wfull = reinterpret_cast<uint64_t*>(reinterpret_cast<unsigned char*>(corr_s) + (kFold ? 0 : C::corr_bytes(T)));
    uint64_t* wempty = wfull + WS;
    uint64_t* xfull = wempty + WS;
    uint64_t* xempty = xfull + XS;
    uint64_t* a_full = xempty + XS;
    uint64_t* a_empty = a_full + AB;
    uint64_t* done = a_empty + AB;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

    if (tid == 0) {
        for (int i = 0; i < WS; ++i) {
            mbar_init(&wfull[i], 1);
            mbar_init(&wempty[i], 4);  // the set of dequantising warps of that stage
        }
        for (int i = 0; i < XS; ++i) {
            mbar_init(&xfull[i], 1);
            mbar_init(&xempty[i], 1 + 4);  // the MMA commit and the four auxiliary (folding: dequantising) warps
        }
        for (int i = 0; i < AB; ++i) {
            mbar_init(&a_full[i], 4);
            mbar_init(&a_empty[i], 1);
        }
        mbar_init(done, 1);
        fence_mbar_init();
        s_abort = 0;
        s_last = 0;
        s_fold = 0;
    }
    if (warp == R::kMma) {
        tmem_alloc(tmem_slot, kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    int wissued = 0, xissued = 0;
    if (warp == R::kWProducer) {
        if (lane == 0) {
            // the weights do not depend on the previous kernels: no dependency wait
            const uint64_t pol = policy_evict_first();
            for (int it = 0; it < nst; ++it) {
                const int slot = it % WS;
                if (it >= WS && (s_abort || !mbar_wait(&wempty[slot], ((it / WS) - 1) & 1, L.status))) {
                    s_abort = 1;
                    break;
                }
                const int64_t kb0 = kb_begin + static_cast<int64_t>(it) * SKB;
                const int n = static_cast<int>(imin64(SKB, kb_end - kb0));
                mbar_arrive_expect_tx(&wfull[slot], static_cast<uint32_t>(n * 4096));
                bulk_g2s_stream(wring + slot * C::kWStage, L.wq + (rt * L.KB + kb0) * 1024,
                                static_cast<uint32_t>(n * 4096), &wfull[slot], pol);
                ++wissued;
            }
        }
    } else if (warp == R::kXProducer) {
        pdl_wait();  // the tokens (and their routing) are the previous kernels' output
        // with a routed token, each stage also brings the blocks' dW segments (fold lists)
        const uint8_t* lists = kFold ? L.fold : L.dseg;
        const uint32_t* listoff = kFold ? L.foldoff : L.dsegoff;
        const bool segs = dslot > 0 && lists != nullptr && (P.route_all || *L.nrouted > 0);
        // the split's list offsets, loaded by the whole warp before the first stage needs them
        const bool pre = segs && nkb < kMaxDoff;
        if (pre)
            for (int j = lane; j <= nkb; j += 32) s_doff[j] = listoff[rt * L.KB + kb_begin + j];
        __syncwarp();
        if (lane == 0) {
            if (kFold) s_fold = segs ? 1 : 0;  // published by the first stage's arrive
            for (int it = 0; it < nst; ++it) {
                const int xs = it % XS;
                if (it >= XS && (s_abort || !mbar_wait(&xempty[xs], ((it / XS) - 1) & 1, L.status))) {
                    s_abort = 1;
                    break;
                }
                const int64_t kb0 = kb_begin + static_cast<int64_t>(it) * SKB;
                const int n = static_cast<int>(imin64(SKB, kb_end - kb0));
                auto doff = [&](int64_t kb) {
                    return pre ? s_doff[kb - kb_begin] : listoff[rt * L.KB + kb];
                };
                uint32_t dbytes = 0;
                if (segs) dbytes = doff(kb0 + n) - doff(kb0);
                mbar_arrive_expect_tx(&xfull[xs], static_cast<uint32_t>(n * xbb) + dbytes);
                for (int k = 0; k < n; ++k)
                    tma_load_2d(xring + xs * xsb + k * xbb, &P.xmap, static_cast<int>(P.x_col0 + (kb0 + k) * 64), 0,
                                &xfull[xs]);
                if (segs) {
                    for (int k = 0; k < n; ++k) {
                        const uint32_t o0 = doff(kb0 + k), o1 = doff(kb0 + k + 1);
                        bulk_g2s(dring + (xs * SKB + k) * dslot, lists + o0, o1 - o0, &xfull[xs]);
                    }
                }
                ++xissued;
            }
        }
    } else if (warp == R::kMma) {
        const uint32_t idesc = idesc_f16_f32(128, Tp);
        bool ok = true;
        bool fo = false;  // folding: the routed tokens' products on A' as well
        for (int u = 0; u < nst && ok; ++u) {
            const int xs = u % XS, b = u % AB;
            ok = __all_sync(0xffffffffu, mbar_wait(&xfull[xs], (u / XS) & 1, L.status));
            if (ok) ok = __all_sync(0xffffffffu, mbar_wait(&a_full[b], (u / AB) & 1, L.status));
            if (!ok) break;
            tc_fence_after();
            if (kFold && u == 0) fo = s_fold != 0;
            const int n = nkb - u * SKB < SKB ? nkb - u * SKB : SKB;
            const uint32_t a0 = tmem + kAcol + b * SKB * kBlkCols;
            const unsigned char* xb = xring + xs * xsb;
            if (elect_one()) {
                for (int k = 0; k < n; ++k) {
                    const uint64_t bd = desc_kmajor_sw128(xb + k * xbb);
#pragma unroll
                    for (int i = 0; i < 4; ++i)  // K step i: 16 columns = 32 B further along the rows
                        tc_mma_ts(tmem, a0 + k * kBlkCols + i * 8, bd + static_cast<uint64_t>(2 * i), idesc,
                                  (u | k | i) ? 1u : 0u);
                    if (kFold && fo) {
#pragma unroll
                        for (int i = 0; i < 4; ++i)
                            tc_mma_ts(tmem + 64, a0 + k * kBlkCols + CPB + i * 8, bd + static_cast<uint64_t>(2 * i),
                                      idesc, (u | k | i) ? 1u : 0u);
                    }
                }
                tc_commit(&a_empty[b]);
                tc_commit(&xempty[xs]);
            }
            __syncwarp();
        }
        if (!ok && lane == 0) s_abort = 1;
        if (elect_one()) tc_commit(done);  // also after an abort, so that the TMEM can be released
        __syncwarp();
    } else if (warp < R::kDq) {
        const int qw = warp & 3, set = warp >> 2;  // lane quadrant, stage set
        const uint32_t lane_addr = static_cast<uint32_t>(32 * qw) << 16;
        bool fo = false;
        for (int u = set; u < nst; u += R::kSets) {
            const int ws = u % WS, b = u % AB, xs = u % XS;
            if (!mbar_wait(&wfull[ws], (u / WS) & 1, L.status)) {
                s_abort = 1;
                break;
            }
            if (kFold && (u == set || fo)) {  // the stage's fold lists (and whether there are any) come with its tokens
                if (!mbar_wait(&xfull[xs], (u / XS) & 1, L.status)) {
                    s_abort = 1;
                    break;
                }
                if (u == set) fo = s_fold != 0;
            }
            const int n = nkb - u * SKB < SKB ? nkb - u * SKB : SKB;
            uint4 wv[SKB][2];  // [block][tile 2w, 2w + 1]
#pragma unroll
            for (int k = 0; k < SKB; ++k)
#pragma unroll
                for (int q = 0; q < 2; ++q)
                    if (k < n)
                        wv[k][q] = *reinterpret_cast<const uint4*>(wring + ws * C::kWStage + k * 4096 +
                                                                   (2 * qw + q) * 512 + lane * 16);
            __syncwarp();
            if (lane == 0) mbar_arrive(&wempty[ws]);
            if (u >= AB && !mbar_wait(&a_empty[b], ((u / AB) - 1) & 1, L.status)) {
                s_abort = 1;
                break;
            }
            tc_fence_after();
#pragma unroll
            for (int k = 0; k < SKB; ++k) {
#pragma unroll
                for (int q = 0; q < 2; ++q) {
                    if (k < n) {
                        const uint32_t words[4] = {wv[k][q].x, wv[k][q].y, wv[k][q].z, wv[k][q].w};
                        const uint32_t col = tmem + lane_addr + (static_cast<uint32_t>(16 * q) << 16) + kAcol +
                                             (b * SKB + k) * kBlkCols;
                        uint32_t h[4][4];
#pragma unroll
                        for (int st = 0; st < 4; ++st) {
                            dequant_word(words[st], h[st]);
                            tc_st_16x256b(col + st * 8, h[st][0], h[st][2], h[st][1], h[st][3]);
                        }
                        if (kFold && fo) {
                            // A' = (q - 8) + dW/s: this lane's entries of 16-row tile 2 warp + q
                            const unsigned char* lst = dring + (xs * SKB + k) * dslot;
                            const uint16_t* offs = reinterpret_cast<const uint16_t*>(lst) + (2 * qw + q) * 33 + lane;
                            const uint32_t* ent = reinterpret_cast<const uint32_t*>(lst + kFoldHdr);
                            const int e1 = offs[1];
                            for (int e = offs[0]; e < e1; ++e) {
                                const uint32_t w = ent[e];
                                fold_add(h, static_cast<int>((w >> 5) & 15u), static_cast<int>((w >> 9) & 1u),
                                         static_cast<uint16_t>(w >> 16));
                            }
#pragma unroll
                            for (int st = 0; st < 4; ++st)
                                tc_st_16x256b(col + CPB + st * 8, h[st][0], h[st][2], h[st][1], h[st][3]);
                        }
                    }
                }
            }
            tc_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                // the stage's fold lists are read (or none were loaded): release the token slot before
                // the MMA can run, so the slot's phase completes before another set reaches stage u + XS
                if (kFold) mbar_arrive(&xempty[xs]);
                mbar_arrive(&a_full[b]);
            }
        }
    } else {
        // ---- auxiliary warps: thread `at` owns row `at` of the tile; dW of the routed tokens
        const int at = 32 * (warp & 3) + lane;
        const int64_t row = rt * 128 + at;
        float* corr = corr_s + at * (T + 1);  // by position in the routed list
        pdl_wait();
        if (at == 0) s_nr = P.route_all ? T : *L.nrouted;
        if (at < T) s_pos[at] = -1;
        aux_bar();
        const int nr = s_nr;
        if (at < nr) {
            const int tk = P.route_all ? at : L.ridx[at];
            s_ridx[at] = tk;
            s_pos[tk] = at;
        }
        if (!kFold)  // folding: no dW sums (their shared memory is not allocated)
            for (int i = 0; i < nr; ++i) corr[i] = 0.0f;
        aux_bar();
        // the first kRegTok routed tokens' sums stay in registers (the x values of an entry are all
        // loaded before the FMAs); any further ones are added in shared memory
        constexpr int kRegTok = 16;
        float cr[kRegTok];
        int tk[kRegTok];
#pragma unroll
        for (int j = 0; j < kRegTok; ++j) {
            cr[j] = 0.0f;
            tk[j] = j < nr ? s_ridx[j] : 0;
        }
        auto add_entry = [&](const unsigned char* blk, int c, float v) {
            float xv[kRegTok];
#pragma unroll
            for (int j = 0; j < kRegTok; ++j) xv[j] = j < nr ? staged_x(blk, tk[j], c) : 0.0f;
#pragma unroll
            for (int j = 0; j < kRegTok; ++j) cr[j] = __fmaf_rn(xv[j], v, cr[j]);
            for (int i = kRegTok; i < nr; ++i) corr[i] = __fmaf_rn(staged_x(blk, s_ridx[i], c), v, corr[i]);
        };
        const bool segs = !kFold && dslot > 0 && L.dseg != nullptr && nr > 0;
        // without segments: this row's CSR entries in the split, one entry loaded ahead of its use
        int64_t e = 0, e_end = 0;
        if (!kFold && !segs && nr > 0 && row < L.N && L.nnz > 0) {
            e = L.rowptr[row];
            e_end = L.rowptr[row + 1];
            if (ks > 1) {
                e = lower_bound_u16(L.col, e, e_end, kb_begin * 64);
                e_end = lower_bound_u16(L.col, e, e_end, kb_end * 64);
            }
        }
        int64_t nc = e < e_end ? static_cast<int64_t>(L.col[e]) : INT64_MAX;
        int nv = e < e_end ? static_cast<int>(L.val[e]) : 0;
        for (int u = 0; u < (kFold ? 0 : nst); ++u) {  // folding: the dequantising warps apply dW
            const int xs = u % XS;
            if (!mbar_wait(&xfull[xs], (u / XS) & 1, L.status)) {
                s_abort = 1;
                break;
            }
            const int n = nkb - u * SKB < SKB ? nkb - u * SKB : SKB;
            if (segs) {
                for (int k = 0; k < n; ++k) {
                    const unsigned char* sg = dring + (xs * SKB + k) * dslot;
                    const uint16_t* ro = reinterpret_cast<const uint16_t*>(sg);
                    const uint16_t* en = reinterpret_cast<const uint16_t*>(sg + 272);
                    const unsigned char* blk = xring + xs * xsb + k * xbb;
                    for (int q = ro[at]; q < ro[at + 1]; ++q) {
                        const uint32_t w = en[q];
                        const int c = static_cast<int>(w & 63u);
                        add_entry(blk, c, __fmul_rn(static_cast<float>(static_cast<int8_t>(w >> 6)), L.ds));
                    }
                }
            }
            const int64_t cend = (kb_begin + static_cast<int64_t>(u) * SKB + n) * 64;
            while (nc < cend) {
                const int64_t rel = nc - kb_begin * 64 - static_cast<int64_t>(u) * SKB * 64;
                const unsigned char* blk = xring + xs * xsb + static_cast<int>(rel >> 6) * xbb;
                const int c = static_cast<int>(rel & 63);
                const float v = __fmul_rn(static_cast<float>(nv), L.ds);
                ++e;
                nc = e < e_end ? static_cast<int64_t>(L.col[e]) : INT64_MAX;  // the next entry, loaded ahead
                nv = e < e_end ? static_cast<int>(L.val[e]) : 0;
                add_entry(blk, c, v);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&xempty[xs]);
        }
#pragma unroll
        for (int j = 0; j < kRegTok; ++j)
            if (!kFold && j < nr) corr[j] = cr[j];
    }

    // ---- epilogue (auxiliary warps): y = acc * s + dW of routed tokens
    if (warp >= R::kAux0) {
        const int at = 32 * (warp & 3) + lane;
        const int64_t row = rt * 128 + at;
        const float* corr = corr_s + at * (T + 1);
        const float sc = row < L.N ? __ldg(L.scale + row) : 0.0f;
        // the producer's condition for the fold lists (route_all: s_nr = T)
        const bool fo = kFold && dslot > 0 && L.fold != nullptr && s_nr > 0;
        const bool ok = mbar_wait(done, 0, L.status);
        if (!ok) s_abort = 1;
        tc_fence_after();
        const uint32_t lane_base = tmem + (static_cast<uint32_t>(32 * (warp & 3)) << 16);
#pragma unroll 1
        for (int t0 = 0; t0 < Tp; t0 += 16) {
            uint32_t d[16], d2[16];
            tc_ld16(lane_base + t0, d);
            if (fo) tc_ld16(lane_base + 64 + t0, d2);
            tc_wait_ld();
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                const int t = t0 + j;
                if (t >= T) break;
                const int p = s_pos[t];
                float v;
                if (kFold) {
                    v = __fmul_rn(__uint_as_float(fo && p >= 0 ? d2[j] : d[j]), sc);
                } else {
                    const float base = __fmul_rn(__uint_as_float(d[j]), sc);
                    v = p >= 0 ? __fadd_rn(base, corr[p]) : base;
                }
                if (ks == 1) {
                    if (row < L.N && !s_abort) {
                        const int64_t oi = static_cast<int64_t>(t) * L.N + row;
                        if (L.partial_out) reinterpret_cast<float*>(L.y)[oi] = v;
                        else store_output(L.y, L.y_dtype, oi, v, L.bias, row);
                    }
                } else {
                    L.partial[((rt * ks + split) * T + t) * 128 + at] = v;
                }
            }
        }
    }
    __syncwarp();  // single-lane roles rejoin their warp before the warp-wide TMEM release below
    tc_fence_before();
    __syncthreads();
    if (warp == R::kMma) {
        if (s_abort) mbar_wait(done, 0, nullptr, kDrainNs);
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
    if (s_abort && warp == R::kWProducer && lane == 0)
        for (int it = wissued > WS ? wissued - WS : 0; it < wissued; ++it)
            mbar_wait(&wfull[it % WS], (it / WS) & 1, nullptr, kDrainNs);
    if (s_abort && warp == R::kXProducer && lane == 0)
        for (int it = xissued > XS ? xissued - XS : 0; it < xissued; ++it)
            mbar_wait(&xfull[it % XS], (it / XS) & 1, nullptr, kDrainNs);
    if (ks == 1) return;

    // ---- column splits: the last CTA of the row tile adds the splits in order and writes y
    if (tid == 0) {
        __threadfence();
        const unsigned ticket = atomicAdd(L.rtcount + rt, 1u);
        s_last = (ticket == static_cast<unsigned>(ks - 1)) ? 1 : 0;
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    // every thread of the CTA: items of 4 consecutive rows of one token, the splits' rows loaded
    // four splits at a time and added in split order
    const float* pr = L.partial + (rt * ks * T) * 128;
    const int items = T * 32;
    for (int it2 = tid; it2 < items && !s_abort; it2 += R::kThreads) {
        const int t = it2 >> 5, r4 = (it2 & 31) * 4;
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int s0 = 0; s0 < ks; s0 += 4) {
            float4 lv[4];
#pragma unroll
            for (int j = 0; j < 4; ++j)
                lv[j] = s0 + j < ks ? __ldcg(reinterpret_cast<const float4*>(pr + ((s0 + j) * T + t) * 128 + r4))
                                    : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
            for (int j = 0; j < 4; ++j)
                if (s0 + j < ks) {
                    v.x = __fadd_rn(v.x, lv[j].x);
                    v.y = __fadd_rn(v.y, lv[j].y);
                    v.z = __fadd_rn(v.z, lv[j].z);
                    v.w = __fadd_rn(v.w, lv[j].w);
                }
        }
        const float o[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const int64_t row = rt * 128 + r4 + q;
            if (row < L.N) {
                const int64_t oi = static_cast<int64_t>(t) * L.N + row;
                if (L.partial_out) reinterpret_cast<float*>(L.y)[oi] = o[q];
                else store_output(L.y, L.y_dtype, oi, o[q], L.bias, row);
            }
        }
    }
    if (tid == 0) L.rtcount[rt] = 0u;
}

// ---------------------------------------------------------------- host side

// dW segments of the 9..64-token GEMM: per (128-row tile, 64-column block), the u16 offsets of the
// tile's 128 rows (and the end) into u16 entries (column in the block | value << 6), each row's
// columns ascending as in the CSR.  Built from the layer's CSR (local columns, ascending per row).
cudaError_t build_dw_segments(Layer& L, const uint32_t* srp, const uint16_t* scol, const int8_t* sval) {
    if (L.nnz == 0) return cudaSuccess;
    const int64_t RT = L.Np / 128, KB = L.KB;
    std::vector<uint32_t> off(static_cast<size_t>(RT * KB + 1), 0);
    std::vector<uint8_t> blob;
    std::vector<uint32_t> cur(128), end(128);
    std::vector<uint16_t> roff(129), ents;
    int64_t maxb = 0;
    for (int64_t rt = 0; rt < RT; ++rt) {
        for (int r = 0; r < 128; ++r) {
            const int64_t row = rt * 128 + r;
            cur[r] = row < L.N ? srp[row] : 0;
            end[r] = row < L.N ? srp[row + 1] : 0;
        }
        for (int64_t kb = 0; kb < KB; ++kb) {
            ents.clear();
            for (int r = 0; r < 128; ++r) {
                roff[r] = static_cast<uint16_t>(ents.size());
                while (cur[r] < end[r] && scol[cur[r]] < (kb + 1) * 64) {
                    const int c = static_cast<int>(scol[cur[r]] - kb * 64);
                    ents.push_back(static_cast<uint16_t>(c | ((static_cast<uint32_t>(static_cast<uint8_t>(sval[cur[r]]))) << 6)));
                    ++cur[r];
                }
            }
            if (ents.size() > 65535) return cudaSuccess;  // u16 offsets cannot describe it: no segments
            roff[128] = static_cast<uint16_t>(ents.size());
            const size_t bytes = 272 + ((ents.size() * 2 + 15) / 16) * 16;
            const size_t at = blob.size();
            blob.resize(at + bytes, 0);
            std::memcpy(&blob[at], roff.data(), 129 * 2);
            if (!ents.empty()) std::memcpy(&blob[at + 272], ents.data(), ents.size() * 2);
            if (blob.size() > 0xFFFFFFFFull) return cudaSuccess;
            off[rt * KB + kb + 1] = static_cast<uint32_t>(blob.size());
            maxb = std::max<int64_t>(maxb, static_cast<int64_t>(bytes));
        }
    }
    cudaError_t e = cudaMalloc(&L.dseg, blob.size());
    if (e == cudaSuccess) e = cudaMalloc(&L.dsegoff, off.size() * 4);
    if (e == cudaSuccess) e = cudaMemcpy(L.dseg, blob.data(), blob.size(), cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMemcpy(L.dsegoff, off.data(), off.size() * 4, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) {
        cudaFree(L.dseg);
        cudaFree(L.dsegoff);
        L.dseg = nullptr;
        L.dsegoff = nullptr;
        return e;
    }
    L.dseg_max = static_cast<int>(maxb);
    L.device_bytes += static_cast<int64_t>(blob.size() + off.size() * 4);
    return cudaSuccess;
}

static PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static std::once_flag once;
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

static int mid_tp(int64_t m) { return static_cast<int>(((m + 15) / 16) * 16); }

static int mid_ctas_per_sm(int64_t m) {
    static std::atomic<int> cache[64][MidCfg::kMaxTok + 1];
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64 || m < 1 || m > MidCfg::kMaxTok) return 1;
    const int have = cache[dev][m].load();
    if (have > 0) return have;
    int ws, xs;
    const int T = static_cast<int>(m), Tp = mid_tp(m);
    mid_stages(T, Tp, MidCfg::kMaxSlot / 4, false, &ws, &xs);
    // shared memory decides (a block's registers and threads fit twice; two CTAs share the 512
    // tensor-memory columns of an SM); the folding variant takes all 512 columns
    const int smem = MidCfg::total_bytes(ws, xs, T, Tp, MidCfg::kMaxSlot / 4, false);
    const int n = m >= kMidFoldMinTokens ? 1 : smem + 2048 <= 112 * 1024 ? 2 : 1;
    cache[dev][m].store(n);
    return n;
}

int mid_ksplit(int64_t rt_total, int64_t kb, int sms, int64_t m) {
    const int64_t wave = static_cast<int64_t>(sms) * mid_ctas_per_sm(m);
    int64_t ks = (wave + rt_total / 2) / rt_total;
    const int64_t kmax = kb / 4 > 0 ? kb / 4 : 1;  // at least four blocks (two stages) per split
    if (ks > kmax) ks = kmax;
    // the last CTA of a row tile reads ks x m partial rows: fewer splits beyond 16 tokens
    const int64_t cap = m <= 16 ? 16 : 8;
    if (ks > cap) ks = cap;
    if (ks < 1) ks = 1;
    return static_cast<int>(ks);
}

cudaError_t launch_mid(const MidArgs& a, cudaStream_t s) {
    const int n = a.n;
    if (n < 1 || n > SC_GROUP_MAX || a.m < 1 || a.m > MidCfg::kMaxTok) return cudaErrorInvalidValue;
    PFN_cuTensorMapEncodeTiled_v12000 encode = tensor_map_encoder();
    if (!encode) return cudaErrorNotSupported;
    const Layer& L0 = *a.layer[0];
    const int T = static_cast<int>(a.m), Tp = mid_tp(a.m);
    cudaError_t e;
    const bool copy = a.x_dtype == SC_BF16 || (reinterpret_cast<uintptr_t>(a.x) & 15u) != 0;
    const void* xf16 = copy ? static_cast<const void*>(a.xconv) : a.x;
    if (!a.routed_in || copy) {
        // route every token (and, for bf16 or unaligned tokens, write their f16 copy)
        MidRouteParams r = {};
        r.x = a.x;
        r.x_dtype = a.x_dtype;
        r.vec_ok = ((reinterpret_cast<uintptr_t>(a.x) & 15u) == 0 && (a.x_stride % 8) == 0) ? 1 : 0;
        r.x_stride = a.x_stride;
        r.r.M = T;
        r.r.nl = a.routed_in ? 0 : n;
        for (int i = 0; i < SC_GROUP_MAX; ++i) {
            const Layer& L = *a.layer[i < n ? i : 0];
            r.r.t4[i] = L.t4;
            r.r.t8[i] = L.t8;
            r.r.mask[i] = a.mask[i < n ? i : 0];
            r.r.ridx[i] = a.ridx[i < n ? i : 0];
            r.r.nrouted[i] = a.nrouted[i < n ? i : 0];
        }
        r.r.route_all = a.route_all;
        r.r.rc = route_consts(a.x_stride);
        r.xcopy = copy ? a.xconv : nullptr;
        r.r.counter = a.counter;
        const size_t row_bytes = static_cast<size_t>((a.x_stride * 2 + 15) / 16 * 16);
        static std::atomic<uint64_t> rflags{0};
        int rdev = 0;
        cudaGetDevice(&rdev);
        if (!(rflags.load() & (1ull << (rdev & 63)))) {
            e = cudaFuncSetAttribute(k_mid_route<256>, cudaFuncAttributeMaxDynamicSharedMemorySize, kRouterMaxRowBytes);
            if (e != cudaSuccess) return e;
            rflags.fetch_or(1ull << (rdev & 63));
        }
        if (row_bytes > static_cast<size_t>(kRouterMaxRowBytes)) return cudaErrorInvalidValue;
        e = launch_pdl(k_mid_route<256>, dim3(static_cast<unsigned>(T)), dim3(256), row_bytes, s, r);
        if (e != cudaSuccess) return e;
    }
    MidParams* Pp = new MidParams();  // large and 64-byte aligned
    MidParams& P = *Pp;
    {
        const cuuint64_t dims[2] = {static_cast<cuuint64_t>(a.x_stride), static_cast<cuuint64_t>(a.m)};
        const cuuint64_t strides[1] = {static_cast<cuuint64_t>(a.x_stride * 2)};
        const cuuint32_t box[2] = {64, static_cast<cuuint32_t>(Tp)};
        const cuuint32_t estr[2] = {1, 1};
        const CUresult r = encode(&P.xmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(xf16), dims, strides,
                                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                  CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (r != CUDA_SUCCESS) {
            delete Pp;
            return cudaErrorInvalidValue;
        }
    }
    P.nl = n;
    P.ks = a.ks;
    P.T = T;
    P.Tp = Tp;
    // from 17 tokens the dequantising warps fold dW/s into a second A (every layer needs its lists);
    // else a dW segment slot: the group's largest segment, if it fits the slot limit
    bool fold = T >= kMidFoldMinTokens;
    int fcap = 0;
    for (int i = 0; i < n; ++i) {
        const Layer& L = *a.layer[i];
        if (L.nnz > 0 && !L.fold) fold = false;
        if (L.fold) fcap = std::max(fcap, L.fold_cap);
    }
    if (fold) {
        P.dslot = fcap;
    } else {
        int dmax = 0;
        bool dok = true;
        for (int i = 0; i < n; ++i) {
            const Layer& L = *a.layer[i];
            if (L.nnz > 0 && !L.dseg) dok = false;
            dmax = std::max(dmax, L.dseg_max);
        }
        P.dslot = (dok && dmax > 0 && dmax <= MidCfg::kMaxSlot) ? dmax : 0;
    }
    mid_stages(T, Tp, P.dslot, fold, &P.wstages, &P.xstages);
    P.route_all = a.route_all;
    P.x_col0 = a.x_col0;
    int ctas = 0;
    int64_t rt_off = 0;
    for (int i = 0; i < n; ++i) {
        const Layer& L = *a.layer[i];
        MidLayer& M = P.L[i];
        M.wq = L.wq;
        M.scale = L.scale;
        M.rowptr = L.rowptr;
        M.col = L.col;
        M.val = L.val;
        M.ds = L.ds;
        M.nnz = L.nnz;
        M.N = L.N;
        M.KB = L.KB;
        M.RT = L.Np / 128;
        M.y = a.y[i];
        M.y_dtype = a.y_dtype;
        M.bias = a.bias[i];
        M.partial_out = a.partial_out;
        M.partial = a.partial + rt_off * a.ks * a.m * 128;
        M.rtcount = a.rtcount + rt_off;
        M.status = L.status;
        M.ridx = a.ridx[i];
        M.nrouted = a.nrouted[i];
        M.dseg = L.dseg;
        M.dsegoff = L.dsegoff;
        M.fold = L.fold;
        M.foldoff = L.foldoff;
        M.cta0 = ctas;
        ctas += static_cast<int>(M.RT * a.ks);
        rt_off += M.RT;
    }
    for (int i = n; i < SC_GROUP_MAX; ++i) {
        P.L[i] = P.L[0];
        P.L[i].cta0 = ctas;
    }
    const int smem = MidCfg::total_bytes(P.wstages, P.xstages, T, Tp, P.dslot, fold);
    static std::atomic<uint64_t> flags[2] = {{0}, {0}};
    int dev = 0;
    cudaGetDevice(&dev);
    const uint64_t bit = 1ull << (dev & 63);
    auto kern = fold ? k_ctarq_mid<true> : k_ctarq_mid<false>;
    e = cudaSuccess;
    if (!(flags[fold ? 1 : 0].load() & bit)) {
        e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 220 * 1024);
        if (e == cudaSuccess) e = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
        if (e == cudaSuccess) flags[fold ? 1 : 0].fetch_or(bit);
    }
    const int threads = fold ? MidRoles<true>::kThreads : MidRoles<false>::kThreads;
    if (e == cudaSuccess) e = launch_pdl(kern, dim3(static_cast<unsigned>(ctas)), dim3(threads), smem, s, P);
    delete Pp;
    return e;
}

}  // namespace sc
