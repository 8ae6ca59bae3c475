// sc_api.cu -- the extern "C" entry points of libsaccade_ctarq.so.
//
// sc_layer_create mirrors SaccadeLinearOp::new (config.rs:76-150): it takes the
// reference-format buffers, validates the dW CSR (the reference would panic on a column
// >= in_features in build_csc, config.rs:176), and builds the device layout.  sc_forward
// mirrors cpu_fwd (op.rs:10-185): router -> base product -> dW for routed tokens -> f16.
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cstring>
#include <limits>
#include <mutex>
#include <string>
#include <vector>

#include "sc_internal.h"

namespace sc {

static thread_local std::string g_last_error;
static std::atomic<int> g_bypass{0};
std::atomic<uint64_t> g_launches{0};

void set_error(const std::string& msg) { g_last_error = msg; }

sc_status cuda_fail(cudaError_t e, const char* what) {
    set_error(std::string(what) + ": " + cudaGetErrorName(e) + " (" + cudaGetErrorString(e) + ")");
    return SC_ECUDA;
}

// Restores the caller's current device on scope exit.
struct DeviceGuard {
    int prev = -1;
    bool ok = false;
    explicit DeviceGuard(int dev) {
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        ok = (prev == dev) || (cudaSetDevice(dev) == cudaSuccess);
    }
    ~DeviceGuard() {
        if (prev >= 0) cudaSetDevice(prev);
    }
};

static int64_t ceil_to(int64_t v, int64_t m) { return (v + m - 1) / m * m; }

static int sm_count(int dev) {
    int n = 148;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    return n > 0 ? n : 148;
}

// Workspace layout.  The first kCounterBytes hold completion counters (the router's at
// offset 0, the split-K row-tile counters after it) at offsets that do not depend on the
// layer or the token count, so one workspace can serve every layer: each call returns the
// counters it used to zero.  Everything after that region is scratch rewritten per call.
// Column splits of the router-fused decode kernel.  The splits of one 128-row tile form a
// thread-block cluster (at most kMaxFusedCluster CTAs) that reduces through distributed shared
// memory.  The split count (= cluster size) for a launch of `rt` row tiles of `kb` column
// blocks: the largest ks whose rt clusters can all be resident at once (one wave: cluster
// packing into the GPCs decides, measured by the occupancy query for two CTAs per SM), with at
// least two column blocks per CTA and each CTA's slice of x within its shared-memory copy.  A
// launch whose weights all fit the rings of one CTA per SM gets half the clusters (about one
// CTA per SM): it then fits beside its neighbour in the stream, whose CTAs hold the other
// slot, and loads all of its weights while that one runs.  0 when no split fits a cluster.
int choose_ksplit(int64_t rt, int64_t kb) {
    const int64_t min_ks = (kb + fused_max_kb(1) - 1) / fused_max_kb(1);
    if (min_ks > kMaxFusedCluster) return 0;
    const bool small = rt * kb * 4096 * 100 <= fused_prefetch_bytes() * SC_FUSED_SMALL_PCT;
    int best = 0;
    for (int ks = 1; ks <= kMaxFusedCluster; ++ks) {
        if (ks < min_ks || (ks > 1 && kb / ks < 2)) continue;
        const int cap = fused_max_active_clusters(ks) / (small ? 2 : 1);
        if (best == 0 || (cap > 0 && rt <= cap)) best = ks;  // larger ks wins while one wave holds
    }
    return best;
}

int fused_ksplit(const Layer& L) { return choose_ksplit(L.Np / 128, L.KB); }

bool use_fused_ks(const Layer& L, int64_t m, int ks) {
    if (L.mode == SC_MODE_EXACT || m > 8 || ks <= 0) return false;
    return (L.KB + ks - 1) / ks <= fused_max_kb(m);  // the x slice fits the CTA's copy
}

bool use_fused(const Layer& L, int64_t m) { return use_fused_ks(L, m, L.ks_fused); }

bool use_mid(const Layer& L, int64_t m) {
    return L.mode != SC_MODE_EXACT && m >= kMidMinTokens && m <= kMidMaxTokens && !use_fused(L, m);
}

// dW blocks of the router-fused decode for `ks` column splits, from the host CSR (columns local
// to the layer, ascending per row): for every (row tile, split), 129 u16 row offsets (272 B), the
// u16 columns relative to the split, then the i8 values, each padded to 16 B; off[rt * ks + sp]
// is the byte offset of a block.  When a block would exceed the kernel's shared-memory copy,
// every CTA of the layer reads its block from global memory instead (`global`).  Left empty (the
// kernel then reads the CSR) when a block holds more entries than u16 offsets describe.
struct DwBlocks {
    uint8_t* blk = nullptr;
    uint32_t* off = nullptr;
    int64_t bytes = 0;
    int global = 0;
};

static cudaError_t build_dw_blocks(const Layer& L, int ks, const uint32_t* srp, const uint16_t* scol,
                                   const int8_t* sval, DwBlocks* out) {
    *out = DwBlocks{};
    if (L.nnz == 0 || ks <= 0) return cudaSuccess;
    const int64_t RT = L.Np / 128;
    std::vector<uint32_t> off(RT * ks + 1, 0);
    std::vector<uint8_t> blob;
    std::vector<uint16_t> roff(129), cols;
    std::vector<int8_t> vals;
    int global = 0;
    for (int64_t rt = 0; rt < RT; ++rt) {
        for (int64_t sp = 0; sp < ks; ++sp) {
            const int64_t bc0 = (L.KB * sp / ks) * 64, bc1 = (L.KB * (sp + 1) / ks) * 64;
            cols.clear();
            vals.clear();
            for (int r = 0; r < 128; ++r) {
                roff[r] = static_cast<uint16_t>(cols.size());
                const int64_t row = rt * 128 + r;
                if (row < L.N) {
                    for (uint32_t q = srp[row]; q < srp[row + 1]; ++q) {
                        if (scol[q] >= bc0 && scol[q] < bc1) {
                            cols.push_back(static_cast<uint16_t>(scol[q] - bc0));
                            vals.push_back(sval[q]);
                        }
                    }
                }
            }
            const size_t n = cols.size();
            if (n > 65535) return cudaSuccess;  // u16 row offsets cannot describe the block
            roff[128] = static_cast<uint16_t>(n);
            const size_t bytes = 272 + ((n * 2 + 15) / 16) * 16 + ((n + 15) / 16) * 16;
            if (static_cast<int64_t>(bytes) > kDwBlockMax) global = 1;
            if (blob.size() + bytes > 0xFFFFFFFFull) return cudaSuccess;  // u32 block offsets
            const size_t at = blob.size();
            blob.resize(at + bytes, 0);
            std::memcpy(&blob[at], roff.data(), 129 * 2);
            if (n) {
                std::memcpy(&blob[at + 272], cols.data(), n * 2);
                std::memcpy(&blob[at + 272 + ((n * 2 + 15) / 16) * 16], vals.data(), n);
            }
            off[rt * ks + sp + 1] = static_cast<uint32_t>(blob.size());
        }
    }
    cudaError_t e = cudaMalloc(&out->blk, blob.size());
    if (e == cudaSuccess) e = cudaMalloc(&out->off, off.size() * 4);
    if (e == cudaSuccess) e = cudaMemcpy(out->blk, blob.data(), blob.size(), cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMemcpy(out->off, off.data(), off.size() * 4, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) {
        cudaFree(out->blk);
        cudaFree(out->off);
        *out = DwBlocks{};
        return e;
    }
    out->bytes = static_cast<int64_t>(blob.size() + off.size() * 4);
    out->global = global;
    return cudaSuccess;
}

WsLayout plan_workspace(const Layer& L, int64_t m) {
    WsLayout w;
    w.Mp = m <= 16 ? 16 : ceil_to(m, 32);
    w.chunk_tokens = 32;
    w.counter = 0;
    w.rtcount = 256;
    size_t off = kCounterBytes;
    auto take = [&](size_t bytes) {
        size_t o = off;
        off = static_cast<size_t>(ceil_to(static_cast<int64_t>(off + bytes), 256));
        return o;
    };
    w.xk = take(static_cast<size_t>(L.KB * 64 * w.Mp * 2));  // [KB][Mp/8][8][8][8] f16
    w.mask = take(static_cast<size_t>(m > 0 ? m : 1));
    w.scores = take(static_cast<size_t>(4 * (m > 0 ? m : 1)));
    w.ridx = take(static_cast<size_t>(4 * (m > 0 ? m : 1)));
    w.nrouted = take(16);
    // one CTA per SM (the ring takes ~200 KB of shared memory): split K so that the
    // 128-row tiles times the splits cover the SMs, with at least one 4-block stage each
    const int64_t RT = L.Np / 128;
    const int64_t target = static_cast<int64_t>(L.sms);
    int64_t ks = (target + RT / 2) / RT;
    ks = std::max<int64_t>(1, std::min<int64_t>(ks, std::min<int64_t>(32, std::max<int64_t>(1, L.KB / 4))));
    if (use_fused(L, m)) {
        w.ksplit = L.ks_fused;  // reduced inside the cluster: no partial buffer
        w.partial = take(16);
    } else if (use_mid(L, m)) {
        // 9..64-token GEMM: split partials, an f16 copy of bf16 (or unaligned) tokens
        const int64_t kfull = L.shard_kind == SC_SHARD_ROWS ? L.fullK : L.K;
        w.mid_ks = mid_ksplit(RT, L.KB, L.sms, m);
        w.partial = take(static_cast<size_t>(w.mid_ks > 1 ? RT * w.mid_ks * m * 128 * 4 : 16));
        w.xconv = take(static_cast<size_t>(m * kfull * 2));
    } else if (L.mode != SC_MODE_EXACT && m >= kGemmMinTokens) {
        // prefill GEMM: x again in routed-first order, that order, split partials
        w.gemm_ks = gemm_ksplit(L, m);
        w.xkp = take(static_cast<size_t>(L.KB * 64 * (w.Mp + 16) * 2));
        w.perm = take(static_cast<size_t>(4 * (w.Mp + 16)));
        const int64_t tiles = RT * ((m + gemm_tile_tokens() - 1) / gemm_tile_tokens() + 1);
        w.partial = take(static_cast<size_t>(w.gemm_ks > 1 ? tiles * w.gemm_ks * gemm_tile_tokens() * 256 * 4 : 16));
    } else {
        w.ksplit = static_cast<int>(ks);
        w.partial = take(static_cast<size_t>(ks > 1 ? RT * ks * 128 * 32 * 4 : 16));
    }
    // a ROWS shard's exchange (sc_forward_split) also needs its slice transposed, [K][tokens to 16],
    // after everything its base product's own layout (an unsharded one, never larger) may use
    if (L.shard_kind == SC_SHARD_ROWS) w.xt = take(static_cast<size_t>(L.KB * 64 * ((m + 15) / 16 * 16) * 2));
    w.total = off;
    return w;
}

// ------------------------------------------------------------------ default workspaces

struct DefaultWs {
    void* ptr = nullptr;
    size_t bytes = 0;
};
static std::mutex g_ws_mu;
static std::vector<DefaultWs> g_ws;

static sc_status default_workspace(int dev, size_t need, void** out) {
    std::lock_guard<std::mutex> lk(g_ws_mu);
    if (static_cast<int>(g_ws.size()) <= dev) g_ws.resize(dev + 1);
    DefaultWs& d = g_ws[dev];
    if (d.bytes < need) {
        cudaError_t e = cudaDeviceSynchronize();
        if (e != cudaSuccess) return cuda_fail(e, "default workspace: synchronize");
        if (d.ptr) cudaFree(d.ptr);
        d.ptr = nullptr;
        d.bytes = 0;
        size_t sz = std::max<size_t>(need, static_cast<size_t>(1) << 20);
        e = cudaMalloc(&d.ptr, sz);
        if (e != cudaSuccess) return cuda_fail(e, "default workspace: cudaMalloc");
        e = cudaMemset(d.ptr, 0, sz);
        if (e != cudaSuccess) return cuda_fail(e, "default workspace: memset");
        d.bytes = sz;
    }
    *out = d.ptr;
    return SC_OK;
}

// ------------------------------------------------------------------ forward

static sc_status forward_impl(const Layer& L, const void* x, int x_dtype, int64_t m, void* y, int y_dtype,
                              const float* bias, uint8_t* mask_out, int32_t* ridx_out, int32_t* nrouted_out,
                              void* ws, size_t ws_bytes, cudaStream_t stream, bool partial,
                              bool base_only = false, bool reuse_route = false) {
    if (m < 0) {
        set_error("sc_forward: negative token count");
        return SC_EINVAL;
    }
    if (m == 0) return SC_OK;
    if (!x || !y) {
        set_error("sc_forward: null x or y");
        return SC_EINVAL;
    }
    if (x_dtype != SC_F16 && x_dtype != SC_BF16) {
        set_error("sc_forward: x dtype must be F16 or BF16");
        return SC_EINVAL;
    }
    if (!partial && y_dtype != SC_F16 && y_dtype != SC_BF16 && y_dtype != SC_F32) {
        set_error("sc_forward: y dtype must be F16, BF16 or F32");
        return SC_EINVAL;
    }
    if ((reinterpret_cast<uintptr_t>(ws) & 255u) != 0) {
        set_error("sc_forward: workspace must be 256-byte aligned");
        return SC_ENONCONTIG;
    }
    const WsLayout w = plan_workspace(L, m);
    if (ws_bytes < w.total) {
        set_error("sc_forward: workspace of " + std::to_string(ws_bytes) + " bytes, need " +
                  std::to_string(w.total));
        return SC_ENOMEM;
    }
    unsigned char* base = static_cast<unsigned char*>(ws);
    const bool bypass_now = !base_only && g_bypass.load() != 0;
    if (use_fused(L, m)) {
        // one launch: router, x staging, base product and dW in the same kernel
        FusedArgs f;
        f.L = &L;
        f.x = x;
        f.x_dtype = x_dtype;
        f.x_stride = L.shard_kind == SC_SHARD_ROWS ? L.fullK : L.K;
        f.x_col0 = L.shard_kind == SC_SHARD_ROWS ? L.col_begin : 0;
        f.m = m;
        f.route_all = bypass_now ? 1 : 0;
        f.y = y;
        f.y_dtype = partial ? SC_F32 : y_dtype;
        f.bias = partial ? nullptr : bias;
        f.partial_out = partial ? 1 : 0;
        f.mask_out = mask_out;
        f.ridx_out = ridx_out;
        f.nrouted_out = nrouted_out;
        f.ws_partial = reinterpret_cast<float*>(base + w.partial);
        f.ws_rtcount = reinterpret_cast<uint32_t*>(base + w.rtcount);
        f.ksplit = w.ksplit;
        f.dwblk = L.dwblk;
        f.dwoff = L.dwoff;
        f.dw_global = L.dw_global;
        cudaError_t e = launch_decode_fused(&f, 1, stream);
        if (e != cudaSuccess) return cuda_fail(e, "fused decode launch");
        return SC_OK;
    }
    if (w.mid_ks > 0) {
        // the 9..64-token tcgen05 GEMM, router and dW in the same launch
        MidArgs a = {};
        a.n = 1;
        a.layer[0] = &L;
        a.x = x;
        a.x_dtype = x_dtype;
        a.x_stride = L.shard_kind == SC_SHARD_ROWS ? L.fullK : L.K;
        a.x_col0 = L.shard_kind == SC_SHARD_ROWS ? L.col_begin : 0;
        a.m = m;
        a.route_all = bypass_now ? 1 : 0;
        a.ks = w.mid_ks;
        a.xconv = reinterpret_cast<uint16_t*>(base + w.xconv);
        a.counter = reinterpret_cast<uint32_t*>(base + w.counter);
        a.mask[0] = mask_out ? mask_out : reinterpret_cast<uint8_t*>(base + w.mask);
        a.ridx[0] = ridx_out ? ridx_out : reinterpret_cast<int32_t*>(base + w.ridx);
        a.nrouted[0] = nrouted_out ? nrouted_out : reinterpret_cast<int32_t*>(base + w.nrouted);
        a.y[0] = y;
        a.y_dtype = partial ? SC_F32 : y_dtype;
        a.bias[0] = partial ? nullptr : bias;
        a.partial_out = partial ? 1 : 0;
        a.partial = reinterpret_cast<float*>(base + w.partial);
        a.rtcount = reinterpret_cast<uint32_t*>(base + w.rtcount);
        cudaError_t e = launch_mid(a, stream);
        if (e != cudaSuccess) return cuda_fail(e, "9..64-token GEMM launch");
        return SC_OK;
    }
    uint16_t* xk = reinterpret_cast<uint16_t*>(base + w.xk);
    uint8_t* mask = mask_out ? mask_out : reinterpret_cast<uint8_t*>(base + w.mask);
    int32_t* ridx = ridx_out ? ridx_out : reinterpret_cast<int32_t*>(base + w.ridx);
    int32_t* nrouted = nrouted_out ? nrouted_out : reinterpret_cast<int32_t*>(base + w.nrouted);
    const bool bypass = bypass_now;

    RouterArgs r;
    r.x = x;
    r.x_dtype = x_dtype;
    r.x_row_stride = L.shard_kind == SC_SHARD_ROWS ? L.fullK : L.K;
    r.x_col0 = L.shard_kind == SC_SHARD_ROWS ? L.col_begin : 0;
    r.M = m;
    r.K = L.K;
    r.Mp = w.Mp;
    r.KB = L.KB;
    r.t4 = L.t4;
    r.t8 = L.t8;
    r.route_all = bypass ? 1 : 0;
    r.xk = xk;
    r.mask = mask;
    r.scores = reinterpret_cast<float*>(base + w.scores);
    r.ridx = ridx;
    r.nrouted = nrouted;
    r.perm = w.gemm_ks > 0 ? reinterpret_cast<int32_t*>(base + w.perm) : nullptr;
    r.counter = reinterpret_cast<uint32_t*>(base + w.counter);
    r.status = L.status;
    cudaError_t e = cudaSuccess;
    if (!reuse_route) {  // else the staged x, routing and token order of the previous call stand
        e = launch_router(r, stream);
        if (e != cudaSuccess) return cuda_fail(e, "router launch");
    }

    DecodeArgs d;
    d.L = &L;
    d.xk = xk;
    d.Mp = w.Mp;
    d.mask = mask;
    d.ridx = ridx;
    d.nrouted = nrouted;
    d.route_all = bypass ? 1 : 0;
    d.dcol_begin = 0;
    d.dcol_end = L.K;
    d.y = y;
    d.y_dtype = partial ? SC_F32 : y_dtype;
    d.bias = partial ? nullptr : bias;
    d.partial_out = partial ? 1 : 0;
    d.ws_partial = reinterpret_cast<float*>(base + w.partial);
    d.ws_rtcount = reinterpret_cast<uint32_t*>(base + w.rtcount);
    if (L.mode == SC_MODE_EXACT) {
        d.tok0 = 0;
        d.ntok = m;
        d.ksplit = 1;
        e = launch_decode_exact(d, bypass ? 1 : 0, stream);
        if (e != cudaSuccess) return cuda_fail(e, "exact kernel launch");
        return SC_OK;
    }
    if (w.gemm_ks > 0) {
        GemmArgs g;
        g.L = &L;
        g.xk = xk;
        g.xkp = reinterpret_cast<uint16_t*>(base + w.xkp);
        g.perm = reinterpret_cast<const int32_t*>(base + w.perm);
        g.nrouted = nrouted;
        g.Mp = w.Mp;
        g.Mpp = w.Mp + 16;
        g.M = m;
        g.route_all = bypass ? 1 : 0;
        g.ks = w.gemm_ks;
        g.partial = reinterpret_cast<float*>(base + w.partial);
        g.tcount = reinterpret_cast<uint32_t*>(base + w.rtcount);
        g.y = y;
        g.y_dtype = partial ? SC_F32 : y_dtype;
        g.bias = partial ? nullptr : bias;
        g.partial_out = partial ? 1 : 0;
        g.skip_gather = reuse_route ? 1 : 0;
        e = launch_gemm(g, stream);
        if (e != cudaSuccess) return cuda_fail(e, "gemm launch");
        return SC_OK;
    }
    for (int64_t t0 = 0; t0 < m; t0 += w.chunk_tokens) {
        d.tok0 = t0;
        d.ntok = std::min<int64_t>(w.chunk_tokens, m - t0);
        d.ksplit = w.ksplit;
        e = launch_decode_tc(d, stream);
        if (e != cudaSuccess) return cuda_fail(e, "decode kernel launch");
    }
    return SC_OK;
}

// ------------------------------------------------------------------ static scratch

// Scratch of sc_forward_static.  The module loader places one copy on every device that
// loads this library's device code, so the call itself allocates nothing.
static __device__ __align__(256) unsigned char g_static_scratch[SC_STATIC_SCRATCH_BYTES];

constexpr int kStaticMaxDevices = 64;
static std::mutex g_static_mu;
static void* g_static_ptr[kStaticMaxDevices] = {};

// Address of the current device's copy of g_static_scratch, looked up on the first call for
// that device (the caller has made it current) and kept for the life of the process.
static sc_status static_scratch(int dev, void** out) {
    if (dev < 0 || dev >= kStaticMaxDevices) {
        set_error("sc_forward_static: device ordinal " + std::to_string(dev) + " out of range");
        return SC_EINVAL;
    }
    std::lock_guard<std::mutex> lk(g_static_mu);
    if (!g_static_ptr[dev]) {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_static_scratch);
        if (e != cudaSuccess) return cuda_fail(e, "sc_forward_static: cudaGetSymbolAddress");
        if (!p || (reinterpret_cast<uintptr_t>(p) & 255u) != 0) {
            set_error("sc_forward_static: static scratch is not 256-byte aligned");
            return SC_EDEVICE;
        }
        g_static_ptr[dev] = p;
    }
    *out = g_static_ptr[dev];
    return SC_OK;
}

}  // namespace sc

using namespace sc;

struct sc_layer {
    Layer L;
};

struct sc_group {
    std::vector<const sc_layer*> layers;
    int ksplit = 0;                 // column splits of the group's one-launch decode
    std::vector<DwBlocks> own;      // dW blocks built for `ksplit` (empty: the layer's own serve)
    ~sc_group() {
        for (DwBlocks& b : own) {
            cudaFree(b.blk);
            cudaFree(b.off);
        }
    }
};

extern "C" {

int sc_abi_version(void) { return SC_ABI_VERSION; }

const char* sc_op_name(void) { return "fused_c_tarq_saccade_linear"; }

size_t sc_last_error(char* buf, size_t len) {
    const std::string& s = g_last_error;
    if (buf && len > 0) {
        size_t n = std::min(len - 1, s.size());
        std::memcpy(buf, s.data(), n);
        buf[n] = '\0';
    }
    return s.size();
}

void sc_set_bypass_c_tarq(int on) { g_bypass.store(on ? 1 : 0); }
uint64_t sc_launch_count(void) { return g_launches.load(); }

void sc_test_drop_weight_copy(int on) { set_drop_weight_copy(on); }
int sc_is_c_tarq_bypassed(void) { return g_bypass.load(); }

static void free_layer(Layer& L) {
    cudaFree(L.wq);
    cudaFree(L.scale);
    cudaFree(L.rowptr);
    cudaFree(L.col);
    cudaFree(L.val);
    cudaFree(L.status);
    cudaFree(L.dwblk);
    cudaFree(L.dwoff);
    cudaFree(L.fold);
    cudaFree(L.foldoff);
    cudaFree(L.dseg);
    cudaFree(L.dsegoff);
    L.dseg = nullptr;
    L.dsegoff = nullptr;
    L.dwblk = nullptr;
    L.dwoff = nullptr;
    L.fold = nullptr;
    L.foldoff = nullptr;
    L.wq = nullptr;
    L.scale = nullptr;
    L.rowptr = nullptr;
    L.col = nullptr;
    L.val = nullptr;
    L.status = nullptr;
}

sc_status sc_layer_create(const sc_layer_desc* desc, sc_layer** out) {
    if (!desc || !out) {
        set_error("sc_layer_create: null argument");
        return SC_EINVAL;
    }
    *out = nullptr;
    const int64_t N = desc->out_features, K = desc->in_features;
    if (N <= 0 || K <= 0 || K % 8 != 0) {
        set_error("sc_layer_create: need out_features > 0 and in_features a positive multiple of 8");
        return SC_EINVAL;
    }
    if (!desc->packed_base || !desc->scale_base) {
        set_error("sc_layer_create: packed_base and scale_base are required");
        return SC_EINVAL;
    }
    const int64_t nnz_in = desc->delta_nnz;
    if (nnz_in < 0 || (nnz_in > 0 && (!desc->delta_row_ptrs || !desc->delta_col_indices || !desc->delta_values))) {
        set_error("sc_layer_create: delta_nnz > 0 needs row_ptrs, col_indices and values");
        return SC_EINVAL;
    }
    if (desc->mode < SC_MODE_FAST || desc->mode > SC_MODE_FAST_TC8) {
        set_error("sc_layer_create: unknown mode");
        return SC_EINVAL;
    }
    Layer L;
    L.device = desc->device;
    L.mode = desc->mode;
    L.fullN = N;
    L.fullK = K;
    L.t4 = desc->t4;
    L.t8 = desc->t8;
    L.shard_kind = desc->shard_kind;
    int64_t r0 = 0, r1 = N, c0 = 0, c1 = K;
    if (desc->shard_kind != SC_SHARD_NONE && desc->shard_end > desc->shard_begin) {
        // an explicit range: whole heads, or the intermediate slice shared with the next layer
        const int64_t b = desc->shard_begin, en = desc->shard_end;
        if (desc->shard_kind == SC_SHARD_COLUMNS) {
            if (b < 0 || en > N || b % 16 != 0 || (en % 16 != 0 && en != N)) {
                set_error("sc_layer_create: COLUMNS range must lie in [0, N) on multiples of 16");
                return SC_EINVAL;
            }
            r0 = b;
            r1 = en;
        } else if (desc->shard_kind == SC_SHARD_ROWS) {
            if (b < 0 || en > K || b % 64 != 0 || (en % 64 != 0 && en != K)) {
                set_error("sc_layer_create: ROWS range must lie in [0, K) on multiples of 64");
                return SC_EINVAL;
            }
            c0 = b;
            c1 = en;
        } else {
            set_error("sc_layer_create: unknown shard kind");
            return SC_EINVAL;
        }
    } else if (desc->shard_kind != SC_SHARD_NONE) {
        const int n = desc->shard_count, i = desc->shard_index;
        if (n <= 0 || i < 0 || i >= n) {
            set_error("sc_layer_create: bad shard index/count");
            return SC_EINVAL;
        }
        if (desc->shard_kind == SC_SHARD_COLUMNS) {
            r0 = std::min<int64_t>(N, ceil_to(N * i / n, 16));
            r1 = std::min<int64_t>(N, ceil_to(N * (i + 1) / n, 16));
            if (i == n - 1) r1 = N;
        } else if (desc->shard_kind == SC_SHARD_ROWS) {
            c0 = std::min<int64_t>(K, ceil_to(K * i / n, 64));
            c1 = std::min<int64_t>(K, ceil_to(K * (i + 1) / n, 64));
            if (i == n - 1) c1 = K;
        } else {
            set_error("sc_layer_create: unknown shard kind");
            return SC_EINVAL;
        }
        if (r1 <= r0 || c1 <= c0) {
            set_error("sc_layer_create: shard is empty");
            return SC_EINVAL;
        }
    }
    L.row_begin = r0;
    L.col_begin = c0;
    L.N = r1 - r0;
    L.K = c1 - c0;
    if (ceil_to(L.N, 128) / 128 > kMaxRowTiles) {
        set_error("sc_layer_create: out_features per shard above " + std::to_string(kMaxRowTiles * 128));
        return SC_EUNSUPPORTED;
    }
    if (L.K > 65536) {
        set_error("sc_layer_create: in_features per shard above 65536 (u16 dW columns)");
        return SC_EUNSUPPORTED;
    }
    L.Np = ceil_to(L.N, 128);
    L.Kp = ceil_to(L.K, 64);
    L.KB = L.Kp / 64;

    DeviceGuard guard(L.device);
    if (!guard.ok) {
        set_error("sc_layer_create: cannot select device " + std::to_string(L.device));
        return SC_ECUDA;
    }
    L.sms = sm_count(L.device);
    cudaError_t e;
    const bool on_dev = desc->buffers_on_device != 0;
    const int64_t kw_full = K / 8;

    // ---- dW CSR: validate and slice on the host (load time only)
    std::vector<uint32_t> rp(N + 1, 0);
    std::vector<uint32_t> ci(static_cast<size_t>(nnz_in));
    std::vector<uint8_t> cv(static_cast<size_t>(nnz_in));
    if (nnz_in > 0) {
        const cudaMemcpyKind kind = on_dev ? cudaMemcpyDeviceToHost : cudaMemcpyHostToHost;
        if ((e = cudaMemcpy(rp.data(), desc->delta_row_ptrs, (N + 1) * 4, kind)) != cudaSuccess ||
            (e = cudaMemcpy(ci.data(), desc->delta_col_indices, nnz_in * 4, kind)) != cudaSuccess ||
            (e = cudaMemcpy(cv.data(), desc->delta_values, nnz_in, kind)) != cudaSuccess)
            return cuda_fail(e, "sc_layer_create: reading dW");
        if (rp[0] != 0 || static_cast<int64_t>(rp[N]) != nnz_in) {
            set_error("sc_layer_create: delta_row_ptrs must start at 0 and end at delta_nnz");
            return SC_EINVAL;
        }
        for (int64_t r = 0; r < N; ++r) {
            if (rp[r + 1] < rp[r]) {
                set_error("sc_layer_create: delta_row_ptrs not monotone");
                return SC_EINVAL;
            }
            for (uint32_t q = rp[r]; q < rp[r + 1]; ++q) {
                if (static_cast<int64_t>(ci[q]) >= K) {
                    set_error("sc_layer_create: delta column index >= in_features");
                    return SC_EINVAL;
                }
            }
        }
        // The reference adds a row's corrections in CSC order: ascending column, and for a
        // repeated (row, column) in CSR order (config.rs:177-193, op.rs:156-167).  A stable
        // per-row sort by column reproduces that order for any CSR the caller passes.
        std::vector<uint32_t> perm;
        for (int64_t r = 0; r < N; ++r) {
            const uint32_t lo = rp[r], hi = rp[r + 1];
            bool sorted = true;
            for (uint32_t q = lo + 1; q < hi; ++q) sorted = sorted && ci[q - 1] <= ci[q];
            if (sorted) continue;
            perm.resize(hi - lo);
            for (uint32_t q = lo; q < hi; ++q) perm[q - lo] = q;
            std::stable_sort(perm.begin(), perm.end(), [&](uint32_t a, uint32_t b) { return ci[a] < ci[b]; });
            std::vector<uint32_t> c2(hi - lo);
            std::vector<uint8_t> v2(hi - lo);
            for (uint32_t q = 0; q < hi - lo; ++q) {
                c2[q] = ci[perm[q]];
                v2[q] = cv[perm[q]];
            }
            std::copy(c2.begin(), c2.end(), ci.begin() + lo);
            std::copy(v2.begin(), v2.end(), cv.begin() + lo);
        }
    }
    std::vector<uint32_t> srp(L.N + 1, 0);
    std::vector<uint16_t> scol;
    std::vector<int8_t> sval;
    for (int64_t r = 0; r < L.N; ++r) {
        srp[r] = static_cast<uint32_t>(scol.size());
        if (nnz_in > 0) {
            for (uint32_t q = rp[r0 + r]; q < rp[r0 + r + 1]; ++q) {
                const int64_t c = ci[q];
                if (c >= c0 && c < c1) {
                    scol.push_back(static_cast<uint16_t>(c - c0));
                    sval.push_back(static_cast<int8_t>(cv[q]));
                }
            }
        }
    }
    srp[L.N] = static_cast<uint32_t>(scol.size());
    L.nnz = static_cast<int64_t>(scol.size());
    {
        const uint16_t dsb = desc->delta_scale;
        // f16 -> f32 on the host (exact), matching config.rs:197 `s_cpu...[0].to_f32()`
        const uint32_t sign = (dsb & 0x8000u) << 16, ex = (dsb >> 10) & 0x1Fu, man = dsb & 0x3FFu;
        float f;
        if (ex == 0) {
            f = static_cast<float>(man) * 5.9604644775390625e-08f;
            if (sign) f = -f;
        } else {
            uint32_t bits = (ex == 0x1F) ? (sign | 0x7F800000u | (man << 13)) : (sign | ((ex - 15u + 127u) << 23) | (man << 13));
            std::memcpy(&f, &bits, 4);
        }
        L.ds = f;
    }

    // ---- allocations
    const int64_t wq_words = L.Np * L.KB * 8;
    auto alloc = [&](void** p, size_t bytes) { return cudaMalloc(p, bytes > 0 ? bytes : 16); };
    if ((e = alloc(reinterpret_cast<void**>(&L.wq), wq_words * 4)) != cudaSuccess ||
        (e = alloc(reinterpret_cast<void**>(&L.scale), L.Np * 4)) != cudaSuccess ||
        (e = alloc(reinterpret_cast<void**>(&L.rowptr), (L.N + 1) * 4)) != cudaSuccess ||
        (e = alloc(reinterpret_cast<void**>(&L.col), (L.nnz + 8) * 2)) != cudaSuccess ||
        (e = alloc(reinterpret_cast<void**>(&L.val), L.nnz + 16)) != cudaSuccess ||
        (e = alloc(reinterpret_cast<void**>(&L.status), 16)) != cudaSuccess) {
        free_layer(L);
        return cuda_fail(e, "sc_layer_create: cudaMalloc");
    }
    L.device_bytes = wq_words * 4 + L.Np * 4 + (L.N + 1) * 4 + (L.nnz + 8) * 2 + (L.nnz + 16);

    // ---- base weights and scales: stage this shard's rows on the device, then repack
    uint32_t* tmp_packed = nullptr;
    uint16_t* tmp_scale = nullptr;
    const uint32_t* src_packed = desc->packed_base + r0 * kw_full;
    const uint16_t* src_scale = desc->scale_base + r0;
    if (!on_dev) {
        if ((e = cudaMalloc(&tmp_packed, L.N * kw_full * 4)) != cudaSuccess ||
            (e = cudaMalloc(&tmp_scale, L.N * 2)) != cudaSuccess ||
            (e = cudaMemcpy(tmp_packed, src_packed, L.N * kw_full * 4, cudaMemcpyHostToDevice)) != cudaSuccess ||
            (e = cudaMemcpy(tmp_scale, src_scale, L.N * 2, cudaMemcpyHostToDevice)) != cudaSuccess) {
            cudaFree(tmp_packed);
            cudaFree(tmp_scale);
            free_layer(L);
            return cuda_fail(e, "sc_layer_create: staging weights");
        }
        src_packed = tmp_packed;
        src_scale = tmp_scale;
    }
    e = launch_repack(src_packed, kw_full, 0, c0 / 8, L, 0);
    if (e == cudaSuccess) e = launch_scales(src_scale, 0, L, 0);
    if (e == cudaSuccess)
        e = cudaMemcpy(L.rowptr, srp.data(), (L.N + 1) * 4, cudaMemcpyHostToDevice);
    if (e == cudaSuccess && L.nnz > 0) e = cudaMemcpy(L.col, scol.data(), L.nnz * 2, cudaMemcpyHostToDevice);
    if (e == cudaSuccess && L.nnz > 0) e = cudaMemcpy(L.val, sval.data(), L.nnz, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMemset(L.status, 0, 16);
    if (e == cudaSuccess) {
        // dW blocks of the router-fused decode kernel
        L.ks_fused = fused_ksplit(L);
        DwBlocks b;
        e = build_dw_blocks(L, L.ks_fused, srp.data(), scol.data(), sval.data(), &b);
        L.dwblk = b.blk;
        L.dwoff = b.off;
        L.dw_global = b.global;
        L.device_bytes += b.bytes;
    }
    if (e == cudaSuccess && L.nnz > 0) {
        // dW/s lists of the prefill GEMM, from the widened row scales
        std::vector<float> hs(static_cast<size_t>(L.Np));
        e = cudaMemcpy(hs.data(), L.scale, L.Np * 4, cudaMemcpyDeviceToHost);
        if (e == cudaSuccess) e = build_fold_lists(L, srp.data(), scol.data(), sval.data(), hs.data());
        if (e == cudaSuccess) e = build_dw_segments(L, srp.data(), scol.data(), sval.data());
    }
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    cudaFree(tmp_packed);
    cudaFree(tmp_scale);
    if (e != cudaSuccess) {
        free_layer(L);
        return cuda_fail(e, "sc_layer_create: device layout");
    }
    {
        // look up sc_forward_static's scratch array now, so that its first call on this device
        // neither loads the module (which places the array) nor takes the lookup's lock
        void* scratch = nullptr;
        const sc_status st = static_scratch(L.device, &scratch);
        if (st != SC_OK) {
            free_layer(L);
            return st;
        }
    }
    sc_layer* layer = new sc_layer;
    layer->L = L;
    *out = layer;
    return SC_OK;
}

void sc_layer_destroy(sc_layer* layer) {
    if (!layer) return;
    DeviceGuard guard(layer->L.device);
    free_layer(layer->L);
    delete layer;
}

sc_status sc_layer_get_info(const sc_layer* layer, sc_layer_info* info) {
    if (!layer || !info) {
        set_error("sc_layer_get_info: null argument");
        return SC_EINVAL;
    }
    const Layer& L = layer->L;
    info->out_features = L.N;
    info->in_features = L.K;
    info->row_begin = L.row_begin;
    info->col_begin = L.col_begin;
    info->full_out_features = L.fullN;
    info->full_in_features = L.fullK;
    info->delta_nnz = L.nnz;
    info->device_bytes = L.device_bytes;
    info->t4 = L.t4;
    info->t8 = L.t8;
    info->mode = L.mode;
    info->device = L.device;
    return SC_OK;
}

sc_status sc_layer_set_thresholds(sc_layer* layer, float t4, float t8) {
    if (!layer) {
        set_error("sc_layer_set_thresholds: null layer");
        return SC_EINVAL;
    }
    layer->L.t4 = t4;
    layer->L.t8 = t8;
    return SC_OK;
}

sc_status sc_layer_set_mode(sc_layer* layer, int mode) {
    if (!layer || mode < SC_MODE_FAST || mode > SC_MODE_FAST_TC8) {
        set_error("sc_layer_set_mode: bad argument");
        return SC_EINVAL;
    }
    layer->L.mode = mode;
    return SC_OK;
}

sc_status sc_layer_check(sc_layer* layer, void* stream) {
    if (!layer) {
        set_error("sc_layer_check: null layer");
        return SC_EINVAL;
    }
    DeviceGuard guard(layer->L.device);
    uint32_t st = 0;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    cudaError_t e = cudaMemcpyAsync(&st, layer->L.status, 4, cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return cuda_fail(e, "sc_layer_check");
    if (st == DEV_OK) return SC_OK;
    cudaMemsetAsync(layer->L.status, 0, 4, s);
    cudaStreamSynchronize(s);
    if (st == DEV_TIMEOUT) {
        set_error("device wait timed out inside a C-TARQ kernel");
        return SC_ETIMEOUT;
    }
    set_error("device recorded a bad index");
    return SC_EDEVICE;
}

size_t sc_workspace_size(const sc_layer* layer, int64_t m) {
    if (!layer || m < 0) return 0;
    return plan_workspace(layer->L, m).total;
}

sc_status sc_forward_ws(const sc_layer* layer, const void* x, int x_dtype, int64_t m, void* y, int y_dtype,
                        const float* bias, uint8_t* mask_out, int32_t* routed_idx_out, int32_t* n_routed_out,
                        void* workspace, size_t workspace_bytes, void* stream) {
    if (!layer) {
        set_error("sc_forward: null layer");
        return SC_EINVAL;
    }
    if (layer->L.shard_kind == SC_SHARD_ROWS) {
        set_error("sc_forward: a ROWS shard produces partial sums; use sc_forward_partial");
        return SC_EINVAL;
    }
    DeviceGuard guard(layer->L.device);
    if (!guard.ok) return cuda_fail(cudaErrorInvalidDevice, "sc_forward: set device");
    return forward_impl(layer->L, x, x_dtype, m, y, y_dtype, bias, mask_out, routed_idx_out, n_routed_out,
                        workspace, workspace_bytes, static_cast<cudaStream_t>(stream), false);
}

sc_status sc_forward(const sc_layer* layer, const void* x, int x_dtype, int64_t m, void* y, int y_dtype,
                     const float* bias, uint8_t* mask_out, int32_t* routed_idx_out, int32_t* n_routed_out,
                     void* stream) {
    if (!layer) {
        set_error("sc_forward: null layer");
        return SC_EINVAL;
    }
    if (m <= 0) return m == 0 ? SC_OK : (set_error("sc_forward: negative token count"), SC_EINVAL);
    DeviceGuard guard(layer->L.device);
    void* ws = nullptr;
    const size_t need = plan_workspace(layer->L, m).total;
    sc_status st = default_workspace(layer->L.device, need, &ws);
    if (st != SC_OK) return st;
    return sc_forward_ws(layer, x, x_dtype, m, y, y_dtype, bias, mask_out, routed_idx_out, n_routed_out, ws,
                         need, stream);
}

sc_status sc_forward_partial(const sc_layer* layer, const void* x, int x_dtype, int64_t m, float* y_partial,
                             uint8_t* mask_out, int32_t* routed_idx_out, int32_t* n_routed_out, void* workspace,
                             size_t workspace_bytes, void* stream) {
    if (!layer) {
        set_error("sc_forward_partial: null layer");
        return SC_EINVAL;
    }
    DeviceGuard guard(layer->L.device);
    void* ws = workspace;
    size_t wsb = workspace_bytes;
    if (!ws) {
        wsb = plan_workspace(layer->L, m).total;
        sc_status st = default_workspace(layer->L.device, wsb, &ws);
        if (st != SC_OK) return st;
    }
    return forward_impl(layer->L, x, x_dtype, m, y_partial, SC_F32, nullptr, mask_out, routed_idx_out,
                        n_routed_out, ws, wsb, static_cast<cudaStream_t>(stream), true);
}

sc_status sc_finalize(const float* acc, int64_t m, int64_t n, void* y, int y_dtype, const float* bias,
                      void* stream) {
    if (!acc || !y || m < 0 || n <= 0 || (y_dtype != SC_F16 && y_dtype != SC_BF16 && y_dtype != SC_F32)) {
        set_error("sc_finalize: bad argument");
        return SC_EINVAL;
    }
    cudaError_t e = launch_finalize(acc, m, n, y, y_dtype, bias, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "sc_finalize launch");
    return SC_OK;
}

size_t sc_split_exchange_floats(const sc_layer* layer, int64_t m) {
    if (!layer || m < 0) return 0;
    return static_cast<size_t>(2 * m * layer->L.N + 3 * m);
}

sc_status sc_forward_split(const sc_layer* layer, const void* x, int x_dtype, int64_t m, float* exchange,
                           void* workspace, size_t workspace_bytes, void* stream) {
    if (!layer || !exchange || m < 0) {
        set_error("sc_forward_split: bad argument");
        return SC_EINVAL;
    }
    if (layer->L.shard_kind != SC_SHARD_ROWS) {
        set_error("sc_forward_split: the layer is not a ROWS shard");
        return SC_EINVAL;
    }
    if (m == 0) return SC_OK;
    if (x_dtype != SC_F16 && x_dtype != SC_BF16) {
        set_error("sc_forward_split: x dtype must be F16 or BF16");
        return SC_EINVAL;
    }
    DeviceGuard guard(layer->L.device);
    if (!guard.ok) return cuda_fail(cudaErrorInvalidDevice, "sc_forward_split: set device");
    // the base product of the slice alone: the layer as an unsharded [N, K_slice] matrix whose
    // thresholds (NaN) route no token
    Layer B = layer->L;
    B.shard_kind = SC_SHARD_NONE;
    B.t4 = B.t8 = std::numeric_limits<float>::quiet_NaN();
    void* ws = workspace;
    size_t wsb = workspace_bytes;
    const size_t need = plan_workspace(layer->L, m).total;
    if (!ws) {
        wsb = need;
        sc_status st = default_workspace(B.device, wsb, &ws);
        if (st != SC_OK) return st;
    } else if (wsb < need || (reinterpret_cast<uintptr_t>(ws) & 255u) != 0) {
        set_error("sc_forward_split: workspace of " + std::to_string(wsb) + " bytes (256-byte aligned), need " +
                  std::to_string(need));
        return SC_ENOMEM;
    }
    const cudaStream_t s = static_cast<cudaStream_t>(stream);
    sc_status st = forward_impl(B, x, x_dtype, m, exchange, SC_F32, nullptr, nullptr, nullptr, nullptr, ws, wsb, s,
                                true, true);
    if (st != SC_OK) return st;
    const int64_t mn = m * layer->L.N;
    uint16_t* xt = reinterpret_cast<uint16_t*>(static_cast<unsigned char*>(ws) + plan_workspace(layer->L, m).xt);
    cudaError_t e = launch_split_extras(layer->L, x, x_dtype, m, exchange + mn, exchange + 2 * mn, xt, s);
    if (e != cudaSuccess) return cuda_fail(e, "sc_forward_split launch");
    return SC_OK;
}

sc_status sc_finalize_split(const sc_layer* layer, const float* exchange, int64_t m, int ranks, void* y, int y_dtype,
                            const float* bias, uint8_t* mask_out, uint32_t* undecided_out, void* stream) {
    if (!layer || !exchange || !y || m < 0 || ranks < 1 ||
        (y_dtype != SC_F16 && y_dtype != SC_BF16 && y_dtype != SC_F32)) {
        set_error("sc_finalize_split: bad argument");
        return SC_EINVAL;
    }
    if (layer->L.shard_kind != SC_SHARD_ROWS) {
        set_error("sc_finalize_split: the layer is not a ROWS shard");
        return SC_EINVAL;
    }
    if (m == 0) return SC_OK;
    DeviceGuard guard(layer->L.device);
    if (!guard.ok) return cuda_fail(cudaErrorInvalidDevice, "sc_finalize_split: set device");
    cudaError_t e = launch_split_finalize(layer->L, exchange, m, ranks, g_bypass.load() != 0 ? 1 : 0, y, y_dtype,
                                          bias, mask_out, undecided_out, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "sc_finalize_split launch");
    return SC_OK;
}

sc_status sc_group_create(sc_layer* const* layers, int count, sc_group** out) {
    if (!out || !layers || count < 1 || count > SC_GROUP_MAX) {
        set_error("sc_group_create: need 1.." + std::to_string(SC_GROUP_MAX) + " layers");
        return SC_EINVAL;
    }
    *out = nullptr;
    for (int i = 0; i < count; ++i) {
        if (!layers[i]) {
            set_error("sc_group_create: null layer");
            return SC_EINVAL;
        }
        const Layer& L = layers[i]->L;
        const Layer& L0 = layers[0]->L;
        if (L.device != L0.device || L.K != L0.K || L.fullK != L0.fullK || L.col_begin != L0.col_begin) {
            set_error("sc_group_create: layers of a group share the device and the input columns");
            return SC_EINVAL;
        }
        if (L.shard_kind == SC_SHARD_ROWS) {
            set_error("sc_group_create: ROWS shards produce partial sums; group them through sc_forward_partial");
            return SC_EINVAL;
        }
    }
    sc_group* g = new sc_group;
    g->layers.assign(layers, layers + count);
    g->own.resize(count);
    const Layer& L0 = layers[0]->L;
    DeviceGuard guard(L0.device);
    if (!guard.ok) {
        delete g;
        return cuda_fail(cudaErrorInvalidDevice, "sc_group_create: set device");
    }
    int64_t rt = 0;
    for (int i = 0; i < count; ++i) rt += layers[i]->L.Np / 128;
    g->ksplit = choose_ksplit(rt, L0.KB);
    for (int i = 0; i < count; ++i) {
        const Layer& L = layers[i]->L;
        if (L.nnz == 0 || g->ksplit == L.ks_fused || g->ksplit <= 0) continue;
        std::vector<uint32_t> srp(L.N + 1);
        std::vector<uint16_t> scol(L.nnz);
        std::vector<int8_t> sval(L.nnz);
        cudaError_t e = cudaMemcpy(srp.data(), L.rowptr, (L.N + 1) * 4, cudaMemcpyDeviceToHost);
        if (e == cudaSuccess) e = cudaMemcpy(scol.data(), L.col, L.nnz * 2, cudaMemcpyDeviceToHost);
        if (e == cudaSuccess) e = cudaMemcpy(sval.data(), L.val, L.nnz, cudaMemcpyDeviceToHost);
        if (e == cudaSuccess) e = build_dw_blocks(L, g->ksplit, srp.data(), scol.data(), sval.data(), &g->own[i]);
        if (e != cudaSuccess) {
            delete g;
            return cuda_fail(e, "sc_group_create: dW blocks");
        }
    }
    *out = g;
    return SC_OK;
}

void sc_group_destroy(sc_group* group) { delete group; }

}  // extern "C"

// One launch pair of the integer GEMM for every layer of a group (2..64 tokens): the workspace
// carve-up (offsets from the base) and its total.
struct MidGroupPlan {
    bool use = false;
    int ks = 0;
    int64_t rt = 0;
    size_t xconv = 0, mask = 0, ridx = 0, nrouted = 0, partial = 0, total = 0;
};

// single: a group of one layer plans too (sc_forward_group runs a lone layer through sc_forward_ws)
static MidGroupPlan plan_mid_group(const sc_group* g, int64_t m, bool single = false) {
    MidGroupPlan p;
    const int n = static_cast<int>(g->layers.size());
    const Layer& L0 = g->layers[0]->L;
    bool ok = n > 1 || (single && n == 1);
    for (int i = 0; i < n && ok; ++i) ok = use_mid(g->layers[i]->L, m);
    if (!ok) return p;
    for (int i = 0; i < n; ++i) p.rt += g->layers[i]->L.Np / 128;
    if (p.rt > kMaxRowTiles) return p;
    p.ks = mid_ksplit(p.rt, L0.KB, L0.sms, m);
    size_t off = kCounterBytes;
    auto take = [&](size_t bytes) {
        size_t o = off;
        off = static_cast<size_t>(ceil_to(static_cast<int64_t>(off + bytes), 256));
        return o;
    };
    p.xconv = take(static_cast<size_t>(m * L0.K * 2));
    p.mask = take(static_cast<size_t>(SC_GROUP_MAX * ceil_to(m, 16)));
    p.ridx = take(static_cast<size_t>(SC_GROUP_MAX * 4 * m));
    p.nrouted = take(static_cast<size_t>(SC_GROUP_MAX * 16));
    p.partial = take(static_cast<size_t>(p.ks > 1 ? p.rt * p.ks * m * 128 * 4 : 16));
    p.total = off;
    p.use = true;
    return p;
}

// The 9..64-token launch of a group (plan mp): the routing into the caller's arrays where given,
// else into the workspace; routed_in: the caller's arrays hold the routing already.
static sc_status forward_group_mid(const sc_group* group, const MidGroupPlan& mp, const void* x, int x_dtype,
                                   int64_t m, void* const* y, int y_dtype, const float* const* bias,
                                   uint8_t* const* mask, int32_t* const* ridx, int32_t* const* nrouted, bool routed_in,
                                   void* workspace, cudaStream_t s, const char* who) {
    const int n = static_cast<int>(group->layers.size());
    unsigned char* base = static_cast<unsigned char*>(workspace);
    MidArgs a = {};
    a.n = n;
    for (int i = 0; i < n; ++i) {
        if (!y[i]) {
            set_error(std::string(who) + ": null output " + std::to_string(i));
            return SC_EINVAL;
        }
        a.layer[i] = &group->layers[i]->L;
        a.mask[i] = (mask && mask[i]) ? mask[i] : base + mp.mask + i * ceil_to(m, 16);
        a.ridx[i] = (ridx && ridx[i]) ? ridx[i] : reinterpret_cast<int32_t*>(base + mp.ridx) + i * m;
        a.nrouted[i] = (nrouted && nrouted[i]) ? nrouted[i] : reinterpret_cast<int32_t*>(base + mp.nrouted) + i * 4;
        a.y[i] = y[i];
        a.bias[i] = bias ? bias[i] : nullptr;
    }
    a.x = x;
    a.x_dtype = x_dtype;
    a.x_stride = group->layers[0]->L.K;
    a.x_col0 = 0;
    a.m = m;
    a.route_all = g_bypass.load() != 0 ? 1 : 0;
    a.routed_in = routed_in ? 1 : 0;
    a.ks = mp.ks;
    a.xconv = reinterpret_cast<uint16_t*>(base + mp.xconv);
    a.y_dtype = y_dtype;
    a.partial_out = 0;
    a.partial = reinterpret_cast<float*>(base + mp.partial);
    a.counter = reinterpret_cast<uint32_t*>(base);
    a.rtcount = reinterpret_cast<uint32_t*>(base + 256);
    const cudaError_t e = launch_mid(a, s);
    if (e != cudaSuccess) return cuda_fail(e, (std::string(who) + ": 9..64-token GEMM launch").c_str());
    return SC_OK;
}

namespace sc {
int group_layers(const sc_group* g, const Layer** out) {
    const int n = std::min(static_cast<int>(g->layers.size()), SC_GROUP_MAX);
    for (int i = 0; i < n; ++i) out[i] = &g->layers[i]->L;
    return n;
}

int bypass_on() { return g_bypass.load() != 0 ? 1 : 0; }
}  // namespace sc

extern "C" {

int sc_group_takes_routing(const sc_group* group, int64_t m, size_t workspace_bytes) {
    if (!group || m <= 0) return 0;
    const MidGroupPlan mp = plan_mid_group(group, m, true);
    return (mp.use && workspace_bytes >= mp.total) ? 1 : 0;
}

sc_status sc_forward_group_routed(const sc_group* group, const uint16_t* x, int64_t m, void* const* y, int y_dtype,
                                  const float* const* bias, const uint8_t* const* mask,
                                  const int32_t* const* routed_idx, const int32_t* const* n_routed, void* workspace,
                                  size_t workspace_bytes, void* stream) {
    if (!group || !y || !x || !mask || !routed_idx || !n_routed) {
        set_error("sc_forward_group_routed: null group, x, output or routing array");
        return SC_EINVAL;
    }
    const int n = static_cast<int>(group->layers.size());
    for (int i = 0; i < n; ++i) {
        if (!mask[i] || !routed_idx[i] || !n_routed[i]) {
            set_error("sc_forward_group_routed: null routing of layer " + std::to_string(i));
            return SC_EINVAL;
        }
    }
    if (y_dtype != SC_F16 && y_dtype != SC_BF16 && y_dtype != SC_F32) {
        set_error("sc_forward_group_routed: y dtype must be F16, BF16 or F32");
        return SC_EINVAL;
    }
    if ((reinterpret_cast<uintptr_t>(x) & 15u) != 0) {
        set_error("sc_forward_group_routed: x must be 16-byte aligned");
        return SC_EINVAL;
    }
    const MidGroupPlan mp = plan_mid_group(group, m, true);
    if (!mp.use || !workspace || workspace_bytes < mp.total || (reinterpret_cast<uintptr_t>(workspace) & 255u) != 0) {
        set_error("sc_forward_group_routed: the group does not run the 9..64-token launch for this call "
                  "(sc_group_takes_routing), or the workspace is too small or not 256-byte aligned");
        return SC_EINVAL;
    }
    DeviceGuard guard(group->layers[0]->L.device);
    if (!guard.ok) return cuda_fail(cudaErrorInvalidDevice, "sc_forward_group_routed: set device");
    return forward_group_mid(group, mp, x, SC_F16, m, y, y_dtype, bias, const_cast<uint8_t* const*>(mask),
                             const_cast<int32_t* const*>(routed_idx), const_cast<int32_t* const*>(n_routed), true,
                             workspace, static_cast<cudaStream_t>(stream), "sc_forward_group_routed");
}

size_t sc_group_workspace_size(const sc_group* group, int64_t m) {
    if (!group || m < 0) return 0;
    size_t need = 0;
    for (const sc_layer* l : group->layers) need = std::max(need, plan_workspace(l->L, m).total);
    const MidGroupPlan p = plan_mid_group(group, m, true);
    if (p.use) need = std::max(need, p.total);
    return need;
}

sc_status sc_forward_group(const sc_group* group, const void* x, int x_dtype, int64_t m, void* const* y, int y_dtype,
                           const float* const* bias, uint8_t* const* mask_out, int32_t* const* routed_idx_out,
                           int32_t* const* n_routed_out, void* workspace, size_t workspace_bytes, void* stream) {
    if (!group || !y) {
        set_error("sc_forward_group: null group or output array");
        return SC_EINVAL;
    }
    if (m <= 0) return m == 0 ? SC_OK : (set_error("sc_forward_group: negative token count"), SC_EINVAL);
    const int n = static_cast<int>(group->layers.size());
    const Layer& L0 = group->layers[0]->L;
    DeviceGuard guard(L0.device);
    if (!guard.ok) return cuda_fail(cudaErrorInvalidDevice, "sc_forward_group: set device");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    // one launch when every layer takes the router-fused decode with the same split
    bool one = group->ksplit > 0;
    for (int i = 0; i < n; ++i) {
        const Layer& L = group->layers[i]->L;
        one = one && use_fused_ks(L, m, group->ksplit) && L.mode == L0.mode;
    }
    if (one) {
        if (x_dtype != SC_F16 && x_dtype != SC_BF16) {
            set_error("sc_forward_group: x dtype must be F16 or BF16");
            return SC_EINVAL;
        }
        if (y_dtype != SC_F16 && y_dtype != SC_BF16 && y_dtype != SC_F32) {
            set_error("sc_forward_group: y dtype must be F16, BF16 or F32");
            return SC_EINVAL;
        }
        if (!x) {
            set_error("sc_forward_group: null x");
            return SC_EINVAL;
        }
        const bool bypass_now = g_bypass.load() != 0;
        FusedArgs f[SC_GROUP_MAX];
        for (int i = 0; i < n; ++i) {
            const Layer& L = group->layers[i]->L;
            if (!y[i]) {
                set_error("sc_forward_group: null output " + std::to_string(i));
                return SC_EINVAL;
            }
            FusedArgs& a = f[i];
            a.L = &L;
            a.x = x;
            a.x_dtype = x_dtype;
            a.x_stride = L.K;
            a.x_col0 = 0;
            a.m = m;
            a.route_all = bypass_now ? 1 : 0;
            a.y = y[i];
            a.y_dtype = y_dtype;
            a.bias = bias ? bias[i] : nullptr;
            a.partial_out = 0;
            a.mask_out = mask_out ? mask_out[i] : nullptr;
            a.ridx_out = routed_idx_out ? routed_idx_out[i] : nullptr;
            a.nrouted_out = n_routed_out ? n_routed_out[i] : nullptr;
            a.ws_partial = nullptr;
            a.ws_rtcount = nullptr;
            a.ksplit = group->ksplit;
            const bool own = group->own[i].blk != nullptr;
            const bool layers_fit = group->ksplit == L.ks_fused;
            a.dwblk = own ? group->own[i].blk : layers_fit ? L.dwblk : nullptr;
            a.dwoff = own ? group->own[i].off : layers_fit ? L.dwoff : nullptr;
            a.dw_global = own ? group->own[i].global : layers_fit ? L.dw_global : 0;
        }
        const cudaError_t e = launch_decode_fused(f, n, s);
        if (e != cudaSuccess) return cuda_fail(e, "grouped decode launch");
        return SC_OK;
    }
    const MidGroupPlan mp = plan_mid_group(group, m);
    if (mp.use && workspace && workspace_bytes >= mp.total && (reinterpret_cast<uintptr_t>(workspace) & 255u) == 0) {
        if ((x_dtype != SC_F16 && x_dtype != SC_BF16) || !x ||
            (y_dtype != SC_F16 && y_dtype != SC_BF16 && y_dtype != SC_F32)) {
            set_error("sc_forward_group: bad x / y dtype or null x");
            return SC_EINVAL;
        }
        return forward_group_mid(group, mp, x, x_dtype, m, y, y_dtype, bias, mask_out, routed_idx_out, n_routed_out,
                                 false, workspace, s, "sc_forward_group");
    }
    // prefill GEMM regime: layers reading the same x with the same thresholds share one router and
    // one token gather (their masks are the same); the others reuse what the first left in the workspace
    bool share = n > 1 && workspace && L0.mode != SC_MODE_EXACT && L0.shard_kind != SC_SHARD_ROWS &&
                 g_bypass.load() == 0;
    for (int i = 0; i < n && share; ++i) {
        const Layer& L = group->layers[i]->L;
        share = L.K == L0.K && L.fullK == L0.fullK && L.mode == L0.mode && L.shard_kind == L0.shard_kind &&
                L.t4 == L0.t4 && L.t8 == L0.t8 && !use_fused(L, m) && !use_mid(L, m) && m >= kGemmMinTokens &&
                workspace_bytes >= plan_workspace(L, m).total;
    }
    if (share) {
        for (int i = 0; i < n; ++i) {
            if (!y[i]) {
                set_error("sc_forward_group: null output " + std::to_string(i));
                return SC_EINVAL;
            }
            const sc_status st = forward_impl(group->layers[i]->L, x, x_dtype, m, y[i], y_dtype, bias ? bias[i] : nullptr,
                                              nullptr, nullptr, nullptr, workspace, workspace_bytes, s, false, false,
                                              i > 0);
            if (st != SC_OK) return st;
        }
        const WsLayout w = plan_workspace(L0, m);
        const unsigned char* base = static_cast<const unsigned char*>(workspace);
        for (int i = 0; i < n; ++i) {
            cudaError_t e = cudaSuccess;
            if (mask_out && mask_out[i]) e = cudaMemcpyAsync(mask_out[i], base + w.mask, m, cudaMemcpyDeviceToDevice, s);
            if (e == cudaSuccess && routed_idx_out && routed_idx_out[i])
                e = cudaMemcpyAsync(routed_idx_out[i], base + w.ridx, 4 * m, cudaMemcpyDeviceToDevice, s);
            if (e == cudaSuccess && n_routed_out && n_routed_out[i])
                e = cudaMemcpyAsync(n_routed_out[i], base + w.nrouted, 4, cudaMemcpyDeviceToDevice, s);
            if (e != cudaSuccess) return cuda_fail(e, "sc_forward_group: routing outputs");
        }
        return SC_OK;
    }
    for (int i = 0; i < n; ++i) {
        const sc_status st = sc_forward_ws(group->layers[i], x, x_dtype, m, y[i], y_dtype, bias ? bias[i] : nullptr,
                                           mask_out ? mask_out[i] : nullptr, routed_idx_out ? routed_idx_out[i] : nullptr,
                                           n_routed_out ? n_routed_out[i] : nullptr, workspace, workspace_bytes, stream);
        if (st != SC_OK) return st;
    }
    return SC_OK;
}

sc_status sc_forward_static(const sc_layer* layer, const void* x, int x_dtype, int64_t m, void* y, int y_dtype,
                            const float* bias, uint8_t* mask_out, int32_t* routed_idx_out, int32_t* n_routed_out,
                            void* stream) {
    if (!layer) {
        set_error("sc_forward_static: null layer");
        return SC_EINVAL;
    }
    if (m <= 0) return m == 0 ? SC_OK : (set_error("sc_forward_static: negative token count"), SC_EINVAL);
    if (layer->L.shard_kind == SC_SHARD_ROWS) {
        set_error("sc_forward_static: a ROWS shard produces partial sums; use sc_forward_partial");
        return SC_EINVAL;
    }
    const size_t need = plan_workspace(layer->L, m).total;
    if (need > static_cast<size_t>(SC_STATIC_SCRATCH_BYTES)) {
        set_error("sc_forward_static: " + std::to_string(m) + " tokens on this layer need " + std::to_string(need) +
                  " bytes of scratch, the static array holds " + std::to_string(SC_STATIC_SCRATCH_BYTES) +
                  "; use sc_forward_ws");
        return SC_EINVAL;
    }
    DeviceGuard guard(layer->L.device);
    if (!guard.ok) return cuda_fail(cudaErrorInvalidDevice, "sc_forward_static: set device");
    void* ws = nullptr;
    sc_status st = static_scratch(layer->L.device, &ws);
    if (st != SC_OK) return st;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    // the completion counters must start at zero
    const cudaError_t e = cudaMemsetAsync(ws, 0, kCounterBytes, s);
    if (e != cudaSuccess) return cuda_fail(e, "sc_forward_static: clear counters");
    return forward_impl(layer->L, x, x_dtype, m, y, y_dtype, bias, mask_out, routed_idx_out, n_routed_out, ws,
                        static_cast<size_t>(SC_STATIC_SCRATCH_BYTES), s, false);
}

}  // extern "C"
