// sc_prep.cu -- load-time conversion of reference-format buffers to the device layout.
//
// The reference keeps the 4-bit base as u32 [N, K/8] with element k at bits 4*(k%8) of
// word k/8 (compress.rs:54-83, read back the same way at op.rs:120-131).  The device
// layout regroups those nibbles so that one coalesced 16-byte load per lane yields four
// ready-made tensor-core A fragments (layout described in sc_internal.h).  The numeric
// content is unchanged: this is a permutation plus padding with q = 0.
#include "sc_device.cuh"
#include "sc_internal.h"

namespace sc {

__global__ void k_repack(const uint32_t* __restrict__ packed, int64_t ref_wpr, int64_t row0, int64_t word0,
                         int64_t N, int64_t K, int64_t KB, int64_t total_words, uint32_t* __restrict__ wq) {
    for (int64_t w = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; w < total_words;
         w += (int64_t)gridDim.x * blockDim.x) {
        const int64_t tile = w / (KB * 128);
        const int64_t rem = w - tile * KB * 128;
        const int64_t kb = rem >> 7;
        const int r2 = static_cast<int>(rem & 127);
        const int lane = r2 >> 2, s = r2 & 3;
        const int g = lane >> 2, c = lane & 3;
        uint32_t out = 0;
#pragma unroll
        for (int p = 0; p < 8; ++p) {
            const int64_t row = tile * 16 + g + ((p & 1) ? 8 : 0);
            const int64_t col = kb * 64 + 16 * s + 2 * c + (((p >> 1) & 1) ? 8 : 0) + (p >> 2);
            uint32_t nib = 8u;
            if (row < N && col < K) {
                const uint32_t word = packed[(row0 + row) * ref_wpr + word0 + (col >> 3)];
                nib = (word >> (4 * (col & 7))) & 0xFu;
            }
            out |= nib << (4 * p);
        }
        wq[w] = out;
    }
}

__global__ void k_scales(const uint16_t* __restrict__ scale_f16, int64_t row0, int64_t N, int64_t Np,
                         float* __restrict__ scale) {
    for (int64_t r = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; r < Np; r += (int64_t)gridDim.x * blockDim.x)
        scale[r] = r < N ? __half2float(__ushort_as_half(scale_f16[row0 + r])) : 0.0f;
}

cudaError_t launch_repack(const uint32_t* packed, int64_t ref_words_per_row, int64_t row0, int64_t word0,
                          const Layer& L, cudaStream_t s) {
    const int64_t total = (L.Np / 16) * L.KB * 128;
    const int threads = 256;
    const int64_t blocks = (total + threads - 1) / threads;
    k_repack<<<static_cast<unsigned>(blocks < 65535 * 16 ? blocks : 65535 * 16), threads, 0, s>>>(
        packed, ref_words_per_row, row0, word0, L.N, L.K, L.KB, total, L.wq);
    return cudaGetLastError();
}

cudaError_t launch_scales(const uint16_t* scale_f16, int64_t row0, const Layer& L, cudaStream_t s) {
    const int threads = 256;
    const int64_t blocks = (L.Np + threads - 1) / threads;
    k_scales<<<static_cast<unsigned>(blocks), threads, 0, s>>>(scale_f16, row0, L.N, L.Np, L.scale);
    return cudaGetLastError();
}

}  // namespace sc
