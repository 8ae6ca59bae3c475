// sc_prep.cu -- load-time conversion of reference-format buffers to the device layout.
//
// The reference keeps the 4-bit base as u32 [N, K/8] with element k at bits 4*(k%8) of
// word k/8 (compress.rs:54-83, read back the same way at op.rs:120-131).  The device
// layout regroups those nibbles into 128-row x 64-column blocks of 4 KB (eight 16-row
// tiles x 32 lanes x 4 words) so that one 16-byte load per lane yields, per 16-column
// step, a word holding rows g and g+8 of the lane's tile at columns 4c..4c+3 (g = lane/4,
// c = lane%4).  That word is an mma.sync A fragment (with the K order permuted inside the
// step, mirrored by the B fragment) and also a tcgen05.st.16x256b operand (natural K order
// in TMEM).  The numeric content is unchanged: a permutation plus padding with q = 0.
#include "sc_device.cuh"
#include "sc_internal.h"

namespace sc {

__global__ void k_repack(const uint32_t* __restrict__ packed, int64_t ref_wpr, int64_t row0, int64_t word0,
                         int64_t N, int64_t K, int64_t KB, int64_t total_words, uint32_t* __restrict__ wq) {
    for (int64_t w = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; w < total_words;
         w += (int64_t)gridDim.x * blockDim.x) {
        const int64_t rt = w / (KB * 1024);
        const int64_t rem = w - rt * KB * 1024;
        const int64_t kb = rem >> 10;
        const int r2 = static_cast<int>(rem & 1023);
        const int tile = r2 >> 7, lane = (r2 >> 2) & 31, s = r2 & 3;
        const int g = lane >> 2, c = lane & 3;
        const int64_t row_g = rt * 128 + tile * 16 + g;
        const int64_t k0 = kb * 64 + 16 * s + 4 * c;
        uint32_t out = 0;
#pragma unroll
        for (int p = 0; p < 8; ++p) {
            const int64_t row = row_g + (p & 1) * 8;
            const int64_t col = k0 + ((p >> 1) & 1) * 2 + (p >> 2);
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
    const int64_t total = L.Np * L.KB * 8;
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
