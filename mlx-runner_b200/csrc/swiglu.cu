// swiglu.cu - gate / up weight pairing and the unfused SwiGLU step.
//
// The reference's MLP (src/model.zig:905-915 mlpForwardQ) runs two
// quantized linears on the same x, g = x.Wg^T and u = x.Wu^T, then
// silu(g) * u, each step a bf16 array.  The fused form keeps one resident
// weight whose rows interleave the two tensors in 64-row blocks, so every
// 128-row tile of the decode and prefill kernels holds 64 gate rows and
// their 64 up rows and the epilogue writes silu(g) * u directly.  Moving
// whole packed rows (codes and scale bytes) keeps the quantisation bit for
// bit: groups run along K.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>

#include "formats.cuh"
#include "internal.h"

namespace qmm {
namespace {

// dst row r: block b = r / 128, j = r % 128; j < 64 -> gate row 64 b + j,
// else up row 64 b + j - 64 (rows >= n_half are skipped).  One thread per
// 16-byte word of a row (pitch is a multiple of 16) or per byte otherwise.
__global__ void interleave_rows_kernel(const uint8_t* __restrict__ gate, const uint8_t* __restrict__ up,
                                       int64_t pitch, int64_t n_half, int64_t rows, uint8_t* __restrict__ dst) {
    const bool vec = (pitch & 15) == 0;
    const int64_t per_row = vec ? pitch / 16 : pitch;
    const int64_t total = rows * per_row;
    for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = t / per_row, w = t % per_row;
        const int64_t b = r / 128, j = r % 128;
        const int64_t src_row = 64 * b + (j < 64 ? j : j - 64);
        if (src_row >= n_half) continue;
        const uint8_t* src = (j < 64 ? gate : up) + src_row * pitch;
        if (vec)
            reinterpret_cast<uint4*>(dst + r * pitch)[w] = reinterpret_cast<const uint4*>(src)[w];
        else
            dst[r * pitch + w] = src[w];
    }
}

__global__ void swiglu_apply_kernel(const uint16_t* __restrict__ y, int64_t ldy, int64_t m, int64_t n_half,
                                    uint16_t* __restrict__ h, int64_t ldh) {
    const int64_t total = m * n_half;
    for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
        const int64_t row = t / n_half, c = t % n_half;
        const int64_t yc = (c / 64) * 128 + (c % 64);
        const float g = bf16_to_f32(y[row * ldy + yc]), u = bf16_to_f32(y[row * ldy + yc + 64]);
        h[row * ldh + c] = swiglu_bf16(g, u);
    }
}

unsigned grid_for(int64_t work) {
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    return (unsigned)std::max<int64_t>(1, std::min<int64_t>((work + 255) / 256, (int64_t)sms * 8));
}

}  // namespace

int launch_interleave_rows(const uint8_t* gate, const uint8_t* up, int64_t pitch, int64_t n_half, int64_t npad,
                           uint8_t* dst, cudaStream_t stream) {
    if (n_half <= 0) return QMM_OK;
    const int64_t rows = 2 * npad;
    const int64_t work = rows * ((pitch & 15) == 0 ? pitch / 16 : pitch);
    interleave_rows_kernel<<<grid_for(work), 256, 0, stream>>>(gate, up, pitch, n_half, rows, dst);
    QMM_CUDA_TRY(cudaGetLastError());
    return QMM_OK;
}

int launch_swiglu_apply(const uint16_t* y, int64_t ldy, int64_t m, int64_t n_half, uint16_t* h, int64_t ldh,
                        cudaStream_t stream) {
    if (m <= 0 || n_half <= 0) return QMM_OK;
    swiglu_apply_kernel<<<grid_for(m * n_half), 256, 0, stream>>>(y, ldy, m, n_half, h, ldh);
    QMM_CUDA_TRY(cudaGetLastError());
    return QMM_OK;
}

}  // namespace qmm
