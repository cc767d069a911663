// dequant.cu - W = decode(code) * decode(scale), written as bf16 or fp32.
//
// Counterpart of mlx_dequantize (src/mlx.zig:274) as the reference's test
// calls it (src/model.zig:1593: no biases, no global scale).  Each thread
// expands one 16-byte code chunk of a row; the values are exact products
// (a 4-bit or 2-bit significand times a power of two or an E4M3 scale), so
// the fp32 output is bit-exact and the bf16 output is exact whenever the
// value is inside bf16's range.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>

#include "formats.cuh"
#include "internal.h"

namespace qmm {
namespace {

template <int FMT, bool BF16>
__global__ void __launch_bounds__(256) dequant_kernel(const uint8_t* __restrict__ codes, int64_t ldc,
                                                      const uint8_t* __restrict__ scales, int64_t lds,
                                                      int64_t n, int64_t k, void* __restrict__ out) {
    constexpr int kCodesPerChunk = FMT == kMXFP8 ? 16 : 32;
    const int64_t chunks = (k + kCodesPerChunk - 1) / kCodesPerChunk;
    const int64_t total = n * chunks;
    for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < total;
         t += (int64_t)gridDim.x * blockDim.x) {
        const int64_t row = t / chunks, c = t % chunks;
        const uint8_t* cp = codes + row * ldc + c * 16;
        const int64_t k0 = c * kCodesPerChunk;
        const int nvalid = (k - k0) < kCodesPerChunk ? (int)(k - k0) : kCodesPerChunk;
        float v[kCodesPerChunk];
        if constexpr (FMT == kMXFP8) {
            const float s = ue8m0_to_f32(scales[row * lds + k0 / 32]);
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const uint32_t w = *reinterpret_cast<const uint32_t*>(cp + 4 * q);
                uint32_t h[2];
                e4m3x4_to_f16x2(w, h);
                float2 a = f16x2_to_float2(h[0]), b = f16x2_to_float2(h[1]);
                v[4 * q + 0] = a.x * s; v[4 * q + 1] = a.y * s;
                v[4 * q + 2] = b.x * s; v[4 * q + 3] = b.y * s;
            }
        } else {
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                if (8 * q >= nvalid) break;
                const float s = ue4m3_to_f32(scales[row * lds + (k0 + 8 * q) / 16]);
                const uint32_t w = *reinterpret_cast<const uint32_t*>(cp + 4 * q);
                uint32_t h[4];
                e2m1x8_to_f16x2(w, h);
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    float2 a = f16x2_to_float2(h[i]);
                    v[8 * q + 2 * i] = a.x * s;
                    v[8 * q + 2 * i + 1] = a.y * s;
                }
            }
        }
        if constexpr (BF16) {
            uint16_t* o = static_cast<uint16_t*>(out) + row * k + k0;
            for (int i = 0; i < nvalid; i += 2)
                *reinterpret_cast<uint32_t*>(o + i) = f32x2_to_bf16x2(v[i], v[i + 1]);
        } else {
            float* o = static_cast<float*>(out) + row * k + k0;
            for (int i = 0; i < nvalid; ++i) o[i] = v[i];
        }
    }
}

__global__ void f32_to_bf16_kernel(const float* __restrict__ in, int64_t rows, int64_t cols, int64_t ld_in,
                                   uint16_t* __restrict__ out, int64_t ld_out) {
    const int64_t total = rows * cols;
    for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < total;
         t += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = t / cols, c = t % cols;
        out[r * ld_out + c] = f32_to_bf16(in[r * ld_in + c]);
    }
}

}  // namespace

int launch_f32_to_bf16(const float* in, int64_t rows, int64_t cols, int64_t ld_in, uint16_t* out, int64_t ld_out,
                       cudaStream_t stream) {
    const int64_t total = rows * cols;
    if (total == 0) return QMM_OK;
    const unsigned grid = (unsigned)std::min<int64_t>((total + 255) / 256, 1184);
    f32_to_bf16_kernel<<<grid, 256, 0, stream>>>(in, rows, cols, ld_in, out, ld_out);
    QMM_CUDA_TRY(cudaGetLastError());
    return QMM_OK;
}

int launch_dequant(int fmt, const uint8_t* codes, int64_t ldc, const uint8_t* scales, int64_t lds,
                   int64_t n, int64_t k, void* out, bool out_bf16, cudaStream_t stream) {
    if (n == 0 || k == 0) return QMM_OK;
    int dev = 0;
    QMM_CUDA_TRY(cudaGetDevice(&dev));
    DeviceInfo info;
    if (int rc = device_info(dev, &info)) return rc;
    const int64_t per = fmt == kMXFP8 ? 16 : 32;
    const int64_t total = n * ((k + per - 1) / per);
    const int64_t want = (total + 255) / 256;
    const unsigned grid = (unsigned)std::min<int64_t>(want, (int64_t)info.sms * 16);
    if (fmt == kMXFP8) {
        if (out_bf16) dequant_kernel<kMXFP8, true><<<grid, 256, 0, stream>>>(codes, ldc, scales, lds, n, k, out);
        else dequant_kernel<kMXFP8, false><<<grid, 256, 0, stream>>>(codes, ldc, scales, lds, n, k, out);
    } else {
        if (out_bf16) dequant_kernel<kNVFP4, true><<<grid, 256, 0, stream>>>(codes, ldc, scales, lds, n, k, out);
        else dequant_kernel<kNVFP4, false><<<grid, 256, 0, stream>>>(codes, ldc, scales, lds, n, k, out);
    }
    QMM_CUDA_TRY(cudaGetLastError());
    return QMM_OK;
}

}  // namespace qmm
