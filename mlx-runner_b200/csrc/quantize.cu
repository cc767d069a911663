// quantize.cu - fp32 / bf16 W [N, K] -> MLX packed codes + scales on the GPU.
//
// Counterpart of mlx_quantize (src/mlx.zig:278, called by the reference's
// qmm test at src/model.zig:1577 with no global scale); the rules are in
// quantize.cuh.  Output is MLX's layout: codes [N, K*bits/8] bytes (the U32
// [N, K*bits/32] array, LSB-first), scales U8 [N, K/group].
//
// HBM-bound: every value is read once (4 or 2 bytes) and written as one code
// (1 byte or half a byte) plus a scale byte per group.  A lane takes four
// consecutive values of a row (one 16-byte or 8-byte load), so a warp reads
// 512 (fp32) or 256 (bf16) contiguous bytes per step; the lanes of one group
// (4 for nvfp4's 16 values, 8 for mxfp8's 32) combine their maxima with
// shuffles, and each lane stores its four codes as one 2- or 4-byte word.
// Groups never straddle rows or warps: K/4 is a multiple of the lanes per
// group and warps start on multiples of 32 lanes.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>

#include "internal.h"
#include "quantize.cuh"

namespace qmm {
namespace {

template <bool BF16, bool VEC>
__device__ __forceinline__ void load4(const void* __restrict__ w, int64_t off, float (&v)[4]) {
    if constexpr (BF16) {
        const uint16_t* p = static_cast<const uint16_t*>(w) + off;
        if constexpr (VEC) {
            const uint2 q = __ldg(reinterpret_cast<const uint2*>(p));
            v[0] = __uint_as_float(q.x << 16);
            v[1] = __uint_as_float(q.x & 0xFFFF0000u);
            v[2] = __uint_as_float(q.y << 16);
            v[3] = __uint_as_float(q.y & 0xFFFF0000u);
        } else {
#pragma unroll
            for (int i = 0; i < 4; ++i) v[i] = __uint_as_float(static_cast<uint32_t>(__ldg(p + i)) << 16);
        }
    } else {
        const float* p = static_cast<const float*>(w) + off;
        if constexpr (VEC) {
            const float4 q = __ldg(reinterpret_cast<const float4*>(p));
            v[0] = q.x; v[1] = q.y; v[2] = q.z; v[3] = q.w;
        } else {
#pragma unroll
            for (int i = 0; i < 4; ++i) v[i] = __ldg(p + i);
        }
    }
}

template <int FMT, bool BF16, bool VEC>
__global__ void __launch_bounds__(256) quantize_kernel(const void* __restrict__ w, int64_t ldw, int64_t n,
                                                       int64_t k, uint8_t* __restrict__ codes,
                                                       uint8_t* __restrict__ scales) {
    constexpr int kLanesPerGroup = FMT == kMXFP8 ? 8 : 4;
    const int64_t cpr = k / 4;                         // 4-value chunks per row
    const int64_t total = n * cpr;
    const int lane = threadIdx.x & 31;
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    // base is the warp's first chunk (a multiple of 32): the loop is warp-uniform.
    for (int64_t base = static_cast<int64_t>(blockIdx.x) * blockDim.x + (threadIdx.x & ~31); base < total;
         base += stride) {
        const int64_t t = base + lane;
        const bool valid = t < total;                  // whole groups are valid or not
        float v[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        int64_t row = 0, c = 0;
        if (valid) {
            row = t / cpr;
            c = t - row * cpr;
            load4<BF16, VEC>(w, row * ldw + c * 4, v);
        }
        float amax = 0.0f;
#pragma unroll
        for (int i = 0; i < 4; ++i) amax = quant::max_skip_nan(amax, fabsf(v[i]));
#pragma unroll
        for (int o = 1; o < kLanesPerGroup; o <<= 1)
            amax = quant::max_skip_nan(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, o));
        if (!valid) continue;
        if constexpr (FMT == kMXFP8) {
            const int x = quant::mx_shared_exp(amax);
            const float inv = quant::pow2f(-x);
            uint32_t word = 0;
#pragma unroll
            for (int i = 0; i < 4; ++i) word |= quant::encode_e4m3(quant::mul_rn(v[i], inv)) << (8 * i);
            *reinterpret_cast<uint32_t*>(codes + row * k + c * 4) = word;
            if ((lane & (kLanesPerGroup - 1)) == 0) scales[row * (k / 32) + c / 8] = static_cast<uint8_t>(x + 127);
        } else {
            const uint32_t sq = quant::encode_e4m3(quant::div_rn(amax, 6.0f));
            const float sd = quant::e4m3_value(sq);
            uint32_t half = 0;
#pragma unroll
            for (int i = 0; i < 4; ++i) half |= quant::nvfp4_code(v[i], sd) << (4 * i);
            *reinterpret_cast<uint16_t*>(codes + row * (k / 2) + c * 2) = static_cast<uint16_t>(half);
            if ((lane & (kLanesPerGroup - 1)) == 0) scales[row * (k / 16) + c / 4] = static_cast<uint8_t>(sq);
        }
    }
}

template <int FMT, bool BF16>
void launch_one(bool vec, unsigned grid, const void* w, int64_t ldw, int64_t n, int64_t k, uint8_t* codes,
                uint8_t* scales, cudaStream_t s) {
    if (vec) quantize_kernel<FMT, BF16, true><<<grid, 256, 0, s>>>(w, ldw, n, k, codes, scales);
    else quantize_kernel<FMT, BF16, false><<<grid, 256, 0, s>>>(w, ldw, n, k, codes, scales);
}

}  // namespace

int launch_quantize(int fmt, const void* w, bool w_bf16, int64_t ldw, int64_t n, int64_t k, uint8_t* codes,
                    uint8_t* scales, cudaStream_t stream) {
    if (n == 0) return QMM_OK;
    int dev = 0;
    QMM_CUDA_TRY(cudaGetDevice(&dev));
    DeviceInfo info;
    if (int rc = device_info(dev, &info)) return rc;
    if (int rc = check_device_buffer(w, dev, "w")) return rc;
    if (int rc = check_device_buffer(codes, dev, "codes")) return rc;
    if (int rc = check_device_buffer(scales, dev, "scales")) return rc;
    const int64_t chunks = n * (k / 4);
    const int64_t want = (chunks + 255) / 256;
    const unsigned grid = static_cast<unsigned>(std::min<int64_t>(want, static_cast<int64_t>(info.sms) * 8));
    // Vector loads need every row's first value on a 16-byte (fp32) or 8-byte
    // (bf16) boundary; chunk offsets inside a row keep it.
    const int64_t align = w_bf16 ? 8 : 16, esize = w_bf16 ? 2 : 4;
    const bool vec = (reinterpret_cast<uintptr_t>(w) % align) == 0 && (ldw * esize) % align == 0;
    if (fmt == kMXFP8) {
        if (w_bf16) launch_one<kMXFP8, true>(vec, grid, w, ldw, n, k, codes, scales, stream);
        else launch_one<kMXFP8, false>(vec, grid, w, ldw, n, k, codes, scales, stream);
    } else {
        if (w_bf16) launch_one<kNVFP4, true>(vec, grid, w, ldw, n, k, codes, scales, stream);
        else launch_one<kNVFP4, false>(vec, grid, w, ldw, n, k, codes, scales, stream);
    }
    QMM_CUDA_TRY(cudaGetLastError());
    return QMM_OK;
}

}  // namespace qmm
