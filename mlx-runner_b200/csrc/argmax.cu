// argmax.cu - greedy sampling over bf16 logits rows (the unfused path of
// qmm_lm_head_argmax; the decode kernel fuses the same arithmetic into its
// epilogue).
//
// src/sample.zig:162-170 (sampleToken, temp == 0): id = argmax of the row
// (mlx_argmax_axis), lp = logprobOf(row, id) (sample.zig:69-79) = logit[id]
// minus logsumexp(row).  Here: the index of the largest value, the lowest
// index among equal values and NaN above every number; logsumexp as max +
// log(sum exp(l - max)) in fp32, rounded to bf16 like the bf16 array the
// reference reads back, and lp = logit[id] - that value in fp32.
#include <cuda_runtime.h>

#include <cstdint>

#include "formats.cuh"
#include "internal.h"

namespace qmm {
namespace {

constexpr int kThreads = 1024;

__device__ __forceinline__ unsigned long long rank_key(float v, uint32_t idx) {
    const uint32_t u = __float_as_uint(v);
    const uint32_t ord = (v != v) ? 0xFFFFFFFFu : ((u & 0x80000000u) ? ~u : (u | 0x80000000u));
    return ((unsigned long long)ord << 32) | (0xFFFFFFFFu - idx);
}

__global__ void __launch_bounds__(kThreads) argmax_rows_kernel(const uint16_t* __restrict__ logits, int64_t ldl,
                                                               int64_t n, int32_t* __restrict__ ids,
                                                               float* __restrict__ lp) {
    __shared__ unsigned long long s_key[kThreads / 32];
    __shared__ float s_m[kThreads / 32], s_s[kThreads / 32];
    const uint16_t* row = logits + (int64_t)blockIdx.x * ldl;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    unsigned long long key = 0;
    float mx = -INFINITY;
    for (int64_t i = threadIdx.x; i < n; i += kThreads) {
        const float v = bf16_to_f32(row[i]);
        key = max(key, rank_key(v, (uint32_t)i));
        mx = fmaxf(mx, v);
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
        key = max(key, __shfl_xor_sync(0xFFFFFFFFu, key, o));
        mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, o));
    }
    if (lane == 0) { s_key[warp] = key; s_m[warp] = mx; }
    __syncthreads();
    if (warp == 0) {
        key = s_key[lane];
        mx = s_m[lane];
#pragma unroll
        for (int o = 16; o; o >>= 1) {
            key = max(key, __shfl_xor_sync(0xFFFFFFFFu, key, o));
            mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, o));
        }
        if (lane == 0) { s_key[0] = key; s_m[0] = mx; }
    }
    __syncthreads();
    key = s_key[0];
    mx = s_m[0];
    float s = 0.0f;
    if (mx != -INFINITY)
        for (int64_t i = threadIdx.x; i < n; i += kThreads) s += expf(bf16_to_f32(row[i]) - mx);
#pragma unroll
    for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xFFFFFFFFu, s, o);
    __syncthreads();
    if (lane == 0) s_s[warp] = s;
    __syncthreads();
    if (threadIdx.x == 0) {
        float tot = 0.0f;
        for (int w = 0; w < kThreads / 32; ++w) tot += s_s[w];
        const uint32_t idx = 0xFFFFFFFFu - (uint32_t)(key & 0xFFFFFFFFu);
        ids[blockIdx.x] = (int32_t)idx;
        if (lp) {
            const float lse = bf16_to_f32(f32_to_bf16(mx + logf(tot)));
            lp[blockIdx.x] = bf16_to_f32(row[idx]) - lse;
        }
    }
}

}  // namespace

int launch_argmax_rows(const uint16_t* logits, int64_t ldl, int64_t m, int64_t n, int32_t* ids, float* lp,
                       cudaStream_t stream) {
    if (m <= 0 || n <= 0) return QMM_OK;
    argmax_rows_kernel<<<(unsigned)m, kThreads, 0, stream>>>(logits, ldl, n, ids, lp);
    QMM_CUDA_TRY(cudaGetLastError());
    return QMM_OK;
}

}  // namespace qmm
