// gemv.cu - split-K quantized GEMV for M <= 8 (decode, MTP verify), sm_100a.
//
// y[m, n] = sum_k x[m, k] * dequant(W)[n, k]  with W in mxfp8 or nvfp4.
// The reference reaches this through qlinear (src/model.zig:244-258) with
// M = 1 (decode, src/engine.zig:428-455) and M = 2..3 (MTP verify,
// src/engine.zig:548, :656).  The op is HBM-bound: every code byte is read
// once, so the kernel is built to keep enough 16-byte loads in flight:
//   - a warp owns R weight rows; lane l streams 16-byte code chunks
//     l, l+32, ... of each row with non-allocating vector loads, so one warp
//     load instruction covers 512 contiguous bytes of a row;
//   - the R rows share each x slice (L1-resident), cutting x traffic by R;
//   - codes are widened with the sm_100 cvt.f16x2.{e4m3x2,e2m1x2}
//     instructions, multiplied into packed fp32 (FFMA2) partial sums per
//     scale group, and each group partial is scaled once (fp32 accumulate);
//   - split-K: the S CTAs of a thread-block cluster take disjoint K ranges
//     of the same rows and reduce their partials through distributed shared
//     memory (no global workspace, no atomics, fixed summation order).
#include <cooperative_groups.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <mutex>

#include "formats.cuh"
#include "internal.h"

namespace cg = cooperative_groups;

namespace qmm {
namespace {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kMaxM = 8;

struct GemvParams {
    const uint8_t* __restrict__ codes;
    const uint8_t* __restrict__ scales;
    const uint16_t* __restrict__ x;
    uint16_t* __restrict__ y;
    float* __restrict__ yf;  // fp32 output (row-parallel partials) when non-null
    int64_t ldc, lds, ldx, ldy;
    int n, k;
    int row_bytes;     // K * bits / 8
    int chunks;        // ceil(row_bytes / 16)
    int chunks_per_split;
};

__device__ __forceinline__ uint4 ld_stream16(const uint8_t* p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
    return v;
}

__device__ __forceinline__ uint32_t ld_stream4(const uint8_t* p) {
    uint32_t v;
    asm volatile("ld.global.nc.L1::no_allocate.u32 %0, [%1];" : "=r"(v) : "l"(p));
    return v;
}

// One 16-byte code chunk of a row; `bytes` valid bytes (16, or 8 for the
// ragged end of an nvfp4 row).  Missing bytes read as zero codes (0.0).
template <bool VEC16>
__device__ __forceinline__ uint4 load_chunk(const uint8_t* p, int bytes) {
    if (VEC16 && bytes == 16) return ld_stream16(p);
    uint4 v = make_uint4(0, 0, 0, 0);
    v.x = ld_stream4(p);
    v.y = ld_stream4(p + 4);
    if (bytes == 16) {
        v.z = ld_stream4(p + 8);
        v.w = ld_stream4(p + 12);
    }
    return v;
}

// 8 consecutive bf16 of x -> 4 float2.
template <bool VEC16>
__device__ __forceinline__ void load_x8(const uint16_t* p, float2 (&xf)[4]) {
    uint32_t u[4];
    if (VEC16) {
        uint4 v = __ldg(reinterpret_cast<const uint4*>(p));
        u[0] = v.x; u[1] = v.y; u[2] = v.z; u[3] = v.w;
    } else {
        const uint32_t* q = reinterpret_cast<const uint32_t*>(p);
#pragma unroll
        for (int i = 0; i < 4; ++i) u[i] = __ldg(q + i);
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) xf[i] = bf16x2_to_float2(u[i]);
}

__device__ __forceinline__ void store_out(const GemvParams& p, int m, int row, float v) {
    if (p.yf) p.yf[(int64_t)m * p.ldy + row] = v;
    else p.y[(int64_t)m * p.ldy + row] = f32_to_bf16(v);
}

__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) { return __ffma2_rn(a, b, c); }

// 8 codes of one row (as 4 f16x2 pairs) against 8 x values for M rows.
template <int M>
__device__ __forceinline__ void dot8(const uint32_t (&h)[4], const float2 (&xf)[M][4],
                                     float2 (&part)[M]) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        float2 w = f16x2_to_float2(h[i]);
#pragma unroll
        for (int m = 0; m < M; ++m) part[m] = ffma2(w, xf[m][i], part[m]);
    }
}

template <int FMT, int M, int R, bool VEC16>
__global__ void __launch_bounds__(kThreads) gemv_kernel(GemvParams p) {
    constexpr int RB = kWarps * R;  // rows per CTA
    __shared__ float part_smem[RB * M];

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int row0 = blockIdx.x * RB + warp * R;
    const int split = blockIdx.y, nsplit = gridDim.y;
    const int c_begin = split * p.chunks_per_split;
    const int c_end = min(p.chunks, c_begin + p.chunks_per_split);

    const uint8_t* crow[R];
    const uint8_t* srow[R];
    bool rvalid[R];
#pragma unroll
    for (int r = 0; r < R; ++r) {
        rvalid[r] = (row0 + r) < p.n;
        const int64_t rr = rvalid[r] ? (row0 + r) : 0;
        crow[r] = p.codes + rr * p.ldc;
        srow[r] = p.scales + rr * p.lds;
    }

    float acc[R][M];
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
        for (int m = 0; m < M; ++m) acc[r][m] = 0.f;

    for (int c = c_begin + lane; c < c_end; c += 32) {
        const int bytes = min(16, p.row_bytes - c * 16);
        uint4 w[R];
#pragma unroll
        for (int r = 0; r < R; ++r)
            w[r] = rvalid[r] ? load_chunk<VEC16>(crow[r] + (int64_t)c * 16, bytes)
                             : make_uint4(0, 0, 0, 0);
        if constexpr (FMT == kMXFP8) {
            // 16 codes = half of one 32-code group.
            float s[R];
#pragma unroll
            for (int r = 0; r < R; ++r) s[r] = scale_to_f32<FMT>(__ldg(srow[r] + (c >> 1)));
            float2 part[R][M];
#pragma unroll
            for (int r = 0; r < R; ++r)
#pragma unroll
                for (int m = 0; m < M; ++m) part[r][m] = make_float2(0.f, 0.f);
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                float2 xf[M][4];
#pragma unroll
                for (int m = 0; m < M; ++m)
                    load_x8<VEC16>(p.x + (int64_t)m * p.ldx + (int64_t)c * 16 + h * 8, xf[m]);
#pragma unroll
                for (int r = 0; r < R; ++r) {
                    uint32_t hw[4];
                    uint32_t lo[2], hi[2];
                    e4m3x4_to_f16x2(h ? w[r].z : w[r].x, lo);
                    e4m3x4_to_f16x2(h ? w[r].w : w[r].y, hi);
                    hw[0] = lo[0]; hw[1] = lo[1]; hw[2] = hi[0]; hw[3] = hi[1];
                    dot8<M>(hw, xf, part[r]);
                }
            }
#pragma unroll
            for (int r = 0; r < R; ++r)
#pragma unroll
                for (int m = 0; m < M; ++m) acc[r][m] = fmaf(part[r][m].x + part[r][m].y, s[r], acc[r][m]);
        } else {
            // 32 codes = two 16-code groups (the second may be past K).
#pragma unroll
            for (int g = 0; g < 2; ++g) {
                if (g == 1 && bytes < 16) break;
                float s[R];
#pragma unroll
                for (int r = 0; r < R; ++r) s[r] = scale_to_f32<FMT>(__ldg(srow[r] + 2 * c + g));
                float2 part[R][M];
#pragma unroll
                for (int r = 0; r < R; ++r)
#pragma unroll
                    for (int m = 0; m < M; ++m) part[r][m] = make_float2(0.f, 0.f);
#pragma unroll
                for (int j = 0; j < 2; ++j) {
                    float2 xf[M][4];
#pragma unroll
                    for (int m = 0; m < M; ++m)
                        load_x8<VEC16>(p.x + (int64_t)m * p.ldx + (int64_t)c * 32 + g * 16 + j * 8, xf[m]);
#pragma unroll
                    for (int r = 0; r < R; ++r) {
                        const uint32_t word = (g == 0) ? (j == 0 ? w[r].x : w[r].y)
                                                       : (j == 0 ? w[r].z : w[r].w);
                        uint32_t hw[4];
                        e2m1x8_to_f16x2(word, hw);
                        dot8<M>(hw, xf, part[r]);
                    }
                }
#pragma unroll
                for (int r = 0; r < R; ++r)
#pragma unroll
                    for (int m = 0; m < M; ++m)
                        acc[r][m] = fmaf(part[r][m].x + part[r][m].y, s[r], acc[r][m]);
            }
        }
    }

    // Lane reduction (butterfly: every lane ends with every sum).
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
        for (int m = 0; m < M; ++m) {
            float v = acc[r][m];
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, off);
            acc[r][m] = v;
        }
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
        for (int m = 0; m < M; ++m)
            if (lane == ((r * M + m) & 31)) part_smem[(warp * R + r) * M + m] = acc[r][m];

    // Cross-split reduction through distributed shared memory: CTA q of the
    // cluster sums slice q of the block's outputs over all S partials, in
    // rank order, and writes them as bf16.
    constexpr int kOut = RB * M;
    if (nsplit == 1) {
        __syncthreads();
        for (int t = threadIdx.x; t < kOut; t += kThreads) {
            const int row = blockIdx.x * RB + t / M, m = t % M;
            if (row < p.n) store_out(p, m, row, part_smem[t]);
        }
        return;
    }
    cg::cluster_group cluster = cg::this_cluster();
    cluster.sync();
    const int per = (kOut + nsplit - 1) / nsplit;
    const int t0 = split * per, t1 = min(kOut, t0 + per);
    for (int t = t0 + threadIdx.x; t < t1; t += kThreads) {
        float v = 0.f;
        for (int q = 0; q < nsplit; ++q) v += cluster.map_shared_rank(part_smem, q)[t];
        const int row = blockIdx.x * RB + t / M, m = t % M;
        if (row < p.n) store_out(p, m, row, v);
    }
    cluster.sync();  // keep this CTA's shared memory alive until peers are done
}

template <int FMT, int M, bool VEC16>
int launch_m(const GemvParams& p, int rows_per_warp_hint, int nsplit, cudaStream_t stream) {
    (void)rows_per_warp_hint;
    constexpr int R = (M <= 1) ? 8 : (M <= 4 ? 4 : 2);   // M = 2 with 8 rows needs > 128 registers
    constexpr int RB = kWarps * R;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)((p.n + RB - 1) / RB), (unsigned)nsplit, 1);
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 1;
    attr[0].val.clusterDim.y = (unsigned)nsplit;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    QMM_CUDA_TRY(cudaLaunchKernelEx(&cfg, gemv_kernel<FMT, M, R, VEC16>, p));
    return QMM_OK;
}

template <int FMT, bool VEC16>
int launch_fmt(const GemvParams& p, int m, int nsplit, cudaStream_t stream) {
    switch (m) {
        case 1: return launch_m<FMT, 1, VEC16>(p, 0, nsplit, stream);
        case 2: return launch_m<FMT, 2, VEC16>(p, 0, nsplit, stream);
        case 3: return launch_m<FMT, 3, VEC16>(p, 0, nsplit, stream);
        case 4: return launch_m<FMT, 4, VEC16>(p, 0, nsplit, stream);
        case 5: return launch_m<FMT, 5, VEC16>(p, 0, nsplit, stream);
        case 6: return launch_m<FMT, 6, VEC16>(p, 0, nsplit, stream);
        case 7: return launch_m<FMT, 7, VEC16>(p, 0, nsplit, stream);
        case 8: return launch_m<FMT, 8, VEC16>(p, 0, nsplit, stream);
    }
    return set_error(QMM_ERR_BAD_SHAPE, "gemv: m=%d outside 1..8", m);
}

inline int rows_per_warp(int m) { return (m <= 1) ? 8 : (m <= 4 ? 4 : 2); }

// Number of K-splits (cluster size): the smallest power of two giving at
// least ~4 CTAs per SM, while each lane keeps >= 2 chunks per split.
int choose_splits(int64_t n, int chunks, int m, int sms) {
    const int64_t rb = (int64_t)kWarps * rows_per_warp(m);
    const int64_t row_blocks = (n + rb - 1) / rb;
    int s = 1;
    while (s < 8 && row_blocks * s < 4LL * sms && chunks / (2 * s) >= 64) s *= 2;
    return s;
}

}  // namespace

int gemv_max_m() { return kMaxM; }

int launch_gemv(const QmmArgs& a, cudaStream_t stream) {
    if (a.m < 1 || a.m > kMaxM) return set_error(QMM_ERR_BAD_SHAPE, "gemv: m=%lld outside 1..8", (long long)a.m);
    if (a.n > INT32_MAX || a.k > INT32_MAX) return set_error(QMM_ERR_BAD_SHAPE, "gemv: n or k too large");
    int dev = 0;
    QMM_CUDA_TRY(cudaGetDevice(&dev));
    DeviceInfo info;
    if (int rc = device_info(dev, &info)) return rc;
    GemvParams p;
    p.codes = a.codes; p.scales = a.scales; p.x = a.x; p.y = a.y; p.yf = a.yf;
    p.ldc = a.ldc; p.lds = a.lds; p.ldx = a.ldx; p.ldy = a.ldy;
    p.n = (int)a.n; p.k = (int)a.k;
    const int bits = a.fmt == kMXFP8 ? 8 : 4;
    p.row_bytes = (int)(a.k * bits / 8);
    p.chunks = (p.row_bytes + 15) / 16;
    const int nsplit = choose_splits(a.n, p.chunks, (int)a.m, info.sms);
    p.chunks_per_split = (p.chunks + nsplit - 1) / nsplit;
    const bool vec16 = (reinterpret_cast<uintptr_t>(a.codes) % 16 == 0) && (a.ldc % 16 == 0) &&
                       (reinterpret_cast<uintptr_t>(a.x) % 16 == 0) && (a.ldx % 8 == 0);
    if (a.fmt == kMXFP8)
        return vec16 ? launch_fmt<kMXFP8, true>(p, (int)a.m, nsplit, stream)
                     : launch_fmt<kMXFP8, false>(p, (int)a.m, nsplit, stream);
    return vec16 ? launch_fmt<kNVFP4, true>(p, (int)a.m, nsplit, stream)
                 : launch_fmt<kNVFP4, false>(p, (int)a.m, nsplit, stream);
}

}  // namespace qmm
