// tensor_peak.cu - measured dense tcgen05 MMA rates of this GPU, the roofline
// denominators of the prefill GEMMs.
//
// The exact prefill path (gemm.cu) dequantises W to bf16 and runs
// tcgen05.mma kind::f16; the x-quantised path (gemm_bs.cu) feeds the packed
// codes themselves to the block-scaled kinds.  Their peaks differ by 2x / 4x
// on paper, so each fraction is reported against the rate of its own kind,
// measured here rather than taken from a datasheet:
//   kind::f16                    bf16 x bf16, K = 16 per instruction
//   kind::mxf8f6f4.block_scale   E4M3 x E4M3, UE8M0 scale per 32, K = 32
//   kind::mxf4nvf4.block_scale   E2M1 x E2M1, UE4M3 scale per 16, K = 64
// One CTA per SM, one thread issuing back-to-back M = 128 x N = 256 MMAs on
// resident shared-memory tiles into one TMEM accumulator; the caller times
// the launch.  Operand values do not change the rate; the scale factors in
// TMEM are set to 1.0 so the sums stay finite.
#include <cuda_runtime.h>

#include <cstdint>

#include "internal.h"

namespace qmm {
namespace {

constexpr int kPM = 128, kPN = 256;
constexpr int kARowBytes = 64;                      // two 32-byte k-steps per row
constexpr int kABytes = kPM * kARowBytes;           // 8 KB
constexpr int kBBytes = kPN * kARowBytes;           // 16 KB
constexpr int kSfaCol = 256, kSfbCol = 320;         // TMEM columns of the scale factors
constexpr uint64_t kPeakTimeoutNs = 4000000000ull;

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ uint64_t now_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}

// K-major, 64-byte swizzle shared-memory descriptor (8-row atoms of 512
// bytes), version 1: the layout gemm.cu's tiles use.
__device__ __forceinline__ uint64_t desc64(uint32_t saddr) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr >> 4) & 0x3FFF);
    d |= (uint64_t)1 << 16;
    d |= (uint64_t)(512 >> 4) << 32;
    d |= (uint64_t)1 << 46;
    d |= (uint64_t)4 << 61;
    return d;
}

// Instruction descriptors, M = 128, N = 256, K-major A and B, fp32 D.
//   kind::f16: D fp32 (bit 4), A / B bf16 (bits 7 / 10), N >> 3 at 17, M >> 4 at 24.
//   block-scaled kinds: A / B format at bits 7-9 / 10-12 (mxf8f6f4: E4M3 = 0;
//   mxf4nvf4: E2M1 = 1), scale type at bit 23 (UE8M0 = 1, UE4M3 = 0), scale
//   factor ids (bits 4-5, 29-30) 0, dense K (bit 31) 0.
constexpr uint32_t kIdescF16 = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(kPN >> 3) << 17) |
                               ((uint32_t)(kPM >> 4) << 24);
constexpr uint32_t kIdescMxf8 = ((uint32_t)(kPN >> 3) << 17) | (1u << 23) | ((uint32_t)(kPM >> 4) << 24);
constexpr uint32_t kIdescNvf4 = (1u << 7) | (1u << 10) | ((uint32_t)(kPN >> 3) << 17) | ((uint32_t)(kPM >> 4) << 24);

__global__ void __launch_bounds__(128, 1) tensor_peak_kernel(int kind, int iters, unsigned int* err) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* a = smem;
    uint8_t* b = smem + kABytes;
    uint64_t* bar = reinterpret_cast<uint64_t*>(smem + kABytes + kBBytes);
    uint32_t* tslot = reinterpret_cast<uint32_t*>(bar + 1);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    // Operands: 0x3C in every byte (bf16 pairs 0x3C3C, E4M3 1.5, E2M1 pairs
    // of -2.0 / 6.0); fixed, finite.
    for (int i = threadIdx.x; i < (kABytes + kBBytes) / 4; i += blockDim.x)
        reinterpret_cast<uint32_t*>(smem)[i] = 0x3C3C3C3Cu;
    if (threadIdx.x == 0) {
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_addr(bar)));
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");   // operands visible to the tensor core
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(smem_addr(tslot))
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = *tslot;

    // Scale factors = 1.0 (UE8M0 0x7F / UE4M3 0x38) in every lane of the
    // scale columns: each warp writes its 32 lanes.
    const uint32_t one = kind == 1 ? 0x7F7F7F7Fu : 0x38383838u;
    const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
#pragma unroll
    for (int c = 0; c < 8; ++c) {
        asm volatile("tcgen05.st.sync.aligned.32x32b.x1.b32 [%0], {%1};" ::"r"(tmem + lane_base + kSfaCol + c),
                     "r"(one) : "memory");
        asm volatile("tcgen05.st.sync.aligned.32x32b.x1.b32 [%0], {%1};" ::"r"(tmem + lane_base + kSfbCol + c),
                     "r"(one) : "memory");
    }
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");

    if (threadIdx.x == 0) {
        const uint32_t aa = smem_addr(a), ba = smem_addr(b);
        const uint32_t sfa = tmem + kSfaCol, sfb = tmem + kSfbCol;
        for (int it = 0; it < iters; ++it) {
#pragma unroll
            for (int ks = 0; ks < 2; ++ks) {
                const uint64_t ad = desc64(aa + ks * 32), bd = desc64(ba + ks * 32);
                const uint32_t acc = (it | ks) ? 1u : 0u;
                if (kind == 0) {
                    asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
                                 "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
                                 ::"r"(tmem), "l"(ad), "l"(bd), "r"(kIdescF16), "r"(acc) : "memory");
                } else if (kind == 1) {
                    asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
                                 "tcgen05.mma.cta_group::1.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%5], [%6], p;\n\t}"
                                 ::"r"(tmem), "l"(ad), "l"(bd), "r"(kIdescMxf8), "r"(acc), "r"(sfa), "r"(sfb)
                                 : "memory");
                } else {
                    asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
                                 "tcgen05.mma.cta_group::1.kind::mxf4nvf4.block_scale.block16 [%0], %1, %2, %3, [%5], [%6], p;\n\t}"
                                 ::"r"(tmem), "l"(ad), "l"(bd), "r"(kIdescNvf4), "r"(acc), "r"(sfa), "r"(sfb)
                                 : "memory");
                }
            }
        }
        asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                     ::"r"(smem_addr(bar)) : "memory");
        // Bounded wait for the last MMA (phase 0 of the barrier).
        const uint64_t t0 = now_ns();
        for (;;) {
            uint32_t ok;
            asm volatile("{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], 0;\n\t"
                         "selp.u32 %0, 1, 0, p;\n\t}" : "=r"(ok) : "r"(smem_addr(bar)) : "memory");
            if (ok) break;
            if (now_ns() - t0 > kPeakTimeoutNs) {
                atomicOr(err, 1u);
                break;
            }
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    if (warp == 0)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tmem) : "memory");
}

}  // namespace
}  // namespace qmm

using namespace qmm;

// Diagnostic entry point (include/qmm.h): one timed launch of `iters`
// back-to-back MMA pairs per SM; *tflops = dense FLOPs / event time.
extern "C" int qmm_tensor_peak(int kind, int64_t iters, void* stream_ptr, double* tflops) {
    if (!tflops) return set_error(QMM_ERR_BAD_ARGUMENT, "tflops is NULL");
    if (kind < 0 || kind > 2)
        return set_error(QMM_ERR_BAD_ARGUMENT, "tensor peak kind %d (0 f16, 1 mxf8f6f4, 2 mxf4nvf4)", kind);
    if (iters < 1 || iters > (1 << 24)) return set_error(QMM_ERR_BAD_ARGUMENT, "iters %lld", (long long)iters);
    cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
    int dev = 0;
    QMM_CUDA_TRY(cudaGetDevice(&dev));
    DeviceInfo info;
    if (int rc = device_info(dev, &info)) return rc;
    // More than half an SM's shared memory: one CTA per SM, so no two CTAs
    // share an SM's tensor core or TMEM.
    const int smem = 120 * 1024;
    QMM_CUDA_TRY(cudaFuncSetAttribute(tensor_peak_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    unsigned int* err = nullptr;
    cudaEvent_t e0 = nullptr, e1 = nullptr;
    auto cleanup = [&]() {
        if (err) cudaFree(err);
        if (e0) cudaEventDestroy(e0);
        if (e1) cudaEventDestroy(e1);
    };
    cudaError_t e;
    if ((e = cudaMalloc(&err, sizeof(unsigned int))) != cudaSuccess ||
        (e = cudaMemsetAsync(err, 0, sizeof(unsigned int), stream)) != cudaSuccess ||
        (e = cudaEventCreate(&e0)) != cudaSuccess || (e = cudaEventCreate(&e1)) != cudaSuccess ||
        (e = cudaEventRecord(e0, stream)) != cudaSuccess) {
        cleanup();
        return cuda_error(e, "tensor peak setup");
    }
    tensor_peak_kernel<<<info.sms, 128, smem, stream>>>(kind, (int)iters, err);
    unsigned int host_err = 0;
    float ms = 0.f;
    if ((e = cudaGetLastError()) != cudaSuccess || (e = cudaEventRecord(e1, stream)) != cudaSuccess ||
        (e = cudaMemcpyAsync(&host_err, err, sizeof(host_err), cudaMemcpyDeviceToHost, stream)) != cudaSuccess ||
        (e = cudaStreamSynchronize(stream)) != cudaSuccess || (e = cudaEventElapsedTime(&ms, e0, e1)) != cudaSuccess) {
        cleanup();
        return cuda_error(e, "tensor peak kernel");
    }
    cleanup();
    if (host_err) return set_error(QMM_ERR_TIMEOUT, "tensor peak kernel: the wait for its last MMA timed out");
    const double k = kind == 0 ? 16 : kind == 1 ? 32 : 64;
    const double flops = (double)info.sms * (double)iters * 2.0 * 2.0 * kPM * kPN * k;
    *tflops = flops / (ms * 1e-3) / 1e12;
    return QMM_OK;
}
