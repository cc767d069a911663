// gemm_bs.cu - x-quantised prefill GEMM on the block-scaled tensor cores
// (tcgen05.mma kind::mxf4nvf4.block_scale.block16), nvfp4 weights.
//
// NOT the parity path.  The exact prefill GEMM (gemm.cu) dequantises W to
// bf16 and keeps x in bf16, so every product is exact; this variant instead
// quantises x to nvfp4 too (E2M1 codes, UE4M3 scale per 16, the same rules
// as qmm_quantize) and feeds both packed operands to the FP4 tensor core, as
// MLX's own block-scaled kernels would on hardware that has them.  The
// weight is used exactly as stored: codes by TMA straight from the
// checkpoint layout, its UE4M3 scales as the A-side scale factors.  The
// result is y = quantize(x) . dequant(W)^T in fp32, rounded to bf16 - about
// 10% relative error from quantising x, which is why it is a separate entry
// point (qmm_run_blockscaled) and never chosen by qmm_run.
//
// Tile: 128 weight rows (MMA M, A operand) x 256 tokens (MMA N, B operand),
// K-blocks of 256 codes (128 bytes per row, one 128-byte swizzle atom).  Per
// K-block the MMA warp copies the block's scale factors from shared memory
// into TMEM (tcgen05.cp 32x128b.warpx4: 4 A atoms, 8 B atoms) and issues
// four K = 64 MMAs.  Scale factors in TMEM: lane r0 of every 32-lane
// quadrant holds, in 32-bit column g of an atom, the four UE4M3 scales
// (k sub-blocks 0-3 of one MMA) of row r0 + 32 g; a shared-memory atom is
// 512 bytes with byte r0 * 16 + g * 4 + s.  Both operands' scales are
// re-tiled into atoms before the GEMM (W once per weight, x per call), so a
// stage's scale factors arrive with one bulk copy each.
// Warp roles (256 threads): 0 TMA producer, 1 MMA issuer, 2 TMEM allocator,
// 4-7 epilogue (tcgen05.ld -> bf16 -> y).  Every wait is bounded.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstdint>
#include <mutex>

#include "formats.cuh"
#include "internal.h"

namespace qmm {

// Bit 2: a bounded wait in the block-scaled GEMM timed out.
__device__ unsigned int g_gemm_bs_error = 0;

namespace {

constexpr int kBsStages = 4;
constexpr int kBsTileW = 128;                 // weight rows per tile (MMA M)
constexpr int kBsTileT = 256;                 // tokens per tile (MMA N)
constexpr int kBsKB = 256;                    // codes per K-block (128 bytes per row)
constexpr int kBsWBytes = kBsTileW * 128;     // 16 KB
constexpr int kBsXBytes = kBsTileT * 128;     // 32 KB
constexpr int kBsAtom = 512;                  // one 128-row scale atom
constexpr int kBsSfaBytes = 4 * kBsAtom;      // 4 MMAs x 1 atom
constexpr int kBsSfbBytes = 8 * kBsAtom;      // 4 MMAs x 2 atoms (256 tokens)
constexpr int kBsStageBytes = kBsWBytes + kBsXBytes + kBsSfaBytes + kBsSfbBytes;   // 54 KB
constexpr int kBsThreads = 256;
constexpr int kBsSmem = 1024 + kBsStages * kBsStageBytes + 256;
constexpr uint32_t kBsSfaCol = 256, kBsSfbCol = 272;   // TMEM columns: D 0-255, SFA 16, SFB 32
constexpr uint64_t kBsTimeoutNs = 2000000000ull;

// kind::mxf4nvf4 instruction descriptor: E2M1 A / B (format 1 at bits 7 /
// 10), UE4M3 scales (bit 23 = 0), N = 256 (>> 3 at 17), M = 128 (>> 4 at 24),
// K-major, dense, scale-factor ids 0.
constexpr uint32_t kBsIdesc = (1u << 7) | (1u << 10) | ((uint32_t)(kBsTileT >> 3) << 17) |
                              ((uint32_t)(kBsTileW >> 4) << 24);

struct BsParams {
    const uint8_t* __restrict__ w_sf;    // W scale atoms [w_tiles][kblocks][4][512]
    const uint8_t* __restrict__ x_sf;    // x scale atoms [t_tiles][kblocks][4][2][512]
    uint16_t* __restrict__ y;
    int64_t ldy;
    int m, n, kblocks, w_tiles, num_tiles;
};

__device__ __forceinline__ uint32_t sm_u32(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }
__device__ __forceinline__ uint64_t bs_now() {
    uint64_t t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}
__device__ __forceinline__ bool bs_try(uint64_t* b, uint32_t parity) {
    uint32_t ok;
    asm volatile("{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
                 "selp.u32 %0, 1, 0, p;\n\t}" : "=r"(ok) : "r"(sm_u32(b)), "r"(parity) : "memory");
    return ok != 0;
}
__device__ __forceinline__ bool bs_wait(uint64_t* b, uint32_t parity, volatile int* abort_flag) {
    if (bs_try(b, parity)) return true;
    const uint64_t t0 = bs_now();
    for (uint32_t i = 1;; ++i) {
        if (bs_try(b, parity)) return true;
        if ((i & 15) == 0) {
            if (*abort_flag) return false;
            if (bs_now() - t0 > kBsTimeoutNs) {
                *abort_flag = 1;
                atomicOr(&g_gemm_bs_error, 4u);
                return false;
            }
        }
    }
}
__device__ __forceinline__ void bs_drain(uint64_t* b, uint32_t parity) {
    const uint64_t t0 = bs_now();
    while (!bs_try(b, parity) && bs_now() - t0 < kBsTimeoutNs) {
    }
}
__device__ __forceinline__ void bs_expect(uint64_t* b, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(sm_u32(b)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void bs_arrive(uint64_t* b) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(sm_u32(b)) : "memory");
}
__device__ __forceinline__ void bs_tma2d(void* dst, const CUtensorMap* map, uint64_t* bar, int x0, int y0) {
    asm volatile("cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
                 " [%0], [%1, {%2, %3}], [%4];"
                 ::"r"(sm_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(x0), "r"(y0), "r"(sm_u32(bar))
                 : "memory");
}
__device__ __forceinline__ void bs_bulk(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 ::"r"(sm_u32(dst)), "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(sm_u32(bar))
                 : "memory");
}
__device__ __forceinline__ void bs_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                 ::"r"(sm_u32(bar)) : "memory");
}
// K-major 128-byte-swizzle operand descriptor (8-row atoms of 1024 bytes).
__device__ __forceinline__ uint64_t bs_desc128(uint32_t saddr) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr >> 4) & 0x3FFF);
    d |= (uint64_t)1 << 16;
    d |= (uint64_t)(1024 >> 4) << 32;
    d |= (uint64_t)1 << 46;
    d |= (uint64_t)2 << 61;
    return d;
}
// A 32-row x 16-byte scale atom (no swizzle; 8-row core matrices of 128
// bytes), the source of tcgen05.cp 32x128b.
__device__ __forceinline__ uint64_t bs_desc_atom(uint32_t saddr) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr >> 4) & 0x3FFF);
    d |= (uint64_t)(128 >> 4) << 16;
    d |= (uint64_t)(128 >> 4) << 32;
    d |= (uint64_t)1 << 46;
    return d;
}
__device__ __forceinline__ void bs_cp_atom(uint32_t tcol, uint64_t sdesc) {
    asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(tcol), "l"(sdesc) : "memory");
}
__device__ __forceinline__ void bs_mma(uint32_t d, uint64_t a, uint64_t b, uint32_t sfa, uint32_t sfb, uint32_t acc) {
    asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
                 "tcgen05.mma.cta_group::1.kind::mxf4nvf4.block_scale.block16 [%0], %1, %2, %3, [%5], [%6], p;\n\t}"
                 ::"r"(d), "l"(a), "l"(b), "r"(kBsIdesc), "r"(acc), "r"(sfa), "r"(sfb) : "memory");
}
__device__ __forceinline__ void bs_ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
        "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__global__ void __launch_bounds__(kBsThreads, 1) qmm_gemm_bs_kernel(const __grid_constant__ CUtensorMap wmap,
                                                                     const __grid_constant__ CUtensorMap xmap,
                                                                     BsParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kBsStages * kBsStageBytes);
    uint64_t* full = bars;                       // stage landed (TMA bytes)
    uint64_t* empty = bars + kBsStages;          // stage consumed (MMA commit)
    uint64_t* tmem_full = bars + 2 * kBsStages;  // accumulator ready (MMA commit)
    uint64_t* tmem_empty = tmem_full + 1;        // accumulator drained (4 epilogue warps)
    uint64_t* drain = tmem_empty + 1;
    volatile int* abort_flag = reinterpret_cast<volatile int*>(drain + 1);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1) + 1;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    auto stage_w = [&](int s) { return smem + s * kBsStageBytes; };
    auto stage_x = [&](int s) { return smem + s * kBsStageBytes + kBsWBytes; };
    auto stage_sfa = [&](int s) { return smem + s * kBsStageBytes + kBsWBytes + kBsXBytes; };
    auto stage_sfb = [&](int s) { return smem + s * kBsStageBytes + kBsWBytes + kBsXBytes + kBsSfaBytes; };

    if (threadIdx.x == 0) {
        for (int s = 0; s < kBsStages; ++s) {
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(sm_u32(&full[s])));
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(sm_u32(&empty[s])));
        }
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(sm_u32(tmem_full)));
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 4;" ::"r"(sm_u32(tmem_empty)));
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(sm_u32(drain)));
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 2) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(sm_u32(tmem_slot))
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    }
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = *tmem_slot;
    const int my_tiles = p.num_tiles > (int)blockIdx.x ? (p.num_tiles - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
    const int total_kb = my_tiles * p.kblocks;

    if (warp == 0) {
        // ---------------- TMA producer ----------------
        if (lane == 0) {
            int last = -1;
            for (int it = 0; it < total_kb; ++it) {
                const int s = it % kBsStages;
                if (!bs_wait(&empty[s], ((uint32_t)(it / kBsStages) & 1u) ^ 1u, abort_flag)) break;
                const int t = (int)blockIdx.x + (it / p.kblocks) * (int)gridDim.x;
                const int kb = it % p.kblocks;
                const int wt = t % p.w_tiles, tt = t / p.w_tiles;
                bs_expect(&full[s], kBsStageBytes);
                bs_tma2d(stage_w(s), &wmap, &full[s], kb * 128, wt * kBsTileW);
                bs_tma2d(stage_x(s), &xmap, &full[s], kb * 128, tt * kBsTileT);
                bs_bulk(stage_sfa(s), p.w_sf + ((int64_t)wt * p.kblocks + kb) * kBsSfaBytes, kBsSfaBytes, &full[s]);
                bs_bulk(stage_sfb(s), p.x_sf + ((int64_t)tt * p.kblocks + kb) * kBsSfbBytes, kBsSfbBytes, &full[s]);
                last = it;
            }
            if (!*abort_flag) {
                // The MMA's commits to every stage used must land before exit.
                for (int it = total_kb; it < total_kb + kBsStages; ++it) {
                    if (it < kBsStages) continue;
                    if (!bs_wait(&empty[it % kBsStages], ((uint32_t)(it / kBsStages) & 1u) ^ 1u, abort_flag)) break;
                }
            }
            if (*abort_flag)
                for (int it = max(0, last - kBsStages + 1); it <= last; ++it)
                    bs_drain(&full[it % kBsStages], (uint32_t)(it / kBsStages) & 1u);
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            int it = 0;
            bool issued = false;
            for (int lt = 0; lt < my_tiles && !*abort_flag; ++lt) {
                if (!bs_wait(tmem_empty, ((uint32_t)lt & 1u) ^ 1u, abort_flag)) break;
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                bool ok = true;
                for (int kb = 0; kb < p.kblocks; ++kb, ++it) {
                    const int s = it % kBsStages;
                    if (!bs_wait(&full[s], (uint32_t)(it / kBsStages) & 1u, abort_flag)) {
                        ok = false;
                        break;
                    }
                    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                    // Scale factors of the block's four MMAs into TMEM (in
                    // order with the MMAs this thread issues after them).
                    const uint32_t sfa = sm_u32(stage_sfa(s)), sfb = sm_u32(stage_sfb(s));
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        bs_cp_atom(tmem + kBsSfaCol + 4 * j, bs_desc_atom(sfa + j * kBsAtom));
                        bs_cp_atom(tmem + kBsSfbCol + 8 * j, bs_desc_atom(sfb + (2 * j) * kBsAtom));
                        bs_cp_atom(tmem + kBsSfbCol + 8 * j + 4, bs_desc_atom(sfb + (2 * j + 1) * kBsAtom));
                    }
                    const uint32_t wa = sm_u32(stage_w(s)), xa = sm_u32(stage_x(s));
#pragma unroll
                    for (int j = 0; j < 4; ++j)
                        bs_mma(tmem, bs_desc128(wa + 32 * j), bs_desc128(xa + 32 * j), tmem + kBsSfaCol + 4 * j,
                               tmem + kBsSfbCol + 8 * j, (kb > 0 || j > 0) ? 1u : 0u);
                    issued = true;
                    bs_commit(&empty[s]);
                }
                if (!ok) break;
                bs_commit(tmem_full);
            }
            if (*abort_flag && issued) {
                bs_commit(drain);
                bs_drain(drain, 0);
            }
        }
    } else if (warp >= 4) {
        // ---------------- epilogue: TMEM -> bf16 -> y ----------------
        const int q = warp & 3;                   // TMEM lanes 32 q .. 32 q + 31 = tile rows
        for (int lt = 0; lt < my_tiles; ++lt) {
            if (!bs_wait(tmem_full, (uint32_t)lt & 1u, abort_flag)) break;
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const int t = (int)blockIdx.x + lt * (int)gridDim.x;
            const int w_row = (t % p.w_tiles) * kBsTileW + q * 32 + lane;
            const int tok0 = (t / p.w_tiles) * kBsTileT;
#pragma unroll 1
            for (int c = 0; c < kBsTileT / 32; ++c) {
                if (tok0 + c * 32 >= p.m) break;      // uniform across the warp
                uint32_t r[32];
                bs_ld32(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(c * 32), r);
                if (w_row < p.n) {
                    uint16_t* yp = p.y + (int64_t)(tok0 + c * 32) * p.ldy + w_row;
                    const int tmax = min(32, p.m - (tok0 + c * 32));
#pragma unroll
                    for (int j = 0; j < 32; ++j)
                        if (j < tmax) yp[(int64_t)j * p.ldy] = f32_to_bf16(__uint_as_float(r[j]));
                }
            }
            asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
            __syncwarp();
            if (lane == 0) bs_arrive(tmem_empty);
        }
    }
    __syncthreads();
    if (warp == 2) {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tmem) : "memory");
    }
}

// Scale bytes [rows][lds] (UE4M3, one per 16 codes) -> atoms
// [row tiles of `tile_rows`][kblocks][4 MMAs][tile_rows / 128][512]: atom
// byte r0 * 16 + g * 4 + s = scale of row 128 h + r0 + 32 g, group
// 16 kb + 4 j + s; zero outside the matrix.
__global__ void sf_atoms_kernel(const uint8_t* __restrict__ src, int64_t lds, int rows, int ngroups,
                                int tile_rows, int kblocks, int64_t total, uint8_t* __restrict__ dst) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int s = (int)(i & 3), g = (int)((i >> 2) & 3), r0 = (int)((i >> 4) & 31);
        int64_t rest = i >> 9;                                  // atom index
        const int halves = tile_rows / 128;
        const int h = (int)(rest % halves);
        rest /= halves;
        const int j = (int)(rest & 3);
        rest >>= 2;
        const int kb = (int)(rest % kblocks);
        const int64_t tile = rest / kblocks;
        const int64_t row = tile * tile_rows + 128 * h + r0 + 32 * g;
        const int64_t grp = (int64_t)kb * 16 + 4 * j + s;
        dst[i] = (row < rows && grp < ngroups) ? src[row * lds + grp] : (uint8_t)0;
    }
}

PFN_cuTensorMapEncodeTiled_v12000 bs_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
    });
    return fn;
}

int launch_sf_atoms(const uint8_t* src, int64_t lds, int64_t rows, int64_t ngroups, int tile_rows, int kblocks,
                    uint8_t* dst, int sms, cudaStream_t s) {
    const int64_t tiles = (rows + tile_rows - 1) / tile_rows;
    const int64_t total = tiles * kblocks * 4 * (tile_rows / 128) * 512;
    const unsigned grid = (unsigned)std::min<int64_t>((total + 255) / 256, (int64_t)sms * 8);
    sf_atoms_kernel<<<grid, 256, 0, s>>>(src, lds, (int)rows, (int)ngroups, tile_rows, kblocks, total, dst);
    QMM_CUDA_TRY(cudaGetLastError());
    return QMM_OK;
}

}  // namespace

int gemm_bs_sf_bytes(int64_t n, int64_t k) {
    const int64_t kblocks = (k + kBsKB - 1) / kBsKB, tiles = (n + kBsTileW - 1) / kBsTileW;
    return (int)std::min<int64_t>(INT32_MAX, tiles * kblocks * kBsSfaBytes);
}

// The library's own stream-ordered pool per device for the per-call x
// scratch.  The device's default pool gives its memory back at every
// synchronisation (release threshold 0), so the next call could pay for
// mapping it again - milliseconds per call; this pool keeps what it has
// reserved (the largest call's scratch) until the process exits, and
// leaves the default pool, which other code may use, as it is.
static int scratch_pool(int dev, cudaMemPool_t* out) {
    static std::mutex mu;
    static cudaMemPool_t pools[64] = {};
    if (dev < 0 || dev >= 64) return set_error(QMM_ERR_BAD_ARGUMENT, "device %d is out of range", dev);
    std::lock_guard<std::mutex> lock(mu);
    if (!pools[dev]) {
        cudaMemPoolProps props = {};
        props.allocType = cudaMemAllocationTypePinned;
        props.handleTypes = cudaMemHandleTypeNone;
        props.location.type = cudaMemLocationTypeDevice;
        props.location.id = dev;
        cudaMemPool_t pool = nullptr;
        QMM_CUDA_TRY(cudaMemPoolCreate(&pool, &props));
        uint64_t keep = UINT64_MAX;
        cudaError_t e = cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &keep);
        if (e != cudaSuccess) {
            cudaMemPoolDestroy(pool);
            return cuda_error(e, "cudaMemPoolSetAttribute(release threshold)");
        }
        pools[dev] = pool;
    }
    *out = pools[dev];
    return QMM_OK;
}

int launch_gemm_blockscaled(const QmmArgs& a, const uint8_t* w_sf, cudaStream_t stream) {
    if (a.fmt != kNVFP4) return set_error(QMM_ERR_BAD_ARGUMENT, "the block-scaled GEMM takes nvfp4 weights");
    if (a.m < 1 || a.n < 1) return QMM_OK;
    if (a.m > INT32_MAX - kBsTileT || a.n > INT32_MAX || a.k > INT32_MAX)
        return set_error(QMM_ERR_BAD_SHAPE, "block-scaled GEMM: dimensions exceed 32-bit indices");
    const auto ca = reinterpret_cast<uintptr_t>(a.codes);
    if ((ca & 15) || (a.ldc & 15))
        return set_error(QMM_ERR_BAD_ARGUMENT, "block-scaled GEMM: code rows must be 16-byte aligned");
    int dev = 0;
    QMM_CUDA_TRY(cudaGetDevice(&dev));
    DeviceInfo info;
    if (int rc = device_info(dev, &info)) return rc;
    auto enc = bs_encoder();
    if (!enc || info.smem_optin < (size_t)kBsSmem)
        return set_error(QMM_ERR_CUDA, "block-scaled GEMM: TMA encoder or shared memory unavailable");
    const int64_t m = a.m, n = a.n, k = a.k, ngroups = k / 16, kblocks = (k + kBsKB - 1) / kBsKB;
    const int64_t t_tiles = (m + kBsTileT - 1) / kBsTileT, w_tiles = (n + kBsTileW - 1) / kBsTileW;
    // x quantised per call into stream-ordered scratch: codes [M, K/2] (the
    // TMA source), row-major scales, then their atoms.
    const int64_t xc_bytes = m * (k / 2), xs_bytes = m * ngroups;
    const int64_t xsf_bytes = t_tiles * kblocks * kBsSfbBytes;
    const int64_t off_s = (xc_bytes + 255) / 256 * 256, off_sf = off_s + (xs_bytes + 255) / 256 * 256;
    uint8_t* scratch = nullptr;
    cudaMemPool_t pool = nullptr;
    if (int rc0 = scratch_pool(dev, &pool)) return rc0;
    QMM_CUDA_TRY(cudaMallocFromPoolAsync(reinterpret_cast<void**>(&scratch), (size_t)(off_sf + xsf_bytes), pool, stream));
    uint8_t* xcodes = scratch;
    uint8_t* xscales = scratch + off_s;
    uint8_t* xsf = scratch + off_sf;
    int rc = launch_quantize(kNVFP4, a.x, true, a.ldx, m, k, xcodes, xscales, stream);
    if (rc == QMM_OK) rc = launch_sf_atoms(xscales, ngroups, m, ngroups, kBsTileT, (int)kblocks, xsf, info.sms, stream);
    CUtensorMap wmap, xmap;
    if (rc == QMM_OK) {
        const cuuint64_t gdim[2] = {(cuuint64_t)(k / 2), (cuuint64_t)n};
        const cuuint64_t gstride[1] = {(cuuint64_t)a.ldc};
        const cuuint32_t box[2] = {128, (cuuint32_t)kBsTileW};
        const cuuint32_t es[2] = {1, 1};
        if (enc(&wmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t*>(a.codes), gdim, gstride, box, es,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            rc = set_error(QMM_ERR_CUDA, "cuTensorMapEncodeTiled(W codes) failed");
    }
    if (rc == QMM_OK) {
        const cuuint64_t gdim[2] = {(cuuint64_t)(k / 2), (cuuint64_t)m};
        const cuuint64_t gstride[1] = {(cuuint64_t)(k / 2)};
        const cuuint32_t box[2] = {128, (cuuint32_t)kBsTileT};
        const cuuint32_t es[2] = {1, 1};
        if ((k / 2) % 16)
            rc = set_error(QMM_ERR_BAD_SHAPE, "block-scaled GEMM: K must be a multiple of 32");
        else if (enc(&xmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, xcodes, gdim, gstride, box, es,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            rc = set_error(QMM_ERR_CUDA, "cuTensorMapEncodeTiled(x codes) failed");
    }
    if (rc == QMM_OK) {
        static bool configured[64] = {false};
        if (dev < 64 && !configured[dev]) {
            cudaError_t e = cudaFuncSetAttribute(qmm_gemm_bs_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kBsSmem);
            if (e != cudaSuccess) rc = cuda_error(e, "cudaFuncSetAttribute(gemm_bs)");
            else configured[dev] = true;
        }
    }
    if (rc == QMM_OK) {
        BsParams p;
        p.w_sf = w_sf;
        p.x_sf = xsf;
        p.y = a.y;
        p.ldy = a.ldy;
        p.m = (int)m;
        p.n = (int)n;
        p.kblocks = (int)kblocks;
        p.w_tiles = (int)w_tiles;
        const int64_t tiles = w_tiles * t_tiles;
        p.num_tiles = (int)std::min<int64_t>(tiles, INT32_MAX);
        const int grid = (int)std::min<int64_t>(tiles, info.sms);
        qmm_gemm_bs_kernel<<<grid, kBsThreads, kBsSmem, stream>>>(wmap, xmap, p);
        cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) rc = cuda_error(e, "qmm_gemm_bs_kernel");
    }
    cudaError_t e = cudaFreeAsync(scratch, stream);
    if (rc == QMM_OK && e != cudaSuccess) rc = cuda_error(e, "cudaFreeAsync(block-scaled scratch)");
    return rc;
}

int make_gemm_bs_weight_sf(const QmmArgs& a, uint8_t** out, cudaStream_t stream) {
    int dev = 0;
    QMM_CUDA_TRY(cudaGetDevice(&dev));
    DeviceInfo info;
    if (int rc = device_info(dev, &info)) return rc;
    const int64_t kblocks = (a.k + kBsKB - 1) / kBsKB, tiles = (a.n + kBsTileW - 1) / kBsTileW;
    const int64_t bytes = tiles * kblocks * kBsSfaBytes;
    uint8_t* sf = nullptr;
    QMM_CUDA_TRY(cudaMalloc(&sf, (size_t)bytes));
    if (int rc = launch_sf_atoms(a.scales, a.lds, a.n, a.k / 16, kBsTileW, (int)kblocks, sf, info.sms, stream)) {
        cudaFree(sf);
        return rc;
    }
    *out = sf;
    return QMM_OK;
}

cudaError_t gemm_bs_take_error(unsigned int* v, cudaStream_t s) {
    unsigned int zero = 0;
    cudaError_t e = cudaMemcpyFromSymbolAsync(v, g_gemm_bs_error, sizeof(*v), 0, cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e == cudaSuccess && *v) {
        e = cudaMemcpyToSymbolAsync(g_gemm_bs_error, &zero, sizeof(zero), 0, cudaMemcpyHostToDevice, s);
        if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    }
    return e;
}

}  // namespace qmm
