// gemm.cu - prefill quantized GEMM on the sm_100a tensor cores (tcgen05).
//
// y[M, N] = x[M, K] . dequant(W)[N, K]^T for M > 8 (prefill chunks, the
// reference's 2048-token chunks of src/engine.zig:19, :367-382, and whole
// 32k prompts), W in mxfp8 or nvfp4, x / y bf16, fp32 accumulation.
//
// Precision: W is dequantised exactly into bf16 (an E4M3 or E2M1 value
// times its scale has at most 4 + 0 or 2 + 4 significant bits) and x stays
// bf16, so every product is exact and the kind::f16 MMA accumulates in
// fp32 - the same arithmetic as the fp64 oracle up to fp32 summation.
// (Quantising x to FP8/FP4 for the block-scaled MMA kinds would add
// 2-10% error per element, far outside the 2e-3 tolerance.)
//
// The expensive step is the dequantisation (the fp8/fp4 -> f16 conversions
// run at a quarter of the fp32 rate on sm_100), so the tile is shaped to
// dequantise each code once per 512 tokens, the k-blocks are 64 wide (16
// codes per dequant thread per hand-over), and x - re-read from L2 by every
// weight tile - is split across a CTA pair.  Two CTAs of a cluster (one per
// SM, persistent) compute y^T tiles of 256 weight rows x 512 tokens with
// tcgen05.mma.cta_group::2: per 64-wide k-block, each CTA dequantises its
// own 128 weight rows (its half of the M = 256 A operand) and loads its
// 128-token half of each of the two 256-token B operands, so a CTA moves
// 32 KB of x per k-block instead of 64 KB.  The pair's leader (cluster rank
// 0) issues two MMAs of 256 x 256 x 16 per k16 step; each CTA's TMEM holds
// its 128 rows x 512 tokens in fp32 (all 512 columns).  Warp roles (24
// warps, both CTAs):
//   warp 0      TMA producer: this CTA's x halves [2 x 128 tokens x 64 k],
//               128B swizzle, counted on the leader's full_x barrier
//   warp 1      MMA issuer (leader only): tcgen05.mma.cta_group::2 kind::f16
//   warp 2      TMEM allocator (512 columns in each CTA, cta_group::2)
//   warp 3      TMA producer: W code tiles [128 rows x 64 k] (own ring)
//   warps 4-7   epilogue: tcgen05.ld -> bf16 -> y (coalesced 64-byte rows)
//   warps 8-23  dequant: 16 codes per thread per k-block from the code ring,
//               scale bytes prefetched from global memory, decoded with
//               cvt.{e4m3x2,e2m1x2}, written as bf16 into the A tile in the
//               UMMA K-major 128B-swizzle layout
// Pipelines (mbarriers): kStages stages of {x halves, W tile}.  On the
// leader: full_x (both CTAs' TMA bytes), full_w (both CTAs' 16 dequant
// warps), tmem_empty (both CTAs' 4 epilogue warps).  In each CTA: empty and
// tmem_full (the leader's MMA commits, one per CTA), and the code ring's
// cfull (TMA bytes) / cempty (16 dequant warps).  TMA / dequant keep
// prefetching the next tile while the epilogue drains the accumulator.
// Every wait is bounded by %globaltimer: a wait that gives up raises the
// CTA's abort flag and the device error word, every role then drains its
// in-flight TMA / MMA work, and the pair meets at a cluster barrier before
// TMEM is freed (the host reads the word with qmm_device_status).  No load
// uses cluster multicast.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <cstdint>
#include <mutex>

#include "formats.cuh"
#include "internal.h"

namespace qmm {

// Bit 0: a bounded wait in the GEMM timed out (read by qmm_device_status).
__device__ unsigned int g_device_error = 0;

namespace {

constexpr int kStages = 4;
constexpr int kBK = 64;                     // k per stage (128 bytes of bf16: one 128B swizzle row)
constexpr int kTileW = 128;                 // weight rows per CTA (half the pair's MMA M)
constexpr int kPairW = 2 * kTileW;          // weight rows per pair tile (MMA M)
constexpr int kHalfT = 256;                 // tokens per MMA (MMA N)
constexpr int kTileT = 2 * kHalfT;          // tokens per tile
constexpr int kCtaT = kHalfT / 2;           // tokens of one MMA's B operand held by each CTA
constexpr int kThreads = 768;
constexpr int kXHalfBytes = kCtaT * kBK * 2;    // 16 KB
constexpr int kXBytes = 2 * kXHalfBytes;        // 32 KB per CTA per stage
constexpr int kWBytes = kTileW * kBK * 2;       // 16 KB
constexpr int kCodeRingBytes = 16384;
// SwiGLU epilogue: a gate-row warp and its up-row warp swap half of each
// 32 x 32 fp32 accumulator chunk (rows padded to 17 words), both ways.
constexpr int kXchBytes = 2 * 2 * 32 * 17 * 4;
constexpr int kSmemBytes = kStages * (kXBytes + kWBytes) + kCodeRingBytes + 1024 /*align*/ +
                           1024 /*barriers + flags*/ + kXchBytes;
constexpr int kDequantWarps = 16;
constexpr int kEpiWarps = 4;
constexpr uint64_t kTimeoutNs = 2000000000ull;  // 2 s per wait

struct GemmParams {
    const uint8_t* __restrict__ codes;
    const uint8_t* __restrict__ scales;
    uint16_t* __restrict__ y;
    int64_t ldc, lds, ldy;
    int m, n, k;
    int kblocks, w_tiles, num_tiles;
    // > 0: W rows are gate / up interleaved in 64-row blocks and y receives
    // silu(g) * u, tile rows 0-63 -> y columns [64 tile, 64 tile + 64).
    int swiglu_n;
};

// ---- PTX wrappers --------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ uint64_t globaltimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}
__device__ __forceinline__ void mbar_init(uint64_t* b, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(b)), "r"(count));
}
__device__ __forceinline__ void mbar_arrive(uint64_t* b) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(b)) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* b, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(b)), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* b, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok) : "r"(smem_u32(b)), "r"(parity) : "memory");
    return ok != 0;
}
// Bounded wait for the phase with the given parity.  False = gave up (the
// abort flag is raised, by this thread if it timed out).
__device__ __forceinline__ bool mbar_wait(uint64_t* b, uint32_t parity, volatile int* abort_flag) {
    if (mbar_try_wait(b, parity)) return true;
    const uint64_t t0 = globaltimer();
    for (uint32_t i = 1;; ++i) {
        if (mbar_try_wait(b, parity)) return true;
        if ((i & 15) == 0) {
            if (*abort_flag) return false;
            if (globaltimer() - t0 > kTimeoutNs) {
                *abort_flag = 1;
                atomicOr(&g_device_error, 1u);
                return false;
            }
        }
    }
}
// Bounded wait used on drain paths (no abort check; gives up after the limit).
__device__ __forceinline__ void mbar_drain(uint64_t* b, uint32_t parity) {
    const uint64_t t0 = globaltimer();
    while (!mbar_try_wait(b, parity) && globaltimer() - t0 < kTimeoutNs) {
    }
}
__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int x0, int y0) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3}], [%4];"
        ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(x0), "r"(y0), "r"(smem_u32(bar))
        : "memory");
}
// ---- CTA pair (cluster of 2) ------------------------------------------------------
__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ uint32_t cluster_id() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
    return r;
}
__device__ __forceinline__ uint32_t cluster_count() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%nclusterid.x;" : "=r"(r));
    return r;
}
// Shared::cluster address of this CTA's object `p` as it lies in CTA `rank`.
__device__ __forceinline__ uint32_t mapa(const void* p, uint32_t rank) {
    uint32_t a;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(a) : "r"(smem_u32(p)), "r"(rank));
    return a;
}
// Arrive on a barrier of either CTA of the pair (cluster address).
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t caddr) {
    asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(caddr) : "memory");
}
__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// x half into this CTA's shared memory, the bytes counted on the leader's
// barrier (cluster address `lead_bar`).  No multicast.
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* map, uint32_t lead_bar, int x0, int y0) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3}], [%4];"
        ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(x0), "r"(y0), "r"(lead_bar)
        : "memory");
}
// One MMA of the pair: D (each CTA's TMEM, its 128 rows) += A (each CTA's
// 128 rows) x B (each CTA's half of the N columns).  Issued by the leader.
__device__ __forceinline__ void mma_bf16_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                              uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(d_tmem), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate) : "memory");
}
// Arrive on barrier `caddr` (cluster address, either CTA) when every pair
// MMA this thread issued so far has completed.
__device__ __forceinline__ void mma_commit_pair(uint32_t caddr) {
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                 ::"r"(caddr) : "memory");
}
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
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

// UMMA shared-memory descriptor: K-major, 128-byte swizzle (8-row atoms of
// 1024 bytes, SBO), version 1 (sm_100).  The 16-byte chunk c of row r of a
// tile sits at r * 128 + ((c ^ (r & 7)) * 16) (tile base 1024-aligned); a
// k16 step advances the start address by 32 bytes within the row.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr >> 4) & 0x3FFF);
    d |= (uint64_t)1 << 16;                    // LBO (unused for swizzled K-major)
    d |= (uint64_t)(1024 >> 4) << 32;          // SBO: 8 rows x 128 bytes
    d |= (uint64_t)1 << 46;                    // descriptor version
    d |= (uint64_t)2 << 61;                    // SWIZZLE_128B
    return d;
}

// kind::f16 instruction descriptor: bf16 A/B, fp32 D, K-major A and B,
// M = 256 (the pair), N = 256.
constexpr uint32_t kIdesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(kHalfT >> 3) << 17) |
                            ((uint32_t)(kPairW >> 4) << 24);

// ---- W code tiles --------------------------------------------------------------
// [128 rows x 64 k] per k-block, by TMA into their own ring: 64 bytes per row
// (mxfp8, 64B swizzle) or 32 bytes (nvfp4, 32B swizzle).
template <int FMT> struct CodeTile;
template <> struct CodeTile<kMXFP8> {
    static constexpr int kRowBytes = 64;
    static constexpr CUtensorMapSwizzle kSwizzle = CU_TENSOR_MAP_SWIZZLE_64B;
};
template <> struct CodeTile<kNVFP4> {
    static constexpr int kRowBytes = 32;
    static constexpr CUtensorMapSwizzle kSwizzle = CU_TENSOR_MAP_SWIZZLE_32B;
};

// Scale byte of a thread's 16 codes (k [kk, kk + 16) of one row: one nvfp4
// group, half an mxfp8 group), prefetched
// ahead from global memory in the checkpoint layout; 0 outside the matrix.
template <int FMT>
__device__ __forceinline__ uint32_t load_scale(const GemmParams& p, int row, int kk) {
    if (row >= p.n || kk >= p.k) return 0;
    return __ldg(p.scales + (int64_t)row * p.lds + kk / (FMT == kMXFP8 ? 32 : 16));
}

// Row r's 16 codes for k quarter q (codes [16q, 16q + 16) of the k-block):
// mxfp8 one 16-byte chunk of a 64-byte row (64B swizzle: chunk ^= (r >> 1) & 3),
// nvfp4 8 bytes of a 32-byte row (32B swizzle: chunk ^= (r >> 2) & 1).
template <int FMT>
__device__ __forceinline__ uint4 read_codes(const uint8_t* tile, int r, int q) {
    if constexpr (FMT == kMXFP8) {
        return *reinterpret_cast<const uint4*>(tile + r * 64 + ((q ^ ((r >> 1) & 3)) << 4));
    } else {
        const uint2 v = *reinterpret_cast<const uint2*>(tile + r * 32 + (((q >> 1) ^ ((r >> 2) & 1)) << 4) + (q & 1) * 8);
        return make_uint4(v.x, v.y, 0u, 0u);
    }
}

__device__ __forceinline__ uint32_t bf16x2_mul(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}

// 8 codes -> 8 bf16 (one 16-byte chunk), exact.
template <int FMT>
__device__ __forceinline__ uint4 dequant8(uint2 c, uint32_t sbyte) {
    if constexpr (FMT == kMXFP8) {
        const float s = ue8m0_to_f32(sbyte);
        uint32_t o[4];
        const uint32_t w[2] = {c.x, c.y};
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            uint32_t h[2];
            e4m3x4_to_f16x2(w[i], h);
            const float2 a = f16x2_to_float2(h[0]), b = f16x2_to_float2(h[1]);
            o[2 * i] = f32x2_to_bf16x2(a.x * s, a.y * s);
            o[2 * i + 1] = f32x2_to_bf16x2(b.x * s, b.y * s);
        }
        return make_uint4(o[0], o[1], o[2], o[3]);
    } else {
        // An E2M1 value v decodes exactly to f16; moving its exponent and
        // mantissa fields down by 3 bits gives the bf16 bit pattern of
        // v * 2^-112 (the f16 exponent field read with bf16's bias; zero
        // stays zero, E2M1 has no Inf/NaN).  One bf16 multiply by
        // s * 2^112 then yields v * s exactly (<= 6 significant bits,
        // magnitudes 2^-10 .. 2688), NaN scales included.
        const uint16_t sb = f32_to_bf16(ue4m3_to_f32(sbyte) * 0x1p112f);
        const uint32_t s2 = (uint32_t)sb * 0x10001u;
        uint32_t h[4], o[4];
        e2m1x8_to_f16x2(c.x, h);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint32_t t = ((h[i] & 0x7FFF7FFFu) >> 3) | (h[i] & 0x80008000u);
            o[i] = bf16x2_mul(t, s2);
        }
        return make_uint4(o[0], o[1], o[2], o[3]);
    }
}

template <int FMT>
__global__ void __launch_bounds__(kThreads, 1) qmm_gemm_kernel(const __grid_constant__ CUtensorMap xmap,
                                                                const __grid_constant__ CUtensorMap cmap,
                                                                GemmParams p) {
    constexpr int kCBytes = kTileW * CodeTile<FMT>::kRowBytes;   // one code tile
    constexpr int kCStages = kCodeRingBytes / kCBytes;
    extern __shared__ uint8_t smem_raw[];
    // Both CTAs of the pair carve the same layout from the same aligned base,
    // so one shared-memory offset names a tile in either CTA (the pair MMA
    // reads A and B at the leader's descriptor offsets in both).
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* smem_x = smem;                                   // kStages x 16 KB
    uint8_t* smem_w = smem + kStages * kXBytes;               // kStages x 8 KB
    uint8_t* smem_c = smem_w + kStages * kWBytes;             // kCStages code tiles (32 KB)
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem_c + kCodeRingBytes);
    uint64_t* full_x = bars;                                  // leader: both CTAs' x bytes
    uint64_t* full_w = bars + kStages;                        // leader: both CTAs' dequant warps
    uint64_t* empty = bars + 2 * kStages;                     // each CTA: MMA commit
    uint64_t* tmem_full = bars + 3 * kStages;                 // each CTA: MMA commit
    uint64_t* tmem_empty = tmem_full + 1;                     // leader: both CTAs' epilogue warps
    uint64_t* drain = tmem_empty + 1;
    uint64_t* cfull = drain + 1;                              // kCStages
    uint64_t* cempty = cfull + kCStages;                      // kCStages
    volatile int* abort_flag = reinterpret_cast<volatile int*>(cempty + kCStages);
    uint32_t* tmem_base_slot = reinterpret_cast<uint32_t*>(cempty + kCStages) + 1;
    uint64_t* xch_full = cempty + kCStages + 1;               // SwiGLU hand-over: up chunk written
    uint64_t* xch_empty = xch_full + 1;                       // ... and read
    float* smem_xch = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(bars) + 1024);
    static_assert((3 * kStages + 3 + 2 * 16 + 1 + 2) * 8 <= 1024, "barrier area");
    static_assert(kStages * (kXBytes + kWBytes) + kCodeRingBytes + 1024 + kXchBytes + 1024 <= kSmemBytes,
                  "shared-memory carve-up exceeds the allocation");
    static_assert(kCStages * kCBytes == kCodeRingBytes && kCStages <= 16, "code ring size");

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_rank();                     // 0: leader (issues the MMAs)
    const int pair = (int)cluster_id(), npairs = (int)cluster_count();

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&full_x[s], 1);
            mbar_init(&full_w[s], 2 * kDequantWarps);
            mbar_init(&empty[s], 1);
        }
        for (int s = 0; s < kCStages; ++s) {
            mbar_init(&cfull[s], 1);
            mbar_init(&cempty[s], kDequantWarps);
        }
        mbar_init(tmem_full, 1);
        mbar_init(tmem_empty, 2 * kEpiWarps);
        mbar_init(drain, 1);
        mbar_init(xch_full, kEpiWarps);
        mbar_init(xch_empty, kEpiWarps);
        *abort_flag = 0;
        fence_barrier_init();
    }
    if (warp == 2) {
        asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], 512;"
                     ::"r"(smem_u32(tmem_base_slot)) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
        tc_fence_before();
    }
    // Both CTAs' barriers are initialised and their TMEM allocated before
    // either CTA signals the other.
    __syncthreads();
    cluster_sync();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_base_slot;

    const int my_tiles = p.num_tiles > pair ? (p.num_tiles - 1 - pair) / npairs + 1 : 0;
    const int total_kb = my_tiles * p.kblocks;
    // Weight rows of this CTA's half of tile t; first token of tile t.
    auto w_row0 = [&](int t) { return (t % p.w_tiles) * kPairW + (int)rank * kTileW; };
    auto tok_0 = [&](int t) { return (t / p.w_tiles) * kTileT; };

    if (warp == 0) {
        // ---------------- TMA producer (this CTA's x halves) ----------------
        if (lane == 0) {
            int last = -1;
            for (int it = 0; it < total_kb; ++it) {
                const int s = it % kStages;
                const uint32_t ph = (uint32_t)(it / kStages) & 1u;
                if (!mbar_wait(&empty[s], ph ^ 1u, abort_flag)) break;
                const int t = pair + (it / p.kblocks) * npairs;
                const int kb = it % p.kblocks;
                const int tok0 = tok_0(t) + (int)rank * kCtaT;
                if (rank == 0) mbar_expect_tx(&full_x[s], 2 * kXBytes);   // both CTAs' bytes
                const uint32_t lead = mapa(&full_x[s], 0);
                tma_load_2d_pair(smem_x + s * kXBytes, &xmap, lead, kb * kBK, tok0);
                tma_load_2d_pair(smem_x + s * kXBytes + kXHalfBytes, &xmap, lead, kb * kBK, tok0 + kHalfT);
                last = it;
            }
            if (!*abort_flag) {
                // Producer tail: the MMA's last commits to every stage's empty
                // barrier must land before the CTA exits.
                for (int it = total_kb; it < total_kb + kStages; ++it) {
                    if (it < kStages) continue;          // stage never used
                    if (!mbar_wait(&empty[it % kStages], ((uint32_t)(it / kStages) & 1u) ^ 1u, abort_flag)) break;
                }
            }
            if (*abort_flag && last >= 0) {
                // Let every TMA still in flight land before the CTA exits.
                // The leader waits for its full_x phases (bounded: a phase the
                // other CTA never filled gives up).  The other CTA's copies
                // signal the leader's barrier, so it waits a fixed 100 us - an
                // 8 KB copy lands in microseconds.
                if (rank == 0) {
                    for (int it = max(0, last - kStages + 1); it <= last; ++it)
                        mbar_drain(&full_x[it % kStages], (uint32_t)(it / kStages) & 1u);
                } else {
                    const uint64_t t0 = globaltimer();
                    while (globaltimer() - t0 < 100000ull) {
                    }
                }
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer (leader) ----------------
        if (lane == 0 && rank == 0) {
            int it = 0;
            bool issued_any = false;
            for (int lt = 0; lt < my_tiles && !*abort_flag; ++lt) {
                if (!mbar_wait(tmem_empty, ((uint32_t)lt & 1u) ^ 1u, abort_flag)) break;
                tc_fence_after();
                bool ok = true;
                for (int kb = 0; kb < p.kblocks; ++kb, ++it) {
                    const int s = it % kStages;
                    const uint32_t ph = (uint32_t)(it / kStages) & 1u;
                    if (!mbar_wait(&full_x[s], ph, abort_flag) || !mbar_wait(&full_w[s], ph, abort_flag)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t xa = smem_u32(smem_x + s * kXBytes);
                    const uint32_t wa = smem_u32(smem_w + s * kWBytes);
#pragma unroll
                    for (int k16 = 0; k16 < kBK / 16; ++k16) {
                        const uint32_t acc = (kb > 0 || k16 > 0) ? 1u : 0u;
                        const uint64_t ad = sw128_desc(wa + k16 * 32);
                        mma_bf16_pair(tmem_base, ad, sw128_desc(xa + k16 * 32), kIdesc, acc);
                        mma_bf16_pair(tmem_base + kHalfT, ad, sw128_desc(xa + kXHalfBytes + k16 * 32), kIdesc, acc);
                    }
                    issued_any = true;
                    mma_commit_pair(mapa(&empty[s], 0));
                    mma_commit_pair(mapa(&empty[s], 1));
                }
                if (!ok) break;
                mma_commit_pair(mapa(tmem_full, 0));
                mma_commit_pair(mapa(tmem_full, 1));
            }
            if (*abort_flag && issued_any) {
                // Wait (bounded) for every MMA issued so far before TMEM is freed.
                mma_commit_pair(mapa(drain, 0));
                mbar_drain(drain, 0);
            }
        }
    } else if (warp == 3) {
        // ---------------- TMA producer (W code tiles) ----------------
        if (lane == 0) {
            int last = -1;
            for (int it = 0; it < total_kb; ++it) {
                const int s = it % kCStages;
                const uint32_t ph = (uint32_t)(it / kCStages) & 1u;
                if (!mbar_wait(&cempty[s], ph ^ 1u, abort_flag)) break;
                const int t = pair + (it / p.kblocks) * npairs;
                const int kb = it % p.kblocks;
                mbar_expect_tx(&cfull[s], kCBytes);
                tma_load_2d(smem_c + s * kCBytes, &cmap, &cfull[s], kb * CodeTile<FMT>::kRowBytes, w_row0(t));
                last = it;
            }
            // Every fill must land before the CTA exits (the dequant warps
            // consume them all on the normal path; bounded on abort).
            for (int it = max(0, last - kCStages + 1); it <= last; ++it)
                mbar_drain(&cfull[it % kCStages], (uint32_t)(it / kCStages) & 1u);
        }
    } else if (warp >= 4 && warp < 8) {
        // ---------------- epilogue: TMEM -> bf16 -> y ----------------
        const int q = warp & 3;                     // TMEM lanes 32q .. 32q + 31
        // SwiGLU: gate-row warp q (rows 0-63) and up-row warp q + 2 (rows
        // 64-127) swap halves of each 32-token chunk through shared memory
        // - the up warp sends tokens 0-15, the gate warp tokens 16-31 - and
        // each computes silu(g) * u for its 16 tokens.  Counted hand-overs
        // on two mbarriers, every wait bounded.
        const bool up_warp = q >= 2;
        float* x_out = smem_xch + ((q & 1) * 2 + (up_warp ? 0 : 1)) * 32 * 17;
        const float* x_in = smem_xch + ((q & 1) * 2 + (up_warp ? 1 : 0)) * 32 * 17;
        const uint32_t lead_tmem_empty = mapa(tmem_empty, 0);
        uint32_t xc = 0;
        bool live = true;
        for (int lt = 0; lt < my_tiles && live; ++lt) {
            if (!mbar_wait(tmem_full, (uint32_t)lt & 1u, abort_flag)) break;
            tc_fence_after();
            const int t = pair + lt * npairs;
            const int w_row = w_row0(t) + q * 32 + lane;
            const int tok0 = tok_0(t);
#pragma unroll 1
            for (int c = 0; c < kTileT / 32; ++c) {
                if (tok0 + c * 32 >= p.m) break;        // uniform across the warp
                uint32_t r[32];
                tmem_ld32(tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(c * 32), r);
                if (p.swiglu_n > 0) {
                    const int tmax = min(32, p.m - (tok0 + c * 32));
                    const int j0 = up_warp ? 16 : 0;       // this warp's tokens j0 .. j0 + 15
                    if (!mbar_wait(xch_empty, (xc & 1u) ^ 1u, abort_flag)) { live = false; break; }
#pragma unroll
                    for (int j = 0; j < 16; ++j) x_out[lane * 17 + j] = __uint_as_float(up_warp ? r[j] : r[16 + j]);
                    __syncwarp();
                    if (lane == 0) mbar_arrive(xch_full);
                    if (!mbar_wait(xch_full, xc & 1u, abort_flag)) { live = false; break; }
                    // This CTA's 128 rows are one interleaved gate / up block.
                    const int64_t hc = (int64_t)(w_row0(t) / kTileW) * 64 + (q & 1) * 32 + lane;
                    if (hc < p.swiglu_n) {
                        uint16_t* hp = p.y + (int64_t)(tok0 + c * 32) * p.ldy + hc;
#pragma unroll
                        for (int j = 0; j < 16; j += 2) {
                            const float m0 = __uint_as_float(up_warp ? r[16 + j] : r[j]);
                            const float m1 = __uint_as_float(up_warp ? r[17 + j] : r[j + 1]);
                            const float o0 = x_in[lane * 17 + j], o1 = x_in[lane * 17 + j + 1];
                            const uint32_t hv = up_warp ? swiglu_bf16x2(o0, o1, m0, m1) : swiglu_bf16x2(m0, m1, o0, o1);
                            if (j0 + j < tmax) hp[(int64_t)(j0 + j) * p.ldy] = (uint16_t)(hv & 0xFFFFu);
                            if (j0 + j + 1 < tmax) hp[(int64_t)(j0 + j + 1) * p.ldy] = (uint16_t)(hv >> 16);
                        }
                    }
                    __syncwarp();
                    if (lane == 0) mbar_arrive(xch_empty);
                    ++xc;
                    continue;
                }
                if (w_row < p.n) {
                    uint16_t* yp = p.y + (int64_t)(tok0 + c * 32) * p.ldy + w_row;
                    const int tmax = min(32, p.m - (tok0 + c * 32));
#pragma unroll
                    for (int j = 0; j < 32; ++j)
                        if (j < tmax) yp[(int64_t)j * p.ldy] = f32_to_bf16(__uint_as_float(r[j]));
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(lead_tmem_empty);
        }
    } else if (warp >= 8) {
        // ---------------- dequant: codes -> bf16 A tiles ----------------
        // A warp covers 8 rows x 4 k-quarters: the four lanes of a row share
        // its scale byte (one sector per row), and the warp's code reads and
        // W-tile writes are contiguous 128 / 256 / 512-byte runs.
        const int r = (warp - 8) * 8 + (lane >> 2); // row within the tile
        const int qd = lane & 3;                    // k quarter of the block: codes [16 qd, 16 qd + 16)
        auto coords = [&](int it, int* row, int* kk) {
            const int t = pair + (it / p.kblocks) * npairs;
            *row = w_row0(t) + r;
            *kk = (it % p.kblocks) * kBK + 16 * qd;
        };
        const uint32_t lead_full_w0 = mapa(&full_w[0], 0);
        // Scale bytes are prefetched four k-blocks ahead.
        uint32_t sc[4];
        int row, kk;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            sc[i] = 0;
            if (i < total_kb) {
                coords(i, &row, &kk);
                sc[i] = load_scale<FMT>(p, row, kk);
            }
        }
        // This thread's two 16-byte bf16 chunks of a W tile row (128B swizzle).
        const uint32_t w_off0 = (uint32_t)(r * 128 + (((2 * qd) ^ (r & 7)) << 4));
        const uint32_t w_off1 = (uint32_t)(r * 128 + (((2 * qd + 1) ^ (r & 7)) << 4));
        for (int it = 0; it < total_kb; ++it) {
            const uint32_t cur = sc[0];
            sc[0] = sc[1];
            sc[1] = sc[2];
            sc[2] = sc[3];
            sc[3] = 0;
            if (it + 4 < total_kb) {
                coords(it + 4, &row, &kk);
                sc[3] = load_scale<FMT>(p, row, kk);
            }
            const int s = it % kStages;
            const uint32_t ph = (uint32_t)(it / kStages) & 1u;
            const int cs = it % kCStages;
            if (!mbar_wait(&cfull[cs], (uint32_t)(it / kCStages) & 1u, abort_flag)) break;
            const uint4 codes = read_codes<FMT>(smem_c + cs * kCBytes, r, qd);
            __syncwarp();
            if (lane == 0) mbar_arrive(&cempty[cs]);
            // Codes outside the matrix are zero (TMA fill) and their scale
            // byte reads as 0, so the chunk is exactly zero.
            const uint4 o0 = FMT == kMXFP8 ? dequant8<FMT>(make_uint2(codes.x, codes.y), cur)
                                           : dequant8<FMT>(make_uint2(codes.x, 0u), cur);
            const uint4 o1 = FMT == kMXFP8 ? dequant8<FMT>(make_uint2(codes.z, codes.w), cur)
                                           : dequant8<FMT>(make_uint2(codes.y, 0u), cur);
            if (!mbar_wait(&empty[s], ph ^ 1u, abort_flag)) break;
            *reinterpret_cast<uint4*>(smem_w + s * kWBytes + w_off0) = o0;
            *reinterpret_cast<uint4*>(smem_w + s * kWBytes + w_off1) = o1;
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(lead_full_w0 + (uint32_t)(s * sizeof(uint64_t)));
        }
    }

    // The pair meets before TMEM is freed: the leader's MMAs write the other
    // CTA's TMEM and read its shared memory, and the other CTA's arrives and
    // copies target the leader's barriers.
    __syncthreads();
    cluster_sync();
    if (warp == 2) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, 512;" ::"r"(tmem_base) : "memory");
    }
}

// ---- host side --------------------------------------------------------------------

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
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

template <int FMT>
int launch_fmt(const QmmArgs& a, const GemmParams& p, const CUtensorMap& map, int pairs, cudaStream_t stream) {
    // Code tiles: u8 [N rows, K*bits/8 bytes] with row stride ldc, box
    // [128 rows x 64 k], swizzled to match read_codes().
    CUtensorMap cmap;
    const cuuint64_t cdim[2] = {(cuuint64_t)(a.k * (FMT == kMXFP8 ? 8 : 4) / 8), (cuuint64_t)a.n};
    const cuuint64_t cstride[1] = {(cuuint64_t)a.ldc};
    const cuuint32_t cbox[2] = {(cuuint32_t)CodeTile<FMT>::kRowBytes, (cuuint32_t)kTileW};
    const cuuint32_t ces[2] = {1, 1};
    CUresult cr = encode_fn()(&cmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t*>(a.codes), cdim, cstride,
                              cbox, ces, CU_TENSOR_MAP_INTERLEAVE_NONE, CodeTile<FMT>::kSwizzle,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (cr != CUDA_SUCCESS) return set_error(QMM_ERR_CUDA, "cuTensorMapEncodeTiled(codes) failed (%d)", (int)cr);
    static bool configured[64] = {false};
    int dev = 0;
    QMM_CUDA_TRY(cudaGetDevice(&dev));
    if (dev < 64 && !configured[dev]) {
        QMM_CUDA_TRY(cudaFuncSetAttribute(qmm_gemm_kernel<FMT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          kSmemBytes));
        configured[dev] = true;
    }
    // Pairs of CTAs (clusters of 2), at most as many pairs as fit on the
    // device at once (a GPC with an odd number of free SMs leaves one idle).
    static int max_pairs[64] = {0};
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = kSmemBytes;
    cfg.stream = stream;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (dev < 64 && max_pairs[dev] == 0) {
        cfg.gridDim = dim3((unsigned)(2 * pairs));
        int n = 0;
        QMM_CUDA_TRY(cudaOccupancyMaxActiveClusters(&n, qmm_gemm_kernel<FMT>, &cfg));
        if (n < 1) return set_error(QMM_ERR_CUDA, "no CTA pair of the prefill GEMM fits on the device");
        max_pairs[dev] = n;
    }
    const int npairs = dev < 64 ? std::min(pairs, max_pairs[dev]) : 1;
    cfg.gridDim = dim3((unsigned)(2 * npairs));
    QMM_CUDA_TRY(cudaLaunchKernelEx(&cfg, qmm_gemm_kernel<FMT>, map, cmap, p));
    return QMM_OK;
}

}  // namespace

int launch_gemm(const QmmArgs& a, cudaStream_t stream, bool* handled) {
    *handled = false;
    // Envelope: 16-byte aligned x rows and code rows (TMA), 32-bit indices.
    const auto x_addr = reinterpret_cast<uintptr_t>(a.x);
    const auto c_addr = reinterpret_cast<uintptr_t>(a.codes);
    if ((x_addr & 15) || ((a.ldx * 2) & 15) || (c_addr & 15) || (a.ldc & 15)) return QMM_OK;
    if (a.m > INT32_MAX - kTileT || a.n > INT32_MAX || a.k > INT32_MAX || a.m < 1) return QMM_OK;
    auto encode = encode_fn();
    if (!encode) return set_error(QMM_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
    int dev = 0;
    QMM_CUDA_TRY(cudaGetDevice(&dev));
    DeviceInfo info;
    if (int rc = device_info(dev, &info)) return rc;
    if (info.smem_optin < (size_t)kSmemBytes) return QMM_OK;

    // x tiles: bf16 [M rows, K] with row stride ldx, box [128 rows x 64 k], 128B swizzle.
    CUtensorMap map;
    const cuuint64_t gdim[2] = {(cuuint64_t)a.k, (cuuint64_t)a.m};
    const cuuint64_t gstride[1] = {(cuuint64_t)(a.ldx * 2)};
    const cuuint32_t box[2] = {(cuuint32_t)kBK, (cuuint32_t)kCtaT};
    const cuuint32_t estride[2] = {1, 1};
    CUresult cr = encode(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<uint16_t*>(a.x), gdim, gstride, box,
                         estride, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (cr != CUDA_SUCCESS) return set_error(QMM_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)cr);

    GemmParams p;
    p.codes = a.codes; p.scales = a.scales; p.y = a.y;
    p.ldc = a.ldc; p.lds = a.lds; p.ldy = a.ldy;
    p.m = (int)a.m; p.n = (int)a.n; p.k = (int)a.k;
    p.kblocks = (p.k + kBK - 1) / kBK;
    p.w_tiles = (p.n + kPairW - 1) / kPairW;
    p.swiglu_n = (int)a.swiglu_n;
    if (a.swiglu_n > 0 && (a.n % kTileW)) return QMM_OK;   // gate / up tiles are whole 64 + 64 blocks
    const int64_t tiles = (int64_t)p.w_tiles * ((p.m + kTileT - 1) / kTileT);
    if (tiles > INT32_MAX) return QMM_OK;
    p.num_tiles = (int)tiles;
    const int pairs = (int)std::min<int64_t>(tiles, info.sms / 2);
    int rc = a.fmt == kMXFP8 ? launch_fmt<kMXFP8>(a, p, map, pairs, stream)
                             : launch_fmt<kNVFP4>(a, p, map, pairs, stream);
    if (rc == QMM_OK) *handled = true;
    return rc;
}

}  // namespace qmm

// Device-side status of bounded waits since the last call: QMM_ERR_TIMEOUT
// if any kernel gave up a wait (the word is cleared).  Synchronizes `stream`.
extern "C" int qmm_device_status(void* stream) {
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    unsigned int v = 0, zero = 0;
    QMM_CUDA_TRY(cudaMemcpyFromSymbolAsync(&v, qmm::g_device_error, sizeof(v), 0, cudaMemcpyDeviceToHost, s));
    QMM_CUDA_TRY(cudaStreamSynchronize(s));
    if (v) {
        QMM_CUDA_TRY(cudaMemcpyToSymbolAsync(qmm::g_device_error, &zero, sizeof(zero), 0, cudaMemcpyHostToDevice, s));
        QMM_CUDA_TRY(cudaStreamSynchronize(s));
    }
    unsigned int v2 = 0, v3 = 0;
    QMM_CUDA_TRY(qmm::gemv_tc_take_error(&v2, s));
    QMM_CUDA_TRY(qmm::gemm_bs_take_error(&v3, s));
    v |= v3;
    if (v2) qmm::gemv_tc_mark_workspaces_dirty();   // stream-K counters may be left set
    if (v | v2) return qmm::set_error(QMM_ERR_TIMEOUT, "a device-side wait timed out (flags 0x%x)", v | v2);
    return QMM_OK;
}
