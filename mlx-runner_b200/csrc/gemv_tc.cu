// gemv_tc.cu - decode / MTP-verify quantized GEMM for M <= 8 on resident
// weights: TMA-fed, tensor-core (mma.sync f16) math, stream-K balanced.
//
// y[m, n] = sum_k x[m, k] * dequant(W)[n, k], M <= 8 (decode M = 1,
// src/engine.zig:428-455; MTP verify M = 2..3, src/engine.zig:548, :656).
// The op streams W once and is bound by HBM, so the kernel is shaped around
// keeping HBM busy with few instructions per code:
//   - persistent grid (one CTA per SM); the work is (128-row block, K-chunk
//     of 256 code bytes per row) units laid out row-block-major and split
//     evenly across CTAs (stream-K), so every SM streams the same number of
//     bytes whatever N and K are;
//   - a producer warp streams each unit's codes with two 2D TMAs (128 rows x
//     128 bytes, 128-byte swizzle), its scales with one bulk copy (from the
//     per-unit scale tiles made at weight creation) and the x chunk with
//     256-element 2D TMAs, into a 4-stage ring: 128 KB of codes in flight per
//     SM without spending registers;
//   - three converter warps turn the x chunk (on a barrier of its own, an L2
//     hit) into f16 B fragments after an exact power-of-two scaling into f16
//     range (per x row and chunk), so every x value within 2^29 of the
//     chunk's largest is represented exactly;
//   - 16 consumer warps (8 groups of 16 rows x 2 halves of the unit's k
//     range) run mma.sync.m16n8k16 (f16 in, fp32 accumulate) with the weight
//     codes widened by cvt.f16x2.e2m1x2 / .e4m3x2 (exact), one 32-bit word at
//     a time.  nvfp4 for M <= 2: the x operand is block-diagonal, each MMA
//     column holds one group, and the group scale multiplies the fp32 sums;
//     nvfp4 for M > 2: scales multiply the f16 codes (E2M1 x UE4M3 is exact in
//     f16); mxfp8 scales (any power of two) are applied in fp32 to per-group
//     partial sums;
//   - one kernel instantiation per epilogue: y (bf16, or fp32 partials), the
//     SwiGLU pair, greedy sampling, or the row-parallel exchange;
//   - rows of a block split between CTAs are summed by the last CTA to
//     finish them, in CTA order (deterministic), through a small fp32
//     scratch owned by the weight; the counters are reset by that CTA.  One
//     thread per CTA fences (per-thread fences stall under HBM load) and the
//     final sum issues every contributor's loads at once.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <atomic>
#include <cstdint>
#include <cstdlib>
#include <map>
#include <mutex>
#include <utility>

#include "formats.cuh"
#include "internal.h"

namespace qmm {

// Bit 1: a bounded wait in this kernel timed out (read by qmm_device_status).
__device__ unsigned int g_gemv_tc_error = 0;

namespace {

constexpr int kRows = 128;                 // rows per unit (8 warps x 16)
constexpr int kBox = kRows * 128;          // one 2D TMA box: 128 rows x 128 code bytes
constexpr int kXRows = 8;                  // x rows staged per unit (M padded to 8)
constexpr int kConverters = 3;             // x-converter warps (tokens m = v, v + 3, v + 6)
constexpr int kConsumers = 16;             // 8 row groups x 2 k halves
constexpr int kFirstConsumer = 1 + kConverters;  // warp index of consumer 0
constexpr int kThreads = (1 + kConverters + kConsumers) * 32;  // producer, converters, consumers
constexpr uint64_t kTimeoutNs = 2000000000ull;

// A unit is 128 rows x kBoxes 128-byte code boxes per row; the ring holds
// kStages units (about 147 KB of weights in flight).  Two-box units for
// both formats: one-box nvfp4 units (twice as many, an 8-stage ring) halve
// the stream-K imbalance between CTAs but measured slower (cfg2 M = 1
// 15.3 -> 16.6 us): the per-unit barrier and hand-over cost dominates.
// Consumer split of a unit: NKS k slices x (8 / NRG) warps of NRG row groups
// (16 rows each), NKS * 8 / NRG = 16 warps.  nvfp4 takes kNvSlices k slices;
// mxfp8 two.  More k slices share each x-fragment load among more row groups
// per warp, at the cost of a (NKS - 1)-way shared-memory reduction per flush
// and twice the code registers per warp: four slices measured slower than two
// (cfg2 M = 1 15.4 -> 15.9 us, the lm_head 132 -> 141 us).
constexpr int kNvSlices = 2;

template <int FMT> struct Cfg;
template <> struct Cfg<kMXFP8> {
    static constexpr int kBoxes = 2;
    static constexpr int KC = 128 * kBoxes;   // codes per row per unit
    static constexpr int SB = KC / 32;        // scale bytes per row per unit
    static constexpr int kStages = 4;
};
template <> struct Cfg<kNVFP4> {
    static constexpr int kBoxes = 2;
    static constexpr int KC = 256 * kBoxes;
    static constexpr int SB = KC / 16;
    static constexpr int kStages = 8 / kBoxes;
};

struct TcParams {
    const uint8_t* __restrict__ scales_tiled;  // [row_blocks][kchunks][128][SB]
    uint16_t* __restrict__ y;
    float* __restrict__ yf;                    // when set: fp32 output (row-parallel partials)
    float* __restrict__ partial;               // [grid][2][128][8]
    unsigned int* __restrict__ counters;       // [row_blocks]
    int64_t ldy;
    int m, n, k;
    int kchunks, row_blocks, units;
    int gap;                                   // empty schedule slots after each row block (flush_slots)
    // > 0: gate / up rows interleaved in 64-row blocks; y gets silu(g) * u
    // for swiglu_n columns (row block rb -> columns [64 rb, 64 rb + 64)).
    int swiglu_n;
    // Greedy sampling (am_ids set): per x row the index of the largest bf16
    // output and (am_lp) its log-probability; y is written only when set.
    // am_keys [8] and am_done are zero between calls (the last CTA resets
    // them); am_part [row_blocks][8][2] holds (max, sum exp(y - max)) of
    // each 64-row half block.
    int32_t* am_ids;
    float* am_lp;
    unsigned long long* am_keys;
    float2* am_part;
    unsigned int* am_done;
    // Row-parallel exchange (tp_n > 1): final row-block sums go to every
    // rank's receive slot over NVLink and are added there in rank order.
    int l2_prefetch;   // 1: prefetch the CTA's weight range beyond the ring into L2 up front
    int tp_n, tp_rank, tp_max_rb;
    int64_t tp_cap;
    float* tp_recv[kMaxTpRanks];
    unsigned int* tp_flags[kMaxTpRanks];
    unsigned int* tp_gen;
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ uint64_t gtimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}
__device__ __forceinline__ void mbar_init(uint64_t* b, uint32_t c) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(b)), "r"(c));
}
__device__ __forceinline__ void mbar_arrive(uint64_t* b) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(b)) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* b, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(b)), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try(uint64_t* b, uint32_t parity) {
    uint32_t ok;
    asm volatile("{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
                 "selp.u32 %0, 1, 0, p;\n\t}" : "=r"(ok) : "r"(smem_u32(b)), "r"(parity) : "memory");
    return ok != 0;
}
__device__ __forceinline__ bool mbar_wait(uint64_t* b, uint32_t parity, volatile int* abort_flag) {
    if (mbar_try(b, parity)) return true;
    const uint64_t t0 = gtimer();
    for (uint32_t i = 1;; ++i) {
        if (mbar_try(b, parity)) return true;
        if ((i & 15) == 0) {
            if (*abort_flag) return false;
            if (gtimer() - t0 > kTimeoutNs) {
                *abort_flag = 1;
                atomicOr(&g_gemv_tc_error, 2u);
                return false;
            }
        }
    }
}
__device__ __forceinline__ void tma_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int x0, int y0) {
    asm volatile("cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
                 " [%0], [%1, {%2, %3}], [%4];"
                 ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(x0), "r"(y0), "r"(smem_u32(bar))
                 : "memory");
}
__device__ __forceinline__ void bulk_1d(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}
// L2 prefetch of a 2D TMA box / a contiguous range (no shared memory, no
// barrier): the bytes are in L2 when the matching load is issued later.
__device__ __forceinline__ void tma_prefetch_2d(const CUtensorMap* map, int x0, int y0) {
    asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global [%0, {%1, %2}];"
                 ::"l"(reinterpret_cast<uint64_t>(map)), "r"(x0), "r"(y0) : "memory");
}
__device__ __forceinline__ void bulk_prefetch_l2(const void* src, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(reinterpret_cast<uint64_t>(src)), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void named_sync(int id, int threads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
                 "{%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
                 : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
                 : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Order-preserving 64-bit key of (value, index): larger values rank higher,
// NaN above +inf, and among equal values the lower index.
__device__ __forceinline__ unsigned long long rank_key(float v, uint32_t idx) {
    const uint32_t u = __float_as_uint(v);
    const uint32_t ord = (v != v) ? 0xFFFFFFFFu : ((u & 0x80000000u) ? ~u : (u | 0x80000000u));
    return ((unsigned long long)ord << 32) | (0xFFFFFFFFu - idx);
}

// (M, S) <- the log-sum-exp merge of (M, S) and (m, s), S counted at M.
__device__ __forceinline__ void lse_merge(float& M, float& S, float m, float s) {
    if (m == -INFINITY) return;
    if (M == -INFINITY) { M = m; S = s; return; }
    const float mx = fmaxf(M, m);
    S = S * expf(M - mx) + s * expf(m - mx);
    M = mx;
}

__device__ __forceinline__ uint32_t hmul2u(uint32_t a, uint32_t b) {
    __half2 r = __hmul2(*reinterpret_cast<__half2*>(&a), *reinterpret_cast<__half2*>(&b));
    return *reinterpret_cast<uint32_t*>(&r);
}

// x layout of the B fragments (nvfp4; mxfp8 always uses kXlTokens):
//   kXlTokens   column n of an mma = x row n; the group scale multiplies the
//               weight fragment (f16) before the mma.  Any M <= 8.
//   kXlGroups2  column n = 2 q + t: group slot q (the quad lane whose codes
//               the k rows hold) x x row t.  The block-diagonal x makes each
//               accumulator column one group's partial sum, scaled after the
//               mma in fp32.  M <= 2.
//               (Measured slower than kXlTokens at M = 3, 4: a two-mma form,
//               n = 4 q + t, and a one-mma form with two group slots of four
//               x rows, the slot's two lanes swapping half their code words.)
constexpr int kXlTokens = 0, kXlGroups2 = 1;

// Epilogue of a finished row block: y (bf16, or fp32 partial sums), the
// SwiGLU pair, greedy sampling, or the row-parallel exchange over NVLink.
// One kernel instantiation each keeps the plain decode kernel free of the
// others' code and registers.
constexpr int kEpiPlain = 0, kEpiSwiglu = 1, kEpiArgmax = 2, kEpiTp = 3;

// Where a unit's scales come from:
//   kScaleTiled  the per-unit [128 rows][SB] tiles made at weight creation
//                (one bulk copy per unit);
//   kScaleCkpt   the checkpoint's U8 [N, K/group] tensor itself (stateless
//                calls): a 2D TMA box of 128 rows; for mxfp8 the box is 16
//                bytes wide (the TMA minimum) and the unit's 8 bytes start at
//                (kc & 1) * 8 inside it.
constexpr int kScaleTiled = 0, kScaleCkpt = 1;

template <int FMT, int SRC> struct ScaleLayout {
    static constexpr int SB = Cfg<FMT>::SB;
    static constexpr int kStride = (SRC == kScaleCkpt && FMT == kMXFP8) ? 16 : SB;   // smem row stride
    static constexpr int kBytes = kRows * kStride;                                    // per stage
};

template <int FMT, int XL, int EPI, int SRC>
__global__ void __launch_bounds__(kThreads, 1) qmm_gemv_tc_kernel(const __grid_constant__ CUtensorMap cmap,
                                                                   const __grid_constant__ CUtensorMap xmap,
                                                                   const __grid_constant__ CUtensorMap smap,
                                                                   TcParams p) {
    constexpr int KC = Cfg<FMT>::KC;
    constexpr int kStages = Cfg<FMT>::kStages;
    constexpr int kCodeBytes = Cfg<FMT>::kBoxes * kBox;    // one unit's codes
    constexpr int SB = ScaleLayout<FMT, SRC>::kStride;     // bytes per row of a staged scale tile
    constexpr int kScaleBytes = ScaleLayout<FMT, SRC>::kBytes;
    constexpr int kXRawBytes = kXRows * KC * 2;
    constexpr int kXfBytes = kXRows * KC * 2;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* s_codes = smem;                                          // kStages x 16 KB (1024-aligned)
    uint8_t* s_scales = s_codes + kStages * kCodeBytes;               // kStages x kScaleBytes
    uint8_t* s_xraw = s_scales + kStages * kScaleBytes;               // kStages x kXRawBytes
    uint8_t* s_xf = s_xraw + kStages * kXRawBytes;                    // kStages x kXfBytes
    float* s_xs = reinterpret_cast<float*>(s_xf + kStages * kXfBytes);  // kStages x 8
    constexpr int NKS = FMT == kNVFP4 ? kNvSlices : 2;    // k slices per unit
    constexpr int NRG = NKS / 2;                          // row groups per consumer warp
    float* s_red = s_xs + kStages * 8;                    // (NKS - 1) x 128 x 8 (k-slice sums)
    uint64_t* bars = reinterpret_cast<uint64_t*>(s_red + (NKS - 1) * kRows * 8);
    uint64_t* full = bars;                  // weight tiles (codes + scales) landed
    uint64_t* xready = bars + kStages;      // f16 x fragments written
    uint64_t* empty = bars + 2 * kStages;   // every consumer is done with the stage
    uint64_t* xfull = bars + 3 * kStages;   // raw x chunk landed
    volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 4 * kStages);
    volatile int* s_last = abort_flag + 1;
    volatile unsigned int* s_epoch = reinterpret_cast<volatile unsigned int*>(abort_flag + 2);
    // Row-parallel: row blocks this CTA pushed, finished after its last unit
    // ([0] = count, then (row block, epoch) pairs).
    volatile int* s_tp_list = abort_flag + 4;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // Static schedule over slots: each row block is its kchunks units then
    // p.gap empty slots (the cost of the flush that follows it), and CTA j
    // owns slots [V j / G, V (j + 1) / G), i.e. the units in them.  A CTA
    // whose range holds a row-block boundary therefore takes fewer units.
    // Unit u belongs to CTA owner(u).  32-bit division when the products fit
    // (64-bit division is a long software sequence).
    // The helpers recompute the slot count from p and gridDim (a few integer
    // operations per call, at flush time) so that it holds no register
    // through the unit loop (held, it cost the M <= 2 kernel spills and
    // 0.4 us per launch).
    auto slot_count = [&]() -> int64_t { return (int64_t)p.row_blocks * (p.kchunks + p.gap); };
    auto fits32 = [&]() -> bool { return (uint64_t)(slot_count() + 1) * gridDim.x < (1ull << 32); };
    auto unit_of_slot = [&](int64_t v) -> int {          // first unit at or after slot v
        if (p.gap == 0) return (int)v;
        const unsigned kcg = (unsigned)(p.kchunks + p.gap);
        const unsigned rb = (unsigned)v / kcg, o = (unsigned)v - rb * kcg;
        return (int)(rb * (unsigned)p.kchunks + min(o, (unsigned)p.kchunks));
    };
    auto first_unit = [&](int j) -> int {
        const int64_t V = slot_count();
        return unit_of_slot(fits32() ? (int64_t)(((unsigned)V * (unsigned)j) / gridDim.x) : (V * j) / gridDim.x);
    };
    auto owner = [&](int u) -> int {
        const int64_t V = slot_count();
        const int64_t v = p.gap == 0 ? u : (int64_t)(u / p.kchunks) * (p.kchunks + p.gap) + u % p.kchunks;
        return fits32() ? (int)(((unsigned)(v + 1) * gridDim.x - 1u) / (unsigned)V)
                        : (int)(((v + 1) * gridDim.x - 1) / V);
    };
    const int u0 = first_unit((int)blockIdx.x);
    const int u1 = first_unit((int)blockIdx.x + 1);
    const int nunits = u1 - u0;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&xfull[s], 1);
            mbar_init(&xready[s], kConverters);
            mbar_init(&empty[s], kConsumers);
        }
        *abort_flag = 0;
        s_tp_list[0] = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    // A dependent grid (the next decode call) may start on SMs this grid frees.
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

    if (warp == 0) {
        // ---------------- producer ----------------
        if (lane == 0) {
            // Weight bytes of a unit (codes + scales) and, on a barrier of its
            // own, its x chunk: M rows of 256-element boxes (an L2 hit after
            // the first CTA), converted while the weights are still in flight.
            // Units are issued in order, so their (row block, chunk) advance by
            // one step each: no division per unit.
            int w_rb = u0 / p.kchunks, w_kc = u0 - w_rb * p.kchunks, x_kc = w_kc;
            auto issue_w = [&](int i) {
                const int s = i % kStages;
                mbar_expect_tx(&full[s], kCodeBytes + kScaleBytes);
#pragma unroll
                for (int b = 0; b < Cfg<FMT>::kBoxes; ++b)
                    tma_2d(s_codes + s * kCodeBytes + b * kBox, &cmap, &full[s], (w_kc * Cfg<FMT>::kBoxes + b) * 128,
                           w_rb * kRows);
                if constexpr (SRC == kScaleCkpt)
                    tma_2d(s_scales + s * kScaleBytes, &smap, &full[s], (w_kc * Cfg<FMT>::SB) & ~15, w_rb * kRows);
                else
                    bulk_1d(s_scales + s * kScaleBytes, p.scales_tiled + (int64_t)(u0 + i) * kScaleBytes,
                            kScaleBytes, &full[s]);
                if (++w_kc == p.kchunks) { w_kc = 0; ++w_rb; }
            };
            auto issue_x = [&](int i) {
                const int s = i % kStages;
                mbar_expect_tx(&xfull[s], (uint32_t)(KC / 256) * (uint32_t)p.m * 512u);
#pragma unroll
                for (int xb = 0; xb < KC / 256; ++xb)   // x rows of the chunk, 256 elements per box
                    tma_2d(s_xraw + s * kXRawBytes + xb * p.m * 512, &xmap, &xfull[s], x_kc * KC + 256 * xb, 0);
                if (++x_kc == p.kchunks) x_kc = 0;
            };
            // The first ring of weight tiles streams before the wait on the
            // previous grid (programmatic dependent launch): only x (and the
            // outputs, written after x is consumed) depend on earlier kernels.
            // The rest of this CTA's weight range is prefetched into L2 as
            // well, so HBM streams this launch's weights while the previous
            // launch finishes (its tail and stream-K fix-up); every weight
            // byte is still read from HBM once.
            const int pre = min(kStages, nunits);
            for (int i = 0; i < pre; ++i) issue_w(i);
            if (p.l2_prefetch) {
                int f_rb = w_rb, f_kc = w_kc;
                for (int i = pre; i < nunits; ++i) {
                    for (int b = 0; b < Cfg<FMT>::kBoxes; ++b)
                        tma_prefetch_2d(&cmap, (f_kc * Cfg<FMT>::kBoxes + b) * 128, f_rb * kRows);
                    if constexpr (SRC == kScaleCkpt)
                        tma_prefetch_2d(&smap, (f_kc * Cfg<FMT>::SB) & ~15, f_rb * kRows);
                    else
                        bulk_prefetch_l2(p.scales_tiled + (int64_t)(u0 + i) * kScaleBytes, kScaleBytes);
                    if (++f_kc == p.kchunks) { f_kc = 0; ++f_rb; }
                }
            }
            asm volatile("griddepcontrol.wait;" ::: "memory");
            for (int i = 0; i < pre; ++i) issue_x(i);
            int last = pre - 1;
            for (int i = pre; i < nunits; ++i) {
                const uint32_t ph = (uint32_t)(i / kStages) & 1u;
                if (!mbar_wait(&empty[i % kStages], ph ^ 1u, abort_flag)) break;
                issue_w(i);
                issue_x(i);
                last = i;
            }
            // Drain: every stage's last fill must land, and every consumer
            // must be done, before the CTA can exit.
            for (int i = max(0, last - kStages + 1); i <= last; ++i) {
                const uint64_t t0 = gtimer();
                while (!mbar_try(&full[i % kStages], (uint32_t)(i / kStages) & 1u) && gtimer() - t0 < kTimeoutNs) {
                }
                while (!mbar_try(&xfull[i % kStages], (uint32_t)(i / kStages) & 1u) && gtimer() - t0 < kTimeoutNs) {
                }
            }
        }
    } else if (warp < kFirstConsumer) {
        // ---------------- x converters ----------------
        // Warp cv converts x rows m = cv, cv + 3, cv + 6 (m < M).  B-fragment slots of x
        // rows >= M are zero for the whole launch and their x-scale factors 1
        // (their accumulator columns are never stored).
        const int cv = warp - 1, ct = threadIdx.x - 32;
        for (int off = ct * 16; off < kStages * kXfBytes; off += kConverters * 32 * 16)
            *reinterpret_cast<uint4*>(s_xf + off) = make_uint4(0, 0, 0, 0);
        for (int t = ct; t < kStages * 8; t += kConverters * 32) s_xs[t] = 1.0f;
        named_sync(2, kConverters * 32);
        for (int i = 0; i < nunits; ++i) {
            const int s = i % kStages;
            const uint32_t ph = (uint32_t)(i / kStages) & 1u;
            if (!mbar_wait(&xfull[s], ph, abort_flag)) break;
            const uint16_t* raw = reinterpret_cast<const uint16_t*>(s_xraw + s * kXRawBytes);
            float* xs = s_xs + s * 8;
            // Lane L owns x elements [E L, E L + E) of every row of the chunk
            // (E = KC / 32): amax over the chunk -> exponent e, x scaled by
            // 2^-e into [2^14, 2^15), converted to f16 and stored into the
            // B-fragment slot that element run belongs to.  Slots of rows
            // m >= M stay zero (cleared once before the first unit).
            // The raw chunk arrives as 256-element TMA boxes of M rows:
            // element (m, k) sits at box k / 256, row m, column k % 256.
            constexpr int E = KC / 32;             // 16 (nvfp4) or 8 (mxfp8)
            uint8_t* xf = s_xf + s * kXfBytes;
            const int k0 = E * lane;
            const uint16_t* rbase = raw + (k0 >> 8) * (p.m * 256) + (k0 & 255);
            for (int m = cv; m < p.m; m += kConverters) {
                float v[E];
                uint32_t w[E / 2];
#pragma unroll
                for (int q = 0; q < E / 8; ++q) {
                    const uint4 r = *reinterpret_cast<const uint4*>(rbase + m * 256 + 8 * q);
                    w[4 * q] = r.x; w[4 * q + 1] = r.y; w[4 * q + 2] = r.z; w[4 * q + 3] = r.w;
                }
                // Largest |x| of the chunk from the bf16 bit patterns (magnitude
                // order = integer order; a NaN sorts above every finite value).
                uint32_t mx = 0;
#pragma unroll
                for (int i = 0; i < E / 2; ++i) {
                    const float2 f = bf16x2_to_float2(w[i]);
                    v[2 * i] = f.x;
                    v[2 * i + 1] = f.y;
                    mx = max(mx, max(w[i] & 0x7FFFu, (w[i] >> 16) & 0x7FFFu));
                }
                mx = __reduce_max_sync(0xFFFFFFFFu, mx);
                int ex = 0;
                if (mx != 0) {
                    ex = (int)((mx >> 7) & 0xFF) - 127 - 14;
                    ex = max(-100, min(100, ex));
                }
                const float inv = __uint_as_float((uint32_t)(127 - ex) << 23);
                if (lane == 0) xs[m] = __uint_as_float((uint32_t)(127 + ex) << 23);
                uint32_t h[E / 2];
#pragma unroll
                for (int i = 0; i < E / 2; ++i) {
                    __half2 hv = __floats2half2_rn(v[2 * i] * inv, v[2 * i + 1] * inv);
                    h[i] = *reinterpret_cast<uint32_t*>(&hv);
                }
                if constexpr (FMT == kNVFP4) {
                    // run R = k / 8 of 8 elements -> super-step su = R / 16,
                    // quad c = (R / 4) % 4, step pair jp = 4 su + R % 4.  The
                    // B-fragment lane is 4 n + c for the run's mma column n.
#pragma unroll
                    for (int q = 0; q < Cfg<FMT>::kBoxes; ++q) {
                        const int R = Cfg<FMT>::kBoxes * lane + q, jp = 4 * (R >> 4) + (R & 3), c = (R >> 2) & 3;
                        int bl;
                        if constexpr (XL == kXlTokens) bl = 4 * m + c;              // n = m
                        else bl = 9 * c + 4 * m;                                     // n = 2 c + m
                        *reinterpret_cast<uint4*>(xf + (jp * 32 + bl) * 16) =
                            make_uint4(h[4 * q], h[4 * q + 1], h[4 * q + 2], h[4 * q + 3]);
                    }
                } else {
                    // run R = k / 4 of 4 elements -> step j = R / 4 (slot j / 2,
                    // half j % 2), quad c = R % 4.
#pragma unroll
                    for (int q = 0; q < 2; ++q) {
                        const int R = 2 * lane + q, j = R >> 2, c = R & 3;
                        *reinterpret_cast<uint2*>(xf + ((j >> 1) * 32 + 4 * m + c) * 16 + (j & 1) * 8) =
                            make_uint2(h[2 * q], h[2 * q + 1]);
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&xready[s]);
        }
    } else {
        // ---------------- consumers ----------------
        // Warp cw owns row groups rg0 .. rg0 + NRG - 1 (16 rows each) of every
        // unit over k slice kh of NKS (super-steps kh, kh + NKS, ... of the
        // unit's 128-code super-steps).
        const int cw = warp - kFirstConsumer, kh = cw / (8 / NRG), rg0 = (cw % (8 / NRG)) * NRG;
        const int g = lane >> 2, c = lane & 3;
        // MMA row slot g computes tile row 16 rg + (g >> 1) + 4 (g & 1) (and
        // that + 8).  A quarter-warp phase of a 16-byte shared load covers
        // the lanes of two consecutive slots; with the TMA's 128-byte swizzle
        // (chunk ^= row & 7) rows 4 apart hit disjoint banks, where adjacent
        // rows would collide on the same 16 (a 2-way conflict on every code
        // load).  Outputs, scales and partial sums all follow r0 / r1.
        int r0[NRG], r1[NRG];
#pragma unroll
        for (int j = 0; j < NRG; ++j) {
            r0[j] = 16 * (rg0 + j) + ((g >> 1) | ((g & 1) << 2));
            r1[j] = r0[j] + 8;
        }
        float acc[NRG][4];
#pragma unroll
        for (int j = 0; j < NRG; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;
        int cur_rb = -1, first_rb = -1, rb_first_unit = 0;
        // Row-parallel exchange of row block rb (final fp32 sums in s_red,
        // [128 rows][8 columns]).  tp_push writes them to this rank's slot of
        // every rank's receive buffer and one thread releases them with a
        // flag per rank (the barrier orders every thread's stores before it);
        // the CTA then carries on with its units.  After its last unit,
        // tp_complete waits - for at most kTimeoutNs - until every rank's
        // flag for each pushed block carries its epoch, and sums the block
        // over ranks in rank order into y.  Epochs count per row block on the
        // device, so graph replays stay in step; two receive parities let a
        // rank run one call ahead of the others.
        constexpr int kTpList = 16;
        auto tp_push = [&](int rb) {
            const int t = threadIdx.x - kFirstConsumer * 32;
            const int P = p.tp_n, me = p.tp_rank;
            if (t == 0) *s_epoch = p.tp_gen[rb] + 1u;
            named_sync(1, kConsumers * 32);
            const unsigned int epoch = *s_epoch;
            const int64_t par = epoch & 1u;
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                const int idx = t + 512 * e, col = idx & 7, row = rb * kRows + (idx >> 3);
                if (row < p.n && col < p.m) {
                    const float v = s_red[idx];
                    const int64_t off = (par * P + me) * p.tp_cap + (int64_t)col * p.n + row;
#pragma unroll
                    for (int r = 0; r < kMaxTpRanks; ++r)
                        if (r < P) p.tp_recv[r][off] = v;
                }
            }
            named_sync(1, kConsumers * 32);
            if (t == 0) {
                // One system-scope release fence, then relaxed flag stores:
                // the fence and each later strong store form a release
                // pattern (the barrier above ordered every thread's pushes
                // before the fence), so the P flags cost one fence, not P.
                asm volatile("fence.acq_rel.sys;" ::: "memory");
#pragma unroll
                for (int r = 0; r < kMaxTpRanks; ++r)
                    if (r < P)
                        asm volatile("st.relaxed.sys.global.u32 [%0], %1;"
                                     ::"l"(p.tp_flags[r] + me * p.tp_max_rb + rb), "r"(epoch) : "memory");
                p.tp_gen[rb] = epoch;
                const int n_list = s_tp_list[0];
                s_tp_list[1 + 2 * n_list] = rb;
                s_tp_list[2 + 2 * n_list] = (int)epoch;
                s_tp_list[0] = n_list + 1;
            }
            named_sync(1, kConsumers * 32);       // s_red / s_epoch / the list are reused
        };
        auto tp_complete = [&]() {
            const int t = threadIdx.x - kFirstConsumer * 32;
            const int P = p.tp_n, me = p.tp_rank;
            const int n_list = s_tp_list[0];
            if (t == 0) {
                const uint64_t t0 = gtimer();
                bool timed_out = false;
                for (int q = 0; q < n_list && !timed_out; ++q) {
                    const int rb = s_tp_list[1 + 2 * q];
                    const unsigned int epoch = (unsigned int)s_tp_list[2 + 2 * q];
                    for (int src = 0; src < P && !timed_out; ++src) {
                        for (;;) {
                            unsigned int f;
                            asm volatile("ld.acquire.sys.global.u32 %0, [%1];"
                                         : "=r"(f) : "l"(p.tp_flags[me] + src * p.tp_max_rb + rb) : "memory");
                            if (f == epoch) break;
                            if (gtimer() - t0 > kTimeoutNs) {
                                atomicOr(&g_gemv_tc_error, 2u);
                                timed_out = true;
                                break;
                            }
                        }
                    }
                }
            }
            named_sync(1, kConsumers * 32);
            for (int q = 0; q < n_list; ++q) {
                const int rb = s_tp_list[1 + 2 * q];
                const int64_t par = (unsigned int)s_tp_list[2 + 2 * q] & 1u;
                // Every rank's value of both outputs is loaded before any is
                // added (2 P loads in flight instead of a chain of 2 P round
                // trips), then summed in rank order.
                float v[2][kMaxTpRanks];
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                    const int idx = t + 512 * e, col = idx & 7, row = rb * kRows + (idx >> 3);
                    const bool ok = row < p.n && col < p.m;
#pragma unroll
                    for (int src = 0; src < kMaxTpRanks; ++src)
                        v[e][src] = ok && src < P
                                        ? __ldcg(p.tp_recv[me] + (par * P + src) * p.tp_cap + (int64_t)col * p.n + row)
                                        : 0.f;
                }
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                    const int idx = t + 512 * e, col = idx & 7, row = rb * kRows + (idx >> 3);
                    if (row < p.n && col < p.m) {
                        float sum = 0.f;
#pragma unroll
                        for (int src = 0; src < kMaxTpRanks; ++src)
                            if (src < P) sum += v[e][src];
                        p.y[(int64_t)col * p.ldy + row] = f32_to_bf16(sum);
                    }
                }
            }
        };
        // A row block finished inside a flush: push it, or - when the list is
        // full - push and complete it at once (all threads see the same count).
        auto tp_finish = [&](int rb) {
            if (s_tp_list[0] < kTpList) {
                tp_push(rb);
            } else {
                tp_complete();
                named_sync(1, kConsumers * 32);
                if (threadIdx.x == kFirstConsumer * 32) s_tp_list[0] = 0;
                named_sync(1, kConsumers * 32);
                tp_push(rb);
            }
        };
        // Gate / up row block rb, final sums in s_red [128 rows][8 columns]:
        // rows 0-63 are gate rows 64 rb + r, rows 64-127 their up rows.
        auto swiglu_out = [&](int rb) {
            const int t = threadIdx.x - kFirstConsumer * 32;
            const int r = t & 63, col = t >> 6;
            const int64_t hc = (int64_t)rb * 64 + r;
            if (col < p.m && hc < p.swiglu_n)
                p.y[(int64_t)col * p.ldy + hc] = swiglu_bf16(s_red[r * 8 + col], s_red[(r + 64) * 8 + col]);
        };
        // Greedy-sampling epilogue of row block rb (final sums in s_red): the
        // bf16 outputs (to y when set), one rank key per x row into am_keys,
        // and (max, sum exp) of each 64-row half into am_part.  Threads
        // 64 col .. 64 col + 63 take x row col: two warps, rows r, r + 64.
        auto argmax_out = [&](int rb) {
            const int t = threadIdx.x - kFirstConsumer * 32;
            const int col = t >> 6, half = (t >> 5) & 1;
            unsigned long long key = 0;
            float l[2], mx = -INFINITY;
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                const int rl = half * 32 + lane + 64 * e;   // rows 0-31 / 32-63 (+64)
                const int row = rb * kRows + rl;
                const bool ok = row < p.n && col < p.m;
                const uint16_t b = f32_to_bf16(s_red[rl * 8 + col]);
                if (ok && p.y) p.y[(int64_t)col * p.ldy + row] = b;
                l[e] = ok ? bf16_to_f32(b) : -INFINITY;
                if (ok) key = max(key, rank_key(l[e], (uint32_t)row));
                mx = fmaxf(mx, l[e]);
            }
#pragma unroll
            for (int o = 16; o; o >>= 1) {
                key = max(key, __shfl_xor_sync(0xFFFFFFFFu, key, o));
                mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, o));
            }
            float sum = mx == -INFINITY ? 0.0f : expf(l[0] - mx) + expf(l[1] - mx);
#pragma unroll
            for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xFFFFFFFFu, sum, o);
            if (lane == 0 && col < p.m) {
                if (key) atomicMax(&p.am_keys[col], key);
                p.am_part[((int64_t)rb * 8 + col) * 2 + half] = make_float2(mx, sum);
            }
        };
        // After this CTA's last flush: the last CTA of the grid to get here
        // (acq_rel count; each CTA's writes are ordered before its count by
        // the barrier) merges the half-block (max, sum) pairs of each x row
        // in a fixed order, writes the id and log-probability and resets the
        // keys and the count for the next call.
        auto argmax_finish = [&]() {
            const int t = threadIdx.x - kFirstConsumer * 32;
            named_sync(1, kConsumers * 32);
            if (t == 0) {
                unsigned prev;
                asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(prev) : "l"(p.am_done) : "memory");
                const int last = prev == gridDim.x - 1 ? 1 : 0;
                if (last) *p.am_done = 0u;
                *s_last = last;
            }
            named_sync(1, kConsumers * 32);
            if (!*s_last) return;
            const int col = t >> 6, j = t & 63;
            float M = -INFINITY, S = 0.0f;
            if (col < p.m) {
                // Eight loads in flight per batch (the pairs are an L2 round
                // trip each; one at a time they cost tens of microseconds on
                // the 248320-row head), merged in index order.
                const int total = 2 * p.row_blocks;
                for (int i0 = j; i0 < total; i0 += 64 * 8) {
                    float2 ps[8];
#pragma unroll
                    for (int q = 0; q < 8; ++q) {
                        const int i = i0 + 64 * q;
                        ps[q] = i < total ? __ldcg(&p.am_part[((int64_t)(i >> 1) * 8 + col) * 2 + (i & 1)])
                                          : make_float2(-INFINITY, 0.0f);
                    }
#pragma unroll
                    for (int q = 0; q < 8; ++q) lse_merge(M, S, ps[q].x, ps[q].y);
                }
            }
#pragma unroll
            for (int o = 16; o; o >>= 1) {
                const float m2 = __shfl_xor_sync(0xFFFFFFFFu, M, o), s2 = __shfl_xor_sync(0xFFFFFFFFu, S, o);
                lse_merge(M, S, m2, s2);
            }
            if (lane == 0) {
                s_red[(col * 2 + (j >> 5)) * 2] = M;
                s_red[(col * 2 + (j >> 5)) * 2 + 1] = S;
            }
            named_sync(1, kConsumers * 32);
            if (j == 0 && col < p.m) {
                lse_merge(M, S, s_red[(col * 2 + 1) * 2], s_red[(col * 2 + 1) * 2 + 1]);
                const unsigned long long key = __ldcg(&p.am_keys[col]);
                p.am_keys[col] = 0ull;
                const uint32_t ord = (uint32_t)(key >> 32);
                const uint32_t idx = 0xFFFFFFFFu - (uint32_t)(key & 0xFFFFFFFFu);
                const float lid = ord == 0xFFFFFFFFu ? __uint_as_float(0x7FC00000u)
                                  : __uint_as_float((ord & 0x80000000u) ? (ord & 0x7FFFFFFFu) : ~ord);
                p.am_ids[col] = (int32_t)idx;
                if (p.am_lp) p.am_lp[col] = lid - bf16_to_f32(f32_to_bf16(M + logf(S)));
            }
        };
        // Counter step of row block rb after this CTA wrote its partial: the
        // last contributor to arrive sums every contributor's partial.
        auto arrive_partial = [&](int rb) {
            constexpr bool to_smem = EPI != kEpiPlain;
            // The barrier orders the CTA's partial writes before thread 64's
            // gpu-scope fence, which then releases them with the counter
            // update; the last arriver's fence acquires the other CTAs' writes
            // for every thread past the next barrier.  (One fence per CTA:
            // fences by every thread stall for microseconds under HBM load.)
            named_sync(1, kConsumers * 32);
            if (threadIdx.x == kFirstConsumer * 32) {
                // CTAs covering rb: owner(first unit) .. owner(last unit).  The
                // acq_rel add releases this CTA's partial (ordered before it by
                // the barrier) and, for the last arriver, acquires the others'.
                const int ifirst = owner(rb * p.kchunks), ilast = owner(rb * p.kchunks + p.kchunks - 1);
                unsigned prev;
                asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;"
                             : "=r"(prev) : "l"(p.counters + rb) : "memory");
                const int last = (prev == (unsigned)(ilast - ifirst)) ? 1 : 0;
                if (last) p.counters[rb] = 0;
                *s_last = last;
            }
            named_sync(1, kConsumers * 32);
            if (*s_last) {
                // Sum the contributors' partials in CTA order.  Each of the 512
                // consumer threads owns 2 of the block's 128 x 8 outputs and
                // keeps 8 contributor loads in flight per batch.
                const int ifirst = owner(rb * p.kchunks), ilast = owner(rb * p.kchunks + p.kchunks - 1);
                const int t = threadIdx.x - kFirstConsumer * 32;
                // Contributor j wrote rb into its slot 0 when rb is its first row
                // block.  Every contributor after ifirst begins inside rb; ifirst
                // used slot 1 if its range began in an earlier row block.
                const int slot_first = first_unit(ifirst) < rb * p.kchunks ? 1 : 0;
                float v[2] = {0.f, 0.f};
                for (int j0 = ifirst; j0 <= ilast; j0 += 8) {
                    float ld[8][2];
#pragma unroll
                    for (int q = 0; q < 8; ++q) {
                        const int j = j0 + q;
                        ld[q][0] = ld[q][1] = 0.f;
                        if (j <= ilast) {
                            const int jslot = j == ifirst ? slot_first : 0;
                            const float* src = p.partial + ((int64_t)j * 2 + jslot) * kRows * 8;
                            ld[q][0] = __ldcg(src + t);
                            ld[q][1] = __ldcg(src + t + 512);
                        }
                    }
#pragma unroll
                    for (int q = 0; q < 8; ++q) {
                        v[0] += ld[q][0];
                        v[1] += ld[q][1];
                    }
                }
                if (to_smem) {
                    // s_red is free here (its last reader was the kh add above).
                    s_red[t] = v[0];
                    s_red[t + 512] = v[1];
                } else {
#pragma unroll
                    for (int e = 0; e < 2; ++e) {
                        const int idx = t + 512 * e, rl = idx >> 3, col = idx & 7;
                        const int row = rb * kRows + rl;
                        if (row < p.n && col < p.m) {
                            if (p.yf) p.yf[(int64_t)col * p.ldy + row] = v[e];
                            else p.y[(int64_t)col * p.ldy + row] = f32_to_bf16(v[e]);
                        }
                    }
                }
            }
            named_sync(1, kConsumers * 32);       // s_red / s_last are reused by the next flush
            if constexpr (EPI == kEpiSwiglu || EPI == kEpiArgmax) {
                if (*s_last) {
                    if constexpr (EPI == kEpiSwiglu) swiglu_out(rb);
                    else argmax_out(rb);
                    named_sync(1, kConsumers * 32);
                }
            }
            if constexpr (EPI == kEpiTp) {
                if (*s_last) tp_finish(rb);
            }
        };
        auto flush = [&](int rb, bool complete) {
            if constexpr (XL == kXlGroups2) {
                // Lanes c of a quad hold x rows 0, 1 over group slot c: add the
                // slots (fixed butterfly order); lane c = 0 then holds columns 0, 1.
#pragma unroll
                for (int j = 0; j < NRG; ++j)
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        acc[j][i] += __shfl_xor_sync(0xFFFFFFFFu, acc[j][i], 1);
                        acc[j][i] += __shfl_xor_sync(0xFFFFFFFFu, acc[j][i], 2);
                        if (c != 0) acc[j][i] = 0.f;
                    }
            }
            // rows r0 / r1 of block rb, x rows (columns) 2c, 2c + 1.  The k
            // slices kh > 0 hand their sums to kh = 0, which adds them in
            // slice order (fixed order).
            auto red_at = [&](int j, int i) { return (i < 2 ? r0[j] : r1[j]) * 8 + 2 * c + (i & 1); };
            if (kh > 0) {
#pragma unroll
                for (int j = 0; j < NRG; ++j)
#pragma unroll
                    for (int i = 0; i < 4; ++i) s_red[(kh - 1) * kRows * 8 + red_at(j, i)] = acc[j][i];
            }
            named_sync(1, kConsumers * 32);
            if (kh == 0) {
#pragma unroll
                for (int q = 1; q < NKS; ++q)
#pragma unroll
                    for (int j = 0; j < NRG; ++j)
#pragma unroll
                        for (int i = 0; i < 4; ++i) acc[j][i] += s_red[(q - 1) * kRows * 8 + red_at(j, i)];
            }
            constexpr bool to_smem = EPI != kEpiPlain;
            if (complete && to_smem) {
                // The kh = 0 threads rewrite slice 1's entries (each its own)
                // with the final sums: s_red[0 .. 1023] is then the block's
                // [128 rows][8].
                if (kh == 0) {
#pragma unroll
                    for (int j = 0; j < NRG; ++j)
#pragma unroll
                        for (int i = 0; i < 4; ++i) s_red[red_at(j, i)] = acc[j][i];
                }
                named_sync(1, kConsumers * 32);
                if constexpr (EPI == kEpiSwiglu) swiglu_out(rb);
                if constexpr (EPI == kEpiArgmax) argmax_out(rb);
                if constexpr (EPI == kEpiTp) {
                    tp_finish(rb);
                } else {
                    named_sync(1, kConsumers * 32);   // s_red is reused by the next flush
                }
                return;
            }
            if (complete) {
                if (kh == 0) {
#pragma unroll
                    for (int j = 0; j < NRG; ++j)
#pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            const int row = rb * kRows + (i < 2 ? r0[j] : r1[j]), col = 2 * c + (i & 1);
                            if (row < p.n && col < p.m) {
                                if (p.yf) p.yf[(int64_t)col * p.ldy + row] = acc[j][i];
                                else p.y[(int64_t)col * p.ldy + row] = f32_to_bf16(acc[j][i]);
                            }
                        }
                }
                named_sync(1, kConsumers * 32);   // s_red is reused by the next flush
                return;
            }
            const int slot = (rb == first_rb) ? 0 : 1;
            float* part = p.partial + ((int64_t)blockIdx.x * 2 + slot) * kRows * 8;
            if (kh == 0) {
#pragma unroll
                for (int j = 0; j < NRG; ++j)
#pragma unroll
                    for (int i = 0; i < 4; ++i) part[red_at(j, i)] = acc[j][i];
            }
            arrive_partial(rb);
        };
        // nvfp4 unit with group-slot x columns (kXlGroups2): the codes enter
        // the mma unscaled (E2M1 -> f16 is exact); each half super-step (jp
        // 0-1: the chunk's first 16 codes, jp 2-3: the last 16) fills
        // accumulators whose column 2c + t is group slot c of x row t, which
        // the group scales of rows r0 / r1 then weight in fp32.
        auto consume_groups = [&](const uint8_t* cs, const uint8_t* ss, const uint8_t* xf, float xs0, float xs1) {
            float u[NRG][4];
#pragma unroll
            for (int j = 0; j < NRG; ++j) u[j][0] = u[j][1] = u[j][2] = u[j][3] = 0.f;
#pragma unroll
            for (int si = 0; si < 2 * Cfg<FMT>::kBoxes / NKS; ++si) {
                const int su = kh + NKS * si;
                const uint8_t* cb = cs + (su >> 1) * kBox;
                const int ch = (4 * su + c) & 7;
                uint32_t wa[NRG][4], wb[NRG][4];
                float2 sa0[NRG], sa1[NRG];
#pragma unroll
                for (int j = 0; j < NRG; ++j) {
                    const uint4 w0 = *reinterpret_cast<const uint4*>(cb + r0[j] * 128 + ((ch ^ (r0[j] & 7)) << 4));
                    const uint4 w1 = *reinterpret_cast<const uint4*>(cb + r1[j] * 128 + ((ch ^ (r1[j] & 7)) << 4));
                    wa[j][0] = w0.x; wa[j][1] = w0.y; wa[j][2] = w0.z; wa[j][3] = w0.w;
                    wb[j][0] = w1.x; wb[j][1] = w1.y; wb[j][2] = w1.z; wb[j][3] = w1.w;
                    // Scales of group slot c (its two halves) for rows r0 and r1.
                    sa0[j] = f16x2_to_float2(e4m3x2_to_f16x2(*reinterpret_cast<const uint16_t*>(ss + r0[j] * SB + 8 * su + 2 * c)));
                    sa1[j] = f16x2_to_float2(e4m3x2_to_f16x2(*reinterpret_cast<const uint16_t*>(ss + r1[j] * SB + 8 * su + 2 * c)));
                }
#pragma unroll
                for (int half = 0; half < 2; ++half) {
                    float da[NRG][4], db[NRG][4];
#pragma unroll
                    for (int j = 0; j < NRG; ++j)
#pragma unroll
                        for (int i = 0; i < 4; ++i) da[j][i] = db[j][i] = 0.f;
#pragma unroll
                    for (int jq = 0; jq < 2; ++jq) {
                        const int jp = 2 * half + jq;
                        // One x-fragment load feeds every row group of the warp.
                        const uint4 bx = *reinterpret_cast<const uint4*>(xf + ((su * 4 + jp) * 32 + lane) * 16);
#pragma unroll
                        for (int j = 0; j < NRG; ++j) {
                            // Word jp of rows r0 / r1 (8 codes each) widened just
                            // before its mmas: 8 live f16 pairs instead of 32.
                            uint32_t ha[4], hb[4];
                            e2m1x8_to_f16x2(wa[j][jp], ha);
                            e2m1x8_to_f16x2(wb[j][jp], hb);
                            const uint32_t a0[4] = {ha[0], hb[0], ha[1], hb[1]};
                            const uint32_t a1[4] = {ha[2], hb[2], ha[3], hb[3]};
                            mma16816(da[j], a0, bx.x, bx.y);
                            mma16816(db[j], a1, bx.z, bx.w);
                        }
                    }
#pragma unroll
                    for (int j = 0; j < NRG; ++j) {
                        const float fa0 = half ? sa0[j].y : sa0[j].x, fa1 = half ? sa1[j].y : sa1[j].x;
                        u[j][0] = fmaf(da[j][0] + db[j][0], fa0, u[j][0]);
                        u[j][1] = fmaf(da[j][1] + db[j][1], fa0, u[j][1]);
                        u[j][2] = fmaf(da[j][2] + db[j][2], fa1, u[j][2]);
                        u[j][3] = fmaf(da[j][3] + db[j][3], fa1, u[j][3]);
                    }
                }
            }
#pragma unroll
            for (int j = 0; j < NRG; ++j) {
                acc[j][0] = fmaf(u[j][0], xs0, acc[j][0]);
                acc[j][1] = fmaf(u[j][1], xs1, acc[j][1]);
                acc[j][2] = fmaf(u[j][2], xs0, acc[j][2]);
                acc[j][3] = fmaf(u[j][3], xs1, acc[j][3]);
            }
        };
        int next_rb = u0 / p.kchunks, next_kc = u0 - next_rb * p.kchunks;   // advanced per unit
        for (int i = 0; i < nunits; ++i) {
            const int rb = next_rb, kc = next_kc;
            if (++next_kc == p.kchunks) { next_kc = 0; ++next_rb; }
            if (rb != cur_rb) {
                if (cur_rb >= 0) flush(cur_rb, rb_first_unit == 0);   // a row block ends inside this CTA
                cur_rb = rb;
                if (first_rb < 0) first_rb = rb;
                rb_first_unit = kc;
#pragma unroll
                for (int j = 0; j < NRG; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;
            }
            const int s = i % kStages;
            const uint32_t ph = (uint32_t)(i / kStages) & 1u;
            // A wait that gives up leaves the unit uncomputed but keeps the
            // warp in step with the others (the named barriers in flush must
            // match); the device error word tells the host the output is void.
            const bool live = mbar_wait(&full[s], ph, abort_flag) && mbar_wait(&xready[s], ph, abort_flag);
            if (live) {
            const uint8_t* cs = s_codes + s * kCodeBytes;
            const uint8_t* ss = s_scales + s * kScaleBytes;
            const uint8_t* xf = s_xf + s * kXfBytes;
            const float* xs = s_xs + s * 8;
            // x rows of this lane's accumulator columns.
            const int t0 = XL == kXlTokens ? 2 * c : 0;
            const float xs0 = xs[t0], xs1 = xs[t0 + 1];
            if constexpr (FMT == kNVFP4 && XL != kXlTokens) {
                consume_groups(cs, ss, xf, xs0, xs1);
            } else if constexpr (FMT == kNVFP4) {
                // Two accumulators per row group (first / second mma of each
                // word) keep two mma chains in flight per row group.
                float d0[NRG][4], d1[NRG][4];
#pragma unroll
                for (int j = 0; j < NRG; ++j)
#pragma unroll
                    for (int i = 0; i < 4; ++i) d0[j][i] = d1[j][i] = 0.f;
#pragma unroll
                for (int si = 0; si < 2 * Cfg<FMT>::kBoxes / NKS; ++si) {
                    const int su = kh + NKS * si;        // this warp's 128-k super-steps of the unit
                    // 16 bytes (32 codes) of rows r0 and r1: box su / 2, chunk
                    // (4 su + c) % 8 of the 128-byte row, 128B-swizzled.
                    const uint8_t* cb = cs + (su >> 1) * kBox;
                    const int ch = (4 * su + c) & 7;
                    uint32_t wa[NRG][4], wb[NRG][4], slo[NRG][2], shi[NRG][2];
#pragma unroll
                    for (int j = 0; j < NRG; ++j) {
                        const uint4 w0 = *reinterpret_cast<const uint4*>(cb + r0[j] * 128 + ((ch ^ (r0[j] & 7)) << 4));
                        const uint4 w1 = *reinterpret_cast<const uint4*>(cb + r1[j] * 128 + ((ch ^ (r1[j] & 7)) << 4));
                        wa[j][0] = w0.x; wa[j][1] = w0.y; wa[j][2] = w0.z; wa[j][3] = w0.w;
                        wb[j][0] = w1.x; wb[j][1] = w1.y; wb[j][2] = w1.z; wb[j][3] = w1.w;
                        // Scales: 2 groups of 16 codes per row.
                        const uint32_t sb0 = *reinterpret_cast<const uint16_t*>(ss + r0[j] * SB + 8 * su + 2 * c);
                        const uint32_t sb1 = *reinterpret_cast<const uint16_t*>(ss + r1[j] * SB + 8 * su + 2 * c);
                        const uint32_t s0 = e4m3x2_to_f16x2((uint16_t)sb0), s1 = e4m3x2_to_f16x2((uint16_t)sb1);
                        slo[j][0] = __byte_perm(s0, 0, 0x1010); shi[j][0] = __byte_perm(s0, 0, 0x3232);
                        slo[j][1] = __byte_perm(s1, 0, 0x1010); shi[j][1] = __byte_perm(s1, 0, 0x3232);
                    }
#pragma unroll
                    for (int jp = 0; jp < 4; ++jp) {
                        const uint4 bx = *reinterpret_cast<const uint4*>(xf + ((su * 4 + jp) * 32 + lane) * 16);
#pragma unroll
                        for (int j = 0; j < NRG; ++j) {
                            // Word jp of rows r0 / r1 widened and scaled just before
                            // its mmas: ha[b] = f16x2 of byte 4 jp + b (codes 2b, 2b + 1).
                            uint32_t ha[4], hb[4];
                            e2m1x8_to_f16x2(wa[j][jp], ha);
                            e2m1x8_to_f16x2(wb[j][jp], hb);
                            const uint32_t sa = jp < 2 ? slo[j][0] : shi[j][0], sbv = jp < 2 ? slo[j][1] : shi[j][1];
#pragma unroll
                            for (int b2 = 0; b2 < 4; ++b2) {
                                ha[b2] = hmul2u(ha[b2], sa);
                                hb[b2] = hmul2u(hb[b2], sbv);
                            }
                            // step j = 2 jp + jj uses bytes 2j (codes 4j, 4j+1) and 2j + 1.
                            const uint32_t a0[4] = {ha[0], hb[0], ha[1], hb[1]};
                            const uint32_t a1[4] = {ha[2], hb[2], ha[3], hb[3]};
                            mma16816(d0[j], a0, bx.x, bx.y);
                            mma16816(d1[j], a1, bx.z, bx.w);
                        }
                    }
                }
#pragma unroll
                for (int j = 0; j < NRG; ++j) {
                    acc[j][0] = fmaf(d0[j][0] + d1[j][0], xs0, acc[j][0]);
                    acc[j][1] = fmaf(d0[j][1] + d1[j][1], xs1, acc[j][1]);
                    acc[j][2] = fmaf(d0[j][2] + d1[j][2], xs0, acc[j][2]);
                    acc[j][3] = fmaf(d0[j][3] + d1[j][3], xs1, acc[j][3]);
                }
            } else {
                // mxfp8: step j covers k [16j, 16j + 16) (one half group);
                // thread c owns bytes 16j + 4c .. + 3 of each row.
                const int soff = (SRC == kScaleCkpt) ? (kc & 1) * 8 : 0;   // the unit's 8 bytes in a 16-byte box row
                const uint32_t sw0 = *reinterpret_cast<const uint32_t*>(ss + r0[0] * SB + soff + 4 * kh);
                const uint32_t sw1 = *reinterpret_cast<const uint32_t*>(ss + r1[0] * SB + soff + 4 * kh);
#pragma unroll
                for (int gi = 0; gi < 4; ++gi) {
                    const int grp = 4 * kh + gi;         // this warp's four 32-code groups
                    float d[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        const int j = 2 * grp + h;
                        const uint8_t* cb = cs + (j >> 3) * kBox;
                        const uint32_t wa = *reinterpret_cast<const uint32_t*>(
                            cb + r0[0] * 128 + (((j & 7) ^ (r0[0] & 7)) << 4) + 4 * c);
                        const uint32_t wb = *reinterpret_cast<const uint32_t*>(
                            cb + r1[0] * 128 + (((j & 7) ^ (r1[0] & 7)) << 4) + 4 * c);
                        uint32_t a[4];
                        a[0] = e4m3x2_to_f16x2((uint16_t)(wa & 0xFFFF));
                        a[1] = e4m3x2_to_f16x2((uint16_t)(wb & 0xFFFF));
                        a[2] = e4m3x2_to_f16x2((uint16_t)(wa >> 16));
                        a[3] = e4m3x2_to_f16x2((uint16_t)(wb >> 16));
                        const uint2 b = *reinterpret_cast<const uint2*>(xf + ((grp * 32 + lane) * 16) + h * 8);
                        mma16816(d, a, b.x, b.y);
                    }
                    const float sc0 = ue8m0_to_f32((sw0 >> (8 * gi)) & 0xFF);
                    const float sc1 = ue8m0_to_f32((sw1 >> (8 * gi)) & 0xFF);
                    acc[0][0] = fmaf(d[0], sc0 * xs0, acc[0][0]);
                    acc[0][1] = fmaf(d[1], sc0 * xs1, acc[0][1]);
                    acc[0][2] = fmaf(d[2], sc1 * xs0, acc[0][2]);
                    acc[0][3] = fmaf(d[3], sc1 * xs1, acc[0][3]);
                }
            }
            }  // live
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);
            if (i == nunits - 1) {
                const bool complete = (kc == p.kchunks - 1) && (rb_first_unit == 0);
                flush(rb, complete);
            }
        }
        if constexpr (EPI == kEpiTp) tp_complete();
        if constexpr (EPI == kEpiArgmax) argmax_finish();
    }
    __syncthreads();
}

// ---- per-weight preparation -----------------------------------------------------

__global__ void retile_scales_kernel(const uint8_t* __restrict__ src, int64_t lds, int n, int ngroups,
                                     int kchunks, int row_blocks, int sb, uint8_t* __restrict__ dst) {
    // dst[((rb * kchunks + kc) * 128 + r) * sb + b] = src[(rb*128 + r) * lds + kc * sb + b] (0 outside).
    const int64_t total = (int64_t)row_blocks * kchunks * kRows * sb;
    for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
        const int b = (int)(t % sb);
        int64_t rest = t / sb;
        const int r = (int)(rest % kRows);
        rest /= kRows;
        const int kc = (int)(rest % kchunks);
        const int rb = (int)(rest / kchunks);
        const int row = rb * kRows + r, grp = kc * sb + b;
        dst[t] = (row < n && grp < ngroups) ? src[(int64_t)row * lds + grp] : (uint8_t)0;
    }
}

PFN_cuTensorMapEncodeTiled_v12000 encoder() {
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

template <int FMT, int SRC = kScaleTiled>
constexpr int smem_bytes() {
    return 1024 + Cfg<FMT>::kStages * (Cfg<FMT>::kBoxes * kBox + ScaleLayout<FMT, SRC>::kBytes +
                                       2 * kXRows * Cfg<FMT>::KC * 2 + 8 * 4) +
           ((FMT == kNVFP4 ? kNvSlices : 2) - 1) * kRows * 8 * 4 + 512;
}

using GemvTcKernel = void (*)(CUtensorMap, CUtensorMap, CUtensorMap, TcParams);

// Up-front L2 prefetch of each CTA's weight range beyond its ring: off unless
// QMM_L2_PREFETCH=1 (measured slower on config 2 and the lm_head).
int l2_prefetch_enabled() {
    static const int on = [] {
        const char* e = getenv("QMM_L2_PREFETCH");
        return (e && e[0] == '1') ? 1 : 0;
    }();
    return on;
}

// Empty schedule slots after each row block (TcParams::gap).  A CTA whose
// unit range holds a row-block boundary flushes that block mid-stream (the
// k-slice hand-over, the partial write and the counter step), which costs
// about one unit's time while the other CTAs stream on; counting it as
// kFlushSlots units gives those CTAs that many fewer units.  Off when a CTA
// would own fewer than kFlushSlots + 2 slots: a shorter range could then
// lie entirely in a gap and own no unit.
constexpr int kFlushSlots = 1;
int flush_slots(int64_t units, int64_t row_blocks, int64_t grid) {
    return units + row_blocks * kFlushSlots >= grid * (kFlushSlots + 2) ? kFlushSlots : 0;
}

// CTAs of a launch: stream-K over every SM, except for short rows.  With at
// most kShortChunks units per row block (a K-shard of an 8-way split, say)
// and fewer row blocks than SMs, one CTA per row block needs no stream-K
// fix-up at all, which measured faster than spreading the units over every
// SM ([5120, 2176] nvfp4, M = 1: 7.7 -> 6.2 us); at 9 units per row block it
// measured slower (8.7 -> 9.7 us).  Every launch path uses this rule, so a
// shape gets the same work split - and the same bits - whichever entry point
// runs it.
constexpr int kShortChunks = 5;
int64_t decode_grid(int64_t units, int64_t row_blocks, int64_t kchunks, int64_t sms) {
    if (kchunks <= kShortChunks && row_blocks < sms) return row_blocks;
    return std::min<int64_t>(units, sms);
}

// Kernel for a format, M, epilogue and scale source, with its dynamic shared
// memory configured once per device.  nvfp4 takes the group-slot x layout
// for M <= 2 (the scale leaves the per-code path); QMM_XL=0 keeps the token
// layout (for A/B runs).  Checkpoint-layout scales (stateless calls) come
// with the plain epilogue only.
int pick_kernel(int fmt, int64_t m, int epi, int src, int dev, GemvTcKernel* fn, int* smem) {
    static const bool tokens_only = [] {
        const char* e = getenv("QMM_XL");
        return e && e[0] == '0';
    }();
    // One table row per (format / layout), one column per epilogue, then the
    // checkpoint-scale plain kernels.
    static const GemvTcKernel table[3][5] = {
        {qmm_gemv_tc_kernel<kMXFP8, kXlTokens, kEpiPlain, kScaleTiled>,
         qmm_gemv_tc_kernel<kMXFP8, kXlTokens, kEpiSwiglu, kScaleTiled>,
         qmm_gemv_tc_kernel<kMXFP8, kXlTokens, kEpiArgmax, kScaleTiled>,
         qmm_gemv_tc_kernel<kMXFP8, kXlTokens, kEpiTp, kScaleTiled>,
         qmm_gemv_tc_kernel<kMXFP8, kXlTokens, kEpiPlain, kScaleCkpt>},
        {qmm_gemv_tc_kernel<kNVFP4, kXlGroups2, kEpiPlain, kScaleTiled>,
         qmm_gemv_tc_kernel<kNVFP4, kXlGroups2, kEpiSwiglu, kScaleTiled>,
         qmm_gemv_tc_kernel<kNVFP4, kXlGroups2, kEpiArgmax, kScaleTiled>,
         qmm_gemv_tc_kernel<kNVFP4, kXlGroups2, kEpiTp, kScaleTiled>,
         qmm_gemv_tc_kernel<kNVFP4, kXlGroups2, kEpiPlain, kScaleCkpt>},
        {qmm_gemv_tc_kernel<kNVFP4, kXlTokens, kEpiPlain, kScaleTiled>,
         qmm_gemv_tc_kernel<kNVFP4, kXlTokens, kEpiSwiglu, kScaleTiled>,
         qmm_gemv_tc_kernel<kNVFP4, kXlTokens, kEpiArgmax, kScaleTiled>,
         qmm_gemv_tc_kernel<kNVFP4, kXlTokens, kEpiTp, kScaleTiled>,
         qmm_gemv_tc_kernel<kNVFP4, kXlTokens, kEpiPlain, kScaleCkpt>},
    };
    if (src == kScaleCkpt && epi != kEpiPlain)
        return set_error(QMM_ERR_BAD_ARGUMENT, "checkpoint-layout scales run the plain epilogue only");
    const int row = fmt == kMXFP8 ? 0 : (!tokens_only && m <= 2) ? 1 : 2;
    const int col = src == kScaleCkpt ? 4 : epi;
    if (fmt == kMXFP8)
        *smem = src == kScaleCkpt ? smem_bytes<kMXFP8, kScaleCkpt>() : smem_bytes<kMXFP8>();
    else
        *smem = src == kScaleCkpt ? smem_bytes<kNVFP4, kScaleCkpt>() : smem_bytes<kNVFP4>();
    *fn = table[row][col];
    const int slot = row * 5 + col;
    static std::mutex mu;
    static bool configured[15][64] = {};
    if (dev < 0 || dev >= 64) return set_error(QMM_ERR_BAD_ARGUMENT, "device %d is out of range", dev);
    std::lock_guard<std::mutex> lock(mu);
    if (!configured[slot][dev]) {
        QMM_CUDA_TRY(cudaFuncSetAttribute(*fn, cudaFuncAttributeMaxDynamicSharedMemorySize, *smem));
        configured[slot][dev] = true;
    }
    return QMM_OK;
}

}  // namespace

struct GemvTcState {
    CUtensorMap cmap;
    uint8_t* scales_tiled = nullptr;
    float* partial = nullptr;
    unsigned int* counters = nullptr;
    // Greedy sampling: [8] keys + the CTA count (one allocation), and the
    // half-block (max, sum exp) pairs [row_blocks][8][2].
    unsigned long long* am_keys = nullptr;
    float2* am_part = nullptr;
    int grid = 0, kchunks = 0, row_blocks = 0;
};

int gemv_tc_prepare(qmm_weight* w, cudaStream_t stream) {
    w->tc = nullptr;
    const int fmt = format_of(w->spec);
    const int KC = fmt == kMXFP8 ? Cfg<kMXFP8>::KC : Cfg<kNVFP4>::KC;
    const int SB = fmt == kMXFP8 ? Cfg<kMXFP8>::SB : Cfg<kNVFP4>::SB;
    if (w->n <= 0 || w->n > INT32_MAX || w->k > INT32_MAX) return QMM_OK;
    auto enc = encoder();
    if (!enc) return QMM_OK;
    DeviceInfo info;
    if (int rc = device_info(w->device, &info)) return rc;
    if (info.smem_optin < (size_t)smem_bytes<kNVFP4>()) return QMM_OK;
    GemvTcState* st = new GemvTcState();
    st->kchunks = (int)((w->k + KC - 1) / KC);
    st->row_blocks = (int)((w->n + kRows - 1) / kRows);
    const int64_t units = (int64_t)st->kchunks * st->row_blocks;
    if (units > INT32_MAX) { delete st; return QMM_OK; }
    st->grid = (int)decode_grid(units, st->row_blocks, st->kchunks, info.sms);
    const int64_t row_bytes = w->k * w->spec.bits / 8;
    const cuuint64_t gdim[2] = {(cuuint64_t)row_bytes, (cuuint64_t)w->n};
    const cuuint64_t gstride[1] = {(cuuint64_t)w->ldc};
    const cuuint32_t box[2] = {128, (cuuint32_t)kRows};
    const cuuint32_t es[2] = {1, 1};
    if (enc(&st->cmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, w->codes, gdim, gstride, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS) {
        delete st;
        return QMM_OK;
    }
    const size_t tiled = (size_t)units * kRows * SB;
    auto fail = [&](cudaError_t e, const char* what) {
        cudaFree(st->scales_tiled);
        cudaFree(st->partial);
        cudaFree(st->counters);
        cudaFree(st->am_keys);
        cudaFree(st->am_part);
        delete st;
        return cuda_error(e, what);
    };
    cudaError_t e;
    if ((e = cudaMalloc(&st->scales_tiled, tiled)) != cudaSuccess) return fail(e, "cudaMalloc(scales_tiled)");
    if ((e = cudaMalloc(&st->partial, (size_t)st->grid * 2 * kRows * 8 * sizeof(float))) != cudaSuccess)
        return fail(e, "cudaMalloc(partial)");
    if ((e = cudaMalloc(&st->counters, (size_t)st->row_blocks * sizeof(unsigned int))) != cudaSuccess)
        return fail(e, "cudaMalloc(counters)");
    if ((e = cudaMemsetAsync(st->counters, 0, (size_t)st->row_blocks * sizeof(unsigned int), stream)) != cudaSuccess)
        return fail(e, "cudaMemsetAsync(counters)");
    // Greedy-sampling state: 8 keys + the CTA count, zero between calls.
    if ((e = cudaMalloc(&st->am_keys, 9 * sizeof(unsigned long long))) != cudaSuccess)
        return fail(e, "cudaMalloc(argmax keys)");
    if ((e = cudaMemsetAsync(st->am_keys, 0, 9 * sizeof(unsigned long long), stream)) != cudaSuccess)
        return fail(e, "cudaMemsetAsync(argmax keys)");
    if ((e = cudaMalloc(&st->am_part, (size_t)st->row_blocks * 16 * sizeof(float2))) != cudaSuccess)
        return fail(e, "cudaMalloc(argmax partials)");
    const int64_t total = (int64_t)tiled;
    const unsigned grid = (unsigned)std::min<int64_t>((total + 255) / 256, (int64_t)info.sms * 8);
    retile_scales_kernel<<<grid, 256, 0, stream>>>(w->scales, w->lds, (int)w->n, (int)(w->k / w->spec.group_size),
                                                   st->kchunks, st->row_blocks, SB, st->scales_tiled);
    if ((e = cudaGetLastError()) != cudaSuccess) return fail(e, "retile_scales_kernel");
    w->tc = st;
    return QMM_OK;
}

cudaError_t gemv_tc_take_error(unsigned int* v, cudaStream_t s) {
    unsigned int zero = 0;
    cudaError_t e = cudaMemcpyFromSymbolAsync(v, g_gemv_tc_error, sizeof(*v), 0, cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e == cudaSuccess && *v) {
        e = cudaMemcpyToSymbolAsync(g_gemv_tc_error, &zero, sizeof(zero), 0, cudaMemcpyHostToDevice, s);
        if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    }
    return e;
}

void gemv_tc_release(qmm_weight* w) {
    if (!w->tc) return;
    cudaFree(w->tc->scales_tiled);
    cudaFree(w->tc->partial);
    cudaFree(w->tc->counters);
    cudaFree(w->tc->am_keys);
    cudaFree(w->tc->am_part);
    delete w->tc;
    w->tc = nullptr;
}

int launch_gemv_tc(const qmm_weight* w, const QmmArgs& a, cudaStream_t stream, bool* handled) {
    *handled = false;
    const GemvTcState* st = w->tc;
    if (!st || a.m < 1 || a.m > kXRows) return QMM_OK;
    const auto xa = reinterpret_cast<uintptr_t>(a.x);
    if ((xa & 15) || ((a.ldx * 2) & 15)) return QMM_OK;
    const int fmt = a.fmt;
    CUtensorMap xmap;
    const cuuint64_t gdim[2] = {(cuuint64_t)a.k, (cuuint64_t)a.m};
    const cuuint64_t gstride[1] = {(cuuint64_t)(a.ldx * 2)};
    const cuuint32_t box[2] = {256u, (cuuint32_t)a.m};   // M rows: no zero-filled rows in shared memory
    const cuuint32_t es[2] = {1, 1};
    if (encoder()(&xmap, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<uint16_t*>(a.x), gdim, gstride, box, es,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return QMM_OK;
    TcParams p;
    p.scales_tiled = st->scales_tiled;
    p.y = a.y;
    p.yf = a.yf;
    p.tp_n = 0;
    if (a.tp && a.tp->nranks > 1) {
        p.tp_n = a.tp->nranks;
        p.tp_rank = a.tp->rank;
        p.tp_max_rb = a.tp->max_rb;
        p.tp_cap = a.tp->cap;
        for (int r = 0; r < kMaxTpRanks; ++r) {
            p.tp_recv[r] = a.tp->recv[r];
            p.tp_flags[r] = a.tp->flags[r];
        }
        p.tp_gen = a.tp->gen;
        p.yf = nullptr;
    }
    p.swiglu_n = (int)a.swiglu_n;
    if (a.swiglu_n > 0 && (p.tp_n > 0 || a.yf)) return QMM_OK;   // not combined with the exchange or fp32 output
    p.am_ids = a.argmax_ids;
    p.am_lp = a.argmax_lp;
    p.am_keys = st->am_keys;
    p.am_part = st->am_part;
    p.am_done = reinterpret_cast<unsigned int*>(st->am_keys + 8);
    if (a.argmax_ids && (p.tp_n > 0 || a.yf || a.swiglu_n > 0)) return QMM_OK;
    p.l2_prefetch = l2_prefetch_enabled();
    p.partial = st->partial;
    p.counters = st->counters;
    p.ldy = a.ldy;
    p.m = (int)a.m;
    p.n = (int)a.n;
    p.k = (int)a.k;
    p.kchunks = st->kchunks;
    p.row_blocks = st->row_blocks;
    p.units = st->kchunks * st->row_blocks;
    p.gap = flush_slots(p.units, p.row_blocks, st->grid);
    // Programmatic dependent launch: the kernel may start while the previous
    // kernel on the stream finishes; it streams its first weight tiles, then
    // waits (griddepcontrol.wait) before reading x or writing anything.
    // QMM_NO_PDL=1 launches in plain stream order.
    static const bool pdl = [] {
        const char* e = getenv("QMM_NO_PDL");
        return !(e && e[0] == '1');
    }();
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)st->grid);
    cfg.blockDim = dim3(kThreads);
    cfg.stream = stream;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    GemvTcKernel fn = nullptr;
    int smem = 0;
    const int epi = a.argmax_ids ? kEpiArgmax : a.swiglu_n > 0 ? kEpiSwiglu : p.tp_n > 1 ? kEpiTp : kEpiPlain;
    if (int rc = pick_kernel(fmt, a.m, epi, kScaleTiled, w->device, &fn, &smem)) return rc;
    cfg.dynamicSmemBytes = smem;
    QMM_CUDA_TRY(cudaLaunchKernelEx(&cfg, fn, st->cmap, xmap, st->cmap, p));   // smap unused (tiled scales)
    QMM_CUDA_TRY(cudaGetLastError());
    *handled = true;
    return QMM_OK;
}

// ---- static-scratch variant (allocates nothing) ------------------------------------
//
// The same decode kernel run on the caller's packed weights in the checkpoint
// layout, with every scratch buffer (per-unit scale tiles, stream-K partial
// sums, row-block counters) carved from one file-scope device array instead
// of per-weight allocations.  The array's address is looked up once per
// device (cudaGetSymbolAddress, that device current).  Calls that overlap in
// time on one device share the array and race; after a call the array keeps
// that call's contents.

namespace {
constexpr size_t kStaticScratchBytes = size_t(8) << 20;  // 8 MiB per device
__device__ __align__(256) uint8_t g_static_scratch[kStaticScratchBytes];

int static_scratch_base(int dev, uint8_t** base) {
    static std::mutex mu;
    static uint8_t* addr[64] = {};
    if (dev < 0 || dev >= 64) return set_error(QMM_ERR_BAD_ARGUMENT, "device %d is out of range", dev);
    std::lock_guard<std::mutex> lock(mu);
    if (!addr[dev]) {
        void* p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_static_scratch);
        if (e != cudaSuccess) return cuda_error(e, "cudaGetSymbolAddress(static scratch)");
        addr[dev] = static_cast<uint8_t*>(p);
    }
    *base = addr[dev];
    return QMM_OK;
}
}  // namespace

int launch_gemv_tc_static(const QmmArgs& a, cudaStream_t stream, bool* handled) {
    *handled = false;
    if (a.yf || a.m < 1 || a.m > kXRows) return QMM_OK;
    if (a.n <= 0 || a.n > INT32_MAX || a.k > INT32_MAX) return QMM_OK;
    // TMA envelope: 16-byte aligned x and code rows.
    const auto xa = reinterpret_cast<uintptr_t>(a.x), ca = reinterpret_cast<uintptr_t>(a.codes);
    if ((xa & 15) || ((a.ldx * 2) & 15) || (ca & 15) || (a.ldc & 15)) return QMM_OK;
    auto enc = encoder();
    if (!enc) return QMM_OK;
    int dev = 0;
    QMM_CUDA_TRY(cudaGetDevice(&dev));
    DeviceInfo info;
    if (int rc = device_info(dev, &info)) return rc;
    if (info.smem_optin < (size_t)smem_bytes<kNVFP4>()) return QMM_OK;

    const int fmt = a.fmt;
    const int KC = fmt == kMXFP8 ? Cfg<kMXFP8>::KC : Cfg<kNVFP4>::KC;
    const int SB = fmt == kMXFP8 ? Cfg<kMXFP8>::SB : Cfg<kNVFP4>::SB;
    const int group = fmt == kMXFP8 ? 32 : 16;
    const int64_t kchunks = (a.k + KC - 1) / KC, row_blocks = (a.n + kRows - 1) / kRows;
    const int64_t units = kchunks * row_blocks;
    const int64_t grid = decode_grid(units, row_blocks, kchunks, info.sms);
    auto align256 = [](int64_t v) { return (v + 255) / 256 * 256; };
    const int64_t tiled_bytes = units * kRows * SB;
    const int64_t partial_off = align256(tiled_bytes);
    const int64_t counters_off = align256(partial_off + grid * 2 * kRows * 8 * (int64_t)sizeof(float));
    const int64_t need = counters_off + row_blocks * (int64_t)sizeof(unsigned int);
    if (need > (int64_t)kStaticScratchBytes)
        return set_error(QMM_ERR_OUT_OF_MEMORY,
                         "[%lld, %lld] weight needs %lld bytes of static scratch; the maximum is %zu (8 MiB)",
                         (long long)a.n, (long long)a.k, (long long)need, kStaticScratchBytes);
    uint8_t* base = nullptr;
    if (int rc = static_scratch_base(dev, &base)) return rc;

    CUtensorMap cmap, xmap;
    {
        const cuuint64_t gdim[2] = {(cuuint64_t)(a.k * (fmt == kMXFP8 ? 8 : 4) / 8), (cuuint64_t)a.n};
        const cuuint64_t gstride[1] = {(cuuint64_t)a.ldc};
        const cuuint32_t box[2] = {128, (cuuint32_t)kRows};
        const cuuint32_t es[2] = {1, 1};
        if (enc(&cmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t*>(a.codes), gdim, gstride, box, es,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return QMM_OK;
    }
    {
        const cuuint64_t gdim[2] = {(cuuint64_t)a.k, (cuuint64_t)a.m};
        const cuuint64_t gstride[1] = {(cuuint64_t)(a.ldx * 2)};
        const cuuint32_t box[2] = {256u, (cuuint32_t)a.m};
        const cuuint32_t es[2] = {1, 1};
        if (enc(&xmap, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<uint16_t*>(a.x), gdim, gstride, box, es,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return QMM_OK;
    }

    // The counters must start at zero (a call that gave up a wait can leave
    // them set); the scale tiles are rebuilt from the checkpoint layout.
    unsigned int* counters = reinterpret_cast<unsigned int*>(base + counters_off);
    QMM_CUDA_TRY(cudaMemsetAsync(counters, 0, (size_t)row_blocks * sizeof(unsigned int), stream));
    const unsigned rgrid = (unsigned)std::min<int64_t>((tiled_bytes + 255) / 256, (int64_t)info.sms * 8);
    retile_scales_kernel<<<rgrid, 256, 0, stream>>>(a.scales, a.lds, (int)a.n, (int)(a.k / group), (int)kchunks,
                                                    (int)row_blocks, SB, base);
    QMM_CUDA_TRY(cudaGetLastError());

    TcParams p;
    p.scales_tiled = base;
    p.y = a.y;
    p.yf = nullptr;
    p.tp_n = 0;
    p.swiglu_n = 0;
    p.am_ids = nullptr;
    p.am_lp = nullptr;
    p.l2_prefetch = l2_prefetch_enabled();
    p.partial = reinterpret_cast<float*>(base + partial_off);
    p.counters = counters;
    p.ldy = a.ldy;
    p.m = (int)a.m;
    p.n = (int)a.n;
    p.k = (int)a.k;
    p.kchunks = (int)kchunks;
    p.row_blocks = (int)row_blocks;
    p.units = (int)units;
    p.gap = flush_slots(units, row_blocks, grid);
    GemvTcKernel fn = nullptr;
    int smem = 0;
    if (int rc = pick_kernel(fmt, a.m, kEpiPlain, kScaleTiled, dev, &fn, &smem)) return rc;
    fn<<<(unsigned)grid, kThreads, smem, stream>>>(cmap, xmap, cmap, p);   // smap unused (tiled scales)
    QMM_CUDA_TRY(cudaGetLastError());
    *handled = true;
    return QMM_OK;
}

}  // namespace qmm

// ---- stateless calls on checkpoint-layout tensors ------------------------------
//
// qmm_quantized_matmul (the mlx_quantized_matmul counterpart) runs the same
// decode kernel on the caller's U32 codes and U8 scales as they lie in the
// checkpoint: codes by the 2D TMA boxes of the resident path, scales by 2D
// TMA boxes of the [N, K/group] tensor (no re-tiled copy).  The stream-K
// partial sums and row-block counters live in a workspace owned by the
// library, one per (device, stream), made on the first call on that stream
// and kept until the process exits: calls on one stream are ordered, calls on
// different streams use different workspaces.  The counters return to zero at
// the end of every call; after a kernel that gave up a bounded wait
// (qmm_device_status reports Timeout) every workspace is zeroed again before
// its next use.

namespace qmm {
namespace {

constexpr int64_t kWsMaxRowBlocks = int64_t(1) << 16;   // N up to 8,388,608 rows

struct StreamWorkspace {
    float* partial = nullptr;           // [grid][2][128][8]
    unsigned int* counters = nullptr;   // [kWsMaxRowBlocks]
    int grid = 0;
    uint64_t zeroed_gen = 0;            // dirty generation the counters were zeroed at
};

std::mutex g_ws_mu;
std::map<std::pair<int, cudaStream_t>, StreamWorkspace> g_ws;
std::atomic<uint64_t> g_ws_dirty_gen{1};

int stream_workspace(int dev, cudaStream_t stream, int sms, StreamWorkspace** out) {
    std::lock_guard<std::mutex> lock(g_ws_mu);
    auto it = g_ws.find({dev, stream});
    if (it == g_ws.end()) {
        cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
        QMM_CUDA_TRY(cudaStreamIsCapturing(stream, &cs));
        if (cs != cudaStreamCaptureStatusNone)
            return set_error(QMM_ERR_BAD_ARGUMENT,
                             "the first qmm_quantized_matmul call on a stream allocates its workspace and cannot be "
                             "captured: make one call on this stream before capturing it");
        StreamWorkspace ws;
        ws.grid = sms;
        cudaError_t e = cudaMalloc(&ws.partial, (size_t)sms * 2 * kRows * 8 * sizeof(float));
        if (e == cudaSuccess) e = cudaMalloc(&ws.counters, (size_t)kWsMaxRowBlocks * sizeof(unsigned int));
        if (e != cudaSuccess) {
            cudaFree(ws.partial);
            return cuda_error(e, "cudaMalloc(stateless workspace)");
        }
        it = g_ws.emplace(std::make_pair(dev, stream), ws).first;
    }
    StreamWorkspace& ws = it->second;
    const uint64_t gen = g_ws_dirty_gen.load();
    if (ws.zeroed_gen != gen) {
        QMM_CUDA_TRY(cudaMemsetAsync(ws.counters, 0, (size_t)kWsMaxRowBlocks * sizeof(unsigned int), stream));
        ws.zeroed_gen = gen;
    }
    *out = &ws;
    return QMM_OK;
}

}  // namespace

void gemv_tc_mark_workspaces_dirty() { g_ws_dirty_gen.fetch_add(1); }

int launch_gemv_tc_ckpt(const QmmArgs& a, cudaStream_t stream, bool* handled) {
    *handled = false;
    if (a.yf || a.m < 1 || a.m > kXRows) return QMM_OK;
    if (a.n <= 0 || a.n > INT32_MAX || a.k > INT32_MAX) return QMM_OK;
    const int fmt = a.fmt;
    const int KC = fmt == kMXFP8 ? Cfg<kMXFP8>::KC : Cfg<kNVFP4>::KC;
    const int group = fmt == kMXFP8 ? 32 : 16;
    const int64_t ngroups = a.k / group;
    const int64_t row_blocks = (a.n + kRows - 1) / kRows, kchunks = (a.k + KC - 1) / KC;
    // TMA envelope: 16-byte aligned x / code / scale rows.
    const auto xa = reinterpret_cast<uintptr_t>(a.x), ca = reinterpret_cast<uintptr_t>(a.codes),
               sa = reinterpret_cast<uintptr_t>(a.scales);
    if ((xa & 15) || ((a.ldx * 2) & 15) || (ca & 15) || (a.ldc & 15) || (sa & 15) || (a.lds & 15)) return QMM_OK;
    if (row_blocks > kWsMaxRowBlocks || kchunks * row_blocks > INT32_MAX) return QMM_OK;
    auto enc = encoder();
    if (!enc) return QMM_OK;
    int dev = 0;
    QMM_CUDA_TRY(cudaGetDevice(&dev));
    DeviceInfo info;
    if (int rc = device_info(dev, &info)) return rc;
    if (info.smem_optin < (size_t)smem_bytes<kNVFP4, kScaleCkpt>()) return QMM_OK;
    CUtensorMap cmap, xmap, smap;
    {
        const cuuint64_t gdim[2] = {(cuuint64_t)(a.k * (fmt == kMXFP8 ? 8 : 4) / 8), (cuuint64_t)a.n};
        const cuuint64_t gstride[1] = {(cuuint64_t)a.ldc};
        const cuuint32_t box[2] = {128, (cuuint32_t)kRows};
        const cuuint32_t es[2] = {1, 1};
        if (enc(&cmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t*>(a.codes), gdim, gstride, box, es,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return QMM_OK;
    }
    {
        const cuuint64_t gdim[2] = {(cuuint64_t)a.k, (cuuint64_t)a.m};
        const cuuint64_t gstride[1] = {(cuuint64_t)(a.ldx * 2)};
        const cuuint32_t box[2] = {256u, (cuuint32_t)a.m};
        const cuuint32_t es[2] = {1, 1};
        if (enc(&xmap, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<uint16_t*>(a.x), gdim, gstride, box, es,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return QMM_OK;
    }
    {
        // One unit's scales: 128 rows of SB bytes (nvfp4: 32), or of a 16-byte
        // box holding the unit's 8 bytes (mxfp8).
        const cuuint64_t gdim[2] = {(cuuint64_t)ngroups, (cuuint64_t)a.n};
        const cuuint64_t gstride[1] = {(cuuint64_t)a.lds};
        const cuuint32_t box[2] = {fmt == kMXFP8 ? 16u : (cuuint32_t)Cfg<kNVFP4>::SB, (cuuint32_t)kRows};
        const cuuint32_t es[2] = {1, 1};
        if (enc(&smap, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t*>(a.scales), gdim, gstride, box, es,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return QMM_OK;
    }
    StreamWorkspace* ws = nullptr;
    if (int rc = stream_workspace(dev, stream, info.sms, &ws)) return rc;
    const int64_t units = kchunks * row_blocks;
    const int grid = (int)std::min<int64_t>(decode_grid(units, row_blocks, kchunks, info.sms), ws->grid);
    TcParams p;
    p.scales_tiled = nullptr;
    p.y = a.y;
    p.yf = nullptr;
    p.tp_n = 0;
    p.swiglu_n = 0;
    p.am_ids = nullptr;
    p.am_lp = nullptr;
    p.l2_prefetch = l2_prefetch_enabled();
    p.partial = ws->partial;
    p.counters = ws->counters;
    p.ldy = a.ldy;
    p.m = (int)a.m;
    p.n = (int)a.n;
    p.k = (int)a.k;
    p.kchunks = (int)kchunks;
    p.row_blocks = (int)row_blocks;
    p.units = (int)units;
    p.gap = flush_slots(units, row_blocks, grid);
    GemvTcKernel fn = nullptr;
    int smem = 0;
    if (int rc = pick_kernel(fmt, a.m, kEpiPlain, kScaleCkpt, dev, &fn, &smem)) return rc;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    QMM_CUDA_TRY(cudaLaunchKernelEx(&cfg, fn, cmap, xmap, smap, p));
    QMM_CUDA_TRY(cudaGetLastError());
    *handled = true;
    return QMM_OK;
}

}  // namespace qmm
