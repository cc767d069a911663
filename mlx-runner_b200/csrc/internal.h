// internal.h - host-side declarations shared by the library's translation units.
#pragma once

#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

#include "qmm.h"

struct qmm_weight;

namespace qmm {

// ---- error latch (src/mlx.zig:719-805 restated for a C ABI) --------------
// The first failure since the last qmm_last_error() wins; later ones are
// dropped so follow-on noise cannot hide the cause.  Returns `status`.
int set_error(int status, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
// Translate a CUDA error into QMM_ERR_CUDA / QMM_ERR_OUT_OF_MEMORY + latch.
int cuda_error(cudaError_t e, const char* what);
// The fault-injection hook: true when the armed k-th checked call is this one.
bool fault_hit();

#define QMM_CUDA_TRY(expr)                                            \
    do {                                                              \
        cudaError_t _e = (expr);                                      \
        if (_e != cudaSuccess) return ::qmm::cuda_error(_e, #expr);   \
    } while (0)

// ---- formats ----------------------------------------------------------------
enum Format : int { kMXFP8 = 0, kNVFP4 = 1 };

inline int format_of(const qmm_quant_spec& s) { return s.mode == QMM_MODE_MXFP8 ? kMXFP8 : kNVFP4; }
// Validates (mode, group, bits) against the two supported pairs.
int check_spec(const qmm_quant_spec& s);

// Device properties cached per device (SM count, compute capability).
struct DeviceInfo {
    int sms = 0;
    int major = 0, minor = 0;
    size_t smem_optin = 0;
};
int device_info(int device, DeviceInfo* out);
// QMM_OK when p is NULL, or device / managed memory that device `dev` can
// use; BadArgument (naming `what`) for host memory or another GPU's buffer.
int check_device_buffer(const void* p, int dev, const char* what);

// ---- kernels -----------------------------------------------------------------
// Peer-memory exchange of a row-parallel (K-sharded) decode: every rank's
// final fp32 row-block sums go straight into every rank's receive buffer over
// NVLink and are added there in rank order (gemv_tc.cu).
constexpr int kMaxTpRanks = 8;
struct TpExchange {
    int nranks = 0, rank = 0, max_rb = 0;
    int64_t cap = 0;                           // floats per (parity, source) receive slot
    float* recv[kMaxTpRanks] = {};             // rank r's receive buffer [2][nranks][cap]
    unsigned int* flags[kMaxTpRanks] = {};     // rank r's flags [nranks][max_rb] (epochs)
    unsigned int* gen = nullptr;               // this rank's per-row-block epoch counters [max_rb]
};

// Operands of one y = x . dequant(W)^T call, all device pointers.
struct QmmArgs {
    int fmt;                 // Format
    const uint8_t* codes;    // [n][ldc] bytes, K*bits/8 meaningful per row
    int64_t ldc;             // bytes between code rows
    const uint8_t* scales;   // [n][lds] bytes, K/group per row
    int64_t lds;
    const uint16_t* x;       // bf16 [m][ldx]
    int64_t ldx;             // elements
    uint16_t* y;             // bf16 [m][ldy]
    int64_t ldy;             // elements
    float* yf = nullptr;     // when set: fp32 output [m][ldy] instead of y
    const TpExchange* tp = nullptr;  // when set: row-parallel shard summed across ranks into y
    // When > 0: W rows are gate / up interleaved in 64-row blocks (rows
    // [128 b, 128 b + 64) = gate rows [64 b, 64 b + 64), the next 64 the
    // matching up rows) and y receives silu(gate) * up, [m][swiglu_n].
    int64_t swiglu_n = 0;
    // When set (decode kernel, M <= 8): greedy sampling of each x row -
    // argmax_ids[m] = the index of the largest bf16 output (lowest index
    // among equals, NaN above all), argmax_lp[m] (nullable) = that output
    // minus logsumexp over the row; y (nullable here) still receives the
    // bf16 outputs when set.
    int32_t* argmax_ids = nullptr;
    float* argmax_lp = nullptr;
    int64_t m, n, k;
};

// Greedy sampling over bf16 rows already in memory (the unfused path):
// ids[r] / lp[r] for logits [m][ldl] of n columns, one CTA per row.
int launch_argmax_rows(const uint16_t* logits, int64_t ldl, int64_t m, int64_t n, int32_t* ids, float* lp,
                       cudaStream_t stream);

// Gate / up interleaving of one packed tensor pair (codes or scales, `pitch`
// bytes per row, n_half rows each) into dst [2 * npad][pitch]; rows past
// n_half stay as dst holds them (the caller zeroes them).
int launch_interleave_rows(const uint8_t* gate, const uint8_t* up, int64_t pitch, int64_t n_half, int64_t npad,
                           uint8_t* dst, cudaStream_t stream);
// h[m][n_half] = silu(gate) * up from an interleaved bf16 y [m][ldy] (the
// unfused path for shapes outside the fused kernels' envelope).
int launch_swiglu_apply(const uint16_t* y, int64_t ldy, int64_t m, int64_t n_half, uint16_t* h, int64_t ldh,
                        cudaStream_t stream);

// Split-K GEMV for m <= 8 (decode / MTP verify).  No workspace: the split-K
// partials are reduced through distributed shared memory inside a cluster.
int launch_gemv(const QmmArgs& a, cudaStream_t stream);
int gemv_max_m();

// Dequantize W into out[n][k] (bf16 if out_bf16 else fp32), row stride k.
int launch_dequant(int fmt, const uint8_t* codes, int64_t ldc, const uint8_t* scales,
                   int64_t lds, int64_t n, int64_t k, void* out, bool out_bf16,
                   cudaStream_t stream);

// Quantize w[n][ldw] (fp32, or bf16 when w_bf16) into MLX's packed codes
// [n][k*bits/8] bytes and scales [n][k/group] (quantize.cu).
int launch_quantize(int fmt, const void* w, bool w_bf16, int64_t ldw, int64_t n, int64_t k, uint8_t* codes,
                    uint8_t* scales, cudaStream_t stream);

// Prefill GEMM (m > 8) on the tcgen05 tensor cores.  Returns QMM_OK or an
// error; *handled = false when the shape is outside the kernel's envelope
// (the caller then uses the GEMV path over row blocks).
int launch_gemm(const QmmArgs& a, cudaStream_t stream, bool* handled);

// Route one call to the right kernel family (`w` is the resident weight the
// operands come from, or null for the stateless entry point).
int dispatch(const QmmArgs& a, cudaStream_t stream, const qmm_weight* w = nullptr);

// TMA-fed tensor-core GEMV for resident weights (gemv_tc.cu): per-weight
// state (codes tensor map, per-unit scale tiles, stream-K scratch) is made
// at weight creation; *handled = false when the call is outside its envelope.
struct GemvTcState;
int gemv_tc_prepare(qmm_weight* w, cudaStream_t stream);
void gemv_tc_release(qmm_weight* w);
int launch_gemv_tc(const qmm_weight* w, const QmmArgs& a, cudaStream_t stream, bool* handled);
// The same kernel on checkpoint-layout weights with its scratch in a static
// device array (no allocation); errors if the weight needs more than it holds.
int launch_gemv_tc_static(const QmmArgs& a, cudaStream_t stream, bool* handled);
// The same kernel on checkpoint-layout weights and scales (TMA boxes of the
// caller's tensors) with its stream-K scratch in a per-(device, stream)
// workspace made on the first call on that stream (not during capture).
int launch_gemv_tc_ckpt(const QmmArgs& a, cudaStream_t stream, bool* handled);
// After a kernel gave up a bounded wait: zero every workspace's counters
// before its next use.
void gemv_tc_mark_workspaces_dirty();
// Read and clear the kernel's device-side timeout word (synchronizes s).
cudaError_t gemv_tc_take_error(unsigned int* v, cudaStream_t s);

// x-quantised prefill GEMM on the block-scaled tensor cores (gemm_bs.cu):
// y = quantize_nvfp4(x) . dequant(W)^T.  Not the parity path.  w_sf holds
// the weight's scale atoms (make_gemm_bs_weight_sf, once per weight).
int launch_gemm_blockscaled(const QmmArgs& a, const uint8_t* w_sf, cudaStream_t stream);
int make_gemm_bs_weight_sf(const QmmArgs& a, uint8_t** out, cudaStream_t stream);
cudaError_t gemm_bs_take_error(unsigned int* v, cudaStream_t s);

}  // namespace qmm

// Resident weight (opaque in the C ABI).
struct qmm_weight {
    qmm::GemvTcState* tc = nullptr;  // decode-kernel state, or null
    int device = -1;
    int64_t n = 0, k = 0;
    qmm_quant_spec spec{};
    uint8_t* codes = nullptr;   // device, row stride ldc (multiple of 16 bytes)
    int64_t ldc = 0;
    uint8_t* scales = nullptr;  // device, row stride lds
    int64_t lds = 0;
    int64_t swiglu_n = 0;       // > 0: gate / up pair interleaved in 64-row blocks (qmm_swiglu_weight_create)
    uint8_t* bs_sf = nullptr;   // scale atoms of the block-scaled GEMM, made on its first call
};
