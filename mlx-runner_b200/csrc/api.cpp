// api.cpp - the C ABI: validation, error latch, resident weights, dispatch.
//
// Validation restates what the reference relies on before the arithmetic
// runs: MLX's quantized_matmul shape rules for the two microscaling modes
// (packed U32 [N, K*bits/32], U8 scales [N, K/group], transpose=true, no
// biases; src/model.zig:244-258) and the loader's spec rules
// (src/weights.zig:132-185, in spec.cpp).  Every failure returns a status
// and latches a message (src/mlx.zig:719-805); nothing calls exit().
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <atomic>
#include <vector>

#include "internal.h"

namespace qmm {
namespace {

std::mutex g_err_mu;
int g_err_status = QMM_OK;
char g_err_msg[512] = {0};
std::atomic<bool> g_err_latched{false};

std::atomic<uint64_t> g_fault_remaining{0};
std::atomic<bool> g_fault_fired{false};

std::mutex g_dev_mu;
std::vector<DeviceInfo> g_dev_info;
std::vector<bool> g_dev_known;

}  // namespace

int set_error(int status, const char* fmt, ...) {
    std::lock_guard<std::mutex> lk(g_err_mu);
    if (!g_err_latched.load(std::memory_order_acquire)) {
        va_list ap;
        va_start(ap, fmt);
        std::vsnprintf(g_err_msg, sizeof(g_err_msg), fmt, ap);
        va_end(ap);
        g_err_status = status;
        g_err_latched.store(true, std::memory_order_release);
    }
    return status;
}

int cuda_error(cudaError_t e, const char* what) {
    const int st = (e == cudaErrorMemoryAllocation) ? QMM_ERR_OUT_OF_MEMORY : QMM_ERR_CUDA;
    return set_error(st, "%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}

bool fault_hit() {
    uint64_t cur = g_fault_remaining.load();
    while (cur != 0) {
        if (g_fault_remaining.compare_exchange_weak(cur, cur - 1)) {
            if (cur == 1) {
                g_fault_fired.store(true);
                return true;
            }
            return false;
        }
    }
    return false;
}

int device_info(int device, DeviceInfo* out) {
    std::lock_guard<std::mutex> lk(g_dev_mu);
    if (device < 0) return set_error(QMM_ERR_BAD_ARGUMENT, "bad device %d", device);
    if ((size_t)device >= g_dev_info.size()) {
        g_dev_info.resize(device + 1);
        g_dev_known.resize(device + 1, false);
    }
    if (!g_dev_known[device]) {
        DeviceInfo d;
        QMM_CUDA_TRY(cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, device));
        QMM_CUDA_TRY(cudaDeviceGetAttribute(&d.major, cudaDevAttrComputeCapabilityMajor, device));
        QMM_CUDA_TRY(cudaDeviceGetAttribute(&d.minor, cudaDevAttrComputeCapabilityMinor, device));
        int optin = 0;
        QMM_CUDA_TRY(cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, device));
        d.smem_optin = (size_t)optin;
        g_dev_info[device] = d;
        g_dev_known[device] = true;
    }
    *out = g_dev_info[device];
    if (out->major != 10 || out->minor != 0)
        return set_error(QMM_ERR_NO_DEVICE, "device %d is sm_%d%d; this library is built for sm_100a only",
                         device, out->major, out->minor);
    return QMM_OK;
}

int dispatch(const QmmArgs& a, cudaStream_t stream, const qmm_weight* w) {
    if (a.m == 0 || a.n == 0) return QMM_OK;
    if (a.m <= gemv_max_m()) {
        if (w) {
            bool handled = false;
            if (int rc = launch_gemv_tc(w, a, stream, &handled)) return rc;
            if (handled) return QMM_OK;
        }
        return launch_gemv(a, stream);
    }
    bool handled = false;
    if (!a.yf) {
        if (int rc = launch_gemm(a, stream, &handled)) return rc;
        if (handled) return QMM_OK;
    }
    // Shapes outside the GEMM kernel's envelope: row blocks of the GEMV.
    for (int64_t m0 = 0; m0 < a.m; m0 += gemv_max_m()) {
        QmmArgs b = a;
        b.m = std::min<int64_t>(gemv_max_m(), a.m - m0);
        b.x = a.x + m0 * a.ldx;
        if (a.yf) b.yf = a.yf + m0 * a.ldy;
        else b.y = a.y + m0 * a.ldy;
        if (int rc = launch_gemv(b, stream)) return rc;
    }
    return QMM_OK;
}

namespace {

// Shared checks of x / y against a validated weight geometry.
int check_xy(const void* x, int64_t m, int64_t k, int64_t ldx, const void* y, int64_t n, int64_t ldy) {
    if (m < 0) return set_error(QMM_ERR_BAD_SHAPE, "m=%lld < 0", (long long)m);
    if (m == 0 || n == 0) return QMM_OK;
    if (!x || !y) return set_error(QMM_ERR_BAD_ARGUMENT, "x or y is NULL");
    if (ldx < k) return set_error(QMM_ERR_BAD_SHAPE, "ldx=%lld < k=%lld", (long long)ldx, (long long)k);
    if (ldy < n) return set_error(QMM_ERR_BAD_SHAPE, "ldy=%lld < n=%lld", (long long)ldy, (long long)n);
    if ((reinterpret_cast<uintptr_t>(x) & 3) || (ldx & 1))
        return set_error(QMM_ERR_BAD_ARGUMENT, "x must be 4-byte aligned with an even row stride");
    if (reinterpret_cast<uintptr_t>(y) & 1) return set_error(QMM_ERR_BAD_ARGUMENT, "y is not 2-byte aligned");
    return QMM_OK;
}

int current_device(int* dev) {
    QMM_CUDA_TRY(cudaGetDevice(dev));
    DeviceInfo info;
    return device_info(*dev, &info);
}

// The stateless entry points take raw pointers and launch on the current
// device: each one must be device (or managed) memory that device can use.
// A host pointer, or another GPU's buffer, handed to a kernel or a TMA map
// would fault the device instead of failing the call.
int check_on_device(const void* p, int dev, const char* what) {
    if (!p) return QMM_OK;
    cudaPointerAttributes attr;
    cudaError_t e = cudaPointerGetAttributes(&attr, p);
    if (e != cudaSuccess) {
        cudaGetLastError();   // the query's error must not linger for the next call
        return set_error(QMM_ERR_BAD_ARGUMENT, "%s: not a CUDA pointer (%s)", what, cudaGetErrorString(e));
    }
    if (attr.type == cudaMemoryTypeManaged) return QMM_OK;
    if (attr.type != cudaMemoryTypeDevice)
        return set_error(QMM_ERR_BAD_ARGUMENT, "%s is host memory; the call needs device memory", what);
    if (attr.device != dev)
        return set_error(QMM_ERR_BAD_ARGUMENT, "%s lives on device %d, the current device is %d", what,
                         attr.device, dev);
    return QMM_OK;
}

int check_stateless_ptrs(int dev, const void* x, const void* y, const void* w, const void* scales) {
    if (int rc = check_on_device(x, dev, "x")) return rc;
    if (int rc = check_on_device(y, dev, "y")) return rc;
    if (int rc = check_on_device(w, dev, "w")) return rc;
    return check_on_device(scales, dev, "scales");
}

}  // namespace

int check_device_buffer(const void* p, int dev, const char* what) { return check_on_device(p, dev, what); }
}  // namespace qmm

using namespace qmm;

extern "C" int qmm_abi_version(void) { return QMM_ABI_VERSION; }

extern "C" int qmm_last_error(char* buf, size_t len) {
    std::lock_guard<std::mutex> lk(g_err_mu);
    const int st = g_err_latched.load() ? g_err_status : QMM_OK;
    if (buf && len) {
        if (g_err_latched.load()) std::snprintf(buf, len, "%s", g_err_msg);
        else buf[0] = 0;
    }
    g_err_latched.store(false);
    g_err_status = QMM_OK;
    g_err_msg[0] = 0;
    return st;
}

extern "C" int qmm_error_pending(void) { return g_err_latched.load() ? 1 : 0; }

extern "C" int qmm_fault_arm(uint64_t k) {
    g_fault_fired.store(false);
    g_fault_remaining.store(k);
    return QMM_OK;
}

extern "C" int qmm_fault_fired(void) { return g_fault_fired.load() ? 1 : 0; }

#define QMM_FAULT_POINT(name)                                                   \
    do {                                                                        \
        if (::qmm::fault_hit())                                                 \
            return ::qmm::set_error(QMM_ERR_INJECTED, "%s: injected failure", name); \
    } while (0)

extern "C" int qmm_quantized_matmul(void* y_dev, int64_t ldy, const void* x_dev, int64_t m, int64_t k,
                                    int64_t ldx, const uint32_t* w_dev, int64_t w_rows, int64_t w_cols,
                                    const uint8_t* scales_dev, int64_t s_rows, int64_t s_cols,
                                    const void* biases, bool transpose, qmm_optional_int group_size,
                                    qmm_optional_int bits, const char* mode, void* stream) {
    QMM_FAULT_POINT("qmm_quantized_matmul");
    qmm_quant_spec spec;
    if (int rc = qmm_spec_from_args(group_size, bits, mode, &spec)) return rc;
    if (biases) return set_error(QMM_ERR_BAD_ARGUMENT, "%s takes no biases", mode);
    if (!transpose) return set_error(QMM_ERR_BAD_ARGUMENT, "only transpose=true (W [N, K]) is supported");
    if (k <= 0 || k % spec.group_size)
        return set_error(QMM_ERR_BAD_SHAPE, "k=%lld is not a positive multiple of group %d", (long long)k, spec.group_size);
    if (w_rows < 0 || w_rows != s_rows)
        return set_error(QMM_ERR_BAD_SHAPE, "w rows %lld != scales rows %lld", (long long)w_rows, (long long)s_rows);
    if (w_cols * 32 / spec.bits != k || (w_cols * 32) % spec.bits)
        return set_error(QMM_ERR_BAD_SHAPE, "w cols %lld do not pack k=%lld at %d bits", (long long)w_cols,
                         (long long)k, spec.bits);
    if (s_cols * spec.group_size != k)
        return set_error(QMM_ERR_BAD_SHAPE, "scales cols %lld != k/group = %lld", (long long)s_cols,
                         (long long)(k / spec.group_size));
    const int64_t n = w_rows;
    if (int rc = check_xy(x_dev, m, k, ldx, y_dev, n, ldy)) return rc;
    if (m == 0 || n == 0) return QMM_OK;
    if (!w_dev || !scales_dev) return set_error(QMM_ERR_BAD_ARGUMENT, "w or scales is NULL");
    int dev;
    if (int rc = current_device(&dev)) return rc;
    if (int rc = check_stateless_ptrs(dev, x_dev, y_dev, w_dev, scales_dev)) return rc;
    QmmArgs a;
    a.fmt = format_of(spec);
    a.codes = reinterpret_cast<const uint8_t*>(w_dev);
    a.ldc = w_cols * 4;
    a.scales = scales_dev;
    a.lds = s_cols;
    a.x = static_cast<const uint16_t*>(x_dev);
    a.ldx = ldx;
    a.y = static_cast<uint16_t*>(y_dev);
    a.ldy = ldy;
    a.m = m; a.n = n; a.k = k;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (m <= gemv_max_m()) {
        // Decode / MTP-verify rows: the TMA decode kernel on the tensors as
        // they are; outside its envelope, the cluster split-K GEMV.
        bool handled = false;
        if (int rc = launch_gemv_tc_ckpt(a, s, &handled)) return rc;
        if (handled) return QMM_OK;
    }
    return dispatch(a, s);
}

extern "C" int qmm_quantized_matmul_noalloc(void* y_dev, int64_t ldy, const void* x_dev, int64_t m, int64_t k,
                                            int64_t ldx, const uint32_t* w_dev, int64_t w_rows, int64_t w_cols,
                                            const uint8_t* scales_dev, int64_t s_rows, int64_t s_cols,
                                            const void* biases, bool transpose, qmm_optional_int group_size,
                                            qmm_optional_int bits, const char* mode, void* stream) {
    QMM_FAULT_POINT("qmm_quantized_matmul_noalloc");
    qmm_quant_spec spec;
    if (int rc = qmm_spec_from_args(group_size, bits, mode, &spec)) return rc;
    if (biases) return set_error(QMM_ERR_BAD_ARGUMENT, "%s takes no biases", mode);
    if (!transpose) return set_error(QMM_ERR_BAD_ARGUMENT, "only transpose=true (W [N, K]) is supported");
    if (k <= 0 || k % spec.group_size)
        return set_error(QMM_ERR_BAD_SHAPE, "k=%lld is not a positive multiple of group %d", (long long)k, spec.group_size);
    if (w_rows < 0 || w_rows != s_rows)
        return set_error(QMM_ERR_BAD_SHAPE, "w rows %lld != scales rows %lld", (long long)w_rows, (long long)s_rows);
    if (w_cols * 32 / spec.bits != k || (w_cols * 32) % spec.bits)
        return set_error(QMM_ERR_BAD_SHAPE, "w cols %lld do not pack k=%lld at %d bits", (long long)w_cols,
                         (long long)k, spec.bits);
    if (s_cols * spec.group_size != k)
        return set_error(QMM_ERR_BAD_SHAPE, "scales cols %lld != k/group = %lld", (long long)s_cols,
                         (long long)(k / spec.group_size));
    const int64_t n = w_rows;
    if (int rc = check_xy(x_dev, m, k, ldx, y_dev, n, ldy)) return rc;
    if (m == 0 || n == 0) return QMM_OK;
    if (!w_dev || !scales_dev) return set_error(QMM_ERR_BAD_ARGUMENT, "w or scales is NULL");
    int dev;
    if (int rc = current_device(&dev)) return rc;
    if (int rc = check_stateless_ptrs(dev, x_dev, y_dev, w_dev, scales_dev)) return rc;
    QmmArgs a;
    a.fmt = format_of(spec);
    a.codes = reinterpret_cast<const uint8_t*>(w_dev);
    a.ldc = w_cols * 4;
    a.scales = scales_dev;
    a.lds = s_cols;
    a.x = static_cast<const uint16_t*>(x_dev);
    a.ldx = ldx;
    a.y = static_cast<uint16_t*>(y_dev);
    a.ldy = ldy;
    a.m = m; a.n = n; a.k = k;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    bool handled = false;
    if (int rc = launch_gemv_tc_static(a, s, &handled)) return rc;
    if (handled) return QMM_OK;
    // Outside the decode kernel's envelope (M > 8, unaligned rows): the
    // scratch-free kernels of qmm_quantized_matmul.
    return dispatch(a, s);
}

namespace {

// Upload of one packed weight (codes bit for bit into 16-byte rows, scales
// unchanged); `prepare` adds the decode kernel's per-weight state.
int create_weight(const void* codes, const void* scales, int64_t n, int64_t k, int64_t ldw, int64_t lds,
                  qmm_quant_spec spec, int src_kind, void* stream, bool prepare, qmm_weight** out) {
    if (!out) return set_error(QMM_ERR_BAD_ARGUMENT, "out is NULL");
    *out = nullptr;
    if (int rc = check_spec(spec)) return rc;
    if (n < 0 || k <= 0 || k % spec.group_size)
        return set_error(QMM_ERR_BAD_SHAPE, "bad weight shape [%lld, %lld] for group %d", (long long)n, (long long)k,
                         spec.group_size);
    if (src_kind != QMM_SRC_HOST && src_kind != QMM_SRC_DEVICE)
        return set_error(QMM_ERR_BAD_ARGUMENT, "src_kind %d", src_kind);
    const int64_t row_bytes = k * spec.bits / 8, ngroups = k / spec.group_size;
    if (ldw == 0) ldw = row_bytes;
    if (lds == 0) lds = ngroups;
    if (ldw < row_bytes || lds < ngroups) return set_error(QMM_ERR_BAD_SHAPE, "source row stride too small");
    if (n > 0 && (!codes || !scales)) return set_error(QMM_ERR_BAD_ARGUMENT, "codes or scales is NULL");
    int dev;
    if (int rc = current_device(&dev)) return rc;
    qmm_weight* w = new qmm_weight();
    w->device = dev;
    w->n = n;
    w->k = k;
    w->spec = spec;
    w->ldc = (row_bytes + 15) / 16 * 16;  // 16-byte rows for vector loads
    w->lds = ngroups;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const cudaMemcpyKind kind = src_kind == QMM_SRC_HOST ? cudaMemcpyHostToDevice : cudaMemcpyDeviceToDevice;
    auto fail = [&](cudaError_t e, const char* what) {
        const int rc = cuda_error(e, what);
        cudaFree(w->codes);
        cudaFree(w->scales);
        delete w;
        return rc;
    };
    cudaError_t e;
    if ((e = cudaMalloc(&w->codes, (size_t)std::max<int64_t>(1, w->ldc * n))) != cudaSuccess) return fail(e, "cudaMalloc(codes)");
    if ((e = cudaMalloc(&w->scales, (size_t)std::max<int64_t>(1, w->lds * n))) != cudaSuccess) return fail(e, "cudaMalloc(scales)");
    if (n > 0) {
        if (w->ldc != row_bytes && (e = cudaMemsetAsync(w->codes, 0, (size_t)(w->ldc * n), s)) != cudaSuccess)
            return fail(e, "cudaMemsetAsync(codes)");
        if ((e = cudaMemcpy2DAsync(w->codes, w->ldc, codes, ldw, row_bytes, n, kind, s)) != cudaSuccess)
            return fail(e, "copy codes");
        if ((e = cudaMemcpy2DAsync(w->scales, w->lds, scales, lds, ngroups, n, kind, s)) != cudaSuccess)
            return fail(e, "copy scales");
    }
    if (prepare) {
        if (int rc = gemv_tc_prepare(w, s)) {
            cudaFree(w->codes);
            cudaFree(w->scales);
            delete w;
            return rc;
        }
    }
    if ((e = cudaStreamSynchronize(s)) != cudaSuccess) {
        gemv_tc_release(w);
        return fail(e, "cudaStreamSynchronize");
    }
    *out = w;
    return QMM_OK;
}

}  // namespace

extern "C" int qmm_weight_create(const void* codes, const void* scales, int64_t n, int64_t k, int64_t ldw,
                                 int64_t lds, qmm_quant_spec spec, int src_kind, void* stream,
                                 qmm_weight** out) {
    QMM_FAULT_POINT("qmm_weight_create");
    return create_weight(codes, scales, n, k, ldw, lds, spec, src_kind, stream, true, out);
}

extern "C" int qmm_swiglu_weight_create(const void* gate_codes, const void* gate_scales, const void* up_codes,
                                        const void* up_scales, int64_t n, int64_t k, int64_t ldw, int64_t lds,
                                        qmm_quant_spec spec, int src_kind, void* stream, qmm_weight** out) {
    QMM_FAULT_POINT("qmm_swiglu_weight_create");
    if (!out) return set_error(QMM_ERR_BAD_ARGUMENT, "out is NULL");
    *out = nullptr;
    if (n <= 0) return set_error(QMM_ERR_BAD_SHAPE, "gate/up weight needs n > 0 (got %lld)", (long long)n);
    qmm_weight *wg = nullptr, *wu = nullptr;
    if (int rc = create_weight(gate_codes, gate_scales, n, k, ldw, lds, spec, src_kind, stream, false, &wg)) return rc;
    if (int rc = create_weight(up_codes, up_scales, n, k, ldw, lds, spec, src_kind, stream, false, &wu)) {
        qmm_weight_destroy(wg);
        return rc;
    }
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int64_t npad = (n + 63) / 64 * 64;
    qmm_weight* w = new qmm_weight();
    w->device = wg->device;
    w->n = 2 * npad;
    w->k = k;
    w->spec = spec;
    w->ldc = wg->ldc;
    w->lds = wg->lds;
    w->swiglu_n = n;
    auto fail = [&](int rc) {
        cudaFree(w->codes);
        cudaFree(w->scales);
        delete w;
        qmm_weight_destroy(wg);
        qmm_weight_destroy(wu);
        return rc;
    };
    cudaError_t e;
    if ((e = cudaMalloc(&w->codes, (size_t)(w->ldc * w->n))) != cudaSuccess) return fail(cuda_error(e, "cudaMalloc(codes)"));
    if ((e = cudaMalloc(&w->scales, (size_t)(w->lds * w->n))) != cudaSuccess) return fail(cuda_error(e, "cudaMalloc(scales)"));
    if (npad != n) {
        // Padding rows of the last block: zero codes and scales (outputs 0, never stored).
        if ((e = cudaMemsetAsync(w->codes, 0, (size_t)(w->ldc * w->n), s)) != cudaSuccess)
            return fail(cuda_error(e, "cudaMemsetAsync(codes)"));
        if ((e = cudaMemsetAsync(w->scales, 0, (size_t)(w->lds * w->n), s)) != cudaSuccess)
            return fail(cuda_error(e, "cudaMemsetAsync(scales)"));
    }
    if (int rc = launch_interleave_rows(wg->codes, wu->codes, w->ldc, n, npad, w->codes, s)) return fail(rc);
    if (int rc = launch_interleave_rows(wg->scales, wu->scales, w->lds, n, npad, w->scales, s)) return fail(rc);
    if (int rc = gemv_tc_prepare(w, s)) return fail(rc);
    if ((e = cudaStreamSynchronize(s)) != cudaSuccess) {
        gemv_tc_release(w);
        return fail(cuda_error(e, "cudaStreamSynchronize"));
    }
    qmm_weight_destroy(wg);
    qmm_weight_destroy(wu);
    *out = w;
    return QMM_OK;
}

extern "C" int qmm_shard_range(int64_t n_full, int64_t k_full, qmm_quant_spec spec, int axis, int rank,
                               int nranks, int64_t* row0, int64_t* rows, int64_t* col0, int64_t* cols) {
    if (int rc = check_spec(spec)) return rc;
    if (!row0 || !rows || !col0 || !cols) return set_error(QMM_ERR_BAD_ARGUMENT, "null output");
    if (nranks < 1 || rank < 0 || rank >= nranks)
        return set_error(QMM_ERR_BAD_ARGUMENT, "rank %d of %d", rank, nranks);
    if (n_full < 0 || k_full <= 0 || k_full % spec.group_size)
        return set_error(QMM_ERR_BAD_SHAPE, "bad full weight shape [%lld, %lld]", (long long)n_full,
                         (long long)k_full);
    if (axis == 0) {
        // Column-parallel: contiguous row blocks, sizes differing by at most one.
        const int64_t r0 = n_full * rank / nranks, r1 = n_full * (rank + 1) / nranks;
        *row0 = r0; *rows = r1 - r0; *col0 = 0; *cols = k_full;
        return QMM_OK;
    }
    if (axis != 1) return set_error(QMM_ERR_BAD_ARGUMENT, "axis %d (0 = rows/N, 1 = columns/K)", axis);
    // Row-parallel: equal K slices that start on a group boundary and on a
    // whole U32 word.
    const int64_t unit = std::max<int64_t>(spec.group_size, 32 / spec.bits);
    if (k_full % nranks || (k_full / nranks) % unit)
        return set_error(QMM_ERR_BAD_SHAPE, "k=%lld does not split into %d shards of whole groups/words",
                         (long long)k_full, nranks);
    *row0 = 0; *rows = n_full; *cols = k_full / nranks; *col0 = *cols * rank;
    return QMM_OK;
}

extern "C" int qmm_weight_create_shard(const void* codes, const void* scales, int64_t n_full, int64_t k_full,
                                       qmm_quant_spec spec, int src_kind, int axis, int rank, int nranks,
                                       void* stream, qmm_weight** out) {
    int64_t r0, rows, c0, cols;
    if (int rc = qmm_shard_range(n_full, k_full, spec, axis, rank, nranks, &r0, &rows, &c0, &cols)) return rc;
    const int64_t row_bytes = k_full * spec.bits / 8, ngroups = k_full / spec.group_size;
    const uint8_t* c = static_cast<const uint8_t*>(codes);
    const uint8_t* sc = static_cast<const uint8_t*>(scales);
    return qmm_weight_create(c ? c + r0 * row_bytes + c0 * spec.bits / 8 : nullptr,
                             sc ? sc + r0 * ngroups + c0 / spec.group_size : nullptr, rows, cols, row_bytes,
                             ngroups, spec, src_kind, stream, out);
}

extern "C" int qmm_weight_destroy(qmm_weight* w) {
    if (!w) return QMM_OK;
    int prev = -1;
    cudaGetDevice(&prev);
    if (w->device >= 0) cudaSetDevice(w->device);
    gemv_tc_release(w);
    cudaFree(w->bs_sf);
    cudaError_t e1 = cudaFree(w->codes);
    cudaError_t e2 = cudaFree(w->scales);
    if (prev >= 0) cudaSetDevice(prev);
    delete w;
    if (e1 != cudaSuccess) return cuda_error(e1, "cudaFree(codes)");
    if (e2 != cudaSuccess) return cuda_error(e2, "cudaFree(scales)");
    return QMM_OK;
}

extern "C" int qmm_weight_info(const qmm_weight* w, int64_t* n, int64_t* k, qmm_quant_spec* spec, int* device) {
    if (!w) return set_error(QMM_ERR_BAD_ARGUMENT, "weight is NULL");
    if (n) *n = w->swiglu_n > 0 ? w->swiglu_n : w->n;
    if (k) *k = w->k;
    if (spec) *spec = w->spec;
    if (device) *device = w->device;
    return QMM_OK;
}

namespace {

// The weight's geometry for a launch on the current device, which must be
// the weight's; x and y (either may be NULL) must be memory of that device.
int weight_args(const qmm_weight* w, QmmArgs* a, const void* x, const void* y) {
    if (!w) return set_error(QMM_ERR_BAD_ARGUMENT, "weight is NULL");
    int dev;
    if (int rc = current_device(&dev)) return rc;
    if (dev != w->device)
        return set_error(QMM_ERR_BAD_ARGUMENT, "weight lives on device %d, current device is %d", w->device, dev);
    if (int rc = check_on_device(x, dev, "x")) return rc;
    if (int rc = check_on_device(y, dev, "y")) return rc;
    a->fmt = format_of(w->spec);
    a->codes = w->codes;
    a->ldc = w->ldc;
    a->scales = w->scales;
    a->lds = w->lds;
    a->n = w->n;
    a->k = w->k;
    return QMM_OK;
}

}  // namespace

extern "C" int qmm_run(const qmm_weight* w, const void* x_dev, int64_t m, int64_t ldx, void* y_dev, int64_t ldy,
                       bool transpose, void* stream) {
    QMM_FAULT_POINT("qmm_run");
    if (!transpose) return set_error(QMM_ERR_BAD_ARGUMENT, "only transpose=true (W [N, K]) is supported");
    if (!w) return set_error(QMM_ERR_BAD_ARGUMENT, "weight is NULL");
    if (w->swiglu_n > 0) return set_error(QMM_ERR_BAD_ARGUMENT, "a gate/up weight runs through qmm_swiglu_run");
    if (int rc = check_xy(x_dev, m, w->k, ldx, y_dev, w->n, ldy)) return rc;
    if (m == 0 || w->n == 0) return QMM_OK;
    QmmArgs a;
    if (int rc = weight_args(w, &a, x_dev, y_dev)) return rc;
    a.x = static_cast<const uint16_t*>(x_dev);
    a.ldx = ldx;
    a.y = static_cast<uint16_t*>(y_dev);
    a.ldy = ldy;
    a.m = m;
    return dispatch(a, static_cast<cudaStream_t>(stream), w);
}

extern "C" int qmm_lm_head_argmax(const qmm_weight* w, const void* x_dev, int64_t m, int64_t ldx,
                                  int32_t* ids_dev, float* logprobs_dev, void* logits_dev, int64_t ldl,
                                  void* stream) {
    QMM_FAULT_POINT("qmm_lm_head_argmax");
    if (!w) return set_error(QMM_ERR_BAD_ARGUMENT, "weight is NULL");
    if (w->swiglu_n > 0) return set_error(QMM_ERR_BAD_ARGUMENT, "a gate/up weight has no logits");
    if (m < 0 || m > gemv_max_m())
        return set_error(QMM_ERR_BAD_SHAPE, "greedy sampling takes 0..%d rows (m=%lld)", gemv_max_m(), (long long)m);
    if (m == 0 || w->n == 0) return QMM_OK;
    if (!ids_dev) return set_error(QMM_ERR_BAD_ARGUMENT, "ids is NULL");
    if (logits_dev) {
        if (int rc = check_xy(x_dev, m, w->k, ldx, logits_dev, w->n, ldl)) return rc;
    } else {
        // check_xy with a stand-in output: x alone is validated here.
        if (int rc = check_xy(x_dev, m, w->k, ldx, ids_dev, 1, 1)) return rc;
    }
    if (w->n > INT32_MAX) return set_error(QMM_ERR_BAD_SHAPE, "n=%lld exceeds 32-bit indices", (long long)w->n);
    QmmArgs a;
    if (int rc = weight_args(w, &a, x_dev, logits_dev)) return rc;
    if (int rc = check_on_device(ids_dev, w->device, "ids")) return rc;
    if (int rc = check_on_device(logprobs_dev, w->device, "logprobs")) return rc;
    a.x = static_cast<const uint16_t*>(x_dev);
    a.ldx = ldx;
    a.y = static_cast<uint16_t*>(logits_dev);
    a.ldy = logits_dev ? ldl : w->n;
    a.m = m;
    a.argmax_ids = ids_dev;
    a.argmax_lp = logprobs_dev;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    bool handled = false;
    if (int rc = launch_gemv_tc(w, a, s, &handled)) return rc;
    if (handled) return QMM_OK;
    // Outside the decode kernel's envelope: the logits (the caller's buffer
    // or stream-ordered scratch), then the sampling kernel.
    uint16_t* y = static_cast<uint16_t*>(logits_dev);
    int64_t ldy = ldl;
    if (!y) {
        QMM_CUDA_TRY(cudaMallocAsync(reinterpret_cast<void**>(&y), (size_t)(m * w->n * 2), s));
        ldy = w->n;
    }
    QmmArgs b = a;
    b.argmax_ids = nullptr;
    b.argmax_lp = nullptr;
    b.y = y;
    b.ldy = ldy;
    int rc = dispatch(b, s, w);
    if (rc == QMM_OK) rc = launch_argmax_rows(y, ldy, m, w->n, ids_dev, logprobs_dev, s);
    if (!logits_dev) {
        cudaError_t e = cudaFreeAsync(y, s);
        if (rc == QMM_OK && e != cudaSuccess) rc = cuda_error(e, "cudaFreeAsync");
    }
    return rc;
}

extern "C" int qmm_swiglu_run(const qmm_weight* w, const void* x_dev, int64_t m, int64_t ldx, void* h_dev,
                              int64_t ldh, void* stream) {
    QMM_FAULT_POINT("qmm_swiglu_run");
    if (!w) return set_error(QMM_ERR_BAD_ARGUMENT, "weight is NULL");
    if (w->swiglu_n <= 0) return set_error(QMM_ERR_BAD_ARGUMENT, "not a gate/up weight (qmm_swiglu_weight_create)");
    if (int rc = check_xy(x_dev, m, w->k, ldx, h_dev, w->swiglu_n, ldh)) return rc;
    if (m == 0) return QMM_OK;
    QmmArgs a;
    if (int rc = weight_args(w, &a, x_dev, h_dev)) return rc;
    a.x = static_cast<const uint16_t*>(x_dev);
    a.ldx = ldx;
    a.y = static_cast<uint16_t*>(h_dev);
    a.ldy = ldh;
    a.m = m;
    a.swiglu_n = w->swiglu_n;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    bool handled = false;
    if (m <= gemv_max_m()) {
        if (int rc = launch_gemv_tc(w, a, s, &handled)) return rc;
    } else {
        if (int rc = launch_gemm(a, s, &handled)) return rc;
    }
    if (handled) return QMM_OK;
    // Outside the fused kernels' envelope (unaligned x): the interleaved
    // gate / up outputs into stream-ordered scratch, then the SwiGLU step.
    uint16_t* y = nullptr;
    QMM_CUDA_TRY(cudaMallocAsync(reinterpret_cast<void**>(&y), (size_t)(m * w->n * 2), s));
    QmmArgs b = a;
    b.swiglu_n = 0;
    b.y = y;
    b.ldy = w->n;
    int rc = dispatch(b, s, w);
    if (rc == QMM_OK) rc = launch_swiglu_apply(y, w->n, m, w->swiglu_n, static_cast<uint16_t*>(h_dev), ldh, s);
    cudaError_t e = cudaFreeAsync(y, s);
    if (rc == QMM_OK && e != cudaSuccess) rc = cuda_error(e, "cudaFreeAsync");
    return rc;
}

extern "C" int qmm_linear(const qmm_weight* w, bool has_packed_u32, const void* x_dev, int64_t m, int64_t ldx,
                          void* y_dev, int64_t ldy, void* stream) {
    // src/model.zig:226-228: a packed U32 weight without scales is MissingWeight.
    if (!w && has_packed_u32) return set_error(QMM_ERR_MISSING_WEIGHT, "packed weight has no scales");
    if (!w) return set_error(QMM_ERR_MISSING_WEIGHT, "weight is missing");
    return qmm_run(w, x_dev, m, ldx, y_dev, ldy, true, stream);
}

extern "C" int qmm_run_blockscaled(qmm_weight* w, const void* x_dev, int64_t m, int64_t ldx, void* y_dev,
                                   int64_t ldy, void* stream) {
    QMM_FAULT_POINT("qmm_run_blockscaled");
    if (!w) return set_error(QMM_ERR_BAD_ARGUMENT, "weight is NULL");
    if (w->swiglu_n > 0) return set_error(QMM_ERR_BAD_ARGUMENT, "a gate/up weight runs through qmm_swiglu_run");
    if (w->spec.mode != QMM_MODE_NVFP4)
        return set_error(QMM_ERR_BAD_ARGUMENT, "the block-scaled GEMM takes nvfp4 weights");
    if (int rc = check_xy(x_dev, m, w->k, ldx, y_dev, w->n, ldy)) return rc;
    if (m == 0 || w->n == 0) return QMM_OK;
    if (w->k % 32) return set_error(QMM_ERR_BAD_SHAPE, "block-scaled GEMM: k=%lld is not a multiple of 32",
                                    (long long)w->k);
    QmmArgs a;
    if (int rc = weight_args(w, &a, x_dev, y_dev)) return rc;
    a.x = static_cast<const uint16_t*>(x_dev);
    a.ldx = ldx;
    a.y = static_cast<uint16_t*>(y_dev);
    a.ldy = ldy;
    a.m = m;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (!w->bs_sf) {
        cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
        QMM_CUDA_TRY(cudaStreamIsCapturing(s, &cs));
        if (cs != cudaStreamCaptureStatusNone)
            return set_error(QMM_ERR_BAD_ARGUMENT, "the first qmm_run_blockscaled call on a weight allocates its "
                                                   "scale atoms and cannot be captured");
        if (int rc = make_gemm_bs_weight_sf(a, &w->bs_sf, s)) return rc;
    }
    return launch_gemm_blockscaled(a, w->bs_sf, s);
}

extern "C" int qmm_dequantize(const qmm_weight* w, void* out_dev, int32_t out_dtype, void* stream) {
    QMM_FAULT_POINT("qmm_dequantize");
    if (out_dtype != QMM_DTYPE_BF16 && out_dtype != QMM_DTYPE_F32)
        return set_error(QMM_ERR_UNSUPPORTED_DTYPE, "dequantize output dtype %d (BF16 or F32)", out_dtype);
    QmmArgs a;
    if (int rc = weight_args(w, &a, nullptr, out_dev)) return rc;
    if (w->swiglu_n > 0) return set_error(QMM_ERR_BAD_ARGUMENT, "a gate/up weight has no single dequantized form");
    if (w->n == 0) return QMM_OK;
    if (!out_dev) return set_error(QMM_ERR_BAD_ARGUMENT, "out is NULL");
    return launch_dequant(a.fmt, a.codes, a.ldc, a.scales, a.lds, a.n, a.k, out_dev, out_dtype == QMM_DTYPE_BF16,
                          static_cast<cudaStream_t>(stream));
}

extern "C" int qmm_quantize(const void* w_dev, int32_t w_dtype, int64_t n, int64_t k, int64_t ldw,
                            qmm_optional_int group_size, qmm_optional_int bits, const char* mode,
                            const void* global_scale, uint32_t* codes_dev, uint8_t* scales_dev, void* stream) {
    QMM_FAULT_POINT("qmm_quantize");
    qmm_quant_spec spec;
    if (int rc = qmm_spec_from_args(group_size, bits, mode, &spec)) return rc;
    if (global_scale) return set_error(QMM_ERR_BAD_ARGUMENT, "%s quantize takes no global scale", mode);
    if (w_dtype != QMM_DTYPE_BF16 && w_dtype != QMM_DTYPE_F32)
        return set_error(QMM_ERR_UNSUPPORTED_DTYPE, "quantize input dtype %d (BF16 or F32)", w_dtype);
    if (n < 0) return set_error(QMM_ERR_BAD_SHAPE, "n=%lld < 0", (long long)n);
    if (k <= 0 || k % spec.group_size)
        return set_error(QMM_ERR_BAD_SHAPE, "k=%lld is not a positive multiple of group %d", (long long)k,
                         spec.group_size);
    if (ldw == 0) ldw = k;
    if (ldw < k) return set_error(QMM_ERR_BAD_SHAPE, "ldw=%lld < k=%lld", (long long)ldw, (long long)k);
    if (n == 0) return QMM_OK;
    if (!w_dev || !codes_dev || !scales_dev) return set_error(QMM_ERR_BAD_ARGUMENT, "w, codes or scales is NULL");
    const int64_t esize = w_dtype == QMM_DTYPE_BF16 ? 2 : 4;
    if (reinterpret_cast<uintptr_t>(w_dev) % esize)
        return set_error(QMM_ERR_BAD_ARGUMENT, "w is not %lld-byte aligned", (long long)esize);
    if (reinterpret_cast<uintptr_t>(codes_dev) & 3) return set_error(QMM_ERR_BAD_ARGUMENT, "codes are not 4-byte aligned");
    int dev;
    if (int rc = current_device(&dev)) return rc;
    return launch_quantize(format_of(spec), w_dev, w_dtype == QMM_DTYPE_BF16, ldw, n, k,
                           reinterpret_cast<uint8_t*>(codes_dev), scales_dev, static_cast<cudaStream_t>(stream));
}

// Used by tp.cpp: the row-parallel partial product in fp32.
namespace qmm {
// Row-parallel decode with the cross-rank sum fused into the decode kernel.
// *handled = false (every rank alike: the test depends only on shapes and the
// weight's decode state) when the fused kernel does not apply; x must then
// still meet its alignment on every rank, else this rank reports an error
// (its peers' waits time out and report QMM_ERR_TIMEOUT).
int run_rowparallel_fused(const qmm_weight* w, const TpExchange* ex, const void* x_dev, int64_t m, int64_t ldx,
                          void* y_dev, int64_t ldy, cudaStream_t stream, bool* handled) {
    *handled = false;
    if (!w || !w->tc || m < 1 || m > 8 || m * w->n > ex->cap) return QMM_OK;
    if (int rc = check_xy(x_dev, m, w->k, ldx, y_dev, w->n, ldy)) return rc;
    if ((reinterpret_cast<uintptr_t>(x_dev) & 15) || ((ldx * 2) & 15))
        return set_error(QMM_ERR_BAD_ARGUMENT, "row-parallel decode needs 16-byte aligned x rows");
    QmmArgs a;
    if (int rc = weight_args(w, &a, x_dev, y_dev)) return rc;
    a.x = static_cast<const uint16_t*>(x_dev);
    a.ldx = ldx;
    a.y = static_cast<uint16_t*>(y_dev);
    a.ldy = ldy;
    a.m = m;
    a.tp = ex;
    if (int rc = launch_gemv_tc(w, a, stream, handled)) return rc;
    if (!*handled) return set_error(QMM_ERR_CUDA, "row-parallel decode kernel declined a prepared weight");
    return QMM_OK;
}

int run_partial_f32(const qmm_weight* w, const void* x_dev, int64_t m, int64_t ldx, float* yf, int64_t ldy,
                    cudaStream_t stream) {
    if (int rc = check_xy(x_dev, m, w ? w->k : 0, ldx, yf, w ? w->n : 0, ldy)) return rc;
    QmmArgs a;
    if (int rc = weight_args(w, &a, x_dev, yf)) return rc;
    a.x = static_cast<const uint16_t*>(x_dev);
    a.ldx = ldx;
    a.y = nullptr;
    a.yf = yf;
    a.ldy = ldy;
    a.m = m;
    return dispatch(a, stream, w);
}
}  // namespace qmm
