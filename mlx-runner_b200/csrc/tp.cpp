// tp.cpp - tensor-parallel plumbing: communicator + row-parallel run.
//
// The reference has no distributed backend (--tp is parsed and logged as a
// single-device stub, src/main.zig:210-215, :338-340); the sharding here is
// the one the qmm path needs.  Column-parallel (N) shards need no exchange.
// Row-parallel (K) shards produce partial sums that are added across ranks:
// the partials are kept in fp32 and reduced with one NCCL fp32 all-reduce,
// then rounded to bf16 once, so the result carries a single bf16 rounding
// as on one GPU (adding bf16-rounded partials in bf16 measurably exceeds a
// 2e-3 relative error at 2+ ranks).
//
// For decode shapes (M <= 8, resident weight with decode-kernel state) the
// reduction is fused into the decode kernel: each rank's final fp32 row-block
// sums go over NVLink straight into every rank's receive buffer (CUDA IPC
// mappings exchanged at communicator creation) and are added in rank order -
// one launch, no NCCL call, no separate conversion.  Every rank takes the same
// path: the choice depends only on the communicator (agreed by all ranks at
// creation) and on shapes.  Otherwise: fp32 partials, one NCCL fp32
// all-reduce, one rounding to bf16.  QMM_TP_FUSED=0 disables the fused path.
//
// NCCL is loaded with dlopen on first use (the copy already in the process,
// e.g. torch's, if any; else $QMM_NCCL_LIBRARY; else libnccl.so.2), so the
// library itself loads on machines without NCCL.
#include <dlfcn.h>

#include <cstdlib>
#include <cstring>
#include <mutex>
#include <vector>

#include <nccl.h>

#include "internal.h"

namespace qmm {
int run_partial_f32(const qmm_weight* w, const void* x_dev, int64_t m, int64_t ldx, float* yf, int64_t ldy,
                    cudaStream_t stream);
int launch_f32_to_bf16(const float* in, int64_t rows, int64_t cols, int64_t ld_in, uint16_t* out, int64_t ld_out,
                       cudaStream_t stream);
int run_rowparallel_fused(const qmm_weight* w, const TpExchange* ex, const void* x_dev, int64_t m, int64_t ldx,
                          void* y_dev, int64_t ldy, cudaStream_t stream, bool* handled);
}  // namespace qmm

struct qmm_comm {
    ncclComm_t comm = nullptr;
    int nranks = 0, rank = 0, device = -1;
    float* partial = nullptr;   // fp32 [capacity] partial sums
    int64_t capacity = 0;
    // Fused row-parallel exchange (peer receive buffers mapped over CUDA IPC).
    bool fused = false;
    qmm::TpExchange ex;
    // qmm_tp_comm_create_detached: no NCCL, the other ranks' buffers are local
    // allocations that nothing else writes.
    bool detached = false;
};

namespace {

struct NcclApi {
    ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
    ncclResult_t (*CommInitRank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
    ncclResult_t (*AllReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                              cudaStream_t) = nullptr;
    ncclResult_t (*AllGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
    const char* (*GetErrorString)(ncclResult_t) = nullptr;
    bool ok = false;
};

std::once_flag g_once;
NcclApi g_api;

void load_nccl() {
    void* h = nullptr;
    if (const char* p = std::getenv("QMM_NCCL_LIBRARY")) h = dlopen(p, RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) return;
    g_api.GetUniqueId = reinterpret_cast<decltype(g_api.GetUniqueId)>(dlsym(h, "ncclGetUniqueId"));
    g_api.CommInitRank = reinterpret_cast<decltype(g_api.CommInitRank)>(dlsym(h, "ncclCommInitRank"));
    g_api.CommDestroy = reinterpret_cast<decltype(g_api.CommDestroy)>(dlsym(h, "ncclCommDestroy"));
    g_api.AllReduce = reinterpret_cast<decltype(g_api.AllReduce)>(dlsym(h, "ncclAllReduce"));
    g_api.AllGather = reinterpret_cast<decltype(g_api.AllGather)>(dlsym(h, "ncclAllGather"));
    g_api.GetErrorString = reinterpret_cast<decltype(g_api.GetErrorString)>(dlsym(h, "ncclGetErrorString"));
    g_api.ok = g_api.GetUniqueId && g_api.CommInitRank && g_api.CommDestroy && g_api.AllReduce &&
               g_api.AllGather && g_api.GetErrorString;
}

int nccl(int* rc_out) {
    std::call_once(g_once, load_nccl);
    if (!g_api.ok) {
        *rc_out = qmm::set_error(QMM_ERR_NCCL, "NCCL could not be loaded (set QMM_NCCL_LIBRARY)");
        return 0;
    }
    return 1;
}

int nccl_fail(ncclResult_t r, const char* what) {
    return qmm::set_error(QMM_ERR_NCCL, "%s: %s", what, g_api.GetErrorString ? g_api.GetErrorString(r) : "?");
}

// Frees the fused-exchange resources of c (peer mappings, local buffers).
void release_fused(qmm_comm* c) {
    for (int r = 0; r < c->nranks && r < qmm::kMaxTpRanks; ++r) {
        if (r == c->rank) continue;
        if (c->detached) {
            cudaFree(c->ex.recv[r]);
            cudaFree(c->ex.flags[r]);
            continue;
        }
        if (c->ex.recv[r]) cudaIpcCloseMemHandle(c->ex.recv[r]);
        if (c->ex.flags[r]) cudaIpcCloseMemHandle(c->ex.flags[r]);
    }
    if (c->rank < qmm::kMaxTpRanks) {
        cudaFree(c->ex.recv[c->rank]);
        cudaFree(c->ex.flags[c->rank]);
    }
    cudaFree(c->ex.gen);
    c->ex = qmm::TpExchange();
    c->fused = false;
}

// Collective (every rank calls it in the same order): allocates this rank's
// receive buffer and flags, exchanges CUDA IPC handles with ncclAllGather,
// maps the peers' buffers, and agrees (ncclAllReduce min) on whether every
// rank succeeded.  Returns an error for NCCL failures and when this rank
// cannot hold the exchange's own scratch (then before any collective); a
// failed buffer allocation or IPC mapping on any rank leaves every rank on the
// NCCL path.
int setup_fused(qmm_comm* c, int64_t cap) {
    const int P = c->nranks, me = c->rank;
    const char* env = std::getenv("QMM_TP_FUSED");
    if (P < 2 || P > qmm::kMaxTpRanks || cap <= 0 || (env && env[0] == '0')) return QMM_OK;
    cudaStream_t s = nullptr;
    if (cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking) != cudaSuccess)
        return qmm::set_error(QMM_ERR_CUDA, "setup of the fused exchange: cudaStreamCreate failed");
    // The device buffers of the handle exchange ([P + 1] handle pairs, then the
    // agreement flag).  Without them this rank cannot take part in the
    // collectives below: it fails here, before any of them, and its peers wait
    // in theirs until the caller's own timeout - as for a rank whose
    // ncclCommInitRank failed.
    const size_t hb = sizeof(cudaIpcMemHandle_t) * 2;
    uint8_t* dbuf = nullptr;
    if (cudaMalloc(&dbuf, hb * (P + 1) + sizeof(int)) != cudaSuccess) {
        cudaStreamDestroy(s);
        return qmm::set_error(QMM_ERR_OUT_OF_MEMORY, "setup of the fused exchange: cudaMalloc failed");
    }
    int* dok = reinterpret_cast<int*>(dbuf + hb * (P + 1));
    const int max_rb = (int)((cap + 127) / 128);
    int ok = 1;
    float* recv = nullptr;
    unsigned int* flags = nullptr;
    unsigned int* gen = nullptr;
    ok = ok && cudaMalloc(&recv, (size_t)2 * P * cap * sizeof(float)) == cudaSuccess;
    ok = ok && cudaMalloc(&flags, (size_t)P * max_rb * sizeof(unsigned int)) == cudaSuccess;
    ok = ok && cudaMalloc(&gen, (size_t)max_rb * sizeof(unsigned int)) == cudaSuccess;
    ok = ok && cudaMemset(flags, 0, (size_t)P * max_rb * sizeof(unsigned int)) == cudaSuccess;
    ok = ok && cudaMemset(gen, 0, (size_t)max_rb * sizeof(unsigned int)) == cudaSuccess;
    cudaIpcMemHandle_t mine[2];
    std::memset(mine, 0, sizeof(mine));
    ok = ok && cudaIpcGetMemHandle(&mine[0], recv) == cudaSuccess;
    ok = ok && cudaIpcGetMemHandle(&mine[1], flags) == cudaSuccess;
    // Exchange [P][2 handles] and the success flags: every rank takes part,
    // whatever its own allocations gave (a failed one only sets ok = 0).
    static_assert(sizeof(mine) == 2 * sizeof(cudaIpcMemHandle_t), "two handles per rank");
    int rc = QMM_OK;
    std::vector<uint8_t> all(hb * P);
    cudaMemcpy(dbuf + hb * P, mine, hb, cudaMemcpyHostToDevice);
    cudaMemcpy(dok, &ok, sizeof(int), cudaMemcpyHostToDevice);
    if (ncclResult_t r = g_api.AllGather(dbuf + hb * P, dbuf, hb, ncclUint8, c->comm, s)) rc = nccl_fail(r, "ncclAllGather");
    else if (ncclResult_t r2 = g_api.AllReduce(dok, dok, 1, ncclInt32, ncclMin, c->comm, s)) rc = nccl_fail(r2, "ncclAllReduce");
    cudaStreamSynchronize(s);
    cudaMemcpy(all.data(), dbuf, hb * P, cudaMemcpyDeviceToHost);
    cudaMemcpy(&ok, dok, sizeof(int), cudaMemcpyDeviceToHost);
    c->ex.nranks = P;
    c->ex.rank = me;
    c->ex.max_rb = max_rb;
    c->ex.cap = cap;
    c->ex.recv[me] = recv;
    c->ex.flags[me] = flags;
    c->ex.gen = gen;
    int opened = ok;
    if (ok && rc == QMM_OK) {
        for (int r = 0; r < P; ++r) {
            if (r == me) continue;
            cudaIpcMemHandle_t h[2];
            std::memcpy(h, all.data() + hb * r, hb);
            void* pr = nullptr;
            void* pf = nullptr;
            opened = opened && cudaIpcOpenMemHandle(&pr, h[0], cudaIpcMemLazyEnablePeerAccess) == cudaSuccess;
            if (pr) c->ex.recv[r] = static_cast<float*>(pr);
            opened = opened && cudaIpcOpenMemHandle(&pf, h[1], cudaIpcMemLazyEnablePeerAccess) == cudaSuccess;
            if (pf) c->ex.flags[r] = static_cast<unsigned int*>(pf);
        }
        // Every rank must have mapped every peer.
        cudaMemcpy(dok, &opened, sizeof(int), cudaMemcpyHostToDevice);
        if (ncclResult_t r = g_api.AllReduce(dok, dok, 1, ncclInt32, ncclMin, c->comm, s)) rc = nccl_fail(r, "ncclAllReduce");
        cudaStreamSynchronize(s);
        cudaMemcpy(&opened, dok, sizeof(int), cudaMemcpyDeviceToHost);
    }
    cudaFree(dbuf);
    cudaStreamDestroy(s);
    cudaGetLastError();   // a failed IPC call leaves a sticky-free error; it is handled by `ok`
    c->fused = ok && opened && rc == QMM_OK;
    if (!c->fused) release_fused(c);
    return rc;
}

}  // namespace

using qmm::set_error;

extern "C" int qmm_tp_unique_id(void* id128) {
    int rc = QMM_OK;
    if (!nccl(&rc)) return rc;
    if (!id128) return set_error(QMM_ERR_BAD_ARGUMENT, "id is NULL");
    ncclUniqueId id;
    if (ncclResult_t r = g_api.GetUniqueId(&id)) return nccl_fail(r, "ncclGetUniqueId");
    static_assert(sizeof(ncclUniqueId) == 128, "NCCL unique id is 128 bytes");
    std::memcpy(id128, &id, sizeof(id));
    return QMM_OK;
}

extern "C" int qmm_tp_comm_create(const void* id128, int nranks, int rank, int64_t max_partial_elems,
                                  qmm_comm** out) {
    if (qmm::fault_hit()) return set_error(QMM_ERR_INJECTED, "qmm_tp_comm_create: injected failure");
    if (!id128 || !out) return set_error(QMM_ERR_BAD_ARGUMENT, "id or out is NULL");
    *out = nullptr;
    if (nranks < 1 || rank < 0 || rank >= nranks || max_partial_elems < 0)
        return set_error(QMM_ERR_BAD_ARGUMENT, "rank %d of %d, capacity %lld", rank, nranks,
                         (long long)max_partial_elems);
    int rc = QMM_OK;
    if (!nccl(&rc)) return rc;
    qmm_comm* c = new qmm_comm();
    c->nranks = nranks;
    c->rank = rank;
    if (cudaError_t e = cudaGetDevice(&c->device)) {
        delete c;
        return qmm::cuda_error(e, "cudaGetDevice");
    }
    if (max_partial_elems > 0) {
        if (cudaError_t e = cudaMalloc(&c->partial, (size_t)max_partial_elems * sizeof(float))) {
            delete c;
            return qmm::cuda_error(e, "cudaMalloc(partial)");
        }
        c->capacity = max_partial_elems;
    }
    ncclUniqueId id;
    std::memcpy(&id, id128, sizeof(id));
    if (ncclResult_t r = g_api.CommInitRank(&c->comm, nranks, id, rank)) {
        cudaFree(c->partial);
        delete c;
        return nccl_fail(r, "ncclCommInitRank");
    }
    if (int frc = setup_fused(c, max_partial_elems)) {
        g_api.CommDestroy(c->comm);
        cudaFree(c->partial);
        delete c;
        return frc;
    }
    *out = c;
    return QMM_OK;
}

extern "C" int qmm_tp_comm_create_detached(int nranks, int rank, int64_t max_partial_elems, qmm_comm** out) {
    if (qmm::fault_hit()) return set_error(QMM_ERR_INJECTED, "qmm_tp_comm_create_detached: injected failure");
    if (!out) return set_error(QMM_ERR_BAD_ARGUMENT, "out is NULL");
    *out = nullptr;
    if (nranks < 2 || nranks > qmm::kMaxTpRanks || rank < 0 || rank >= nranks || max_partial_elems <= 0)
        return set_error(QMM_ERR_BAD_ARGUMENT, "rank %d of %d (2..%d ranks), capacity %lld", rank, nranks,
                         qmm::kMaxTpRanks, (long long)max_partial_elems);
    qmm_comm* c = new qmm_comm();
    c->nranks = nranks;
    c->rank = rank;
    c->detached = true;
    c->capacity = max_partial_elems;
    if (cudaError_t e = cudaGetDevice(&c->device)) {
        delete c;
        return qmm::cuda_error(e, "cudaGetDevice");
    }
    // The same buffers setup_fused gives every rank, all on this device.
    const int P = nranks;
    const int64_t cap = max_partial_elems;
    const int max_rb = (int)((cap + 127) / 128);
    const size_t recv_bytes = (size_t)2 * P * cap * sizeof(float), flag_bytes = (size_t)P * max_rb * sizeof(unsigned int);
    cudaError_t e = cudaSuccess;
    for (int r = 0; r < P && e == cudaSuccess; ++r) {
        if ((e = cudaMalloc(&c->ex.recv[r], recv_bytes)) == cudaSuccess &&
            (e = cudaMemset(c->ex.recv[r], 0, recv_bytes)) == cudaSuccess &&
            (e = cudaMalloc(&c->ex.flags[r], flag_bytes)) == cudaSuccess)
            e = cudaMemset(c->ex.flags[r], 0, flag_bytes);
    }
    if (e == cudaSuccess && (e = cudaMalloc(&c->ex.gen, (size_t)max_rb * sizeof(unsigned int))) == cudaSuccess)
        e = cudaMemset(c->ex.gen, 0, (size_t)max_rb * sizeof(unsigned int));
    c->ex.nranks = P;
    c->ex.rank = rank;
    c->ex.max_rb = max_rb;
    c->ex.cap = cap;
    if (e != cudaSuccess) {
        const int rc = qmm::cuda_error(e, "qmm_tp_comm_create_detached");
        release_fused(c);
        delete c;
        return rc;
    }
    c->fused = true;
    *out = c;
    return QMM_OK;
}

extern "C" int qmm_tp_comm_destroy(qmm_comm* c) {
    if (!c) return QMM_OK;
    int rc = QMM_OK;
    if (c->comm && g_api.ok) {
        if (ncclResult_t r = g_api.CommDestroy(c->comm)) rc = nccl_fail(r, "ncclCommDestroy");
    }
    release_fused(c);
    if (c->partial) cudaFree(c->partial);
    delete c;
    return rc;
}

extern "C" int qmm_tp_allreduce_bf16(qmm_comm* c, void* buf_dev, int64_t count, void* stream) {
    if (qmm::fault_hit()) return set_error(QMM_ERR_INJECTED, "qmm_tp_allreduce_bf16: injected failure");
    if (!c) return set_error(QMM_ERR_BAD_ARGUMENT, "comm is NULL");
    if (c->detached) return set_error(QMM_ERR_BAD_ARGUMENT, "a detached communicator has no collectives");
    if (count < 0 || (count > 0 && !buf_dev)) return set_error(QMM_ERR_BAD_ARGUMENT, "bad buffer");
    if (ncclResult_t r = g_api.AllReduce(buf_dev, buf_dev, (size_t)count, ncclBfloat16, ncclSum, c->comm,
                                         static_cast<cudaStream_t>(stream)))
        return nccl_fail(r, "ncclAllReduce(bf16)");
    return QMM_OK;
}

extern "C" int qmm_tp_run_rowparallel(const qmm_weight* w, qmm_comm* c, const void* x_dev, int64_t m, int64_t ldx,
                                      void* y_dev, int64_t ldy, void* stream) {
    if (qmm::fault_hit()) return set_error(QMM_ERR_INJECTED, "qmm_tp_run_rowparallel: injected failure");
    if (!c || !w) return set_error(QMM_ERR_BAD_ARGUMENT, "weight or comm is NULL");
    if (w->swiglu_n > 0) return set_error(QMM_ERR_BAD_ARGUMENT, "a gate/up weight is not row-parallel");
    int64_t n = 0, k = 0;
    qmm_weight_info(w, &n, &k, nullptr, nullptr);
    if (m < 0) return set_error(QMM_ERR_BAD_SHAPE, "m < 0");
    if (m * n > c->capacity)
        return set_error(QMM_ERR_BAD_SHAPE, "m*n=%lld exceeds the communicator's partial buffer (%lld)",
                         (long long)(m * n), (long long)c->capacity);
    if (ldy < n) return set_error(QMM_ERR_BAD_SHAPE, "ldy < n");
    if (m == 0 || n == 0) return QMM_OK;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (c->fused) {
        bool handled = false;
        if (int rc = qmm::run_rowparallel_fused(w, &c->ex, x_dev, m, ldx, y_dev, ldy, s, &handled)) return rc;
        if (handled) return QMM_OK;
    }
    if (c->detached)
        return set_error(QMM_ERR_BAD_ARGUMENT, "a detached communicator runs only the fused decode exchange "
                                               "(M <= 8, a resident decode weight, 16-byte aligned x rows)");
    if (int rc = qmm::run_partial_f32(w, x_dev, m, ldx, c->partial, n, s)) return rc;
    if (ncclResult_t r = g_api.AllReduce(c->partial, c->partial, (size_t)(m * n), ncclFloat32, ncclSum, c->comm, s))
        return nccl_fail(r, "ncclAllReduce(f32)");
    return qmm::launch_f32_to_bf16(c->partial, m, n, n, static_cast<uint16_t*>(y_dev), ldy, s);
}
