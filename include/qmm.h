/*
 * qmm.h - C ABI of the B200 quantized-matmul library (libqmm_b200.so).
 *
 * The library replaces one hot path of mlx-runner: the quantized linear
 * layer that every projection of its model runs through,
 *     y = x . dequant(W)^T
 * for MLX's mxfp8 (E4M3 codes, group 32, UE8M0 scales) and nvfp4 (E2M1
 * codes, group 16, UE4M3 scales) formats on MLX's packed layout: codes
 * U32 [N, K*bits/32] (LSB-first), scales U8 [N, K/group].
 *
 * Conventions shared by every entry point:
 *   - return 0 (QMM_OK) on success or a qmm_status code; the message of the
 *     first failure is latched and can be read with qmm_last_error();
 *   - pointers named *_dev are device pointers of the current CUDA device;
 *     `stream` is a cudaStream_t passed as void* (NULL = legacy stream);
 *   - work is enqueued on `stream` and runs asynchronously; nothing here
 *     synchronizes the device except qmm_weight_create/destroy;
 *   - no entry point ever calls exit() and none falls back to the CPU;
 *   - x and y are bf16 (uint16 bit patterns), row-major with a row stride.
 *
 * Reference interfaces replaced (paths relative to the mlx-runner tree):
 *   src/mlx.zig:265      mlx_quantized_matmul    -> qmm_quantized_matmul, qmm_run
 *   src/mlx.zig:274      mlx_dequantize          -> qmm_dequantize
 *   src/mlx.zig:278      mlx_quantize            -> qmm_quantize
 *   src/mlx.zig:41-51    mlx_optional_int        -> qmm_optional_int
 *   src/mlx.zig:589-595  check (int status)      -> qmm_status return codes
 *   src/mlx.zig:719-805  error latch             -> qmm_last_error, qmm_error_pending
 *   src/mlx.zig:562-595  fault.arm (test hook)   -> qmm_fault_arm
 *   src/weights.zig:23-55  WeightsError, DType, QuantMode, QuantSpec
 *   src/weights.zig:132-185 inferQuantSpec       -> qmm_infer_quant_spec
 *   src/weights.zig:203-353 WeightMap (U32/U8 upload) -> qmm_weight_create
 *   src/model.zig:218-258 namedLinearQ / qlinear -> qmm_linear, qmm_run
 */
#ifndef QMM_B200_H
#define QMM_B200_H

#include <stdbool.h>
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define QMM_ABI_VERSION 1

/* Status codes.  1-9 mirror src/weights.zig:23-33 WeightsError and
 * src/model.zig ModelError.MissingWeight; 20+ are device-side failures. */
typedef enum qmm_status {
    QMM_OK = 0,
    QMM_ERR_BAD_SHAPE = 1,            /* shapes disagree (x K vs W K, group divisibility, ...) */
    QMM_ERR_NONSTANDARD_QUANT = 2,    /* WeightsError.NonstandardQuant  (weights.zig:30) */
    QMM_ERR_INCONSISTENT_QUANT = 3,   /* WeightsError.InconsistentQuant (weights.zig:31) */
    QMM_ERR_AFFINE_UNSUPPORTED = 4,   /* WeightsError.AffineUnsupported (weights.zig:32) */
    QMM_ERR_UNSUPPORTED_DTYPE = 5,    /* WeightsError.UnsupportedDtype  (weights.zig:26) */
    QMM_ERR_BAD_MODE = 6,             /* mode string not "mxfp8"/"nvfp4", or group/bits mismatch */
    QMM_ERR_BAD_ARGUMENT = 7,         /* NULL pointer, transpose=false, biases given, bad stride */
    QMM_ERR_MISSING_WEIGHT = 8,       /* ModelError.MissingWeight (model.zig:220, :228) */
    QMM_ERR_BAD_INDEX_JSON = 10,      /* WeightsError.BadIndexJson      (weights.zig:24) */
    QMM_ERR_BAD_HEADER = 11,          /* WeightsError.BadHeader         (weights.zig:25) */
    QMM_ERR_UNSUPPORTED_LAYOUT = 12,  /* WeightsError.UnsupportedLayout (weights.zig:27) */
    QMM_ERR_MISSING_TENSOR = 13,      /* WeightsError.MissingTensor     (weights.zig:28) */
    QMM_ERR_DUPLICATE_TENSOR = 14,    /* WeightsError.DuplicateTensor   (weights.zig:29) */
    QMM_ERR_IO = 15,                  /* a checkpoint file could not be opened or read */
    QMM_ERR_CUDA = 20,                /* a CUDA runtime/driver call failed */
    QMM_ERR_OUT_OF_MEMORY = 21,       /* device allocation failed */
    QMM_ERR_NCCL = 22,                /* an NCCL call failed or NCCL could not be loaded */
    QMM_ERR_TIMEOUT = 23,             /* a bounded device-side wait gave up */
    QMM_ERR_NO_DEVICE = 24,           /* the current device is not an sm_100 part */
    QMM_ERR_INJECTED = 30             /* failure injected by qmm_fault_arm */
} qmm_status;

/* src/weights.zig:42 QuantMode. */
typedef enum qmm_mode { QMM_MODE_NONE = 0, QMM_MODE_MXFP8 = 1, QMM_MODE_NVFP4 = 2 } qmm_mode;

/* src/weights.zig:35 DType (the safetensors dtypes the loader accepts). */
typedef enum qmm_dtype {
    QMM_DTYPE_BF16 = 0, QMM_DTYPE_F32 = 1, QMM_DTYPE_U32 = 2, QMM_DTYPE_U8 = 3
} qmm_dtype;

/* src/weights.zig:43-55 QuantSpec. */
typedef struct qmm_quant_spec {
    int32_t mode;        /* qmm_mode */
    int32_t group_size;  /* 32 (mxfp8), 16 (nvfp4), 0 (none) */
    int32_t bits;        /* 8 (mxfp8), 4 (nvfp4), 0 (none) */
} qmm_quant_spec;

/* src/weights.zig:56-60 TensorInfo (one safetensors header entry). */
typedef struct qmm_tensor_info {
    const char* name;      /* NUL-terminated tensor name */
    int32_t dtype;         /* qmm_dtype */
    int32_t ndim;
    const int64_t* shape;  /* ndim extents */
} qmm_tensor_info;

/* src/mlx.zig:41-51 mlx_optional_int: same layout (int, then bool). */
typedef struct qmm_optional_int {
    int value;
    bool has_value;
} qmm_optional_int;

typedef struct qmm_weight qmm_weight;  /* opaque, owns device copies of codes + scales */
typedef struct qmm_comm qmm_comm;      /* opaque tensor-parallel communicator (NCCL) */
typedef struct qmm_checkpoint qmm_checkpoint;  /* opaque: an opened sharded safetensors checkpoint */

/* ---- spec inference (pure host; src/weights.zig:132-185) --------------- */

/* Infer (mode, group, bits) from the tensor infos of a whole checkpoint,
 * exactly as inferQuantSpec does: the first "*.scales" decides the ratio
 * r = packed_cols / scale_cols (8 -> mxfp8, 2 -> nvfp4), every scales
 * tensor must agree and every U32 "*.weight" needs its scales.  No scales
 * and no U32/U8 tensor -> mode NONE. */
int qmm_infer_quant_spec(const qmm_tensor_info* infos, int64_t count, qmm_quant_spec* out);

/* Mode string for a spec: "mxfp8" / "nvfp4" (src/weights.zig:47-53; NONE
 * maps to "mxfp8" there too, and is never used for a qmm). */
const char* qmm_mode_str(qmm_quant_spec spec);

/* Resolve mlx_quantized_matmul's (group_size, bits, mode) arguments into a
 * spec; unset optionals take the mode's defaults (32/8, 16/4). */
int qmm_spec_from_args(qmm_optional_int group_size, qmm_optional_int bits, const char* mode,
                       qmm_quant_spec* out);

/* ---- stateless operator (src/mlx.zig:265 mlx_quantized_matmul) ----------- */

/* y[M, N] = x[M, K] . dequant(w, scales)^T on `stream`.
 *   x_dev      bf16 [M, K], row stride ldx (elements)
 *   w_dev      U32  [w_rows = N, w_cols = K*bits/32]
 *   scales_dev U8   [s_rows = N, s_cols = K/group]
 *   biases     must be NULL (mxfp8/nvfp4 are bias-less, src/model.zig:230-232)
 *   transpose  must be true (the only form the reference uses, model.zig:253)
 *   y_dev      bf16 [M, N], row stride ldy (elements)
 * Every pointer must be memory of the current device (checked before any
 * launch: host memory or another GPU's buffer is QMM_ERR_BAD_ARGUMENT).
 * Reads the codes and scales in their checkpoint layout.  For M <= 8 with
 * 16-byte aligned x / code / scale rows it runs qmm_run's tensor-core decode
 * kernel, reading both tensors by TMA; its stream-K scratch (1.2 MB of
 * partial sums, 256 KB of counters) is a workspace the library makes on the
 * first call on each (device, stream) and keeps until the process exits.
 * That first call allocates and so cannot be captured in a CUDA graph (it
 * fails with QMM_ERR_BAD_ARGUMENT inside a capture): make one call on a
 * stream before capturing it.  Calls on different streams never share a
 * workspace.  Other shapes run a workspace-free split-K kernel. */
int qmm_quantized_matmul(void* y_dev, int64_t ldy,
                         const void* x_dev, int64_t m, int64_t k, int64_t ldx,
                         const uint32_t* w_dev, int64_t w_rows, int64_t w_cols,
                         const uint8_t* scales_dev, int64_t s_rows, int64_t s_cols,
                         const void* biases, bool transpose,
                         qmm_optional_int group_size, qmm_optional_int bits, const char* mode,
                         void* stream);

/* Same arguments, result (within the parity tolerance) and errors as
 * qmm_quantized_matmul, for callers that may not allocate device memory.  No
 * counterpart in the reference.  For M <= 8 it runs the tensor-core decode
 * kernel of qmm_run on the checkpoint-layout weights, with that kernel's
 * scratch (per-unit scale tiles, stream-K partial sums, counters) in one
 * static 8 MiB device array per device; cudaMalloc/cudaFree are never called.
 * A weight whose scratch exceeds 8 MiB fails with QMM_ERR_OUT_OF_MEMORY: the
 * scale tiles take N*K/16 (nvfp4) or N*K/32 (mxfp8) bytes and the partial
 * sums 1.2 MB, so N*K up to about 110 M (nvfp4) or 220 M (mxfp8) fits, e.g.
 * [5120, 17408] and [17408, 5120].  Other shapes take the
 * scratch-free kernels of qmm_quantized_matmul.
 *   - the first call on each device looks up the array's address
 *     (cudaGetSymbolAddress): make it before any stream capture begins;
 *   - calls that overlap in time on one device share the array and race:
 *     order them on one stream;
 *   - the array keeps the last call's contents after it returns;
 *   - the address is cached per device for the life of the process: after a
 *     cudaDeviceReset the entry point is unusable until the process restarts. */
int qmm_quantized_matmul_noalloc(void* y_dev, int64_t ldy,
                                 const void* x_dev, int64_t m, int64_t k, int64_t ldx,
                                 const uint32_t* w_dev, int64_t w_rows, int64_t w_cols,
                                 const uint8_t* scales_dev, int64_t s_rows, int64_t s_cols,
                                 const void* biases, bool transpose,
                                 qmm_optional_int group_size, qmm_optional_int bits, const char* mode,
                                 void* stream);

/* ---- resident weights (src/weights.zig:203-353 + src/model.zig:244) ----- */

#define QMM_SRC_HOST   0  /* codes/scales pointers are host memory */
#define QMM_SRC_DEVICE 1  /* codes/scales pointers are device memory (copied) */

/* Upload one quantized weight to the current device: the packed codes are
 * copied bit for bit, the scales once into the kernels' tiled layout, and
 * the split-K workspace is sized here so qmm_run never allocates.
 *   n, k   logical W shape (out features, in features)
 *   ldw    bytes between source code rows   (0: K*bits/8)
 *   lds    bytes between source scale rows  (0: K/group)
 * Blocks until the copies are done. */
int qmm_weight_create(const void* codes, const void* scales, int64_t n, int64_t k,
                      int64_t ldw, int64_t lds, qmm_quant_spec spec, int src_kind,
                      void* stream, qmm_weight** out);

/* Tensor-parallel shard of a full [n_full, k_full] weight: axis 0 takes the
 * rows [rank*n_full/P, (rank+1)*n_full/P) (column-parallel), axis 1 the
 * columns [rank*k_full/P, ...) (row-parallel).  A K-shard must start on a
 * group boundary and a whole U32 word. */
int qmm_weight_create_shard(const void* codes, const void* scales, int64_t n_full,
                            int64_t k_full, qmm_quant_spec spec, int src_kind, int axis,
                            int rank, int nranks, void* stream, qmm_weight** out);

/* The slice qmm_weight_create_shard takes (pure host): rows [*row0, *row0 +
 * *rows) and logical columns [*col0, *col0 + *cols) of the full weight. */
int qmm_shard_range(int64_t n_full, int64_t k_full, qmm_quant_spec spec, int axis, int rank,
                    int nranks, int64_t* row0, int64_t* rows, int64_t* col0, int64_t* cols);

int qmm_weight_destroy(qmm_weight* w);

/* n, k, spec and the device the weight lives on. */
int qmm_weight_info(const qmm_weight* w, int64_t* n, int64_t* k, qmm_quant_spec* spec,
                    int* device);

/* y[M, N] = x[M, K] . dequant(W)^T.  transpose must be true.  Calls on the
 * same handle must be ordered (same stream or externally synchronized):
 * the split-K workspace belongs to the handle. */
int qmm_run(const qmm_weight* w, const void* x_dev, int64_t m, int64_t ldx, void* y_dev,
            int64_t ldy, bool transpose, void* stream);

/* src/model.zig:218-233 namedLinearQ for one projection: `w` NULL with
 * `has_packed_u32` set is MissingWeight (a packed tensor without scales);
 * otherwise it forwards to qmm_run. */
int qmm_linear(const qmm_weight* w, bool has_packed_u32, const void* x_dev, int64_t m,
               int64_t ldx, void* y_dev, int64_t ldy, void* stream);

/* ---- checkpoint loading (src/weights.zig:72-121, :241-352) ----------------- */

/* WeightMap.load's reading of a sharded safetensors checkpoint, headers
 * only: model_dir/model.safetensors.index.json's "weight_map" names the
 * shards (BadIndexJson otherwise), visited in first-appearance order; per
 * shard checkShardFile (weights.zig:241-255) reads the u64 LE header length
 * (0 < n <= 256 MiB, else BadHeader) and parseHeaderJson (:72-121) the
 * entries: dtype BF16 / F32 / U32 / U8 (else UnsupportedDtype), a shape of
 * integers (else BadHeader), "conv1d.weight" ending in a unit dimension
 * (else UnsupportedLayout); here also data_offsets that match the shape and
 * stay inside the file (else BadHeader).  A name in two shards is
 * DuplicateTensor.  The checkpoint's spec comes from qmm_infer_quant_spec
 * over every header.  Names are kept as stored (the reference's name
 * sanitising is model-specific).  An unreadable file is QMM_ERR_IO. */
int qmm_checkpoint_open(const char* model_dir, qmm_checkpoint** out);
int qmm_checkpoint_close(qmm_checkpoint* c);
/* The inferred spec, and a view of every tensor (valid until close). */
int qmm_checkpoint_spec(const qmm_checkpoint* c, qmm_quant_spec* spec);
int qmm_checkpoint_tensors(const qmm_checkpoint* c, const qmm_tensor_info** infos, int64_t* count);
/* One tensor's bytes, as stored, into dst (QMM_SRC_HOST or QMM_SRC_DEVICE
 * memory of at least its size); MissingTensor if absent. */
int qmm_checkpoint_read(const qmm_checkpoint* c, const char* name, void* dst, int64_t dst_bytes,
                        int dst_kind);
/* The quantized linear "<prefix>.weight" (U32 codes) + "<prefix>.scales"
 * (U8) as a resident qmm_weight on the current device (qmm_weight_create:
 * codes bit for bit, scales re-tiled).  A missing .weight is MissingTensor,
 * a missing .scales MissingWeight (model.zig:226-228). */
int qmm_checkpoint_load_linear(const qmm_checkpoint* c, const char* prefix, void* stream,
                               qmm_weight** out);
/* A gate / up pair ("<gate_prefix>", "<up_prefix>") as one SwiGLU weight
 * (qmm_swiglu_weight_create). */
int qmm_checkpoint_load_swiglu(const qmm_checkpoint* c, const char* gate_prefix,
                               const char* up_prefix, void* stream, qmm_weight** out);

/* ---- fused gate / up projection with the SwiGLU epilogue ------------------- */

/* src/model.zig:905-915 mlpForwardQ without its last linear: g = x.Wg^T and
 * u = x.Wu^T (two namedLinearQ calls, model.zig:218-258), silu(g)
 * (model.zig:405-415: sigmoid, then g times it) and silu(g) * u
 * (model.zig:451 mul), each a bf16 array in the reference.  One resident
 * weight holds both tensors: gate and up rows are interleaved in 64-row
 * blocks (whole packed rows and scale rows, so the quantisation is bit for
 * bit), and one kernel writes h = silu(g) * u with the same four bf16
 * roundings.  gate_* and up_* are two [n, k] tensors of one spec (a fused
 * [2n, k] gate_up tensor passes its halves).  qmm_run and qmm_dequantize
 * refuse the result; qmm_weight_info reports n. */
int qmm_swiglu_weight_create(const void* gate_codes, const void* gate_scales,
                             const void* up_codes, const void* up_scales, int64_t n, int64_t k,
                             int64_t ldw, int64_t lds, qmm_quant_spec spec, int src_kind,
                             void* stream, qmm_weight** out);

/* h[M, n] = silu(x.Wg^T) * (x.Wu^T) in bf16.  M <= 8 runs the decode
 * kernel, M > 8 the tcgen05 GEMM, both with the SwiGLU epilogue; x rows
 * that are not 16-byte aligned take the unfused kernels with a
 * stream-ordered scratch of M x 2n bf16. */
int qmm_swiglu_run(const qmm_weight* w, const void* x_dev, int64_t m, int64_t ldx, void* h_dev,
                   int64_t ldh, void* stream);

/* ---- lm_head with greedy sampling ----------------------------------------- */

/* src/model.zig:1300-1310 logitsOf (the lm_head linear over the last M
 * hidden rows) followed, per row, by src/sample.zig:162-170 sampleToken at
 * temp == 0: ids[r] = argmax of the row's bf16 logits (mlx_argmax_axis;
 * here the lowest index among equal values, NaN above every number) and
 * logprobs[r] (nullable) = logprobOf (sample.zig:69-79) = logit[id] -
 * logsumexp(row), the logsumexp computed in fp32 and rounded to bf16 as the
 * reference's bf16 array is.  M <= 8 (decode, MTP verify).  The decode
 * kernel does it in its epilogue, so logits_dev may be NULL (no [M, N]
 * logits are written); when given, it receives them as qmm_run would. */
int qmm_lm_head_argmax(const qmm_weight* w, const void* x_dev, int64_t m, int64_t ldx,
                       int32_t* ids_dev, float* logprobs_dev, void* logits_dev, int64_t ldl,
                       void* stream);

/* src/mlx.zig:274 mlx_dequantize: out[N, K] in bf16 (out_dtype BF16) or fp32
 * (F32).  Every mxfp8/nvfp4 value is exact in fp32; bf16 is exact unless a
 * value leaves bf16's range. */
int qmm_dequantize(const qmm_weight* w, void* out_dev, int32_t out_dtype, void* stream);

/* src/mlx.zig:278 mlx_quantize, as the reference's qmm test calls it
 * (src/model.zig:1577: mode "mxfp8" / "nvfp4", global_scale NULL): w [N, K]
 * (w_dtype F32 or BF16, row stride ldw elements, 0 = K) on the device ->
 * codes U32 [N, K*bits/32] (LSB-first) and scales U8 [N, K/group], dense,
 * on `stream`; (group_size, bits, mode) resolve as in qmm_spec_from_args and
 * global_scale must be NULL.  Per group, amax = the largest magnitude (NaN
 * skipped):
 *   mxfp8 (OCP MX v1.0): X = floor(log2 amax) - 8 clamped to [-127, 127]
 *     (-127 for amax 0, -9 for an infinite amax), scale byte X + 127,
 *     code = E4M3(w * 2^-X);
 *   nvfp4: scale = E4M3(amax / 6), code = E2M1(w / scale) (0 if scale is 0).
 * E4M3 / E2M1 round to nearest even and saturate (448, 6); NaN is 0x7F
 * (E4M3) or sign|7 (E2M1).  Deterministic and bit-identical to the CPU
 * restatement of these rules. */
int qmm_quantize(const void* w_dev, int32_t w_dtype, int64_t n, int64_t k, int64_t ldw,
                 qmm_optional_int group_size, qmm_optional_int bits, const char* mode,
                 const void* global_scale, uint32_t* codes_dev, uint8_t* scales_dev, void* stream);

/* ---- tensor parallel (NCCL over NVLink) ----------------------------------- */

/* 128-byte NCCL unique id, produced on one rank and broadcast by the caller. */
int qmm_tp_unique_id(void* id128);
/* One communicator per rank (current device).  max_partial_elems sizes the
 * fp32 partial-sum buffer of qmm_tp_run_rowparallel (m * n at most), which
 * is allocated here so the run itself never allocates. */
int qmm_tp_comm_create(const void* id128, int nranks, int rank, int64_t max_partial_elems,
                       qmm_comm** out);
int qmm_tp_comm_destroy(qmm_comm* c);
/* Test hook, no reference counterpart (beside the fault hooks of
 * src/mlx.zig:562-595): a communicator of `nranks` ranks (2..8) in which this
 * process is `rank` and the other ranks never run - their receive buffers and
 * flags are local allocations that nothing else writes, and no NCCL is used.
 * qmm_tp_run_rowparallel on it takes the fused decode exchange (M <= 8, a
 * resident weight with decode state, 16-byte aligned x rows; anything else is
 * QMM_ERR_BAD_ARGUMENT), pushes its partial sums, waits the bounded 2 s for the
 * absent ranks, gives up and writes y from what it has; qmm_device_status then
 * reports QMM_ERR_TIMEOUT.  This exercises the device-side failure path on one
 * GPU without a fault or a hang. */
int qmm_tp_comm_create_detached(int nranks, int rank, int64_t max_partial_elems, qmm_comm** out);

/* In-place bf16 sum all-reduce of `count` elements on `stream`. */
int qmm_tp_allreduce_bf16(qmm_comm* c, void* buf_dev, int64_t count, void* stream);

/* Row-parallel projection: y = allreduce_sum(x_shard . W_shard^T), with x_dev
 * this rank's K-slice.  The partials are summed in fp32 and rounded to bf16
 * once.  Column-parallel shards need no collective: use qmm_run on them. */
int qmm_tp_run_rowparallel(const qmm_weight* w, qmm_comm* c, const void* x_dev, int64_t m,
                           int64_t ldx, void* y_dev, int64_t ldy, void* stream);

/* ---- errors and test hooks ------------------------------------------------ */

/* Copy the latched message of the first failure since the last call into
 * buf (NUL-terminated, truncated to len) and clear the latch.  Returns the
 * latched status (QMM_OK if none).  src/mlx.zig:792 takeError. */
int qmm_last_error(char* buf, size_t len);

/* Status of the bounded device-side waits since the last call: QMM_OK, or
 * QMM_ERR_TIMEOUT if a kernel gave up a wait (it then skipped the rest of its
 * work and released its resources; the word is cleared).  Synchronizes
 * `stream`; the reference surfaces asynchronous device failures the same way
 * at its checkError points (src/mlx.zig:858-866). */
int qmm_device_status(void* stream);

/* 1 when a failure is latched (src/mlx.zig:778 errorPending). */
int qmm_error_pending(void);

/* Make the k-th checked entry-point call from now fail with QMM_ERR_INJECTED
 * (k >= 1; 0 disarms).  Mirrors the test-only src/mlx.zig:562-595 fault.arm;
 * the failure is injected on the host before any device work is enqueued. */
int qmm_fault_arm(uint64_t k);
/* 1 if the armed fault fired (src/mlx.zig:581 didFire). */
int qmm_fault_fired(void);

int qmm_abi_version(void);

/* x-quantised prefill on the block-scaled tensor cores - NOT the parity
 * path, no counterpart in the reference's own code (MLX's block-scaled
 * kernels are the closest analogue).  y[M, N] = q(x) . dequant(W)^T, where
 * q(x) quantises each 16-value group of x to nvfp4 by qmm_quantize's rules
 * (E2M1 codes, UE4M3 scale) and the product runs as tcgen05.mma
 * kind::mxf4nvf4.block_scale on the packed codes of both operands, fp32
 * accumulation, bf16 out.  Quantising x costs about 10% relative error, far
 * outside qmm_run's parity bar: callers opt in by calling this entry point.
 * nvfp4 weights only, K a multiple of 32.  The first call on a weight builds
 * its scale-factor tiles (allocates; not inside a graph capture); every call
 * takes its x scratch (about M*K*9/16 bytes) from the stream-ordered
 * allocator. */
int qmm_run_blockscaled(qmm_weight* w, const void* x_dev, int64_t m, int64_t ldx, void* y_dev, int64_t ldy,
                        void* stream);

/* Measurement hook, no counterpart in the reference: the dense tcgen05 MMA
 * rate of the current device for one MMA kind (0 = kind::f16 bf16, 1 =
 * kind::mxf8f6f4 E4M3 with UE8M0 scales per 32, 2 = kind::mxf4nvf4 E2M1 with
 * UE4M3 scales per 16), from one timed launch of `iters` back-to-back
 * 128 x 256 MMA pairs per SM on `stream`; *tflops receives the rate.  These
 * are the roofline denominators of the prefill GEMMs (bench.py).
 * Synchronizes `stream`. */
int qmm_tensor_peak(int kind, int64_t iters, void* stream, double* tflops);

#ifdef __cplusplus
}
#endif
#endif /* QMM_B200_H */
