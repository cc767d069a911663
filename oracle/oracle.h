/*
 * oracle.h - CPU restatement of mlx-runner's quantized linear-layer arithmetic.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the product (the qmm_b200 library,
 * its C ABI or the Python binding) links, loads or calls this code.  Only
 * tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference
 * arm may use it, and there only as the checker or the timed CPU baseline.
 *
 * What it restates (file:line relative to the mlx-runner source tree):
 *   - the operator  y = x . dequant(W)^T  that src/model.zig:244-258 (qlinear)
 *     asks libmlx for via mlx_quantized_matmul(..., transpose=true,
 *     group, bits, mode) with biases = null and no global scale;
 *   - the (mode, group, bits) pairs of src/weights.zig:37-55
 *     (mxfp8 = E4M3 codes, group 32, UE8M0 scale; nvfp4 = E2M1 codes,
 *     group 16, UE4M3 scale);
 *   - the packed shapes of src/weights.zig:154-161: U32 [N, K*bits/32]
 *     codes and U8 [N, K/group] scales.
 *
 * The arithmetic itself lives in third-party libmlx (mlx==0.32.2, pinned by
 * scripts/build-mlx.sh:46), which is not part of the reference tree and
 * cannot be built or run here.  The format definitions restated below are
 * the published ones: OCP Microscaling Formats (MX) v1.0 for E4M3 / UE8M0 /
 * group 32, and NVIDIA's NVFP4 definition for E2M1 / UE4M3 / group 16.
 *
 * Parity status: the decode tables are pinned against an independent
 * implementation (ml_dtypes) by tests/golden; the spec rule and the packed
 * shapes are pinned by the reference's own tests (src/weights.zig:493-541);
 * the integer wiring case of src/model.zig:1561-1609 is pinned exactly.
 * MLX's own quantize/qmm outputs are NOT available, so numeric parity with
 * libmlx itself is unpinned: the quantizer here is a test-data generator
 * that follows the OCP / NVFP4 rules, not a copy of MLX's scale selection.
 *
 * Packing assumption (not pinned by the reference, which fixes only shapes):
 * codes are packed LSB-first into each little-endian U32, so as a byte
 * stream element k of a row is byte k (mxfp8) or nibble (k & 1) of byte k/2,
 * low nibble first (nvfp4).
 */
#ifndef QMM_ORACLE_H
#define QMM_ORACLE_H

#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

enum { ORC_MXFP8 = 1, ORC_NVFP4 = 2 };

/* Scalar format decoders (exact; return NaN for the NaN encodings). */
float orc_decode_e4m3(uint8_t code);
float orc_decode_e2m1(uint8_t nibble);
float orc_decode_ue8m0(uint8_t code);
float orc_decode_ue4m3(uint8_t code);

/* Round-to-nearest-even encoders with saturation to the largest finite value. */
uint8_t orc_encode_e4m3(float v);
uint8_t orc_encode_e2m1(float v);

/* bf16 helpers: round-to-nearest-even, NaN kept quiet. */
uint16_t orc_f32_to_bf16(float v);
float orc_bf16_to_f32(uint16_t b);

/* Quantize fp32 W [N, K] row-major into packed codes (bytes; K*bits/8 per
 * row, identical to the U32 [N, K*bits/32] little-endian buffer) and U8
 * scales [N, K/group].  Returns 0, or -1 on a bad mode/shape. */
int orc_quantize(int mode, const float* w, int64_t n, int64_t k,
                 uint8_t* codes, uint8_t* scales);

/* Dequantize to fp32 W [N, K] (every value is exact in fp32). */
int orc_dequantize(int mode, const uint8_t* codes, const uint8_t* scales,
                   int64_t n, int64_t k, float* out);

/* fp64 dequantise-then-matmul: y[m, n] = sum_k x[m, k] * W[n, k], x in bf16
 * bits [M, K] (row stride ldx), y fp64 [M, N].  OpenMP over N. */
int orc_qmm_f64(int mode, const uint16_t* x, int64_t m, int64_t ldx,
                const uint8_t* codes, const uint8_t* scales, int64_t n, int64_t k,
                double* y);

/* orc_qmm_f64 and, in yabs [M, N], sum_k |x[m, k]| * |W[n, k]| (NaN weights
 * count 0): the scale of the accumulation error, in one pass over W. */
int orc_qmm_f64_abs(int mode, const uint16_t* x, int64_t m, int64_t ldx,
                    const uint8_t* codes, const uint8_t* scales, int64_t n, int64_t k,
                    double* y, double* yabs);

/* The timed CPU baseline: dequantize on the fly, fp32 accumulate, bf16
 * output (RNE) [M, N].  Uses `threads` OpenMP threads (<=0: all). */
int orc_qmm_f32(int mode, const uint16_t* x, int64_t m, int64_t ldx,
                const uint8_t* codes, const uint8_t* scales, int64_t n, int64_t k,
                uint16_t* y, int threads);

int orc_max_threads(void);

#ifdef __cplusplus
}
#endif
#endif
