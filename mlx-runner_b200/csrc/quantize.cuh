// quantize.cuh - the mxfp8 / nvfp4 quantization rules, as host + device code.
//
// Counterpart of mlx_quantize (src/mlx.zig:278) as the reference's qmm test
// calls it (src/model.zig:1577: mode "mxfp8" / "nvfp4", no global scale).
// For every group of `group` consecutive values of a row, with amax the
// largest magnitude of the group (every NaN is skipped, signalling ones too):
//   mxfp8 (OCP MX v1.0): shared exponent X = floor(log2(amax)) - 8, 8 being
//     the largest E4M3 exponent, clamped to UE8M0's [-127, 127]; X = -127
//     when amax = 0 and X = -9 when amax is infinite (frexp's exponent 0);
//     scale byte X + 127; code = E4M3(w * 2^-X).
//   nvfp4: scale byte = E4M3(amax / 6), 6 being the largest E2M1 value;
//     code = E2M1(w / decoded scale), or 0 when the decoded scale is 0.
// E4M3 and E2M1 round to nearest even and saturate at their largest finite
// value (448, 6); NaN encodes as 0x7F (E4M3) and as sign | 7 (E2M1).  Every
// step is exact or one IEEE round-to-nearest fp32 operation (the scaling
// product, the two divisions), so host and device produce the same bytes.
#pragma once

#include <cstdint>
#include <cstring>
#include <cmath>

#if defined(__CUDACC__)
#define QMM_HD __host__ __device__ __forceinline__
#else
#define QMM_HD inline
#endif

namespace qmm {
namespace quant {

QMM_HD uint32_t f32_bits(float v) {
#if defined(__CUDA_ARCH__)
    return __float_as_uint(v);
#else
    uint32_t u;
    std::memcpy(&u, &v, 4);
    return u;
#endif
}

QMM_HD float bits_f32(uint32_t u) {
#if defined(__CUDA_ARCH__)
    return __uint_as_float(u);
#else
    float v;
    std::memcpy(&v, &u, 4);
    return v;
#endif
}

QMM_HD int clz32(uint32_t v) {
#if defined(__CUDA_ARCH__)
    return __clz(static_cast<int>(v));
#else
    return __builtin_clz(v);
#endif
}

// One IEEE round-to-nearest-even product / quotient (never contracted into
// an FMA).
QMM_HD float mul_rn(float a, float b) {
#if defined(__CUDA_ARCH__)
    return __fmul_rn(a, b);
#else
    volatile float r = a * b;
    return r;
#endif
}

QMM_HD float div_rn(float a, float b) {
#if defined(__CUDA_ARCH__)
    return __fdiv_rn(a, b);
#else
    volatile float r = a / b;
    return r;
#endif
}

// Nearest integer, ties to even (the default rounding mode on both sides).
QMM_HD float rint_even(float a) {
#if defined(__CUDA_ARCH__)
    return rintf(a);
#else
    return std::nearbyint(a);
#endif
}

// 2^e as an fp32, e in [-149, 127] (subnormal below -126).
QMM_HD float pow2f(int e) {
    return e >= -126 ? bits_f32(static_cast<uint32_t>(e + 127) << 23) : bits_f32(1u << (e + 149));
}

// floor(log2(a)) of a finite a > 0, subnormals included.
QMM_HD int ilog2f(float a) {
    const uint32_t u = f32_bits(a);
    const int e = static_cast<int>(u >> 23);
    if (e) return e - 127;
    return (31 - clz32(u & 0x7FFFFFu)) - 149;
}

QMM_HD bool is_nan_bits(uint32_t u) { return (u & 0x7FFFFFFFu) > 0x7F800000u; }

// The running maximum of magnitudes: a NaN `a` (quiet or signalling) never
// wins the compare, so amax skips every NaN.
QMM_HD float max_skip_nan(float amax, float a) { return a > amax ? a : amax; }

// fp32 -> E4M3 ("fn": bias 7, max 448, S.1111.111 = NaN).
QMM_HD uint32_t encode_e4m3(float v) {
    const uint32_t u = f32_bits(v);
    if (is_nan_bits(u)) return 0x7Fu;
    const uint32_t s = (u >> 24) & 0x80u;
    const float a = bits_f32(u & 0x7FFFFFFFu);
    if (a >= 448.0f) return s | 0x7Eu;
    if (a == 0.0f) return s;
    int e = ilog2f(a);
    if (e < -6) return s | static_cast<uint32_t>(rint_even(mul_rn(a, 512.0f)));  // quantum 2^-9; 8 = 2^-6
    int q = static_cast<int>(rint_even(mul_rn(a, pow2f(3 - e))));             // 1.mmm in eighths: [8, 16]
    if (q >= 16) { ++e; q = 8; }
    uint32_t code = static_cast<uint32_t>(((e + 7) << 3) | (q - 8));
    if (code > 0x7Eu) code = 0x7Eu;
    return s | code;
}

// fp32 -> E2M1 (magnitudes 0, .5, 1, 1.5, 2, 3, 4, 6; sign in bit 3).
QMM_HD uint32_t encode_e2m1(float v) {
    const uint32_t u = f32_bits(v);
    const uint32_t s = (u >> 28) & 0x8u;
    if (is_nan_bits(u)) return s | 0x7u;
    const float a = bits_f32(u & 0x7FFFFFFFu);
    if (a >= 6.0f) return s | 0x7u;
    if (a == 0.0f) return s;
    int e = ilog2f(a);
    if (e < 0) return s | static_cast<uint32_t>(rint_even(mul_rn(a, 2.0f)));   // quantum 0.5; 2 = 1.0
    int q = static_cast<int>(rint_even(mul_rn(a, pow2f(1 - e))));             // 1.m in halves: [2, 4]
    if (q >= 4) { ++e; q = 2; }
    uint32_t code = static_cast<uint32_t>(((e + 1) << 1) | (q - 2));
    if (code > 7u) code = 7u;
    return s | code;
}

// E4M3 code (not NaN) -> its exact fp32 value.
QMM_HD float e4m3_value(uint32_t c) {
    const int e = static_cast<int>((c >> 3) & 0xFu), m = static_cast<int>(c & 7u);
    const float v = e == 0 ? mul_rn(static_cast<float>(m), pow2f(-9)) : mul_rn(static_cast<float>(8 + m), pow2f(e - 10));
    return (c & 0x80u) ? -v : v;
}

// mxfp8 shared exponent X of a group (amax >= 0, not NaN).
QMM_HD int mx_shared_exp(float amax) {
    if (amax == 0.0f) return -127;
    if (f32_bits(amax) == 0x7F800000u) return -9;
    int x = ilog2f(amax) - 8;
    return x < -127 ? -127 : (x > 127 ? 127 : x);
}

// nvfp4 code of one value under the decoded group scale sd (>= 0).
QMM_HD uint32_t nvfp4_code(float v, float sd) {
    if (!(sd > 0.0f)) return 0u;
    const uint32_t u = f32_bits(v);
    if (is_nan_bits(u)) return ((u >> 28) & 0x8u) | 0x7u;    // NaN / sd keeps the sign of v
    return encode_e2m1(div_rn(v, sd));
}

}  // namespace quant
}  // namespace qmm
