// formats.cuh - device-side decoding of the mxfp8 / nvfp4 element and scale
// formats (sm_100a).  Every conversion here is exact:
//   E4M3 -> f16   (every E4M3 value, subnormals included, is a normal f16)
//   E2M1 -> f16
//   UE8M0 -> f32  2^(e-127), 0xFF -> NaN (e = 0 is the f32 subnormal 2^-127)
//   UE4M3 -> f32  via E4M3
// Codes are packed LSB-first: byte b of a row holds code b (mxfp8) or codes
// 2b (low nibble) and 2b+1 (high nibble) (nvfp4).
#pragma once

#include <cstdint>
#include <cuda_fp16.h>

namespace qmm {

// Two E4M3 codes (low byte = first code) -> f16x2 (low half = first code).
__device__ __forceinline__ uint32_t e4m3x2_to_f16x2(uint16_t v) {
    uint32_t out;
    asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(out) : "h"(v));
    return out;
}

// One byte of two E2M1 codes (low nibble = first code) -> f16x2.
__device__ __forceinline__ uint32_t e2m1x2_to_f16x2(uint32_t byte_in_low_bits) {
    uint32_t out;
    asm("{\n\t.reg .b8 b;\n\t"
        "cvt.u8.u32 b, %1;\n\t"
        "cvt.rn.f16x2.e2m1x2 %0, b;\n\t}"
        : "=r"(out) : "r"(byte_in_low_bits));
    return out;
}

// Four E2M1 code pairs of a 32-bit word -> four f16x2 (in code order).
__device__ __forceinline__ void e2m1x8_to_f16x2(uint32_t w, uint32_t (&out)[4]) {
    asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\t"
        "mov.b32 {b0, b1, b2, b3}, %4;\n\t"
        "cvt.rn.f16x2.e2m1x2 %0, b0;\n\t"
        "cvt.rn.f16x2.e2m1x2 %1, b1;\n\t"
        "cvt.rn.f16x2.e2m1x2 %2, b2;\n\t"
        "cvt.rn.f16x2.e2m1x2 %3, b3;\n\t}"
        : "=r"(out[0]), "=r"(out[1]), "=r"(out[2]), "=r"(out[3]) : "r"(w));
}

// Four E4M3 codes of a 32-bit word -> two f16x2 (in code order).
__device__ __forceinline__ void e4m3x4_to_f16x2(uint32_t w, uint32_t (&out)[2]) {
    out[0] = e4m3x2_to_f16x2(static_cast<uint16_t>(w & 0xFFFFu));
    out[1] = e4m3x2_to_f16x2(static_cast<uint16_t>(w >> 16));
}

__device__ __forceinline__ float2 f16x2_to_float2(uint32_t h) {
    __half2 v = *reinterpret_cast<__half2*>(&h);
    return __half22float2(v);
}

// UE8M0 scale byte -> f32.
__device__ __forceinline__ float ue8m0_to_f32(uint32_t e) {
    if (e == 0xFFu) return __uint_as_float(0x7FC00000u);
    if (e == 0u) return __uint_as_float(0x00400000u);  // 2^-127 (f32 subnormal)
    return __uint_as_float(e << 23);
}

// UE4M3 scale byte -> f32 (decoded as E4M3, sign bit included).
__device__ __forceinline__ float ue4m3_to_f32(uint32_t b) {
    uint32_t h = e4m3x2_to_f16x2(static_cast<uint16_t>(b & 0xFFu));
    return __half2float(__ushort_as_half(static_cast<unsigned short>(h & 0xFFFFu)));
}

template <int FMT>
__device__ __forceinline__ float scale_to_f32(uint32_t b) {
    if constexpr (FMT == 0) return ue8m0_to_f32(b);
    else return ue4m3_to_f32(b);
}

// bf16 pair (low half = first element) -> float2.
__device__ __forceinline__ float2 bf16x2_to_float2(uint32_t u) {
    return make_float2(__uint_as_float(u << 16), __uint_as_float(u & 0xFFFF0000u));
}

// float -> bf16 bits, round to nearest even (NaN stays NaN).
__device__ __forceinline__ uint16_t f32_to_bf16(float f) {
    uint16_t r;
    asm("cvt.rn.bf16.f32 %0, %1;" : "=h"(r) : "f"(f));
    return r;
}

__device__ __forceinline__ uint32_t f32x2_to_bf16x2(float lo, float hi) {
    uint32_t r;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    return r;
}

__device__ __forceinline__ float bf16_to_f32(uint16_t b) { return __uint_as_float((uint32_t)b << 16); }

// silu(g) * u from the fp32 gate / up sums of two outputs (g0, u0) and
// (g1, u1), bf16x2 out (low half = first), with the reference's sequence of
// bf16 arrays (src/model.zig:905-915 mlpForwardQ: g and u are bf16 linear
// outputs; silu (model.zig:405-415) is sigmoid(g) then g * sigmoid(g), each
// a bf16 array; then that times u): g, u and sigmoid(g) are rounded to bf16
// (nearest even), and the two products are bf16 multiplies, which round the
// exact product once - as fp32 products rounded to bf16 would.  The sigmoid
// itself is computed in fp32 to about 2 ulp before its bf16 rounding.
__device__ __forceinline__ uint32_t swiglu_bf16x2(float g0, float g1, float u0, float u1) {
    const uint32_t gb = f32x2_to_bf16x2(g0, g1), ub = f32x2_to_bf16x2(u0, u1);
    const float2 g = bf16x2_to_float2(gb);
    const float s0 = __fdividef(1.0f, 1.0f + __expf(-g.x));
    const float s1 = __fdividef(1.0f, 1.0f + __expf(-g.y));
    const uint32_t sb = f32x2_to_bf16x2(s0, s1);
    uint32_t t, h;
    asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(t) : "r"(gb), "r"(sb));
    asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(h) : "r"(t), "r"(ub));
    return h;
}

__device__ __forceinline__ uint16_t swiglu_bf16(float g, float u) {
    return static_cast<uint16_t>(swiglu_bf16x2(g, 0.0f, u, 0.0f) & 0xFFFFu);
}

}  // namespace qmm
