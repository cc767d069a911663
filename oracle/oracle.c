/*
 * oracle.c - CPU restatement of the mxfp8 / nvfp4 quantized matmul.
 *
 * TEST INFRASTRUCTURE ONLY (see oracle.h): the checker for the CUDA path and
 * the timed CPU baseline.  The product never links or calls it.
 *
 * Reference anchors (mlx-runner tree):
 *   src/model.zig:244-258   qlinear -> mlx_quantized_matmul(x, w, scales,
 *                           biases=null, transpose=true, group, bits, mode)
 *   src/weights.zig:37-55   QuantSpec: mxfp8 = (32, 8), nvfp4 = (16, 4)
 *   src/weights.zig:154-161 packed U32 [N, K*bits/32], U8 scales [N, K/group]
 *   src/model.zig:1561-1609 the reference's only numeric qmm test
 * The element formats follow OCP MX v1.0 (E4M3, UE8M0) and NVFP4 (E2M1,
 * UE4M3 scale); libmlx's own sources (mlx==0.32.2) are not available.
 */
#include "oracle.h"

#include <math.h>
#include <string.h>
#include <stdlib.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* ---- scalar decoders ---------------------------------------------------- */

/* E4M3 ("fn" variant): bias 7, no infinities, S.1111.111 is NaN, max 448. */
float orc_decode_e4m3(uint8_t code) {
    int s = code >> 7, e = (code >> 3) & 0xF, m = code & 7;
    float v;
    if (e == 15 && m == 7) return NAN;
    if (e == 0) v = ldexpf((float)m, -9);                 /* subnormal: m * 2^-9 */
    else v = ldexpf(1.0f + (float)m / 8.0f, e - 7);
    return s ? -v : v;
}

/* E2M1: magnitudes {0, .5, 1, 1.5, 2, 3, 4, 6} and a sign bit (bit 3). */
float orc_decode_e2m1(uint8_t nib) {
    int s = (nib >> 3) & 1, e = (nib >> 1) & 3, m = nib & 1;
    float v = (e == 0) ? 0.5f * (float)m : ldexpf(1.0f + 0.5f * (float)m, e - 1);
    return s ? -v : v;
}

/* UE8M0: 2^(e-127); 0xFF is NaN. */
float orc_decode_ue8m0(uint8_t code) {
    if (code == 0xFF) return NAN;
    return ldexpf(1.0f, (int)code - 127);
}

/* UE4M3 scale byte: decoded as an E4M3 value.  The NVFP4 quantizer only
 * produces non-negative scales (sign bit clear); a set sign bit is decoded
 * as a negative scale rather than silently dropped. */
float orc_decode_ue4m3(uint8_t code) { return orc_decode_e4m3(code); }

/* ---- encoders (test-data generator) ------------------------------------ */

uint8_t orc_encode_e4m3(float v) {
    if (isnan(v)) return 0x7F;
    uint8_t s = signbit(v) ? 0x80 : 0;
    double a = fabs((double)v);
    if (a >= 448.0) return s | 0x7E;                      /* satfinite */
    if (a == 0.0) return s;
    int ex;
    frexp(a, &ex);                                        /* a = f * 2^ex, f in [.5,1) */
    int E = ex - 1;
    if (E < -6) {                                         /* subnormal quantum 2^-9 */
        double n = nearbyint(ldexp(a, 9));
        return s | (uint8_t)n;                            /* n == 8 is 2^-6, code 0x08 */
    }
    double n = nearbyint(ldexp(a, 3 - E));                /* in [8, 16] */
    if (n >= 16.0) { E += 1; n = 8.0; }
    int code = ((E + 7) << 3) | ((int)n - 8);
    if (code > 0x7E) code = 0x7E;
    return s | (uint8_t)code;
}

uint8_t orc_encode_e2m1(float v) {
    uint8_t s = signbit(v) ? 0x8 : 0;
    if (isnan(v)) return s | 0x7;
    double a = fabs((double)v);
    if (a >= 6.0) return s | 0x7;                         /* satfinite */
    int ex;
    if (a == 0.0) return s;
    frexp(a, &ex);
    int E = ex - 1;
    if (E < 0) {                                          /* quantum 0.5 */
        double n = nearbyint(a * 2.0);                    /* 0, 1 or 2 (= 1.0) */
        return s | (uint8_t)n;
    }
    double n = nearbyint(ldexp(a, 1 - E));                /* in [2, 4] */
    if (n >= 4.0) { E += 1; n = 2.0; }
    int code = ((E + 1) << 1) | ((int)n - 2);
    if (code > 7) code = 7;
    return s | (uint8_t)code;
}

uint16_t orc_f32_to_bf16(float v) {
    uint32_t u;
    memcpy(&u, &v, 4);
    if ((u & 0x7FFFFFFFu) > 0x7F800000u) return (uint16_t)((u >> 16) | 0x40);
    u += 0x7FFFu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

float orc_bf16_to_f32(uint16_t b) {
    uint32_t u = (uint32_t)b << 16;
    float v;
    memcpy(&v, &u, 4);
    return v;
}

/* ---- layout helpers ------------------------------------------------------ */

static int spec_of(int mode, int* group, int* bits) {
    if (mode == ORC_MXFP8) { *group = 32; *bits = 8; return 0; }
    if (mode == ORC_NVFP4) { *group = 16; *bits = 4; return 0; }
    return -1;
}

/* Code k of one packed row (LSB-first inside each little-endian U32). */
static inline uint8_t code_at(const uint8_t* row, int bits, int64_t k) {
    if (bits == 8) return row[k];
    return (uint8_t)((row[k >> 1] >> ((k & 1) * 4)) & 0xF);
}

static inline float scale_of(int mode, uint8_t s) {
    return mode == ORC_MXFP8 ? orc_decode_ue8m0(s) : orc_decode_ue4m3(s);
}

static inline float elem_of(int mode, uint8_t c) {
    return mode == ORC_MXFP8 ? orc_decode_e4m3(c) : orc_decode_e2m1(c);
}

/* ---- quantize / dequantize --------------------------------------------- */

int orc_quantize(int mode, const float* w, int64_t n, int64_t k,
                 uint8_t* codes, uint8_t* scales) {
    int group, bits;
    if (spec_of(mode, &group, &bits) || n < 0 || k <= 0 || k % group) return -1;
    const int64_t row_bytes = k * bits / 8, ng = k / group;
    #pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < n; ++r) {
        const float* wr = w + r * k;
        uint8_t* cr = codes + r * row_bytes;
        if (bits == 4) memset(cr, 0, (size_t)row_bytes);
        for (int64_t g = 0; g < ng; ++g) {
            const float* v = wr + g * group;
            float amax = 0.f;
            /* Every NaN is skipped, signalling ones too (a compare, not
             * fmaxf, whose C library may propagate a signalling NaN). */
            for (int i = 0; i < group; ++i) {
                const float a = fabsf(v[i]);
                if (a > amax) amax = a;
            }
            if (mode == ORC_MXFP8) {
                /* OCP MX v1.0: X = 2^(floor(log2(amax)) - emax_elem), emax(E4M3) = 8 */
                int se = -127;
                if (amax > 0.f) {
                    int ex;
                    frexpf(amax, &ex);
                    se = (ex - 1) - 8;
                    if (se < -127) se = -127;
                    if (se > 127) se = 127;
                }
                scales[r * ng + g] = (uint8_t)(se + 127);
                for (int i = 0; i < group; ++i)
                    cr[g * group + i] = orc_encode_e4m3((float)ldexp((double)v[i], -se));
            } else {
                /* NVFP4: scale = amax / 6 rounded to E4M3; codes = RNE(w / scale).
                 * Both divisions are single fp32 operations, so the rounded
                 * inputs of the encoders are reproducible bit for bit. */
                uint8_t sq = orc_encode_e4m3(amax / 6.0f);
                float sd = orc_decode_e4m3(sq);
                scales[r * ng + g] = sq;
                for (int i = 0; i < group; ++i) {
                    uint8_t c = sd > 0.f ? orc_encode_e2m1(v[i] / sd) : 0;
                    int64_t kk = g * group + i;
                    cr[kk >> 1] |= (uint8_t)(c << ((kk & 1) * 4));
                }
            }
        }
    }
    return 0;
}

int orc_dequantize(int mode, const uint8_t* codes, const uint8_t* scales,
                   int64_t n, int64_t k, float* out) {
    int group, bits;
    if (spec_of(mode, &group, &bits) || n < 0 || k <= 0 || k % group) return -1;
    const int64_t row_bytes = k * bits / 8, ng = k / group;
    #pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < n; ++r) {
        const uint8_t* cr = codes + r * row_bytes;
        for (int64_t kk = 0; kk < k; ++kk)
            out[r * k + kk] = elem_of(mode, code_at(cr, bits, kk)) *
                              scale_of(mode, scales[r * ng + kk / group]);
    }
    return 0;
}

/* ---- matmuls ------------------------------------------------------------ */

int orc_qmm_f64(int mode, const uint16_t* x, int64_t m, int64_t ldx,
                const uint8_t* codes, const uint8_t* scales, int64_t n, int64_t k,
                double* y) {
    int group, bits;
    if (spec_of(mode, &group, &bits) || m < 0 || n < 0 || k <= 0 || k % group || ldx < k) return -1;
    const int64_t row_bytes = k * bits / 8, ng = k / group;
    double* xd = (double*)malloc(sizeof(double) * (size_t)(m * k + 1));
    if (!xd) return -1;
    for (int64_t i = 0; i < m; ++i)
        for (int64_t kk = 0; kk < k; ++kk) xd[i * k + kk] = orc_bf16_to_f32(x[i * ldx + kk]);
    int bad = 0;
    #pragma omp parallel
    {
        double* w = (double*)malloc(sizeof(double) * (size_t)k);
        if (!w) {
            #pragma omp atomic write
            bad = 1;
        } else {
            #pragma omp for schedule(static)
            for (int64_t r = 0; r < n; ++r) {
                const uint8_t* cr = codes + r * row_bytes;
                for (int64_t kk = 0; kk < k; ++kk)
                    w[kk] = (double)elem_of(mode, code_at(cr, bits, kk)) *
                            (double)scale_of(mode, scales[r * ng + kk / group]);
                for (int64_t i = 0; i < m; ++i) {
                    const double* xr = xd + i * k;
                    double acc = 0.0;
                    for (int64_t kk = 0; kk < k; ++kk) acc += xr[kk] * w[kk];
                    y[i * n + r] = acc;
                }
            }
            free(w);
        }
    }
    free(xd);
    return bad ? -1 : 0;
}

/* y and sum_k |x| |W| in one pass, for checks at full benchmark sizes (no
 * [N, K] intermediate).  Four partial sums per dot product keep the fp64
 * adds from forming one long dependency chain; in fp64 the order changes the
 * result by ~1e-16 relative, far below every bar the tests apply.  A NaN
 * weight contributes NaN to y and 0 to the absolute sum (as abs_qmm_f64). */
int orc_qmm_f64_abs(int mode, const uint16_t* x, int64_t m, int64_t ldx,
                    const uint8_t* codes, const uint8_t* scales, int64_t n, int64_t k,
                    double* y, double* yabs) {
    int group, bits;
    if (spec_of(mode, &group, &bits) || m < 0 || n < 0 || k <= 0 || k % group || ldx < k) return -1;
    const int64_t row_bytes = k * bits / 8, ng = k / group;
    double* xd = (double*)malloc(sizeof(double) * (size_t)(2 * m * k + 1));
    if (!xd) return -1;
    double* xa = xd + m * k;
    for (int64_t i = 0; i < m; ++i)
        for (int64_t kk = 0; kk < k; ++kk) {
            xd[i * k + kk] = orc_bf16_to_f32(x[i * ldx + kk]);
            xa[i * k + kk] = fabs(xd[i * k + kk]);
        }
    int bad = 0;
    #pragma omp parallel
    {
        double* w = (double*)malloc(sizeof(double) * (size_t)(2 * k));
        if (!w) {
            #pragma omp atomic write
            bad = 1;
        } else {
            double* wa = w + k;
            #pragma omp for schedule(dynamic, 16)
            for (int64_t r = 0; r < n; ++r) {
                const uint8_t* cr = codes + r * row_bytes;
                for (int64_t kk = 0; kk < k; ++kk) {
                    w[kk] = (double)elem_of(mode, code_at(cr, bits, kk)) *
                            (double)scale_of(mode, scales[r * ng + kk / group]);
                    wa[kk] = isnan(w[kk]) ? 0.0 : fabs(w[kk]);
                }
                for (int64_t i = 0; i < m; ++i) {
                    const double* xr = xd + i * k;
                    const double* ar = xa + i * k;
                    double s[4] = {0, 0, 0, 0}, t[4] = {0, 0, 0, 0};
                    int64_t kk = 0;
                    for (; kk + 4 <= k; kk += 4)
                        for (int j = 0; j < 4; ++j) {
                            s[j] += xr[kk + j] * w[kk + j];
                            t[j] += ar[kk + j] * wa[kk + j];
                        }
                    for (; kk < k; ++kk) {
                        s[0] += xr[kk] * w[kk];
                        t[0] += ar[kk] * wa[kk];
                    }
                    y[i * n + r] = (s[0] + s[1]) + (s[2] + s[3]);
                    yabs[i * n + r] = (t[0] + t[1]) + (t[2] + t[3]);
                }
            }
            free(w);
        }
    }
    free(xd);
    return bad ? -1 : 0;
}

int orc_max_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

int orc_qmm_f32(int mode, const uint16_t* x, int64_t m, int64_t ldx,
                const uint8_t* codes, const uint8_t* scales, int64_t n, int64_t k,
                uint16_t* y, int threads) {
    int group, bits;
    if (spec_of(mode, &group, &bits) || m < 0 || n < 0 || k <= 0 || k % group || ldx < k) return -1;
    const int64_t row_bytes = k * bits / 8, ng = k / group;
    if (threads <= 0) threads = orc_max_threads();
    float lut[256];
    for (int c = 0; c < 256; ++c) lut[c] = mode == ORC_MXFP8 ? orc_decode_e4m3((uint8_t)c)
                                                             : orc_decode_e2m1((uint8_t)(c & 0xF));
    float* xf = (float*)malloc(sizeof(float) * (size_t)(m * k + 1));
    if (!xf) return -1;
    for (int64_t i = 0; i < m; ++i)
        for (int64_t kk = 0; kk < k; ++kk) xf[i * k + kk] = orc_bf16_to_f32(x[i * ldx + kk]);
    int bad = 0;
    #pragma omp parallel num_threads(threads)
    {
        float* w = (float*)malloc(sizeof(float) * (size_t)k);
        if (!w) {
            #pragma omp atomic write
            bad = 1;
        } else {
            #pragma omp for schedule(static)
            for (int64_t r = 0; r < n; ++r) {
                const uint8_t* cr = codes + r * row_bytes;
                const uint8_t* sr = scales + r * ng;
                for (int64_t g = 0; g < ng; ++g) {
                    const float s = scale_of(mode, sr[g]);
                    float* wg = w + g * group;
                    if (bits == 8) {
                        const uint8_t* cg = cr + g * group;
                        for (int i = 0; i < group; ++i) wg[i] = lut[cg[i]] * s;
                    } else {
                        const uint8_t* cg = cr + g * (group / 2);
                        for (int i = 0; i < group / 2; ++i) {
                            wg[2 * i] = lut[cg[i] & 0xF] * s;
                            wg[2 * i + 1] = lut[cg[i] >> 4] * s;
                        }
                    }
                }
                for (int64_t i = 0; i < m; ++i) {
                    const float* xr = xf + i * k;
                    float acc = 0.f;
                    #pragma omp simd reduction(+:acc)
                    for (int64_t kk = 0; kk < k; ++kk) acc += xr[kk] * w[kk];
                    y[i * n + r] = orc_f32_to_bf16(acc);
                }
            }
            free(w);
        }
    }
    free(xf);
    return bad ? -1 : 0;
}
