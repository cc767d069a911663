"""ctypes binding of the CPU oracle (oracle.c).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the
cpu_baseline / reference arm of bench.py, as the checker or the timed CPU
baseline.  The product path never imports this module.

The oracle restates the arithmetic behind mlx-runner's
``mlx_quantized_matmul(x, w, scales, null, transpose=true, group, bits, mode)``
(src/model.zig:244-258) for the mxfp8 and nvfp4 formats of
src/weights.zig:37-55; see oracle.h for what is pinned and what is not.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
BUILD = os.path.join(HERE, "_build")
LIB_PATH = os.path.join(BUILD, "liboracle.so")

MXFP8 = 1
NVFP4 = 2
MODES = {"mxfp8": MXFP8, "nvfp4": NVFP4}
SPEC = {"mxfp8": (32, 8), "nvfp4": (16, 4)}


def build(force: bool = False) -> str:
    """Compile oracle.c into _build/liboracle.so with gcc + OpenMP."""
    src = os.path.join(HERE, "oracle.c")
    if (not force and os.path.exists(LIB_PATH)
            and os.path.getmtime(LIB_PATH) >= max(os.path.getmtime(src),
                                                  os.path.getmtime(os.path.join(HERE, "oracle.h")))):
        return LIB_PATH
    os.makedirs(BUILD, exist_ok=True)
    tmp = LIB_PATH + f".tmp{os.getpid()}"
    subprocess.check_call(["gcc", "-O3", "-march=x86-64-v3", "-fopenmp", "-fPIC", "-shared",
                           "-std=c11", "-Wall", "-o", tmp, src, "-lm"])
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = ctypes.CDLL(LIB_PATH)
        u8, f32, i64, vp = ctypes.c_uint8, ctypes.c_float, ctypes.c_int64, ctypes.c_void_p
        for name, arg in (("orc_decode_e4m3", u8), ("orc_decode_e2m1", u8),
                          ("orc_decode_ue8m0", u8), ("orc_decode_ue4m3", u8)):
            fn = getattr(L, name)
            fn.argtypes, fn.restype = [arg], f32
        L.orc_encode_e4m3.argtypes, L.orc_encode_e4m3.restype = [f32], u8
        L.orc_encode_e2m1.argtypes, L.orc_encode_e2m1.restype = [f32], u8
        L.orc_quantize.argtypes = [ctypes.c_int, vp, i64, i64, vp, vp]
        L.orc_dequantize.argtypes = [ctypes.c_int, vp, vp, i64, i64, vp]
        L.orc_qmm_f64.argtypes = [ctypes.c_int, vp, i64, i64, vp, vp, i64, i64, vp]
        L.orc_qmm_f32.argtypes = [ctypes.c_int, vp, i64, i64, vp, vp, i64, i64, vp, ctypes.c_int]
        L.orc_qmm_f64_abs.argtypes = [ctypes.c_int, vp, i64, i64, vp, vp, i64, i64, vp, vp]
        for fn in (L.orc_quantize, L.orc_dequantize, L.orc_qmm_f64, L.orc_qmm_f32, L.orc_qmm_f64_abs):
            fn.restype = ctypes.c_int
        L.orc_max_threads.restype = ctypes.c_int
        _lib = L
    return _lib


def _p(a: np.ndarray) -> int:
    assert a.flags["C_CONTIGUOUS"], "oracle buffers must be C-contiguous"
    return a.ctypes.data


def quantize(w: np.ndarray, mode: str):
    """fp32 W [N, K] -> (U32 codes [N, K*bits/32], U8 scales [N, K/group])."""
    group, bits = SPEC[mode]
    w = np.ascontiguousarray(w, dtype=np.float32)
    n, k = w.shape
    codes = np.zeros((n, k * bits // 32), dtype=np.uint32)
    scales = np.zeros((n, k // group), dtype=np.uint8)
    rc = lib().orc_quantize(MODES[mode], _p(w), n, k, _p(codes), _p(scales))
    if rc:
        raise ValueError(f"orc_quantize rejected shape {w.shape} for {mode}")
    return codes, scales


def dequantize(codes: np.ndarray, scales: np.ndarray, mode: str) -> np.ndarray:
    group, bits = SPEC[mode]
    codes = np.ascontiguousarray(codes, dtype=np.uint32)
    scales = np.ascontiguousarray(scales, dtype=np.uint8)
    n = codes.shape[0]
    k = codes.shape[1] * 32 // bits
    out = np.empty((n, k), dtype=np.float32)
    if lib().orc_dequantize(MODES[mode], _p(codes), _p(scales), n, k, _p(out)):
        raise ValueError("orc_dequantize rejected its arguments")
    return out


def qmm_f64(x_bf16: np.ndarray, codes: np.ndarray, scales: np.ndarray, mode: str) -> np.ndarray:
    """fp64 dequantise-then-matmul; x given as bf16 bits (uint16) [M, K]."""
    group, bits = SPEC[mode]
    x_bf16 = np.ascontiguousarray(x_bf16, dtype=np.uint16)
    codes = np.ascontiguousarray(codes, dtype=np.uint32)
    scales = np.ascontiguousarray(scales, dtype=np.uint8)
    m, k = x_bf16.shape
    n = codes.shape[0]
    assert codes.shape[1] * 32 // bits == k
    y = np.empty((m, n), dtype=np.float64)
    if lib().orc_qmm_f64(MODES[mode], _p(x_bf16), m, k, _p(codes), _p(scales), n, k, _p(y)):
        raise ValueError("orc_qmm_f64 rejected its arguments")
    return y


def qmm_f64_abs(x_bf16: np.ndarray, codes: np.ndarray, scales: np.ndarray, mode: str):
    """(qmm_f64, abs_qmm_f64) in one pass over W without an [N, K]
    intermediate: the checker at full benchmark sizes."""
    group, bits = SPEC[mode]
    x_bf16 = np.ascontiguousarray(x_bf16, dtype=np.uint16)
    codes = np.ascontiguousarray(codes, dtype=np.uint32)
    scales = np.ascontiguousarray(scales, dtype=np.uint8)
    m, k = x_bf16.shape
    n = codes.shape[0]
    assert codes.shape[1] * 32 // bits == k
    y = np.empty((m, n), dtype=np.float64)
    ya = np.empty((m, n), dtype=np.float64)
    if m < 16:
        # Few x rows: one pass over W in C, each row dequantized once.
        if lib().orc_qmm_f64_abs(MODES[mode], _p(x_bf16), m, k, _p(codes), _p(scales), n, k, _p(y), _p(ya)):
            raise ValueError("orc_qmm_f64_abs rejected its arguments")
        return y, ya
    # Many x rows: exact fp32 dequantisation of W in row blocks, then fp64
    # matrix products (every product of a bf16 and a dequantised value is
    # exact in fp64; only the fp64 summation order differs from qmm_f64).
    xd = bf16_bits_to_f32(x_bf16).astype(np.float64)
    xa = np.abs(xd)
    block = max(256, (1 << 25) // max(1, k))
    for r0 in range(0, n, block):
        w = dequantize(codes[r0:r0 + block], scales[r0:r0 + block], mode).astype(np.float64)
        y[:, r0:r0 + block] = xd @ w.T
        np.abs(w, out=w)
        w[np.isnan(w)] = 0.0
        ya[:, r0:r0 + block] = xa @ w.T
    return y, ya


def qmm_f32(x_bf16: np.ndarray, codes: np.ndarray, scales: np.ndarray, mode: str,
            threads: int = 0) -> np.ndarray:
    """The CPU baseline: fp32 accumulate, bf16 bits out [M, N]."""
    group, bits = SPEC[mode]
    x_bf16 = np.ascontiguousarray(x_bf16, dtype=np.uint16)
    codes = np.ascontiguousarray(codes, dtype=np.uint32)
    scales = np.ascontiguousarray(scales, dtype=np.uint8)
    m, k = x_bf16.shape
    n = codes.shape[0]
    y = np.empty((m, n), dtype=np.uint16)
    if lib().orc_qmm_f32(MODES[mode], _p(x_bf16), m, k, _p(codes), _p(scales), n, k, _p(y), threads):
        raise ValueError("orc_qmm_f32 rejected its arguments")
    return y


def max_threads() -> int:
    return int(lib().orc_max_threads())


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(a: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even fp32 -> bf16 bits (NaN kept quiet)."""
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32).astype(np.uint64)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    r[nan] = ((u[nan] >> 16) | 0x40).astype(np.uint16)
    return r


def abs_qmm_f64(x_bf16: np.ndarray, codes: np.ndarray, scales: np.ndarray, mode: str) -> np.ndarray:
    """sum_k |x[m, k]| * |W[n, k]| in fp64: the scale of the accumulation error."""
    xa = np.abs(bf16_bits_to_f32(x_bf16)).astype(np.float32)
    wa = np.abs(dequantize(codes, scales, mode))
    wa = np.nan_to_num(wa, nan=0.0)
    return xa.astype(np.float64) @ wa.astype(np.float64).T


def bf16_ulp(a: np.ndarray) -> np.ndarray:
    """Spacing of bf16 values at |a| (normal range; 2^-133 below it)."""
    a = np.abs(np.asarray(a, dtype=np.float64))
    e = np.floor(np.log2(np.maximum(a, 2.0 ** -126)))
    return np.exp2(e - 7)


def parity_violations(y: np.ndarray, ref: np.ndarray, absref: np.ndarray, ulps: float = 1.0,
                      acc_rel: float = 2.0 ** -20) -> int:
    """Elements where a bf16 result misses the fp64 reference by more than
    `ulps` bf16 ulps plus an fp32-accumulation allowance acc_rel * sum|x||w|.
    Correct rounding alone is within 0.5 ulp."""
    y = np.asarray(y, dtype=np.float64)
    tol = ulps * bf16_ulp(ref) + acc_rel * absref
    bad = ~(np.abs(y - ref) <= tol)
    both_nan = np.isnan(y) & np.isnan(ref)
    return int(np.count_nonzero(bad & ~both_nan))


def rel_frobenius(y: np.ndarray, ref: np.ndarray) -> float:
    y = np.asarray(y, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    den = np.linalg.norm(ref)
    return float(np.linalg.norm(y - ref) / (den if den > 0 else 1.0))


# ---- SwiGLU (src/model.zig:905-915) -----------------------------------------------

def _f64_to_bf16_bits(a: np.ndarray) -> np.ndarray:
    """fp64 -> bf16 bits, one round-to-nearest-even step (no fp32 detour)."""
    a = np.asarray(a, dtype=np.float64)
    out = f32_to_bf16_bits(a.astype(np.float32))
    # Values whose fp32 rounding landed exactly on a bf16 tie would round twice:
    # redo those from the fp64 value.
    f32 = a.astype(np.float32).view(np.uint32)
    tie = (f32 & 0xFFFF) == 0x8000
    if np.any(tie):
        lo = (f32[tie] & 0xFFFF0000).view(np.float32).astype(np.float64)
        hi_bits = ((f32[tie] >> 16) + 1).astype(np.uint16)
        hi = bf16_bits_to_f32(hi_bits).astype(np.float64)
        av = a[tie]
        pick_hi = np.abs(av - hi) < np.abs(av - lo)
        even = ((f32[tie] >> 16) & 1) == 0
        eq = np.abs(av - hi) == np.abs(av - lo)
        pick_hi = pick_hi | (eq & ~even)
        out[tie] = np.where(pick_hi, hi_bits, (f32[tie] >> 16).astype(np.uint16))
    return out


def swiglu_bf16(g_bits: np.ndarray, u_bits: np.ndarray) -> np.ndarray:
    """silu(g) * u over bf16 arrays (bits in, bits out) with the reference's
    sequence of bf16 arrays: sigmoid(g) (model.zig:409), g * sigmoid(g)
    (:412), that * u (:913, mul :451), each rounded to bf16 (nearest even).
    The sigmoid is 1 / (1 + e^-g) in fp64 rounded once; the products of two
    bf16 values are exact in fp64 before their rounding."""
    g = bf16_bits_to_f32(g_bits).astype(np.float64)
    u = bf16_bits_to_f32(u_bits).astype(np.float64)
    with np.errstate(over="ignore", invalid="ignore"):
        s = 1.0 / (1.0 + np.exp(-g))
    sb = bf16_bits_to_f32(_f64_to_bf16_bits(s)).astype(np.float64)
    t = bf16_bits_to_f32(_f64_to_bf16_bits(g * sb)).astype(np.float64)
    return _f64_to_bf16_bits(t * u)


def swiglu_violations(h_bits: np.ndarray, g_ref: np.ndarray, u_ref: np.ndarray, absg: np.ndarray,
                      absu: np.ndarray, acc_rel: float = 2.0 ** -20) -> int:
    """Elements of h = silu(g) * u (bf16 bits) outside the exact composition's
    band: the gate / up sums may each miss by the GEMM bar (1 bf16 ulp +
    acc_rel * sum|x||w|), carried through silu(g) * u by its derivatives,
    plus the four bf16 roundings of the chain (2^-8 relative each), plus the
    fp32 range of the sigmoid: a sigmoid evaluated in fp32 - MLX's of a bf16
    array, or the kernels' - is 0 once e^-g overflows (g < -87.3), where the
    exact value is below 2^-126, so h may miss by |g| |u| 2^-126 there."""
    h = bf16_bits_to_f32(h_bits).astype(np.float64)
    g, u = np.asarray(g_ref, np.float64), np.asarray(u_ref, np.float64)
    with np.errstate(over="ignore", invalid="ignore"):
        sig = 1.0 / (1.0 + np.exp(-g))
    silu = g * sig
    dsilu = sig * (1.0 + g * (1.0 - sig))
    ref = silu * u
    tg = bf16_ulp(g) + acc_rel * absg
    tu = bf16_ulp(u) + acc_rel * absu
    tol = (np.abs(dsilu) * tg * (np.abs(u) + tu) + (np.abs(silu) + np.abs(dsilu) * tg) * tu
           + 4.0 * 2.0 ** -8 * np.abs(ref) + (np.abs(g) + tg) * (np.abs(u) + tu) * 2.0 ** -126 + 2.0 ** -133)
    bad = ~(np.abs(h - ref) <= tol)
    both_nan = np.isnan(h) & np.isnan(ref)
    return int(np.count_nonzero(bad & ~both_nan))


# ---- greedy sampling (src/sample.zig:162-170, :69-79) ----------------------------

def greedy_sample(logits_bits: np.ndarray):
    """Per row of bf16 logits (bits [M, N]): (ids, logprobs).  id = argmax
    (mlx_argmax_axis; the lowest index among equal values, NaN above every
    number); logprob = logit[id] - logsumexp(row), the logsumexp in fp64
    rounded to bf16 (the reference reads a bf16 array back as f32)."""
    l = bf16_bits_to_f32(np.asarray(logits_bits, dtype=np.uint16)).astype(np.float64)
    m, n = l.shape
    ids = np.zeros(m, np.int64)
    lps = np.zeros(m, np.float64)
    for r in range(m):
        row = l[r]
        nan = np.isnan(row)
        ids[r] = int(np.argmax(nan)) if nan.any() else int(np.argmax(row))
        mx = np.nanmax(row) if not nan.all() else np.nan
        with np.errstate(over="ignore", invalid="ignore"):
            lse = mx + np.log(np.sum(np.exp(row - mx)))
        lse_b = bf16_bits_to_f32(_f64_to_bf16_bits(np.array([lse]))).astype(np.float64)[0]
        lps[r] = row[ids[r]] - lse_b
    return ids, lps
