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
        for fn in (L.orc_quantize, L.orc_dequantize, L.orc_qmm_f64, L.orc_qmm_f32):
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
