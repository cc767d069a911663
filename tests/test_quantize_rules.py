"""The library's quantization rules (csrc/quantize.cuh, the arithmetic of
qmm_quantize = src/mlx.zig:278 mlx_quantize) compiled as host code, against
the oracle's quantizer, byte for byte, on the hard cases of quant_cases.py
and on seeded N(0, 0.02^2) weights.  The device build of the same header
differs only in using the IEEE-exact intrinsics (__fmul_rn, __fdiv_rn,
rintf, __clz); the GPU parity test checks the kernel itself."""
import ctypes
import os
import shutil
import subprocess
import tempfile

import numpy as np
import pytest

import oracle
from quant_cases import hard_matrix

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(os.path.dirname(HERE), "mlx-runner_b200", "csrc")


@pytest.fixture(scope="module")
def rules():
    cxx = shutil.which("g++")
    if cxx is None:
        pytest.skip("g++ not available")
    d = tempfile.mkdtemp(prefix="qrules_")
    so = os.path.join(d, "libqrules.so")
    subprocess.check_call([cxx, "-O2", "-std=c++17", "-shared", "-fPIC", f"-I{CSRC}",
                           os.path.join(HERE, "quantize_rules_host.cpp"), "-o", so])
    L = ctypes.CDLL(so)
    L.qr_quantize.argtypes = [ctypes.c_int, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p,
                              ctypes.c_void_p]
    yield L
    shutil.rmtree(d, ignore_errors=True)


def host_quantize(L, w: np.ndarray, mode: str):
    group, bits = oracle.SPEC[mode]
    w = np.ascontiguousarray(w, dtype=np.float32)
    n, k = w.shape
    codes = np.zeros((n, k * bits // 32), dtype=np.uint32)
    scales = np.zeros((n, k // group), dtype=np.uint8)
    assert L.qr_quantize(1 if mode == "mxfp8" else 2, w.ctypes.data, n, k, codes.ctypes.data,
                         scales.ctypes.data) == 0
    return codes, scales


@pytest.mark.parametrize("mode", ["mxfp8", "nvfp4"])
def test_rules_match_oracle_on_hard_cases(rules, mode):
    with np.errstate(over="ignore", invalid="ignore"):
        w = hard_matrix(mode, rows=8192, seed=1)
    c_o, s_o = oracle.quantize(w, mode)
    c_h, s_h = host_quantize(rules, w, mode)
    bad_s = np.argwhere(s_o != s_h)
    assert bad_s.size == 0, f"{bad_s.shape[0]} scale bytes differ, first at {bad_s[0]}"
    bad_c = np.argwhere(c_o != c_h)
    assert bad_c.size == 0, f"{bad_c.shape[0]} code words differ, first at {bad_c[0]}"


@pytest.mark.parametrize("mode", ["mxfp8", "nvfp4"])
def test_rules_match_oracle_on_weights(rules, mode):
    rng = np.random.default_rng(5)
    w = (rng.standard_normal((512, 2048), dtype=np.float32) * 0.02).astype(np.float32)
    c_o, s_o = oracle.quantize(w, mode)
    c_h, s_h = host_quantize(rules, w, mode)
    assert np.array_equal(s_o, s_h) and np.array_equal(c_o, c_h)


def test_hard_cases_cover_every_code(rules):
    """The hard cases reach every E2M1 code in both signs and every E4M3
    code a quantizer can emit (all but NaN's 0x7F / 0xFF)."""
    with np.errstate(over="ignore", invalid="ignore"):
        c8, _ = host_quantize(rules, hard_matrix("mxfp8", rows=8192, seed=1), "mxfp8")
        c4, _ = host_quantize(rules, hard_matrix("nvfp4", rows=8192, seed=1), "nvfp4")
    b8 = set(np.unique(c8.view(np.uint8)).tolist())
    assert set(range(256)) - b8 <= {0xFF}, sorted(set(range(256)) - b8)
    b4 = c4.view(np.uint8)
    nib = set(np.unique(np.concatenate([b4 & 0xF, b4 >> 4])).tolist())
    assert nib == set(range(16))


@pytest.mark.parametrize("idx", [4, 5])
def test_rules_match_independent_fixtures(rules, golden, idx):
    """The rules' decision points (ties, saturation, scale ties, zero / tiny /
    huge groups) against the fixtures of an independent quantizer (numpy +
    ml_dtypes casts, tests/golden/make_golden.py)."""
    case = golden["quant_cases"][idx]
    w = np.asarray(case["w_f32_bits"], dtype=np.uint32).view(np.float32).reshape(case["w_shape"])
    codes, scales = host_quantize(rules, w, case["mode"])
    assert np.array_equal(codes.ravel(), np.asarray(case["codes_u32"], dtype=np.uint32))
    assert np.array_equal(scales.ravel(), np.asarray(case["scales_u8"], dtype=np.uint8))
