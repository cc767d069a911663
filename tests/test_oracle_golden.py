"""The CPU oracle against the committed golden vectors (tests/golden).

Pins the oracle before it is trusted as the checker: exhaustive decode
tables against ml_dtypes, quantized fixtures bit for bit, and the
reference's integer wiring case (src/model.zig:1561-1609) exactly.
"""
import math

import numpy as np
import pytest

import oracle


def _f32(bits):
    return np.asarray(bits, dtype=np.uint32).view(np.float32)


def _same(a: float, b: float) -> bool:
    if math.isnan(a) or math.isnan(b):
        return math.isnan(a) and math.isnan(b)
    return np.float32(a).view(np.uint32) == np.float32(b).view(np.uint32)


def test_e4m3_table_exhaustive(golden):
    L = oracle.lib()
    want = _f32(golden["decode"]["e4m3_f32_bits"])
    for c in range(256):
        assert _same(L.orc_decode_e4m3(c), want[c]), hex(c)


def test_ue8m0_table_exhaustive(golden):
    L = oracle.lib()
    want = _f32(golden["decode"]["ue8m0_f32_bits"])
    for c in range(256):
        assert _same(L.orc_decode_ue8m0(c), want[c]), hex(c)


def test_e2m1_table_exhaustive(golden):
    L = oracle.lib()
    want = _f32(golden["decode"]["e2m1_f32_bits"])
    for c in range(16):
        assert _same(L.orc_decode_e2m1(c), want[c]), hex(c)


def test_ue4m3_is_e4m3(golden):
    L = oracle.lib()
    for c in range(128):
        assert _same(L.orc_decode_ue4m3(c), L.orc_decode_e4m3(c))


def test_encoders_round_trip_every_finite_code():
    L = oracle.lib()
    for c in range(256):
        v = L.orc_decode_e4m3(c)
        if math.isnan(v):
            continue
        got = L.orc_encode_e4m3(v)
        assert _same(L.orc_decode_e4m3(got), v), hex(c)
    for c in range(16):
        v = L.orc_decode_e2m1(c)
        assert _same(L.orc_decode_e2m1(L.orc_encode_e2m1(v)), v)


def test_encoders_saturate_and_tie_to_even():
    L = oracle.lib()
    assert L.orc_decode_e4m3(L.orc_encode_e4m3(1e9)) == 448.0
    assert L.orc_decode_e4m3(L.orc_encode_e4m3(-1e9)) == -448.0
    assert L.orc_decode_e2m1(L.orc_encode_e2m1(7.0)) == 6.0
    assert L.orc_decode_e2m1(L.orc_encode_e2m1(5.0)) == 4.0     # tie -> even
    assert L.orc_decode_e2m1(L.orc_encode_e2m1(0.25)) == 0.0    # tie -> even
    assert L.orc_decode_e2m1(L.orc_encode_e2m1(0.75)) == 1.0    # tie -> even
    assert L.orc_decode_e4m3(L.orc_encode_e4m3(2.0 ** -10)) == 0.0  # half of the smallest subnormal


@pytest.mark.parametrize("idx", range(6))
def test_quantize_dequantize_fixtures(golden, idx):
    """The oracle's quantizer against fixtures made by an independent one
    (numpy + ml_dtypes casts): the reference's integer case, seeded weights
    with planted edge values, and (idx 4, 5) the rules' decision points."""
    case = golden["quant_cases"][idx]
    w = _f32(case["w_f32_bits"]).reshape(case["w_shape"])
    codes, scales = oracle.quantize(w, case["mode"])
    np.testing.assert_array_equal(codes.ravel(), np.asarray(case["codes_u32"], dtype=np.uint32))
    np.testing.assert_array_equal(scales.ravel(), np.asarray(case["scales_u8"], dtype=np.uint8))
    dq = oracle.dequantize(codes, scales, case["mode"])
    np.testing.assert_array_equal(dq.ravel().view(np.uint32),
                                  np.asarray(case["dequant_f32_bits"], dtype=np.uint32))


@pytest.mark.parametrize("mode", ["nvfp4", "mxfp8"])
def test_reference_wiring_case_is_exact(golden, mode):
    """src/model.zig:1561-1609: the integer pattern quantizes exactly, so the
    qmm must equal the integer matmul (the reference allows 0.05)."""
    case = next(c for c in golden["quant_cases"] if c["name"] == f"model_zig_1561_{mode}")
    w = _f32(case["w_f32_bits"]).reshape(case["w_shape"])
    x = _f32(case["x_f32_bits"]).reshape(case["x_shape"])
    codes, scales = oracle.quantize(w, mode)
    np.testing.assert_array_equal(oracle.dequantize(codes, scales, mode), w)
    xb = oracle.f32_to_bf16_bits(x)
    y64 = oracle.qmm_f64(xb, codes, scales, mode)
    np.testing.assert_array_equal(y64.ravel(), np.asarray(case["y_exact"], dtype=np.float64))
    y32 = oracle.bf16_bits_to_f32(oracle.qmm_f32(xb, codes, scales, mode))
    assert np.max(np.abs(y32.ravel() - np.asarray(case["y_exact"]))) < 0.05


@pytest.mark.parametrize("idx", [2, 3])
def test_qmm_oracles_match_fixture(golden, idx):
    case = golden["quant_cases"][idx]
    codes = np.asarray(case["codes_u32"], dtype=np.uint32).reshape(case["w_shape"][0], -1)
    scales = np.asarray(case["scales_u8"], dtype=np.uint8).reshape(case["w_shape"][0], -1)
    x = _f32(case["x_f32_bits"]).reshape(case["x_shape"])
    xb = oracle.f32_to_bf16_bits(x)
    y64 = oracle.qmm_f64(xb, codes, scales, case["mode"])
    want = np.asarray(case["y_f64"]).reshape(y64.shape)
    np.testing.assert_allclose(y64, want, rtol=1e-12, atol=1e-15)
    y32 = oracle.bf16_bits_to_f32(oracle.qmm_f32(xb, codes, scales, case["mode"]))
    # fp32 accumulation + one bf16 rounding: within 1 bf16 ulp of fp64 per
    # element, and no worse than bf16 rounding of the exact result overall.
    absref = oracle.abs_qmm_f64(xb, codes, scales, case["mode"])
    assert oracle.parity_violations(y32, want, absref) == 0
    floor = oracle.rel_frobenius(oracle.bf16_bits_to_f32(oracle.f32_to_bf16_bits(want)), want)
    assert oracle.rel_frobenius(y32, want) <= 1.25 * floor + 1e-4


def test_bf16_rounding_matches_torch():
    torch = pytest.importorskip("torch")
    rng = np.random.default_rng(1)
    a = (rng.standard_normal(10000) * 10.0 ** rng.integers(-30, 30, 10000)).astype(np.float32)
    a[:4] = [np.inf, -np.inf, 0.0, -0.0]
    ours = oracle.f32_to_bf16_bits(a)
    theirs = torch.from_numpy(a).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    np.testing.assert_array_equal(ours, theirs)


def test_swiglu_oracle_sequence():
    """silu(g) * u over bf16 arrays: known values and single RNE rounding."""
    g = oracle.f32_to_bf16_bits(np.array([0.0, 1.0, -1.0, 10.0, -100.0, 3.5], np.float32))
    u = oracle.f32_to_bf16_bits(np.array([2.0, 2.0, 2.0, 0.5, 1.0, -1.0], np.float32))
    h = oracle.bf16_bits_to_f32(oracle.swiglu_bf16(g, u))
    np.testing.assert_array_equal(h, np.array([0.0, 1.4609375, -0.5390625, 5.0, -0.0, -3.390625], np.float32))
    a = np.random.default_rng(0).standard_normal(20000) * 3
    b = oracle._f64_to_bf16_bits(a)
    cand = np.stack([b - 1, b, b + 1]).astype(np.uint16)
    best = np.argmin(np.abs(oracle.bf16_bits_to_f32(cand).astype(np.float64) - a), axis=0)
    assert np.all(best == 1)
    # The band (about 3% here): the exact composition passes, 6% off does not.
    gr = np.array([[0.7, -2.0, 4.0]])
    ur = np.array([[1.5, 0.25, -3.0]])
    ref = gr / (1 + np.exp(-gr)) * ur
    hb = oracle.f32_to_bf16_bits(ref.astype(np.float32))
    zero = np.zeros_like(gr)
    assert oracle.swiglu_violations(hb, gr, ur, zero, zero) == 0
    off = oracle.f32_to_bf16_bits((ref * 1.06).astype(np.float32))
    assert oracle.swiglu_violations(off, gr, ur, zero, zero) == 3
