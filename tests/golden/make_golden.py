"""Generate tests/golden/golden.json - the fixtures that pin the CPU oracle.

Run from the repository root:  python tests/golden/make_golden.py

Sources of truth (none of them is the oracle being checked):
  * decode tables of every E4M3 / UE8M0 code and every E2M1 code, from
    ml_dtypes (float8_e4m3fn, float8_e8m0fnu, float4_e2m1fn) - an
    independent implementation of the OCP MX / NVFP4 element formats;
  * quantized fixtures computed here with numpy + ml_dtypes casts (RNE,
    saturated to the largest finite value), following the same published
    rules the oracle restates (OCP MX v1.0 shared exponent for mxfp8, amax/6
    rounded to E4M3 for nvfp4);
  * the reference's own test vectors:
      - src/model.zig:1566-1569: W[8,32] = (i % 7) - 3, x[2,32] = (i % 5) - 2,
        y = x . W^T must equal the integer matmul (the reference checks
        max abs error < 0.05 against MLX's dequantize, src/model.zig:1606);
      - src/weights.zig:493-541: the shape -> (mode, group, bits) cases of
        inferQuantSpec, including the AffineUnsupported and NonstandardQuant
        rejections.
"""
from __future__ import annotations

import json
import os

import ml_dtypes
import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def f32_bits(a) -> list[int]:
    return np.asarray(a, dtype=np.float32).view(np.uint32).astype(np.int64).tolist()


def decode_tables() -> dict:
    codes = np.arange(256, dtype=np.uint8)
    e4m3 = codes.view(ml_dtypes.float8_e4m3fn).astype(np.float32)
    ue8m0 = codes.view(ml_dtypes.float8_e8m0fnu).astype(np.float32)
    # ml_dtypes stores one E2M1 value per byte; codes 0..15.
    e2m1 = np.arange(16, dtype=np.uint8).view(ml_dtypes.float4_e2m1fn).astype(np.float32)
    return {"e4m3_f32_bits": f32_bits(e4m3), "ue8m0_f32_bits": f32_bits(ue8m0),
            "e2m1_f32_bits": f32_bits(e2m1)}


def quantize_mxfp8(w: np.ndarray):
    n, k = w.shape
    g = w.reshape(n, k // 32, 32).astype(np.float32)
    amax = np.abs(g).max(axis=2)
    _, ex = np.frexp(amax)
    se = np.where(amax > 0, (ex - 1) - 8, -127).clip(-127, 127).astype(np.int32)
    v = np.ldexp(g, -se[..., None]).astype(np.float32)           # exact power-of-two scaling
    c = np.clip(v, -448.0, 448.0).astype(ml_dtypes.float8_e4m3fn).view(np.uint8)
    codes = c.reshape(n, k).copy().view("<u4")                    # byte k -> LSB-first u32
    return codes, (se + 127).astype(np.uint8)


def quantize_nvfp4(w: np.ndarray):
    n, k = w.shape
    g = w.reshape(n, k // 16, 16).astype(np.float32)
    amax = np.abs(g).max(axis=2)
    s = np.clip(amax / np.float32(6.0), 0, 448.0).astype(np.float32)
    sq = s.astype(ml_dtypes.float8_e4m3fn)
    sd = sq.astype(np.float32)
    with np.errstate(divide="ignore", invalid="ignore"):
        v = np.where(sd[..., None] > 0, g / sd[..., None], 0).astype(np.float32)
    c = np.clip(v, -6.0, 6.0).astype(ml_dtypes.float4_e2m1fn).view(np.uint8).reshape(n, k)
    packed = (c[:, 0::2] & 0xF) | ((c[:, 1::2] & 0xF) << 4)       # low nibble = even k
    return packed.astype(np.uint8).copy().view("<u4"), sq.view(np.uint8)


def dequant(codes, scales, mode) -> np.ndarray:
    n = codes.shape[0]
    b = codes.view(np.uint8).reshape(n, -1)
    if mode == "mxfp8":
        vals = b.view(ml_dtypes.float8_e4m3fn).astype(np.float32)
        sc = scales.view(ml_dtypes.float8_e8m0fnu).astype(np.float32)
        return vals * np.repeat(sc, 32, axis=1)
    nib = np.empty((n, b.shape[1] * 2), dtype=np.uint8)
    nib[:, 0::2] = b & 0xF
    nib[:, 1::2] = b >> 4
    vals = nib.view(ml_dtypes.float4_e2m1fn).astype(np.float32)
    sc = scales.view(ml_dtypes.float8_e4m3fn).astype(np.float32)
    return vals * np.repeat(sc, 16, axis=1)


def quant_case(name, w, x, mode):
    codes, scales = (quantize_mxfp8 if mode == "mxfp8" else quantize_nvfp4)(w)
    dq = dequant(codes, scales, mode)
    y = x.astype(np.float64) @ dq.astype(np.float64).T
    return {"name": name, "mode": mode, "w_shape": list(w.shape),
            "w_f32_bits": f32_bits(w.ravel()), "x_f32_bits": f32_bits(x.ravel()),
            "x_shape": list(x.shape),
            "codes_u32": codes.astype(np.int64).ravel().tolist(),
            "scales_u8": scales.astype(np.int64).ravel().tolist(),
            "dequant_f32_bits": f32_bits(dq.ravel()), "y_f64": y.ravel().tolist()}


def rule_rows(mode: str) -> np.ndarray:
    """Hand-picked rows [r, 64] on the quantization rules' decision points: the
    round-to-nearest-even ties of E4M3 (normal and subnormal) and E2M1,
    saturation at 448 / 6, the scale's own ties (amax / 6 between two E4M3
    values), and zero, tiny and huge groups.  No NaN or infinity (their
    encodings are checked against the oracle elsewhere)."""
    rows = []
    pad = lambda v: np.resize(np.asarray(v, dtype=np.float64), 64)
    if mode == "mxfp8":
        # amax 2^8 -> X = 0: the codes are E4M3 of the values themselves.
        ties = [(m + 0.5) / 8 * 2.0 ** e for e in (-6, -1, 0, 3, 7) for m in (8, 9, 14, 15)]
        sub = [(q + 0.5) * 2.0 ** -9 for q in range(8)] + [2.0 ** -10, 3 * 2.0 ** -11]
        g0 = [256.0] + ties[:31]
        g1 = [256.0] + ties[31:] + sub + [-v for v in sub] + [1.0] * 4
        rows.append(pad(g0 + g1[:32]))
        rows.append(pad([500.0, 449.0, 460.0, 464.0, 470.0, 480.0, -449.0, -464.0, 447.0, 440.0] + [1.0] * 22 +
                        [0.0] * 32))                                              # saturation; a zero group
        rows.append(pad([1e-40, -1e-41, 5e-42] + [0.0] * 29 + [3e38, -1e38, 2.5e37] + [1.0] * 29))
        rows.append(pad([2.0 ** (e / 4) for e in range(-40, 24)]))                # amax crossing powers of two
    else:
        ties = [0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 5.5, 0.24, 0.26, 4.9, 5.1, 6.0]
        g = lambda scale: [6.0 * scale] + [t * scale for t in ties] + [-0.75 * scale, -5.0 * scale]
        rows.append(pad(g(1.0) + g(2.0 ** -3) + g(2.0 ** 4) + g(2.0 ** -6)))
        # amax / 6 on E4M3 ties: 1.0625 -> 1.0, 1.1875 -> 1.25, 2^-9 * 1.5 -> 2^-8 (subnormal scale)
        rows.append(pad([6.0 * 1.0625, 1.0, -2.0, 3.0] + [0.5] * 12 + [6.0 * 1.1875, 1.0] + [0.25] * 14 +
                        [6.0 * 1.5 * 2.0 ** -9, 2.0 ** -9] + [0.0] * 14 + [6.0 * 448.0 * 1.01, 1.0] + [3.0] * 14))
        rows.append(pad([1e-4, -2e-5] + [0.0] * 14 + [0.0] * 16 + [1e4, -3e3, 7.0] + [1.0] * 13 +
                        [1e-30, 1e-31] + [0.0] * 14))                             # zero scale, saturated scale
        rows.append(pad([2.0 ** (e / 4) for e in range(-40, 24)]))
    return np.asarray(rows, dtype=np.float32)


def spec_cases() -> list[dict]:
    # src/weights.zig:493-541, restated as (tensor infos, expected) pairs.
    t = lambda name, dtype, shape: {"name": name, "dtype": dtype, "shape": shape}
    return [
        {"ref": "src/weights.zig:495-507 nvfp4",
         "tensors": [t("l.q_proj.weight", "U32", [8, 8]), t("l.q_proj.scales", "U8", [8, 4]),
                     t("l.norm.weight", "BF16", [16])],
         "expect": {"mode": "nvfp4", "group_size": 16, "bits": 4}},
        {"ref": "src/weights.zig:508-517 mxfp8",
         "tensors": [t("l.q_proj.weight", "U32", [8, 32]), t("l.q_proj.scales", "U8", [8, 4])],
         "expect": {"mode": "mxfp8", "group_size": 32, "bits": 8}},
        {"ref": "src/weights.zig:518-524 dense",
         "tensors": [t("l.norm.weight", "BF16", [16])],
         "expect": {"mode": "none", "group_size": 0, "bits": 0}},
        {"ref": "src/weights.zig:525-533 affine (BF16 scales)",
         "tensors": [t("l.q_proj.weight", "U32", [8, 32]), t("l.q_proj.scales", "BF16", [8, 2]),
                     t("l.q_proj.biases", "BF16", [8, 2])],
         "expect": {"error": "AffineUnsupported"}},
        {"ref": "src/weights.zig:534-540 orphan packed weight",
         "tensors": [t("l.q_proj.weight", "U32", [8, 32])],
         "expect": {"error": "NonstandardQuant"}},
    ]


def main() -> None:
    rng = np.random.default_rng(0)
    # src/model.zig:1566-1569 integer pattern (exactly representable after quantization).
    w_int = (np.arange(8 * 32) % 7 - 3).astype(np.float32).reshape(8, 32)
    x_int = (np.arange(2 * 32) % 5 - 2).astype(np.float32).reshape(2, 32)
    cases = []
    for mode in ("nvfp4", "mxfp8"):
        c = quant_case(f"model_zig_1561_{mode}", w_int, x_int, mode)
        c["y_exact"] = (x_int.astype(np.int64) @ w_int.astype(np.int64).T).ravel().tolist()
        cases.append(c)
    # Seeded N(0, 0.02^2) weights with a few planted edge values (zero groups,
    # tiny values that land on subnormal codes, a large outlier per group).
    for mode in ("nvfp4", "mxfp8"):
        w = (rng.standard_normal((16, 64)) * 0.02).astype(np.float32)
        w[0, :32] = 0.0
        w[1, 5] = 1e-7
        w[2, 7] = 3.0
        w[3, :] *= 1e-3
        x = rng.standard_normal((3, 64)).astype(np.float32)
        x = (x.view(np.uint32) & 0xFFFF0000).view(np.float32)  # bf16-exact activations
        cases.append(quant_case(f"seeded_16x64_{mode}", w, x, mode))
    # The rules' decision points (no RNG: appended after the seeded cases).
    for mode in ("nvfp4", "mxfp8"):
        w = rule_rows(mode)
        x = np.resize(np.array([1.0, -0.5, 0.25, 2.0], dtype=np.float32), (2, 64))
        cases.append(quant_case(f"rules_{mode}", w, x, mode))
    out = {"generator": "tests/golden/make_golden.py", "ml_dtypes": ml_dtypes.__version__,
           "numpy": np.__version__, "decode": decode_tables(), "quant_cases": cases,
           "spec_cases": spec_cases()}
    with open(os.path.join(HERE, "golden.json"), "w") as f:
        json.dump(out, f, separators=(",", ":"))
    print("wrote", os.path.join(HERE, "golden.json"))


if __name__ == "__main__":
    main()
