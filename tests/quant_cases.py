"""Hard inputs for the quantizer (fp32 W [rows, 64]): the cases where the
mxfp8 / nvfp4 rules of src/mlx.zig:278 mlx_quantize (restated in the oracle
and in csrc/quantize.cuh) can go wrong - rounding ties, saturation, the
subnormal ranges of E4M3 and fp32, zero / NaN / infinite groups, and random
magnitudes from 1e-44 to 1e38.  Seeded; shared by the CPU rule test and the
GPU parity test."""
from __future__ import annotations

import numpy as np

K = 64  # 2 mxfp8 groups or 4 nvfp4 groups per row


def _f32(bits) -> np.ndarray:
    return np.asarray(bits, dtype=np.uint32).view(np.float32)


def hard_matrix(mode: str, rows: int = 4096, seed: int = 0) -> np.ndarray:
    rng = np.random.default_rng(seed)
    group = 32 if mode == "mxfp8" else 16
    out = np.empty((rows, K), dtype=np.float32)
    specials = _f32([0x7FC00000, 0xFFC00000, 0x7F800001, 0xFFA00000,   # NaNs (quiet / signalling, both signs)
                     0x7F800000, 0xFF800000, 0x80000000, 0x00000000,   # +-inf, -0, +0
                     0x00000001, 0x807FFFFF, 0x00800000, 0x7F7FFFFF])  # subnormal, min normal, max
    e4m3_ties = np.array([(m + 0.5) / 8 * 2.0 ** e for e in range(-6, 9) for m in range(8, 16)] +
                         [(n + 0.5) * 2.0 ** -9 for n in range(8)] + [448.0, 449.0, 464.0, 480.0, 2.0 ** -10],
                         dtype=np.float64)
    e2m1_ties = np.array([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 5.5, 6.0, 6.5, 7.0, 0.24, 0.26], dtype=np.float64)
    for r in range(rows):
        kind = r % 8
        row = rng.standard_normal(K).astype(np.float32)
        if kind == 0:                                   # log-uniform magnitudes per group
            for g in range(0, K, group):
                row[g:g + group] *= np.float32(10.0 ** rng.uniform(-44, 38))
        elif kind == 1:                                 # specials sprinkled into normal groups
            idx = rng.choice(K, size=rng.integers(1, 6), replace=False)
            row[idx] = rng.choice(specials, size=idx.size)
        elif kind == 2:                                 # E4M3 ties under a power-of-two group scale
            x = int(rng.integers(-20, 20))
            vals = rng.choice(e4m3_ties, size=K) * np.where(rng.random(K) < 0.5, -1.0, 1.0)
            row[:] = (vals * 2.0 ** x).astype(np.float32)
            if mode == "mxfp8":
                for g in range(0, K, group):            # amax fixes X: put 2^(x+8) in each group
                    row[g] = np.float32(2.0 ** (x + 8))
        elif kind == 3:                                 # E2M1 ties: amax 6 * 2^j -> scale 2^j exactly
            j = int(rng.integers(-6, 8))
            vals = rng.choice(e2m1_ties, size=K) * np.where(rng.random(K) < 0.5, -1.0, 1.0)
            row[:] = (vals * 2.0 ** j).astype(np.float32)
            for g in range(0, K, group):
                row[g] = np.float32(6.0 * 2.0 ** j)
        elif kind == 4:                                 # all-zero, single-value and tiny-scale groups
            row[:] = 0.0
            choice = r // 8 % 4
            if choice == 1:
                row[rng.integers(K)] = np.float32(rng.standard_normal())
            elif choice == 2:
                row[:] = rng.standard_normal(K).astype(np.float32) * np.float32(1e-3 * 2.0 ** -10)
            elif choice == 3:
                row[:] = _f32(rng.integers(1, 1 << 23, size=K, dtype=np.uint32))  # fp32 subnormals
        elif kind == 5:                                 # huge groups (scale saturation, overflow)
            row *= np.float32(10.0 ** rng.uniform(30, 38.5))
        elif kind == 6:                                 # raw fp32 bit patterns
            row[:] = _f32(rng.integers(0, 1 << 32, size=K, dtype=np.uint64).astype(np.uint32))
        else:                                           # amax / 6 near E4M3 rounding points
            t = rng.choice(e4m3_ties) * 6.0
            row *= np.float32(0.1)
            for g in range(0, K, group):
                row[g] = np.float32(t * (1 if rng.random() < 0.5 else -1))
        out[r] = row
    return out
