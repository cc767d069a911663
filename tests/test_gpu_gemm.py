"""Parity of the tcgen05 prefill GEMM (M > 8) with the CPU oracle (B200).

Same bar as the GEMV tests: within 1 bf16 ulp (+ 2^-20 * sum|x||w|) of the
fp64 dequantise-then-matmul per element; relative Frobenius <= 2e-3 at the
benchmark config sizes.  Full-size configs are checked on sampled rows (every
tile row position is covered by the sample) plus a full-tensor comparison
against torch's bf16 matmul over our exact bf16 dequantisation.
"""
import numpy as np
import pytest

import oracle
import qmm
from test_gpu_qmm import bits, check_parity, make_weight, make_x

pytestmark = pytest.mark.gpu


def sampled_parity(y_gpu, x, codes, scales, mode, rows, frob=2e-3):
    xs = x[rows].contiguous()
    xb = bits(xs)
    ref, absref = oracle.qmm_f64_abs(xb, codes, scales, mode)
    y = oracle.bf16_bits_to_f32(bits(y_gpu[rows]))
    assert oracle.parity_violations(y, ref, absref) == 0
    rf = oracle.rel_frobenius(y, ref)
    assert rf <= frob, rf
    return rf


@pytest.mark.parametrize("mode", ["mxfp8", "nvfp4"])
@pytest.mark.parametrize("m,n,k", [(9, 128, 64), (64, 96, 1024), (255, 200, 512), (256, 256, 2048),
                                   (257, 384, 96), (600, 130, 5120)])
def test_gemm_shapes(cuda_device, mode, m, n, k):
    if k % (32 if mode == "mxfp8" else 16):
        pytest.skip("k not a multiple of the group")
    codes, scales = make_weight(n, k, mode, seed=m + n)
    x = make_x(m, k, seed=k).to(cuda_device)
    w = qmm.QuantizedWeight(codes, scales, mode)
    y = w(x)
    qmm.device_status()
    check_parity(y, x, codes, scales, mode)


@pytest.mark.parametrize("mode", ["mxfp8", "nvfp4"])
def test_gemm_k_tails(cuda_device, mode):
    # K not a multiple of the 64-wide k-block: 32 (mxfp8), 16 / 48 (nvfp4).
    for k in ((96, 160) if mode == "mxfp8" else (80, 112, 144)):
        codes, scales = make_weight(136, k, mode, seed=k)
        x = make_x(300, k, seed=k).to(cuda_device)
        check_parity(qmm.QuantizedWeight(codes, scales, mode)(x), x, codes, scales, mode)


@pytest.mark.parametrize("mode", ["mxfp8", "nvfp4"])
def test_gemm_stateless_matches_handle(cuda_device, mode):
    import torch
    codes, scales = make_weight(384, 1024, mode, seed=7)
    x = make_x(512, 1024, seed=7).to(cuda_device)
    y1 = qmm.QuantizedWeight(codes, scales, mode)(x)
    y2 = qmm.quantized_matmul(x, torch.from_numpy(codes.view(np.int32)).to(cuda_device),
                              torch.from_numpy(scales).to(cuda_device), mode=mode)
    torch.cuda.synchronize()
    assert torch.equal(y1, y2)
    y3 = qmm.QuantizedWeight(codes, scales, mode)(x)
    assert torch.equal(y1, y3)                 # deterministic


@pytest.mark.parametrize("mode", ["mxfp8", "nvfp4"])
def test_gemm_strided_io(cuda_device, mode):
    import torch
    n, k, m = 256, 1024, 300
    codes, scales = make_weight(n, k, mode, seed=11)
    w = qmm.QuantizedWeight(codes, scales, mode)
    xbig = make_x(m, k + 64, seed=3).to(cuda_device)
    x = xbig[:, 32:32 + k]                     # 64-byte offset, ldx = k + 64
    out = torch.full((m, n + 24), 5.0, dtype=torch.bfloat16, device=cuda_device)
    y = out[:, :n]
    qmm.check(qmm.lib().qmm_run(w.handle, x.data_ptr(), m, x.stride(0), y.data_ptr(), y.stride(0), True, None))
    torch.cuda.synchronize()
    assert torch.all(out[:, n:] == 5.0)
    check_parity(y, x.contiguous(), codes, scales, mode)


def _torch_check(y, x, w, tol=2e-3):
    import torch
    deq = w.dequantize(torch.bfloat16)
    ref = (x.float() @ deq.float().T)
    err = (y.float() - ref).norm() / ref.norm()
    assert float(err) < tol, float(err)


@pytest.mark.parametrize("name,mode,m,n,k", [
    ("cfg4 in_proj_qkvz", "mxfp8", 2048, 16384, 5120),
    ("cfg4 in_proj_ba", "mxfp8", 2048, 96, 5120),
    ("cfg4 out_proj", "mxfp8", 2048, 5120, 6144),
    ("cfg4 down", "mxfp8", 2048, 5120, 17408),
    ("cfg3 gate/up", "nvfp4", 2048, 34816, 5120),
])
def test_config_shapes_sampled(cuda_device, name, mode, m, n, k):
    """Benchmark configs 3/4 weight shapes at a 2048-token chunk (the
    reference's prefill chunk), sampled rows against the fp64 oracle."""
    codes, scales = make_weight(n, k, mode, seed=n)
    x = make_x(m, k, seed=n).to(cuda_device)
    w = qmm.QuantizedWeight(codes, scales, mode)
    y = w(x)
    qmm.device_status()
    rows = sorted({0, 1, 255, 256, 511, 1000, m - 1} | set(np.random.default_rng(n).integers(0, m, 9).tolist()))
    sampled_parity(y, x, codes, scales, mode, rows)
    _torch_check(y, x, w)


def sample_rows(m, seed, count=512):
    """`count` distinct seeded token rows: the first and last rows, both sides
    of the 128-, 256- and 512-token tile edges near the start, the middle and
    the end, and seeded random rows for the rest."""
    edges = {0, 1, 127, 128, 255, 256, 511, 512, m // 2 - 1, m // 2, m - 513, m - 512, m - 257, m - 256,
             m - 129, m - 128, m - 2, m - 1}
    rows = {r for r in edges if 0 <= r < m}
    rng = np.random.default_rng(seed)
    while len(rows) < min(count, m):
        rows.update(rng.integers(0, m, count - len(rows)).tolist())
    return sorted(rows)[:count] if len(rows) > count else sorted(rows)


def test_cfg3_full_32k_prefill(cuda_device):
    """Benchmark config 3 at full size: x [32768, 5120], W [34816, 5120] nvfp4;
    512 seeded token rows (every output column) against the fp64 oracle, and
    the whole tensor against torch over the exact bf16 dequantisation."""
    m, n, k = 32768, 34816, 5120
    codes, scales = make_weight(n, k, "nvfp4", seed=0)
    x = make_x(m, k, seed=0).to(cuda_device)
    w = qmm.QuantizedWeight(codes, scales, "nvfp4")
    y = w(x)
    qmm.device_status()
    rows = sample_rows(m, seed=1)
    assert len(rows) == 512
    sampled_parity(y, x, codes, scales, "nvfp4", rows)
    _torch_check(y, x, w)


# Benchmark config 4: the prefill GEMMs of one GDN layer (mxfp8, T = 32768),
# the reference's call sites src/model.zig:1066-1075 (in_proj_qkv|z and b|a,
# concatenated along N), :1230 (out_proj) and :905-915 (gate/up, down).
CFG4 = [("in_proj_qkvz", 16384, 5120), ("in_proj_ba", 96, 5120), ("out_proj", 5120, 6144),
        ("gate_up", 34816, 5120), ("down", 5120, 17408)]


@pytest.mark.parametrize("name,n,k", CFG4, ids=[c[0] for c in CFG4])
def test_cfg4_full_32k_prefill(cuda_device, name, n, k):
    """Each config 4 projection at the benchmarked T = 32768: 512 seeded token
    rows against the fp64 oracle (per element and relative Frobenius) and the
    full tensor against torch over the exact bf16 dequantisation."""
    import torch
    m, mode = 32768, "mxfp8"
    codes, scales = make_weight(n, k, mode, seed=n + k)
    x = make_x(m, k, seed=k).to(cuda_device)
    w = qmm.QuantizedWeight(codes, scales, mode)
    y = w(x)
    qmm.device_status()
    rows = sample_rows(m, seed=n)
    assert len(rows) == 512
    sampled_parity(y, x, codes, scales, mode, rows)
    _torch_check(y, x, w)
    w.close()
    del x, y
    torch.cuda.empty_cache()
