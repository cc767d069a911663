"""The x-quantised block-scaled prefill GEMM (qmm_run_blockscaled: tcgen05.mma
kind::mxf4nvf4 on the packed nvfp4 codes of W and of the quantised x).

Not the parity path, so it has its own bar: its result must be the exact
product of the QUANTISED x with W - x quantised by the oracle's nvfp4 rules
(byte-identical to qmm_quantize), dequantised (every E2M1 x UE4M3 value is
exact in bf16), multiplied in fp64 - within the usual fp32-accumulation band
(1 bf16 ulp + 2^-20 sum|x~||w| per element).  That pins the operand and
scale-factor layouts exactly.  Against the exact product of the bf16 x, the
relative Frobenius error is the cost of quantising x (about 0.1); the test
checks it stays in that range and records it."""
import numpy as np
import pytest

import oracle
import qmm
from test_gpu_qmm import bits, make_weight, make_x

pytestmark = pytest.mark.gpu


def quantized_x_bits(x):
    """bf16 bits of dequant(quantize_nvfp4(x)) for a bf16 tensor x [M, K]."""
    xf = oracle.bf16_bits_to_f32(bits(x)).astype(np.float32)
    c, s = oracle.quantize(xf, "nvfp4")
    xq = oracle.dequantize(c, s, "nvfp4")
    xb = oracle.f32_to_bf16_bits(xq)
    assert np.array_equal(oracle.bf16_bits_to_f32(xb), xq)       # exact in bf16
    return xb


def check_blockscaled(y, x, codes, scales, rows=None):
    xb = bits(x) if rows is None else bits(x[rows])
    xq = quantized_x_bits(x if rows is None else x[rows])
    yb = bits(y) if rows is None else bits(y[rows])
    ref, absref = oracle.qmm_f64_abs(xq, codes, scales, "nvfp4")
    got = oracle.bf16_bits_to_f32(yb)
    bad = oracle.parity_violations(got, ref, absref)
    assert bad == 0, f"{bad} elements off the quantised-x product"
    exact, _ = oracle.qmm_f64_abs(xb, codes, scales, "nvfp4")
    rf = oracle.rel_frobenius(got, exact)
    assert 0.01 < rf < 0.3, rf                                      # the cost of quantising x
    return rf


@pytest.mark.parametrize("m,n,k", [(256, 128, 256), (300, 200, 512), (513, 384, 1056), (64, 136, 5120)])
def test_blockscaled_shapes(cuda_device, m, n, k):
    """Ragged M (not a multiple of 256), ragged N (not of 128), a partial last
    K-block (K = 1056 = 4 x 256 + 32)."""
    codes, scales = make_weight(n, k, "nvfp4", seed=m + n + k)
    w = qmm.QuantizedWeight(codes, scales, "nvfp4")
    x = make_x(m, k, seed=k).to(cuda_device)
    y = w.run_blockscaled(x)
    qmm.device_status()
    check_blockscaled(y, x, codes, scales)
    y2 = w.run_blockscaled(x)                          # second call: cached weight atoms, deterministic
    import torch
    torch.cuda.synchronize()
    assert torch.equal(y.view(torch.int16), y2.view(torch.int16))
    w.close()


def test_blockscaled_config3(cuda_device):
    """Benchmark config 3's shape, x [32768, 5120] . W [34816, 5120]^T, on
    128 seeded token rows against the quantised-x product."""
    m, n, k = 32768, 34816, 5120
    codes, scales = make_weight(n, k, "nvfp4", seed=0)
    w = qmm.QuantizedWeight(codes, scales, "nvfp4")
    x = make_x(m, k, seed=0).to(cuda_device)
    y = w.run_blockscaled(x)
    qmm.device_status()
    rows = sorted(set([0, 255, 256, 16383, m - 1] + np.random.default_rng(2).integers(0, m, 123).tolist()))
    check_blockscaled(y, x, codes, scales, rows=rows)
    w.close()


def test_blockscaled_rejects_mxfp8(cuda_device):
    codes, scales = make_weight(128, 256, "mxfp8", seed=1)
    w = qmm.QuantizedWeight(codes, scales, "mxfp8")
    with pytest.raises(qmm.QmmError) as ei:
        w.run_blockscaled(make_x(8, 256).to(cuda_device))
    assert ei.value.name == "BadArgument"
    w.close()
