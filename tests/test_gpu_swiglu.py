"""Fused gate / up projection with the SwiGLU epilogue (src/model.zig:905-915
up to the down projection) on the B200, through the C ABI.

Bar: h = silu(g) * u per element inside the exact composition's band (the
gate / up sums each within the GEMM bar of 1 bf16 ulp + 2^-20 sum|x||w|,
carried through silu(g) * u, plus the chain's four bf16 roundings), and
nearly always bit-identical to the reference's unfused sequence applied to
the GPU's own bf16 gate / up outputs (the fused kernel rounds g and u the
same way; only an fp32-vs-fp64 sigmoid or a different fp32 summation order
can move a bit).
"""
import numpy as np
import pytest

import oracle
import qmm

pytestmark = pytest.mark.gpu


def make_weight(n, k, mode, seed=0, scale=0.02):
    rng = np.random.default_rng(seed)
    w = (rng.standard_normal((n, k), dtype=np.float32) * scale).astype(np.float32)
    return oracle.quantize(w, mode)


def make_x(m, k, seed=1):
    import torch
    g = torch.Generator().manual_seed(seed)
    return torch.randn((m, k), generator=g, dtype=torch.float32).to(torch.bfloat16)


def bits(t):
    import torch
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def check_swiglu(h, x, gate, up, mode, min_exact):
    """Oracle band (no violations) and agreement with the unfused GPU sequence."""
    import torch
    xb = bits(x)
    g_ref = oracle.qmm_f64(xb, *gate, mode)
    u_ref = oracle.qmm_f64(xb, *up, mode)
    absg = oracle.abs_qmm_f64(xb, *gate, mode)
    absu = oracle.abs_qmm_f64(xb, *up, mode)
    hb = bits(h)
    assert oracle.swiglu_violations(hb, g_ref, u_ref, absg, absu) == 0
    # Unfused: the two linears on the GPU, then the bf16 sequence on the CPU.
    xd = x.cuda() if not x.is_cuda else x
    g = bits(qmm.QuantizedWeight(*gate, mode)(xd))
    u = bits(qmm.QuantizedWeight(*up, mode)(xd))
    unfused = oracle.swiglu_bf16(g, u)
    exact = np.mean(hb == unfused)
    assert exact >= min_exact, exact
    return exact


@pytest.mark.parametrize("mode", ["mxfp8", "nvfp4"])
@pytest.mark.parametrize("m", [1, 2, 3, 4, 5, 8])
def test_swiglu_decode_small(cuda_device, mode, m):
    n, k = 333, 1536                       # n not a multiple of 64: a padded last block
    gate, up = make_weight(n, k, mode, seed=10 + m), make_weight(n, k, mode, seed=20 + m)
    w = qmm.SwiGLUWeight(*gate, *up, mode)
    assert w.n == n and w.k == k
    x = make_x(m, k, seed=m).to(cuda_device)
    check_swiglu(w(x), x, gate, up, mode, min_exact=0.98)


@pytest.mark.parametrize("m", [1, 3])
def test_swiglu_decode_model_shape(cuda_device, m):
    """The model's gate / up pair: [17408, 5120] each, nvfp4 (benchmark config 3's
    fused weight [34816, 5120] is their concatenation)."""
    n, k, mode = 17408, 5120, "nvfp4"
    gate, up = make_weight(n, k, mode, seed=1), make_weight(n, k, mode, seed=2)
    w = qmm.SwiGLUWeight(*gate, *up, mode)
    x = make_x(m, k, seed=m).to(cuda_device)
    check_swiglu(w(x), x, gate, up, mode, min_exact=0.98)


@pytest.mark.parametrize("mode", ["mxfp8", "nvfp4"])
@pytest.mark.parametrize("m", [9, 300, 600])
def test_swiglu_prefill(cuda_device, mode, m):
    n, k = 200, 1024
    gate, up = make_weight(n, k, mode, seed=30 + m), make_weight(n, k, mode, seed=40 + m)
    w = qmm.SwiGLUWeight(*gate, *up, mode)
    x = make_x(m, k, seed=m).to(cuda_device)
    # The GEMM sums every output in the same order as the unfused weights.
    check_swiglu(w(x), x, gate, up, mode, min_exact=0.995)


def test_swiglu_unaligned_x_takes_unfused_path(cuda_device):
    import torch
    n, k, mode = 130, 512, "nvfp4"
    gate, up = make_weight(n, k, mode, seed=5), make_weight(n, k, mode, seed=6)
    w = qmm.SwiGLUWeight(*gate, *up, mode)
    for m in (2, 20):
        xbig = make_x(m, k + 8, seed=m).to(cuda_device)
        x = xbig[:, 2:2 + k]                   # 4-byte aligned rows, not 16
        h = w(x)
        torch.cuda.synchronize()
        check_swiglu(h, x.contiguous(), gate, up, mode, min_exact=0.98)


def test_swiglu_handle_rules(cuda_device):
    import torch
    n, k, mode = 64, 256, "mxfp8"
    gate, up = make_weight(n, k, mode, seed=7), make_weight(n, k, mode, seed=8)
    w = qmm.SwiGLUWeight(*gate, *up, mode)
    x = make_x(1, k).to(cuda_device)
    y = torch.empty((1, n), dtype=torch.bfloat16, device=cuda_device)
    rc = qmm.lib().qmm_run(w.handle, x.data_ptr(), 1, k, y.data_ptr(), n, True, None)
    assert qmm.STATUS_NAMES[rc] == "BadArgument"
    qmm.take_error()
    with pytest.raises(qmm.QmmError):
        w.dequantize()
    plain = qmm.QuantizedWeight(*gate, mode)
    rc = qmm.lib().qmm_swiglu_run(plain.handle, x.data_ptr(), 1, k, y.data_ptr(), n, None)
    assert qmm.STATUS_NAMES[rc] == "BadArgument"
    qmm.take_error()
    # M = 0 is a no-op; the device stays usable.
    w(torch.empty((0, k), dtype=torch.bfloat16, device=cuda_device))
    qmm.device_status()
