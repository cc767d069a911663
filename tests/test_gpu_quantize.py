"""qmm_quantize (src/mlx.zig:278 mlx_quantize, as src/model.zig:1577 calls
it) on the GPU against the oracle's quantizer, byte for byte: the hard cases
(ties, saturation, subnormals, NaN / inf / zero groups), benchmark configs 1
and 2 at full size, bf16 input, strided and unaligned rows; then the
reference's own qmm test (src/model.zig:1561-1609) through quantize ->
quantized_matmul -> dequantize."""
import numpy as np
import pytest

import oracle
import qmm
from quant_cases import hard_matrix

pytestmark = pytest.mark.gpu


def gpu_quantize(w_np, mode, dev, **kw):
    import torch
    codes, scales = qmm.quantize(torch.from_numpy(w_np).to(dev), mode, **kw)
    torch.cuda.synchronize()
    return codes.cpu().numpy().view(np.uint32), scales.cpu().numpy()


def assert_same(got, want, what):
    bad = np.argwhere(got != want)
    assert bad.size == 0, f"{what}: {bad.shape[0]} entries differ, first at {tuple(bad[0])}"


@pytest.mark.parametrize("mode", ["mxfp8", "nvfp4"])
def test_quantize_hard_cases(cuda_device, mode):
    with np.errstate(over="ignore", invalid="ignore"):
        w = hard_matrix(mode, rows=8192, seed=1)
    c, s = gpu_quantize(w, mode, cuda_device)
    c_o, s_o = oracle.quantize(w, mode)
    assert_same(s, s_o, "scales")
    assert_same(c, c_o, "codes")


@pytest.mark.parametrize("idx", [4, 5])
def test_quantize_independent_fixtures(cuda_device, golden, idx):
    """The rules' decision points against the fixtures of an independent
    quantizer (numpy + ml_dtypes casts), byte for byte."""
    case = golden["quant_cases"][idx]
    w = np.asarray(case["w_f32_bits"], dtype=np.uint32).view(np.float32).reshape(case["w_shape"])
    c, s = gpu_quantize(w, case["mode"], cuda_device)
    assert_same(c.ravel(), np.asarray(case["codes_u32"], dtype=np.uint32), "codes")
    assert_same(s.ravel(), np.asarray(case["scales_u8"], dtype=np.uint8), "scales")


@pytest.mark.parametrize("mode,n,k", [("mxfp8", 17408, 5120), ("nvfp4", 5120, 17408)])
def test_quantize_config_shapes(cuda_device, mode, n, k):
    """Benchmark configs 1 and 2: W ~ N(0, 0.02^2) [N, K], seed 0."""
    rng = np.random.default_rng(0)
    w = (rng.standard_normal((n, k), dtype=np.float32) * 0.02).astype(np.float32)
    c, s = gpu_quantize(w, mode, cuda_device)
    c_o, s_o = oracle.quantize(w, mode)
    assert_same(s, s_o, "scales")
    assert_same(c, c_o, "codes")


@pytest.mark.parametrize("mode", ["mxfp8", "nvfp4"])
def test_quantize_bf16_input(cuda_device, mode):
    import torch
    g = torch.Generator().manual_seed(3)
    w = (torch.randn((300, 1024), generator=g) * 0.05).to(torch.bfloat16)
    codes, scales = qmm.quantize(w.to(cuda_device), mode)
    c_o, s_o = oracle.quantize(w.float().numpy(), mode)
    assert_same(scales.cpu().numpy(), s_o, "scales")
    assert_same(codes.cpu().numpy().view(np.uint32), c_o, "codes")


@pytest.mark.parametrize("mode", ["mxfp8", "nvfp4"])
@pytest.mark.parametrize("dtype", ["f32", "bf16"])
@pytest.mark.parametrize("pad,offset", [(4, 0), (1, 0), (3, 1)])
def test_quantize_strided_and_unaligned_rows(cuda_device, mode, dtype, pad, offset):
    """Row stride K + pad starting `offset` elements into the buffer: pad 4 /
    offset 0 keeps the vector loads, the others take the scalar path."""
    import torch
    n, k = 97, 512
    g = torch.Generator().manual_seed(11)
    big = torch.randn((n, k + pad), generator=g) * 0.1
    if dtype == "bf16":
        big = big.to(torch.bfloat16)
    flat = torch.zeros(n * (k + pad) + offset, dtype=big.dtype)
    flat[offset:] = big.reshape(-1)
    dev_flat = flat.to(cuda_device)
    view = dev_flat[offset:].view(n, k + pad)[:, :k]
    codes, scales = qmm.quantize(view, mode)
    c_o, s_o = oracle.quantize(big[:, :k].float().numpy(), mode)
    assert_same(scales.cpu().numpy(), s_o, "scales")
    assert_same(codes.cpu().numpy().view(np.uint32), c_o, "codes")


@pytest.mark.parametrize("mode", ["mxfp8", "nvfp4"])
def test_reference_qmm_test_through_quantize(cuda_device, mode):
    """src/model.zig:1561-1609: W[8, 32] = (i % 7) - 3, x[2, 32] = (i % 5) - 2;
    quantize, quantized_matmul, and an f32 matmul over dequantize agree to
    0.05 (here exactly: the dequantised values are the integers)."""
    import torch
    w = ((np.arange(8 * 32) % 7) - 3).astype(np.float32).reshape(8, 32)
    x = ((np.arange(2 * 32) % 5) - 2).astype(np.float32).reshape(2, 32)
    codes, scales = qmm.quantize(torch.from_numpy(w).to(cuda_device), mode)
    xb = torch.from_numpy(x).to(torch.bfloat16).to(cuda_device)
    y = qmm.quantized_matmul(xb, codes, scales, mode=mode).float().cpu().numpy()
    wt = qmm.QuantizedWeight(codes, scales, mode)
    dq = wt.dequantize(torch.float32).cpu().numpy()
    wt.close()
    ref = x @ dq.T
    assert np.max(np.abs(y - ref)) < 0.05
    assert np.array_equal(dq, w)
    assert np.array_equal(y, x @ w.T)


def test_quantize_in_a_graph_and_on_a_stream(cuda_device):
    """No allocation or synchronisation inside: the call captures into a CUDA
    graph, and a replay writes the same bytes."""
    import torch
    w = torch.randn((256, 2048), device=cuda_device) * 0.02
    codes = torch.empty((256, 2048 * 4 // 32), dtype=torch.int32, device=cuda_device)
    scales = torch.empty((256, 2048 // 16), dtype=torch.uint8, device=cuda_device)
    O = qmm.OptionalInt.of
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())

    def call(st):
        qmm.check(qmm.lib().qmm_quantize(w.data_ptr(), 1, 256, 2048, 2048, O(None), O(None), b"nvfp4", None,
                                         codes.data_ptr(), scales.data_ptr(), st.cuda_stream))
    with torch.cuda.stream(s):
        call(s)
    s.synchronize()
    want_c, want_s = codes.clone(), scales.clone()
    codes.zero_()
    scales.zero_()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=s):
        call(s)
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(codes, want_c) and torch.equal(scales, want_s)
    del graph
