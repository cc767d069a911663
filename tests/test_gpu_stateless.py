"""The stateless entry point (qmm_quantized_matmul, src/mlx.zig:265
mlx_quantized_matmul) on checkpoint-layout tensors for M <= 8: the TMA decode
kernel reading the caller's U32 codes and U8 [N, K/group] scales through 2D
TMA boxes, with its stream-K scratch in a per-stream workspace.

Checked against the fp64 oracle and, bit for bit, against the resident-weight
path (same kernel arithmetic and work split, re-tiled scales): ragged N, a
half-full last K chunk (nvfp4), mxfp8's odd chunks (the unit's scale bytes in
the second half of a 16-byte TMA box), every M in 1..8, two streams at once,
and a CUDA graph captured after the stream's first call."""
import numpy as np
import pytest

import oracle
import qmm
from test_gpu_qmm import check_parity, make_weight, make_x

pytestmark = pytest.mark.gpu


def _dev(codes, scales, dev):
    import torch
    return torch.from_numpy(codes.view(np.int32)).to(dev), torch.from_numpy(scales).to(dev)


# (n, k) with 16-byte scale rows (the kernel's TMA envelope): K = 1536 (3 / 6
# chunks), 4352 (nvfp4: 8.5 chunks, the last one half full; mxfp8 falls back,
# its 136-byte scale rows are not 16-byte aligned), 5632 with N = 257 (ragged
# last row block), and config 2's [5120, 17408].
SHAPES = [(333, 1536), (130, 4352), (257, 5632), (5120, 17408)]


@pytest.mark.parametrize("mode", ["mxfp8", "nvfp4"])
@pytest.mark.parametrize("n,k", SHAPES)
def test_stateless_decode_parity(cuda_device, mode, n, k):
    import torch
    codes, scales = make_weight(n, k, mode, seed=n + k)
    wd, sd = _dev(codes, scales, cuda_device)
    w = qmm.QuantizedWeight(codes, scales, mode)
    for m in range(1, 9):
        x = make_x(m, k, seed=m + k).to(cuda_device)
        y = qmm.quantized_matmul(x, wd, sd, mode=mode)
        y_res = w(x)
        torch.cuda.synchronize()
        check_parity(y, x, codes, scales, mode)
        assert torch.equal(y.view(torch.int16), y_res.view(torch.int16)), (m, "stateless != resident")
    qmm.device_status()
    w.close()


def test_stateless_two_streams(cuda_device):
    """Calls in flight on two streams at once use two workspaces."""
    import torch
    n, k, mode = 5120, 17408, "nvfp4"
    codes, scales = make_weight(n, k, mode, seed=5)
    wd, sd = _dev(codes, scales, cuda_device)
    s1, s2 = torch.cuda.Stream(), torch.cuda.Stream()
    xs = [make_x(2, k, seed=40 + i).to(cuda_device) for i in range(2)]
    ys = [torch.empty((2, n), dtype=torch.bfloat16, device=cuda_device) for _ in range(2)]
    for st in (s1, s2):                                   # first call per stream (workspace)
        with torch.cuda.stream(st):
            qmm.quantized_matmul(xs[0], wd, sd, mode=mode, out=ys[0], stream=st)
    torch.cuda.synchronize()
    for _ in range(20):
        with torch.cuda.stream(s1):
            qmm.quantized_matmul(xs[0], wd, sd, mode=mode, out=ys[0], stream=s1)
        with torch.cuda.stream(s2):
            qmm.quantized_matmul(xs[1], wd, sd, mode=mode, out=ys[1], stream=s2)
    torch.cuda.synchronize()
    for x, y in zip(xs, ys):
        check_parity(y, x, codes, scales, mode)


def test_stateless_graph_capture(cuda_device):
    """After one call on a stream, its calls capture into a CUDA graph whose
    replays give the eager result; a first call inside a capture is refused
    with a clear error instead of allocating there."""
    import torch
    n, k, mode = 2048, 5120, "mxfp8"
    codes, scales = make_weight(n, k, mode, seed=9)
    wd, sd = _dev(codes, scales, cuda_device)
    x = make_x(3, k, seed=9).to(cuda_device)
    y = torch.empty((3, n), dtype=torch.bfloat16, device=cuda_device)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        qmm.quantized_matmul(x, wd, sd, mode=mode, out=y, stream=s)
    s.synchronize()
    eager = y.clone()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        qmm.quantized_matmul(x, wd, sd, mode=mode, out=y, stream=s)
    for _ in range(3):
        y.zero_()
        g.replay()
        torch.cuda.synchronize()
        assert torch.equal(y.view(torch.int16), eager.view(torch.int16))
    check_parity(y, x, codes, scales, mode)
    del g
    fresh = torch.cuda.Stream()
    g2 = torch.cuda.CUDAGraph()
    with pytest.raises(qmm.QmmError) as ei:
        with torch.cuda.graph(g2, stream=fresh):
            qmm.quantized_matmul(x, wd, sd, mode=mode, out=y, stream=fresh)
    assert ei.value.name == "BadArgument" and "before capturing" in str(ei.value)
    del g2
    torch.cuda.synchronize()
    qmm.device_status()
