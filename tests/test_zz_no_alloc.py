"""qmm_quantized_matmul_noalloc: the decode kernel with its scratch in a
static device array.  Results match qmm_quantized_matmul within the parity
tolerance, repeat bit for bit over consecutive calls (the array is rebuilt
each call) and equal qmm_run on a resident copy of the weight (same kernel),
the device's free memory does not move, and a weight whose scratch exceeds
the array is rejected with QMM_ERR_OUT_OF_MEMORY.
"""
import numpy as np
import pytest

import oracle
import qmm

pytestmark = pytest.mark.gpu


def make_case(n, k, m, mode, seed):
    import torch
    rng = np.random.default_rng(seed)
    w = (rng.standard_normal((n, k), dtype=np.float32) * 0.02).astype(np.float32)
    codes, scales = oracle.quantize(w, mode)
    g = torch.Generator().manual_seed(seed + 1)
    x = torch.randn((m, k), generator=g, dtype=torch.float32).to(torch.bfloat16)
    return codes, scales, x


def bits(t):
    import torch
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def rel_diff(a, b):
    fa = oracle.bf16_bits_to_f32(bits(a)).astype(np.float64)
    fb = oracle.bf16_bits_to_f32(bits(b)).astype(np.float64)
    return float(np.linalg.norm(fa - fb) / max(np.linalg.norm(fb), 1e-30))


def oracle_parity(y, x, codes, scales, mode):
    xb = bits(x)
    ref = oracle.qmm_f64(xb, codes, scales, mode)
    absref = oracle.abs_qmm_f64(xb, codes, scales, mode)
    assert oracle.parity_violations(oracle.bf16_bits_to_f32(bits(y)), ref, absref) == 0


CASES = [  # (n, k, m, mode): cfg1 and cfg2 weights, a ragged small one
    (17408, 5120, 1, "mxfp8"),
    (5120, 17408, 4, "nvfp4"),
    (200, 1024, 3, "mxfp8"),
    (328, 2048, 2, "nvfp4"),
]


@pytest.mark.parametrize("n,k,m,mode", CASES)
def test_noalloc_matches_stateless_twice(cuda_device, n, k, m, mode):
    import torch
    codes, scales, x = make_case(n, k, m, mode, seed=n + m)
    wd = torch.from_numpy(codes.view(np.int32)).to(cuda_device)
    sd = torch.from_numpy(scales).to(cuda_device)
    xd = x.to(cuda_device)
    ref = qmm.quantized_matmul(xd, wd, sd, mode=mode)
    y1 = torch.empty_like(ref)
    y2 = torch.full_like(ref, 7.0)
    qmm.quantized_matmul_noalloc(xd, wd, sd, y1, mode=mode)
    qmm.quantized_matmul_noalloc(xd, wd, sd, y2, mode=mode)
    torch.cuda.synchronize()
    qmm.device_status()
    assert rel_diff(y1, ref) <= 2e-3
    assert np.array_equal(bits(y1), bits(y2))
    # Same kernel, grid and unit split as a resident weight's qmm_run.
    h = qmm.QuantizedWeight(codes, scales, mode)
    assert np.array_equal(bits(h.run(xd)), bits(y1))
    h.close()
    if n * k <= 2048 * 2048:
        oracle_parity(y1, x, codes, scales, mode)


def test_noalloc_interleaved_weights_and_free_memory(cuda_device):
    import torch
    a = make_case(5120, 17408, 1, "nvfp4", seed=11)
    b = make_case(17408, 5120, 2, "mxfp8", seed=12)
    dev = []
    for (codes, scales, x), mode in ((a, "nvfp4"), (b, "mxfp8")):
        wd = torch.from_numpy(codes.view(np.int32)).to(cuda_device)
        sd = torch.from_numpy(scales).to(cuda_device)
        xd = x.to(cuda_device)
        ref = qmm.quantized_matmul(xd, wd, sd, mode=mode)
        dev.append((wd, sd, xd, mode, ref, torch.empty_like(ref)))
    for wd, sd, xd, mode, ref, y in dev:  # set-up call on this device
        qmm.quantized_matmul_noalloc(xd, wd, sd, y, mode=mode)
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info(cuda_device)[0]
    for _ in range(2):
        for wd, sd, xd, mode, ref, y in dev:
            y.fill_(0)
            qmm.quantized_matmul_noalloc(xd, wd, sd, y, mode=mode)
            assert rel_diff(y, ref) <= 2e-3
    torch.cuda.synchronize()
    qmm.device_status()
    assert torch.cuda.mem_get_info(cuda_device)[0] == free0


def test_noalloc_rejects_oversize_weight(cuda_device):
    import torch
    n, k = 16384, 16384  # nvfp4 scale tiles alone need 16 MiB
    wd = torch.zeros((n, k // 8), dtype=torch.int32, device=cuda_device)
    sd = torch.zeros((n, k // 16), dtype=torch.uint8, device=cuda_device)
    xd = torch.zeros((1, k), dtype=torch.bfloat16, device=cuda_device)
    y = torch.zeros((1, n), dtype=torch.bfloat16, device=cuda_device)
    with pytest.raises(qmm.QmmError) as ei:
        qmm.quantized_matmul_noalloc(xd, wd, sd, y, mode="nvfp4")
    assert ei.value.status == 21 and "8 MiB" in str(ei.value)
    torch.cuda.synchronize()
