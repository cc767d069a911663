"""The C entry points check, before any launch, that the raw pointers they
are given are memory of the current device: a host pointer (pageable or
pinned) is refused with BadArgument and the device stays usable; with two
GPUs, so is a buffer of the other GPU.  Called through the C ABI directly,
as a Zig or C caller would, past the Python binding's own guards."""
import numpy as np
import pytest

import oracle
import qmm

pytestmark = pytest.mark.gpu

O = qmm.OptionalInt.of


def _status(rc):
    name = qmm.STATUS_NAMES.get(rc, rc)
    qmm.take_error()
    return name


def _stateless(y, x, w, s, m, n, k):
    return qmm.lib().qmm_quantized_matmul(y, n, x, m, k, k, w, n, k // 8, s, n, k // 16, None, True,
                                          O(None), O(None), b"nvfp4", None)


def test_host_pointers_are_refused(cuda_device):
    import torch
    m, n, k = 2, 256, 512
    rng = np.random.default_rng(0)
    codes, scales = oracle.quantize((rng.standard_normal((n, k), dtype=np.float32) * 0.02), "nvfp4")
    wd = torch.from_numpy(codes.view(np.int32)).to(cuda_device)
    sd = torch.from_numpy(scales).to(cuda_device)
    xd = torch.randn((m, k), device=cuda_device).to(torch.bfloat16)
    yd = torch.empty((m, n), device=cuda_device, dtype=torch.bfloat16)
    xh = np.zeros((m, k), dtype=np.uint16)                        # pageable host memory
    yp = torch.empty((m, n), dtype=torch.bfloat16).pin_memory()   # pinned host memory
    cases = {
        "x pageable": (yd.data_ptr(), xh.ctypes.data, wd.data_ptr(), sd.data_ptr()),
        "y pinned": (yp.data_ptr(), xd.data_ptr(), wd.data_ptr(), sd.data_ptr()),
        "w pageable": (yd.data_ptr(), xd.data_ptr(), codes.ctypes.data, sd.data_ptr()),
        "scales pageable": (yd.data_ptr(), xd.data_ptr(), wd.data_ptr(), scales.ctypes.data),
    }
    for what, (y, x, w, s) in cases.items():
        assert _status(_stateless(y, x, w, s, m, n, k)) == "BadArgument", what
        assert _status(qmm.lib().qmm_quantized_matmul_noalloc(
            y, n, x, m, k, k, w, n, k // 8, s, n, k // 16, None, True, O(None), O(None), b"nvfp4",
            None)) == "BadArgument", what
    wt = qmm.QuantizedWeight(codes, scales, "nvfp4")
    assert _status(qmm.lib().qmm_run(wt.handle, xh.ctypes.data, m, k, yd.data_ptr(), n, True, None)) == "BadArgument"
    assert _status(qmm.lib().qmm_run(wt.handle, xd.data_ptr(), m, k, yp.data_ptr(), n, True, None)) == "BadArgument"
    wq = np.zeros((n, k), dtype=np.float32)
    cq = torch.empty((n, k // 8), dtype=torch.int32, device=cuda_device)
    sq = torch.empty((n, k // 16), dtype=torch.uint8, device=cuda_device)
    assert _status(qmm.lib().qmm_quantize(wq.ctypes.data, 1, n, k, k, O(None), O(None), b"nvfp4", None,
                                          cq.data_ptr(), sq.data_ptr(), None)) == "BadArgument"
    # The device is still usable, and the same call on device memory is right.
    qmm.check(_stateless(yd.data_ptr(), xd.data_ptr(), wd.data_ptr(), sd.data_ptr(), m, n, k))
    torch.cuda.synchronize()
    xb = xd.cpu().view(torch.int16).numpy().view(np.uint16)
    ref, absref = oracle.qmm_f64_abs(xb, codes, scales, "nvfp4")
    got = oracle.bf16_bits_to_f32(yd.cpu().view(torch.int16).numpy().view(np.uint16))
    assert oracle.parity_violations(got, ref, absref) == 0
    wt.close()


def test_other_gpu_buffers_are_refused(cuda_device):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    m, n, k = 1, 128, 256
    on1 = {"x": torch.zeros((m, k), dtype=torch.bfloat16, device="cuda:1"),
           "y": torch.zeros((m, n), dtype=torch.bfloat16, device="cuda:1"),
           "w": torch.zeros((n, k // 8), dtype=torch.int32, device="cuda:1"),
           "s": torch.zeros((n, k // 16), dtype=torch.uint8, device="cuda:1")}
    torch.cuda.set_device(0)
    rc = _stateless(on1["y"].data_ptr(), on1["x"].data_ptr(), on1["w"].data_ptr(), on1["s"].data_ptr(), m, n, k)
    assert _status(rc) == "BadArgument"
