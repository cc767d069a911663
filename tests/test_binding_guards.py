"""The ctypes binding refuses, before any library call, tensors that would
make a kernel read or write the wrong memory: host tensors (a host pointer
handed to a kernel faults the device), tensors on another GPU than the
weight, and caller output buffers smaller than the result (the library sees
only their row stride).  CPU only: a stub stands in for a CUDA tensor."""
import types

import pytest

import qmm

torch = pytest.importorskip("torch")


class FakeCuda:
    """Just enough of a CUDA tensor for the guards: device, dtype, shape, strides."""

    def __init__(self, shape, dtype=None, device=0, strides=None, contiguous=True):
        self.is_cuda = True
        self.device = types.SimpleNamespace(index=device, type="cuda")
        self.dtype = dtype or torch.bfloat16
        self.shape = tuple(shape)
        self._strides = strides or (shape[1], 1)
        self._contiguous = contiguous

    def dim(self):
        return len(self.shape)

    def stride(self, i):
        return self._strides[i]

    def is_contiguous(self):
        return self._contiguous


def fake_weight(n=8, k=32, device=0):
    w = qmm.QuantizedWeight.__new__(qmm.QuantizedWeight)
    w.n, w.k, w.device = n, k, device
    w._h = None
    return w


def name_of(excinfo):
    return excinfo.value.name


def test_host_tensors_are_refused():
    x = torch.zeros((1, 32), dtype=torch.bfloat16)
    with pytest.raises(qmm.QmmError) as ei:
        fake_weight().run(x)
    assert name_of(ei) == "BadArgument" and "CUDA" in str(ei.value)
    with pytest.raises(qmm.QmmError) as ei:
        fake_weight().argmax(x)
    assert name_of(ei) == "BadArgument"
    with pytest.raises(qmm.QmmError) as ei:
        qmm.quantize(torch.zeros((8, 32)), "nvfp4")
    assert name_of(ei) == "BadArgument"
    w = torch.zeros((8, 4), dtype=torch.int32)
    s = torch.zeros((8, 2), dtype=torch.uint8)
    with pytest.raises(qmm.QmmError) as ei:
        qmm.quantized_matmul(x, w, s, mode="nvfp4")
    assert name_of(ei) == "BadArgument"
    with pytest.raises(qmm.QmmError) as ei:
        qmm.quantized_matmul_noalloc(x, w, s, torch.zeros((1, 8), dtype=torch.bfloat16), mode="nvfp4")
    assert name_of(ei) == "BadArgument"


def test_other_device_is_refused():
    with pytest.raises(qmm.QmmError) as ei:
        qmm._need_cuda("x", FakeCuda((1, 32), device=1), 0)
    assert "cuda:1" in str(ei.value) and "cuda:0" in str(ei.value)
    qmm._need_cuda("x", FakeCuda((1, 32), device=0), 0)          # same device: accepted


def test_output_buffers_must_hold_the_result():
    ok = FakeCuda((3, 64))
    qmm._check_out(ok, 3, 64, 0)
    qmm._check_out(FakeCuda((4, 80), strides=(96, 1)), 3, 64, 0)   # larger, strided rows: fine
    for bad in (FakeCuda((2, 64)),                                 # too few rows
                FakeCuda((3, 63)),                                 # too few columns
                FakeCuda((3, 64), dtype=torch.float32),            # not bf16
                FakeCuda((3, 64), strides=(1, 3)),                 # column stride != 1
                FakeCuda((3, 64), device=1)):                      # another GPU
        with pytest.raises(qmm.QmmError):
            qmm._check_out(bad, 3, 64, 0)


@pytest.fixture
def current_cuda0(monkeypatch):
    """torch.cuda.current_device() == 0 without a GPU."""
    monkeypatch.setattr(torch.cuda, "current_device", lambda: 0)


def test_packed_tensors_must_be_contiguous_and_together(current_cuda0):
    w = FakeCuda((8, 4), dtype=torch.int32)
    qmm._need_packed(w, FakeCuda((8, 2), dtype=torch.uint8))
    with pytest.raises(qmm.QmmError):
        qmm._need_packed(w, FakeCuda((8, 2), dtype=torch.uint8, device=1))
    with pytest.raises(qmm.QmmError):
        qmm._need_packed(FakeCuda((8, 4), dtype=torch.int32, contiguous=False), FakeCuda((8, 2), dtype=torch.uint8))


def test_packed_tensors_must_have_the_packed_dtypes(current_cuda0):
    """Codes are the U32 words (int32 / uint32) and scales bytes: a float or
    int64 tensor of the right shape would be read as the wrong bytes."""
    s = FakeCuda((8, 2), dtype=torch.uint8)
    qmm._need_packed(FakeCuda((8, 4), dtype=torch.int32), s)
    for bad in (torch.int64, torch.float32, torch.uint8, torch.bfloat16):
        with pytest.raises(qmm.QmmError) as ei:
            qmm._need_packed(FakeCuda((8, 4), dtype=bad), s)
        assert name_of(ei) == "UnsupportedDtype"
    for bad in (torch.int32, torch.float32, torch.int8):
        with pytest.raises(qmm.QmmError) as ei:
            qmm._need_packed(FakeCuda((8, 4), dtype=torch.int32), FakeCuda((8, 2), dtype=bad))
        assert name_of(ei) == "UnsupportedDtype"


def test_stateless_calls_need_the_current_device(monkeypatch):
    """The stateless entry points launch on the current device: tensors that
    all live on cuda:1 while cuda:0 is current are refused, not launched on
    device 0 with device 1's pointers."""
    monkeypatch.setattr(torch.cuda, "current_device", lambda: 0)
    w = FakeCuda((8, 4), dtype=torch.int32, device=1)
    s = FakeCuda((8, 2), dtype=torch.uint8, device=1)
    with pytest.raises(qmm.QmmError) as ei:
        qmm._need_packed(w, s)
    assert name_of(ei) == "BadArgument" and "current device is cuda:0" in str(ei.value)
    monkeypatch.setattr(torch.cuda, "current_device", lambda: 1)
    qmm._need_packed(w, s)                                       # current device 1: accepted
