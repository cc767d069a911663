"""Python binding of libqmm_b200.so - the operator surface of mlx-runner's
quantized linear layer, on B200.

Mirrors the reference's interface for this path:
  * ``quantized_matmul(x, w, scales, biases=None, transpose=True,
    group_size=None, bits=None, mode=...)``  ->  mlx_quantized_matmul
    (src/mlx.zig:265, called by qlinear src/model.zig:244-258);
  * ``infer_quant_spec(tensors)``  ->  inferQuantSpec (src/weights.zig:132-185);
  * ``QuantizedWeight``  ->  a resident packed weight as WeightMap holds it
    (src/weights.zig:203-353), run like namedLinearQ / qlinear;
  * ``QmmError``  ->  the error latch (src/mlx.zig:719-805), raised with the
    reference's error class names.

The arithmetic runs only in the CUDA library: importing this module without
the built library, or calling it without a B200, raises - there is no CPU
fallback.  torch tensors are used purely as device buffers and streams.
"""
from __future__ import annotations

import ctypes
import os
from dataclasses import dataclass
from typing import Iterable, Optional, Sequence

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get("QMM_B200_LIB") or os.path.join(HERE, "_build", "libqmm_b200.so")

QMM_OK = 0
STATUS_NAMES = {
    1: "BadShape", 2: "NonstandardQuant", 3: "InconsistentQuant", 4: "AffineUnsupported",
    5: "UnsupportedDtype", 6: "BadMode", 7: "BadArgument", 8: "MissingWeight",
    10: "BadIndexJson", 11: "BadHeader", 12: "UnsupportedLayout", 13: "MissingTensor", 14: "DuplicateTensor",
    15: "IoError",
    20: "CudaError", 21: "OutOfMemory", 22: "NcclError", 23: "Timeout", 24: "NoDevice",
    30: "Injected",
}
MODE_NONE, MODE_MXFP8, MODE_NVFP4 = 0, 1, 2
MODE_NAMES = {MODE_NONE: "none", MODE_MXFP8: "mxfp8", MODE_NVFP4: "nvfp4"}
DTYPES = {"BF16": 0, "F32": 1, "U32": 2, "U8": 3}
SRC_HOST, SRC_DEVICE = 0, 1

# Every symbol the C ABI (include/qmm.h) exports.
EXPORTS = (
    "qmm_abi_version", "qmm_infer_quant_spec", "qmm_mode_str", "qmm_spec_from_args",
    "qmm_quantized_matmul", "qmm_quantized_matmul_noalloc", "qmm_weight_create", "qmm_weight_create_shard", "qmm_shard_range",
    "qmm_weight_destroy",
    "qmm_weight_info", "qmm_run", "qmm_linear", "qmm_dequantize", "qmm_quantize", "qmm_tp_unique_id",
    "qmm_swiglu_weight_create", "qmm_swiglu_run", "qmm_lm_head_argmax",
    "qmm_checkpoint_open", "qmm_checkpoint_close", "qmm_checkpoint_spec", "qmm_checkpoint_tensors",
    "qmm_checkpoint_read", "qmm_checkpoint_load_linear", "qmm_checkpoint_load_swiglu",
    "qmm_tp_comm_create", "qmm_tp_comm_create_detached", "qmm_tp_comm_destroy", "qmm_tp_allreduce_bf16",
    "qmm_tp_run_rowparallel",
    "qmm_last_error", "qmm_error_pending", "qmm_device_status", "qmm_fault_arm", "qmm_fault_fired",
    "qmm_tensor_peak", "qmm_run_blockscaled",
)


class QmmError(RuntimeError):
    """A non-zero qmm status; ``name`` is the reference's error class."""

    def __init__(self, status: int, message: str):
        self.status = status
        self.name = STATUS_NAMES.get(status, f"Status{status}")
        super().__init__(f"{self.name}: {message}")


class QuantSpec(ctypes.Structure):
    _fields_ = [("mode", ctypes.c_int32), ("group_size", ctypes.c_int32), ("bits", ctypes.c_int32)]

    @property
    def mode_str(self) -> str:
        return MODE_NAMES.get(self.mode, "?")

    def astuple(self):
        return (self.mode_str, self.group_size, self.bits)


class TensorInfo(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char_p), ("dtype", ctypes.c_int32), ("ndim", ctypes.c_int32),
                ("shape", ctypes.POINTER(ctypes.c_int64))]


class OptionalInt(ctypes.Structure):
    _fields_ = [("value", ctypes.c_int), ("has_value", ctypes.c_bool)]

    @classmethod
    def of(cls, v: Optional[int]) -> "OptionalInt":
        return cls(0, False) if v is None else cls(int(v), True)


_lib = None


def lib() -> ctypes.CDLL:
    """Load the library; raise if it has not been built (no fallback)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise ImportError(f"{LIB_PATH} is missing: build it with `python mlx-runner_b200/build.py`")
    L = ctypes.CDLL(LIB_PATH)
    i64, vp, i32 = ctypes.c_int64, ctypes.c_void_p, ctypes.c_int
    L.qmm_infer_quant_spec.argtypes = [ctypes.POINTER(TensorInfo), i64, ctypes.POINTER(QuantSpec)]
    L.qmm_mode_str.argtypes = [QuantSpec]
    L.qmm_mode_str.restype = ctypes.c_char_p
    L.qmm_spec_from_args.argtypes = [OptionalInt, OptionalInt, ctypes.c_char_p, ctypes.POINTER(QuantSpec)]
    L.qmm_quantized_matmul.argtypes = [vp, i64, vp, i64, i64, i64, vp, i64, i64, vp, i64, i64, vp,
                                       ctypes.c_bool, OptionalInt, OptionalInt, ctypes.c_char_p, vp]
    L.qmm_quantized_matmul_noalloc.argtypes = L.qmm_quantized_matmul.argtypes
    L.qmm_weight_create.argtypes = [vp, vp, i64, i64, i64, i64, QuantSpec, i32, vp, ctypes.POINTER(vp)]
    L.qmm_weight_create_shard.argtypes = [vp, vp, i64, i64, QuantSpec, i32, i32, i32, i32, vp,
                                          ctypes.POINTER(vp)]
    L.qmm_shard_range.argtypes = [i64, i64, QuantSpec, i32, i32, i32] + [ctypes.POINTER(i64)] * 4
    L.qmm_weight_destroy.argtypes = [vp]
    L.qmm_weight_info.argtypes = [vp, ctypes.POINTER(i64), ctypes.POINTER(i64), ctypes.POINTER(QuantSpec),
                                  ctypes.POINTER(i32)]
    L.qmm_run.argtypes = [vp, vp, i64, i64, vp, i64, ctypes.c_bool, vp]
    L.qmm_linear.argtypes = [vp, ctypes.c_bool, vp, i64, i64, vp, i64, vp]
    L.qmm_dequantize.argtypes = [vp, vp, ctypes.c_int32, vp]
    L.qmm_quantize.argtypes = [vp, ctypes.c_int32, i64, i64, i64, OptionalInt, OptionalInt, ctypes.c_char_p, vp,
                               vp, vp, vp]
    L.qmm_swiglu_weight_create.argtypes = [vp, vp, vp, vp, i64, i64, i64, i64, QuantSpec, i32, vp,
                                           ctypes.POINTER(vp)]
    L.qmm_swiglu_run.argtypes = [vp, vp, i64, i64, vp, i64, vp]
    L.qmm_lm_head_argmax.argtypes = [vp, vp, i64, i64, vp, vp, vp, i64, vp]
    L.qmm_checkpoint_open.argtypes = [ctypes.c_char_p, ctypes.POINTER(vp)]
    L.qmm_checkpoint_close.argtypes = [vp]
    L.qmm_checkpoint_spec.argtypes = [vp, ctypes.POINTER(QuantSpec)]
    L.qmm_checkpoint_tensors.argtypes = [vp, ctypes.POINTER(ctypes.POINTER(TensorInfo)), ctypes.POINTER(i64)]
    L.qmm_checkpoint_read.argtypes = [vp, ctypes.c_char_p, vp, i64, i32]
    L.qmm_checkpoint_load_linear.argtypes = [vp, ctypes.c_char_p, vp, ctypes.POINTER(vp)]
    L.qmm_checkpoint_load_swiglu.argtypes = [vp, ctypes.c_char_p, ctypes.c_char_p, vp, ctypes.POINTER(vp)]
    L.qmm_tp_unique_id.argtypes = [vp]
    L.qmm_tp_comm_create.argtypes = [vp, i32, i32, i64, ctypes.POINTER(vp)]
    L.qmm_tp_comm_destroy.argtypes = [vp]
    L.qmm_tp_comm_create_detached.argtypes = [i32, i32, i64, ctypes.POINTER(vp)]
    L.qmm_tp_allreduce_bf16.argtypes = [vp, vp, i64, vp]
    L.qmm_tp_run_rowparallel.argtypes = [vp, vp, vp, i64, i64, vp, i64, vp]
    L.qmm_last_error.argtypes = [ctypes.c_char_p, ctypes.c_size_t]
    L.qmm_fault_arm.argtypes = [ctypes.c_uint64]
    L.qmm_device_status.argtypes = [vp]
    L.qmm_tensor_peak.argtypes = [i32, i64, vp, ctypes.POINTER(ctypes.c_double)]
    L.qmm_run_blockscaled.argtypes = [vp, vp, i64, i64, vp, i64, vp]
    for name in EXPORTS:
        fn = getattr(L, name)
        if name != "qmm_mode_str":
            fn.restype = ctypes.c_int
    _lib = L
    return L


def check(rc: int) -> None:
    """Raise QmmError for a non-zero status (src/mlx.zig:589 check)."""
    if rc != QMM_OK:
        buf = ctypes.create_string_buffer(512)
        lib().qmm_last_error(buf, len(buf))
        raise QmmError(rc, buf.value.decode(errors="replace"))


def take_error() -> tuple[int, str]:
    buf = ctypes.create_string_buffer(512)
    st = lib().qmm_last_error(buf, len(buf))
    return st, buf.value.decode(errors="replace")


def device_status(stream=None) -> None:
    """Raise QmmError(Timeout) if a kernel gave up a bounded wait."""
    check(lib().qmm_device_status(_stream_handle(stream)))


TENSOR_KINDS = {"bf16": 0, "mxf8f6f4": 1, "mxf4nvf4": 2}


def tensor_peak(kind: str, iters: int = 1 << 15, stream=None) -> float:
    """Measured dense tcgen05 rate (TFLOP/s) of one MMA kind on the current
    device: "bf16" (kind::f16), "mxf8f6f4" (E4M3, UE8M0 per 32) or
    "mxf4nvf4" (E2M1, UE4M3 per 16)."""
    out = ctypes.c_double()
    check(lib().qmm_tensor_peak(TENSOR_KINDS[kind], iters, _stream_handle(stream), ctypes.byref(out)))
    return out.value


def fault_arm(k: int) -> None:
    lib().qmm_fault_arm(k)


def fault_fired() -> bool:
    return bool(lib().qmm_fault_fired())


# ---- spec inference ---------------------------------------------------------

def infer_quant_spec(tensors: Iterable) -> tuple[str, int, int]:
    """(mode, group_size, bits) for a checkpoint's tensor infos.

    ``tensors`` yields (name, dtype, shape) with dtype one of BF16/F32/U32/U8.
    Raises QmmError(NonstandardQuant / InconsistentQuant / AffineUnsupported)
    exactly where src/weights.zig:132-185 returns those errors.
    """
    items = list(tensors)
    arr = (TensorInfo * max(1, len(items)))()
    keep = []
    for i, (name, dtype, shape) in enumerate(items):
        shp = (ctypes.c_int64 * max(1, len(shape)))(*shape)
        keep.append(shp)
        arr[i] = TensorInfo(name.encode(), DTYPES[dtype], len(shape), shp)
    spec = QuantSpec()
    check(lib().qmm_infer_quant_spec(arr, len(items), ctypes.byref(spec)))
    return spec.astuple()


def spec_from_args(group_size: Optional[int], bits: Optional[int], mode: str) -> QuantSpec:
    spec = QuantSpec()
    check(lib().qmm_spec_from_args(OptionalInt.of(group_size), OptionalInt.of(bits), mode.encode(),
                                   ctypes.byref(spec)))
    return spec


def make_spec(mode: str) -> QuantSpec:
    return spec_from_args(None, None, mode)


def shard_range(n_full: int, k_full: int, mode: str, axis: int, rank: int, nranks: int):
    """(row0, rows, col0, cols) of a tensor-parallel shard (pure host)."""
    out = [ctypes.c_int64() for _ in range(4)]
    check(lib().qmm_shard_range(n_full, k_full, make_spec(mode), axis, rank, nranks,
                                *[ctypes.byref(o) for o in out]))
    return tuple(o.value for o in out)


# ---- torch plumbing -----------------------------------------------------------

def _torch():
    import torch
    return torch


def _stream_handle(stream) -> int:
    torch = _torch()
    if stream is None:
        stream = torch.cuda.current_stream()
    return int(stream.cuda_stream) if hasattr(stream, "cuda_stream") else int(stream)


def _as_2d(x):
    k = x.shape[-1]
    x2 = x.reshape(-1, k)
    if x2.stride(-1) != 1:
        x2 = x2.contiguous()
    return x2


def _need_cuda(name: str, t, device: Optional[int] = None) -> None:
    """Raise unless t is a CUDA tensor (on `device` when given): the library
    hands data_ptr() to kernels, and a host or another GPU's pointer there
    would fault the device instead of failing the call."""
    if not getattr(t, "is_cuda", False):
        raise QmmError(7, f"{name} must be a CUDA tensor (got {getattr(t, 'device', type(t).__name__)})")
    if device is not None and t.device.index != device:
        raise QmmError(7, f"{name} is on cuda:{t.device.index}, the weight on cuda:{device}")


def _check_out(out, rows: int, cols: int, device: Optional[int] = None) -> None:
    """A caller's output buffer must hold [rows, cols] bf16 with unit column
    stride: the library sees only its row stride, not its size."""
    torch = _torch()
    _need_cuda("out", out, device)
    if out.dtype != torch.bfloat16 or out.dim() != 2 or out.stride(1) != 1 or out.shape[0] < rows \
            or out.shape[1] < cols:
        raise QmmError(7, f"out must be bfloat16 [>= {rows}, >= {cols}] with unit column stride, "
                          f"got {tuple(out.shape)} {out.dtype}")


def _need_current(name: str, t) -> None:
    """The stateless entry points launch on the current CUDA device: a tensor
    on another device would hand that device's pointers to this one."""
    cur = _torch().cuda.current_device()
    if t.device.index != cur:
        raise QmmError(7, f"{name} is on cuda:{t.device.index} but the current device is cuda:{cur}; "
                          f"call under `with torch.cuda.device({t.device.index})`")


def _need_packed(w, scales) -> None:
    torch = _torch()
    _need_cuda("w", w)
    _need_cuda("scales", scales, w.device.index)
    _need_current("w", w)
    if w.dim() != 2 or scales.dim() != 2 or not w.is_contiguous() or not scales.is_contiguous():
        raise QmmError(7, "w and scales must be contiguous 2-D tensors (the checkpoint layout)")
    if w.dtype not in (torch.int32, getattr(torch, "uint32", torch.int32)):
        raise QmmError(5, f"w must hold the packed U32 words (int32 or uint32), got {w.dtype}")
    if scales.dtype != torch.uint8:
        raise QmmError(5, f"scales must be uint8, got {scales.dtype}")


def quantized_matmul(x, w, scales, biases=None, transpose: bool = True, group_size: Optional[int] = None,
                     bits: Optional[int] = None, mode: str = "mxfp8", stream=None, out=None):
    """y = x . dequant(w, scales)^T for x bf16 [..., K] on the GPU.

    w: uint32 [N, K*bits/32] and scales: uint8 [N, K/group] CUDA tensors in
    the checkpoint layout (src/weights.zig:154-161).
    """
    torch = _torch()
    if x.dtype != torch.bfloat16:
        raise QmmError(7, f"x must be bfloat16, got {x.dtype}")
    _need_packed(w, scales)
    _need_cuda("x", x, w.device.index)
    x2 = _as_2d(x)
    n = w.shape[0]
    m, k = x2.shape
    if out is not None:
        _check_out(out, m, n, w.device.index)
    y = out if out is not None else torch.empty((m, n), dtype=torch.bfloat16, device=x.device)
    check(lib().qmm_quantized_matmul(
        y.data_ptr(), y.stride(0), x2.data_ptr(), m, k, x2.stride(0),
        w.data_ptr(), w.shape[0], w.shape[1], scales.data_ptr(), scales.shape[0], scales.shape[1],
        None if biases is None else biases.data_ptr(), transpose, OptionalInt.of(group_size),
        OptionalInt.of(bits), mode.encode(), _stream_handle(stream)))
    return y.reshape(*x.shape[:-1], n) if out is None else y


def quantized_matmul_noalloc(x, w, scales, out, biases=None, transpose: bool = True,
                             group_size: Optional[int] = None, bits: Optional[int] = None, mode: str = "mxfp8",
                             stream=None):
    """quantized_matmul into the caller's `out` through the entry point that
    allocates no device memory (its scratch is a static device array; calls
    that overlap on one device race)."""
    torch = _torch()
    if x.dtype != torch.bfloat16:
        raise QmmError(7, f"x must be bfloat16, got {x.dtype}")
    _need_packed(w, scales)
    _need_cuda("x", x, w.device.index)
    x2 = _as_2d(x)
    m, k = x2.shape
    _check_out(out, m, w.shape[0], w.device.index)
    check(lib().qmm_quantized_matmul_noalloc(
        out.data_ptr(), out.stride(0), x2.data_ptr(), m, k, x2.stride(0),
        w.data_ptr(), w.shape[0], w.shape[1], scales.data_ptr(), scales.shape[0], scales.shape[1],
        None if biases is None else biases.data_ptr(), transpose, OptionalInt.of(group_size),
        OptionalInt.of(bits), mode.encode(), _stream_handle(stream)))
    return out


def quantize(w, mode: str = "mxfp8", group_size: Optional[int] = None, bits: Optional[int] = None,
             global_scale=None, stream=None):
    """src/mlx.zig:278 mlx_quantize (as src/model.zig:1577 calls it): w fp32 or
    bf16 [N, K] on the GPU -> (codes, scales) on the same device, codes the
    U32 [N, K*bits/32] words held in an int32 tensor, scales uint8
    [N, K/group]; the layout QuantizedWeight and quantized_matmul take."""
    torch = _torch()
    if w.dtype == torch.float32:
        dt = DTYPES["F32"]
    elif w.dtype == torch.bfloat16:
        dt = DTYPES["BF16"]
    else:
        raise QmmError(5, f"quantize input must be float32 or bfloat16, got {w.dtype}")
    if w.dim() != 2:
        raise QmmError(1, f"quantize takes a 2-D weight, got shape {tuple(w.shape)}")
    _need_cuda("w", w)
    _need_current("w", w)
    if w.stride(1) != 1:
        w = w.contiguous()
    spec = spec_from_args(group_size, bits, mode)
    n, k = w.shape
    codes = torch.empty((n, k * spec.bits // 32), dtype=torch.int32, device=w.device)
    scales = torch.empty((n, k // spec.group_size), dtype=torch.uint8, device=w.device)
    check(lib().qmm_quantize(w.data_ptr(), dt, n, k, w.stride(0), OptionalInt.of(group_size), OptionalInt.of(bits),
                             mode.encode(), None if global_scale is None else global_scale.data_ptr(),
                             codes.data_ptr(), scales.data_ptr(), _stream_handle(stream)))
    return codes, scales


@dataclass
class _Src:
    ptr: int
    kind: int
    keep: object


def _src(a, dtype_name: str) -> _Src:
    """Host numpy array or torch tensor (CPU or CUDA) -> pointer + kind."""
    torch = _torch()
    if isinstance(a, torch.Tensor):
        a = a.contiguous()
        return _Src(a.data_ptr(), SRC_DEVICE if a.is_cuda else SRC_HOST, a)
    import numpy as np
    arr = np.ascontiguousarray(a)
    return _Src(arr.ctypes.data, SRC_HOST, arr)


class QuantizedWeight:
    """A packed weight resident on the current CUDA device.

    Created from the checkpoint tensors (U32 codes [N, K*bits/32], U8 scales
    [N, K/group]); the codes are uploaded bit for bit.
    """

    def __init__(self, codes, scales, mode: str, stream=None, shard: Optional[tuple[int, int, int]] = None):
        self.spec = make_spec(mode)
        c, s = _src(codes, "U32"), _src(scales, "U8")
        n_full = int(codes.shape[0])
        k_full = int(codes.shape[1]) * 32 // self.spec.bits
        h = ctypes.c_void_p()
        if shard is None:
            check(lib().qmm_weight_create(c.ptr, s.ptr, n_full, k_full, 0, 0, self.spec, c.kind,
                                          _stream_handle(stream), ctypes.byref(h)))
        else:
            axis, rank, nranks = shard
            check(lib().qmm_weight_create_shard(c.ptr, s.ptr, n_full, k_full, self.spec, c.kind, axis, rank,
                                                nranks, _stream_handle(stream), ctypes.byref(h)))
        self._h = h
        n, k, dev = ctypes.c_int64(), ctypes.c_int64(), ctypes.c_int()
        check(lib().qmm_weight_info(h, ctypes.byref(n), ctypes.byref(k), None, ctypes.byref(dev)))
        self.n, self.k, self.device = n.value, k.value, dev.value

    @property
    def handle(self) -> ctypes.c_void_p:
        if not self._h:
            raise QmmError(7, "weight was destroyed")
        return self._h

    @property
    def mode(self) -> str:
        return self.spec.mode_str

    def __call__(self, x, out=None, stream=None):
        return self.run(x, out=out, stream=stream)

    def run(self, x, out=None, stream=None):
        torch = _torch()
        if x.dtype != torch.bfloat16:
            raise QmmError(7, f"x must be bfloat16, got {x.dtype}")
        _need_cuda("x", x, self.device)
        x2 = _as_2d(x)
        m = x2.shape[0]
        if out is not None:
            _check_out(out, m, self.n, self.device)
        y = out if out is not None else torch.empty((m, self.n), dtype=torch.bfloat16, device=x.device)
        check(lib().qmm_run(self.handle, x2.data_ptr(), m, x2.stride(0), y.data_ptr(), y.stride(0), True,
                            _stream_handle(stream)))
        return y.reshape(*x.shape[:-1], self.n) if out is None else y

    def run_blockscaled(self, x, out=None, stream=None):
        """y = quantize_nvfp4(x) . dequant(W)^T on the block-scaled FP4 tensor
        cores (qmm_run_blockscaled): NOT the parity path - x is quantised."""
        torch = _torch()
        if x.dtype != torch.bfloat16:
            raise QmmError(7, f"x must be bfloat16, got {x.dtype}")
        _need_cuda("x", x, self.device)
        x2 = _as_2d(x)
        m = x2.shape[0]
        if out is not None:
            _check_out(out, m, self.n, self.device)
        y = out if out is not None else torch.empty((m, self.n), dtype=torch.bfloat16, device=x.device)
        check(lib().qmm_run_blockscaled(self.handle, x2.data_ptr(), m, x2.stride(0), y.data_ptr(), y.stride(0),
                                        _stream_handle(stream)))
        return y.reshape(*x.shape[:-1], self.n) if out is None else y

    def argmax(self, x, logits: bool = False, stream=None):
        """Greedy sampling of each x row through this (lm_head) weight:
        (ids int32 [M], logprobs fp32 [M], logits bf16 [M, N] or None)."""
        torch = _torch()
        if x.dtype != torch.bfloat16:
            raise QmmError(7, f"x must be bfloat16, got {x.dtype}")
        _need_cuda("x", x, self.device)
        x2 = _as_2d(x)
        m = x2.shape[0]
        ids = torch.empty((m,), dtype=torch.int32, device=x.device)
        lp = torch.empty((m,), dtype=torch.float32, device=x.device)
        y = torch.empty((m, self.n), dtype=torch.bfloat16, device=x.device) if logits else None
        check(lib().qmm_lm_head_argmax(self.handle, x2.data_ptr(), m, x2.stride(0), ids.data_ptr(), lp.data_ptr(),
                                       y.data_ptr() if y is not None else None, y.stride(0) if y is not None else 0,
                                       _stream_handle(stream)))
        return ids, lp, y

    def dequantize(self, dtype=None, stream=None):
        torch = _torch()
        dtype = dtype or torch.bfloat16
        code = {torch.bfloat16: DTYPES["BF16"], torch.float32: DTYPES["F32"]}[dtype]
        out = torch.empty((self.n, self.k), dtype=dtype, device=f"cuda:{self.device}")
        check(lib().qmm_dequantize(self.handle, out.data_ptr(), code, _stream_handle(stream)))
        return out

    def close(self) -> None:
        if getattr(self, "_h", None):
            check(lib().qmm_weight_destroy(self._h))
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class SwiGLUWeight(QuantizedWeight):
    """Gate and up projections of one MLP as a single resident weight whose
    run() returns h = silu(x.Wg^T) * (x.Wu^T) (src/model.zig:905-915 up to the
    down projection)."""

    def __init__(self, gate_codes, gate_scales, up_codes, up_scales, mode: str, stream=None):
        self.spec = make_spec(mode)
        gc, gs = _src(gate_codes, "U32"), _src(gate_scales, "U8")
        uc, us = _src(up_codes, "U32"), _src(up_scales, "U8")
        if gc.kind != uc.kind:
            raise QmmError(7, "gate and up tensors must both be host or both device arrays")
        n = int(gate_codes.shape[0])
        k = int(gate_codes.shape[1]) * 32 // self.spec.bits
        h = ctypes.c_void_p()
        check(lib().qmm_swiglu_weight_create(gc.ptr, gs.ptr, uc.ptr, us.ptr, n, k, 0, 0, self.spec, gc.kind,
                                             _stream_handle(stream), ctypes.byref(h)))
        self._h = h
        nn, kk, dev = ctypes.c_int64(), ctypes.c_int64(), ctypes.c_int()
        check(lib().qmm_weight_info(h, ctypes.byref(nn), ctypes.byref(kk), None, ctypes.byref(dev)))
        self.n, self.k, self.device = nn.value, kk.value, dev.value

    def run(self, x, out=None, stream=None):
        torch = _torch()
        if x.dtype != torch.bfloat16:
            raise QmmError(7, f"x must be bfloat16, got {x.dtype}")
        _need_cuda("x", x, self.device)
        x2 = _as_2d(x)
        m = x2.shape[0]
        if out is not None:
            _check_out(out, m, self.n, self.device)
        h = out if out is not None else torch.empty((m, self.n), dtype=torch.bfloat16, device=x.device)
        check(lib().qmm_swiglu_run(self.handle, x2.data_ptr(), m, x2.stride(0), h.data_ptr(), h.stride(0),
                                   _stream_handle(stream)))
        return h.reshape(*x.shape[:-1], self.n) if out is None else h

    def dequantize(self, dtype=None, stream=None):
        raise QmmError(7, "a gate/up weight has no single dequantized form")


def linear(weight: Optional[QuantizedWeight], x, has_packed_u32: bool = True, out=None, stream=None):
    """namedLinearQ (src/model.zig:218-233) for one projection."""
    torch = _torch()
    x2 = _as_2d(x)
    if weight is None:
        check(lib().qmm_linear(None, has_packed_u32, x2.data_ptr(), x2.shape[0], x2.stride(0), None, 0,
                               _stream_handle(stream)))
    if x.dtype != torch.bfloat16:
        raise QmmError(7, f"x must be bfloat16, got {x.dtype}")
    _need_cuda("x", x, weight.device)
    if out is not None:
        _check_out(out, x2.shape[0], weight.n, weight.device)
    y = out if out is not None else torch.empty((x2.shape[0], weight.n), dtype=torch.bfloat16, device=x.device)
    check(lib().qmm_linear(weight.handle, has_packed_u32, x2.data_ptr(), x2.shape[0], x2.stride(0),
                           y.data_ptr(), y.stride(0), _stream_handle(stream)))
    return y


def _adopt(cls, h: ctypes.c_void_p, spec):
    obj = cls.__new__(cls)
    obj.spec = spec
    obj._h = h
    n, k, dev = ctypes.c_int64(), ctypes.c_int64(), ctypes.c_int()
    check(lib().qmm_weight_info(h, ctypes.byref(n), ctypes.byref(k), None, ctypes.byref(dev)))
    obj.n, obj.k, obj.device = n.value, k.value, dev.value
    return obj


class Checkpoint:
    """A sharded safetensors checkpoint opened from its directory
    (src/weights.zig WeightMap.load, headers only until a tensor is read)."""

    def __init__(self, model_dir: str):
        h = ctypes.c_void_p()
        check(lib().qmm_checkpoint_open(os.fsencode(model_dir), ctypes.byref(h)))
        self._h = h

    @property
    def spec(self) -> QuantSpec:
        s = QuantSpec()
        check(lib().qmm_checkpoint_spec(self._h, ctypes.byref(s)))
        return s

    def tensors(self) -> dict:
        """name -> (dtype name, shape) for every tensor of every shard."""
        infos = ctypes.POINTER(TensorInfo)()
        count = ctypes.c_int64()
        check(lib().qmm_checkpoint_tensors(self._h, ctypes.byref(infos), ctypes.byref(count)))
        names = {v: k for k, v in DTYPES.items()}
        out = {}
        for i in range(count.value):
            t = infos[i]
            out[t.name.decode()] = (names[t.dtype], tuple(t.shape[d] for d in range(t.ndim)))
        return out

    def read(self, name: str):
        """The tensor's bytes as a numpy array of its dtype and shape."""
        import numpy as np
        info = self.tensors().get(name)
        if info is None:
            check(lib().qmm_checkpoint_read(self._h, name.encode(), None, 0, SRC_HOST))   # MissingTensor
        dt, shape = info
        np_dt = {"BF16": np.uint16, "F32": np.float32, "U32": np.uint32, "U8": np.uint8}[dt]
        arr = np.empty(shape, dtype=np_dt)
        check(lib().qmm_checkpoint_read(self._h, name.encode(), arr.ctypes.data, arr.nbytes, SRC_HOST))
        return arr

    def linear(self, prefix: str, stream=None) -> QuantizedWeight:
        h = ctypes.c_void_p()
        check(lib().qmm_checkpoint_load_linear(self._h, prefix.encode(), _stream_handle(stream), ctypes.byref(h)))
        return _adopt(QuantizedWeight, h, self.spec)

    def swiglu(self, gate_prefix: str, up_prefix: str, stream=None) -> "SwiGLUWeight":
        h = ctypes.c_void_p()
        check(lib().qmm_checkpoint_load_swiglu(self._h, gate_prefix.encode(), up_prefix.encode(),
                                               _stream_handle(stream), ctypes.byref(h)))
        return _adopt(SwiGLUWeight, h, self.spec)

    def close(self) -> None:
        if getattr(self, "_h", None):
            lib().qmm_checkpoint_close(self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class TPComm:
    """NCCL communicator for row-parallel shards (one per rank / GPU)."""

    def __init__(self, unique_id: bytes, nranks: int, rank: int, max_partial_elems: int):
        buf = ctypes.create_string_buffer(bytes(unique_id), 128)
        h = ctypes.c_void_p()
        check(lib().qmm_tp_comm_create(buf, nranks, rank, max_partial_elems, ctypes.byref(h)))
        self._h = h
        self.nranks, self.rank = nranks, rank

    @staticmethod
    def unique_id() -> bytes:
        buf = ctypes.create_string_buffer(128)
        check(lib().qmm_tp_unique_id(buf))
        return buf.raw

    @classmethod
    def detached(cls, nranks: int, rank: int, max_partial_elems: int) -> "TPComm":
        """Test hook: a communicator whose other ranks never run (no NCCL); the
        fused exchange on it times out and qmm_device_status reports Timeout."""
        obj = cls.__new__(cls)
        h = ctypes.c_void_p()
        check(lib().qmm_tp_comm_create_detached(nranks, rank, max_partial_elems, ctypes.byref(h)))
        obj._h = h
        obj.nranks, obj.rank = nranks, rank
        return obj

    def run_rowparallel(self, weight: QuantizedWeight, x_shard, out=None, stream=None):
        torch = _torch()
        _need_cuda("x_shard", x_shard, weight.device)
        x2 = _as_2d(x_shard)
        if out is not None:
            _check_out(out, x2.shape[0], weight.n, weight.device)
        y = out if out is not None else torch.empty((x2.shape[0], weight.n), dtype=torch.bfloat16,
                                                    device=x_shard.device)
        check(lib().qmm_tp_run_rowparallel(weight.handle, self._h, x2.data_ptr(), x2.shape[0], x2.stride(0),
                                           y.data_ptr(), y.stride(0), _stream_handle(stream)))
        return y

    def allreduce_bf16(self, buf, stream=None):
        _need_cuda("buf", buf)
        check(lib().qmm_tp_allreduce_bf16(self._h, buf.data_ptr(), buf.numel(), _stream_handle(stream)))
        return buf

    def close(self) -> None:
        if getattr(self, "_h", None):
            check(lib().qmm_tp_comm_destroy(self._h))
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
