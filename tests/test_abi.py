"""The C-ABI library on the CPU: it loads, exports every symbol include/qmm.h
declares, validates arguments before touching the device, and mirrors the
reference's error latch (src/mlx.zig:719-805) and fault hook
(src/mlx.zig:562-595).  No kernel runs here."""
import ctypes
import os
import re

import pytest

import qmm

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared():
    txt = open(os.path.join(ROOT, "include", "qmm.h")).read()
    txt = re.sub(r"/\*.*?\*/", "", txt, flags=re.S)
    return sorted(set(re.findall(r"\b(qmm_[a-z0-9_]+)\s*\(", txt)))


def test_header_and_binding_agree():
    assert sorted(qmm.EXPORTS) == _declared()


def test_library_exports_every_declared_symbol():
    L = qmm.lib()
    for name in _declared():
        assert hasattr(L, name), name
    assert L.qmm_abi_version() == 1


def _mm(entry="qmm_quantized_matmul", **kw):
    """qmm_quantized_matmul (or its no-alloc twin, same arguments) with harmless
    defaults (never reaches the device)."""
    a = dict(y=1 << 20, ldy=8, x=1 << 20, m=1, k=32, ldx=32, w=1 << 20, w_rows=8, w_cols=8,
             s=1 << 20, s_rows=8, s_cols=1, biases=None, transpose=True, group=None, bits=None, mode=b"mxfp8")
    a.update(kw)
    return getattr(qmm.lib(), entry)(a["y"], a["ldy"], a["x"], a["m"], a["k"], a["ldx"], a["w"], a["w_rows"],
                                     a["w_cols"], a["s"], a["s_rows"], a["s_cols"], a["biases"], a["transpose"],
                                     qmm.OptionalInt.of(a["group"]), qmm.OptionalInt.of(a["bits"]), a["mode"], None)


def _status(rc):
    qmm.take_error()
    return qmm.STATUS_NAMES.get(rc, rc)


@pytest.mark.parametrize("entry", ["qmm_quantized_matmul", "qmm_quantized_matmul_noalloc"])
def test_validation_before_any_device_work(entry):
    import functools
    _mm_ = functools.partial(_mm, entry)
    qmm.take_error()
    assert _status(_mm_(mode=b"affine")) == "BadMode"
    assert _status(_mm_(group=64)) == "BadMode"
    assert _status(_mm_(biases=1 << 20)) == "BadArgument"
    assert _status(_mm_(transpose=False)) == "BadArgument"
    assert _status(_mm_(k=48)) == "BadShape"                       # not a multiple of group 32
    assert _status(_mm_(w_cols=4)) == "BadShape"                   # packs 16, not k = 32
    assert _status(_mm_(s_cols=2)) == "BadShape"                   # 2 groups for k = 32
    assert _status(_mm_(s_rows=7)) == "BadShape"
    assert _status(_mm_(ldx=16)) == "BadShape"
    assert _status(_mm_(ldy=4)) == "BadShape"
    assert _status(_mm_(x=None)) == "BadArgument"
    assert _status(_mm_(x=(1 << 20) + 2)) == "BadArgument"         # x not 4-byte aligned
    assert _status(_mm_(m=-1)) == "BadShape"
    # nvfp4: k = 16 is valid (one group), w packs 8 codes per word
    assert _status(_mm_(mode=b"nvfp4", k=16, ldx=16, w_cols=2, s_cols=1, ldy=4)) == "BadShape"  # ldy < n = 8


@pytest.mark.parametrize("entry", ["qmm_quantized_matmul", "qmm_quantized_matmul_noalloc"])
def test_empty_inputs_are_noops(entry):
    # m == 0 or n == 0 returns OK without touching the device (or its pointers).
    assert _mm(entry, m=0, x=None, y=None) == 0
    assert _mm(entry, w_rows=0, s_rows=0, w=None, s=None) == 0


def test_error_latch_first_wins_and_clears():
    qmm.take_error()
    assert not qmm.lib().qmm_error_pending()
    _mm(mode=b"nope")
    _mm(transpose=False)
    assert qmm.lib().qmm_error_pending()
    st, msg = qmm.take_error()
    assert qmm.STATUS_NAMES[st] == "BadMode" and "nope" in msg
    assert qmm.take_error() == (0, "")


def test_check_raises_reference_error_names():
    with pytest.raises(qmm.QmmError) as ei:
        qmm.infer_quant_spec([("l.q.weight", "U32", [8, 32]), ("l.q.scales", "BF16", [8, 2])])
    assert ei.value.name == "AffineUnsupported" and "U8" in str(ei.value)


def test_fault_injection_kth_call():
    """fault.arm(k): the k-th checked call fails, earlier ones run normally."""
    qmm.take_error()
    qmm.fault_arm(2)
    assert _status(_mm(mode=b"bad")) == "BadMode"     # call 1: not injected
    assert not qmm.fault_fired()
    assert _status(_mm()) == "Injected"               # call 2: injected before any work
    assert qmm.fault_fired()
    assert _status(_mm(mode=b"bad")) == "BadMode"     # disarmed afterwards
    qmm.fault_arm(0)


def test_weight_create_validates_on_host():
    h = ctypes.c_void_p()
    L = qmm.lib()
    spec = qmm.make_spec("nvfp4")
    rc = L.qmm_weight_create(None, None, 8, 24, 0, 0, spec, 0, None, ctypes.byref(h))
    assert _status(rc) == "BadShape" and not h.value               # k % 16 != 0
    rc = L.qmm_weight_create(None, None, 8, 32, 0, 0, spec, 0, None, ctypes.byref(h))
    assert _status(rc) == "BadArgument"                            # NULL sources
    rc = L.qmm_weight_create(None, None, 8, 32, 0, 0, qmm.QuantSpec(1, 16, 4), 0, None, ctypes.byref(h))
    assert _status(rc) == "BadMode"
    assert _status(L.qmm_linear(None, True, None, 1, 32, None, 8, None)) == "MissingWeight"


def test_no_device_is_an_error_not_a_fallback():
    """Without a GPU every compute entry point fails loudly."""
    torch = pytest.importorskip("torch")
    if torch.cuda.is_available():
        pytest.skip("a GPU is visible")
    rc = _mm()
    assert qmm.STATUS_NAMES[rc] in ("CudaError", "NoDevice")
    qmm.take_error()


def test_next_row_entry_points_validate_on_host():
    """SwiGLU, greedy sampling and checkpoint entry points reject bad arguments
    before any device work."""
    L = qmm.lib()
    h = ctypes.c_void_p()
    spec = qmm.make_spec("nvfp4")
    qmm.take_error()
    rc = L.qmm_swiglu_weight_create(None, None, None, None, 0, 32, 0, 0, spec, 0, None, ctypes.byref(h))
    assert _status(rc) == "BadShape" and not h.value                # n must be > 0
    rc = L.qmm_swiglu_weight_create(None, None, None, None, 8, 24, 0, 0, spec, 0, None, ctypes.byref(h))
    assert _status(rc) == "BadShape"                                # k % 16 != 0
    rc = L.qmm_swiglu_weight_create(None, None, None, None, 8, 32, 0, 0, spec, 0, None, None)
    assert _status(rc) == "BadArgument"                             # no out pointer
    assert _status(L.qmm_swiglu_run(None, None, 1, 32, None, 8, None)) == "BadArgument"
    assert _status(L.qmm_lm_head_argmax(None, None, 1, 32, None, None, None, 0, None)) == "BadArgument"
    assert _status(L.qmm_checkpoint_open(None, ctypes.byref(h))) == "BadArgument"
    assert _status(L.qmm_checkpoint_open(b"/nonexistent-model-dir", ctypes.byref(h))) == "IoError"
    assert not h.value
    assert L.qmm_checkpoint_close(None) == 0
    assert _status(L.qmm_checkpoint_load_linear(None, b"x", None, ctypes.byref(h))) == "BadArgument"


def test_quantize_validates_on_host():
    """qmm_quantize (src/mlx.zig:278) rejects bad arguments before any device
    work, with the reference's error classes."""
    L = qmm.lib()
    O = qmm.OptionalInt.of
    qmm.take_error()
    buf = ctypes.c_void_p(16)   # never dereferenced: every call below fails first
    args = lambda **kw: dict(dict(w=buf, dt=1, n=8, k=32, ldw=0, g=O(None), b=O(None), mode=b"nvfp4", gs=None,
                                  c=buf, s=buf), **kw)

    def call(**kw):
        a = args(**kw)
        return _status(L.qmm_quantize(a["w"], a["dt"], a["n"], a["k"], a["ldw"], a["g"], a["b"], a["mode"], a["gs"],
                                      a["c"], a["s"], None))
    assert call(mode=b"affine") == "BadMode"              # as qmm_spec_from_args for every entry point
    assert call(mode=b"nvfp4", g=O(32)) == "BadMode"
    assert call(gs=buf) == "BadArgument"                 # global_scale is not taken
    assert call(dt=2) == "UnsupportedDtype"              # U32 input
    assert call(k=24) == "BadShape"                      # k % 16
    assert call(mode=b"mxfp8", k=48) == "BadShape"       # k % 32
    assert call(ldw=16) == "BadShape"                    # ldw < k
    assert call(n=-1) == "BadShape"
    assert call(w=None) == "BadArgument"
    assert call(c=ctypes.c_void_p(18)) == "BadArgument"  # codes not 4-byte aligned
    assert call(n=0) == 0                                # empty: nothing to do


def test_detached_comm_validates_on_host():
    L = qmm.lib()
    h = ctypes.c_void_p()
    qmm.take_error()
    assert _status(L.qmm_tp_comm_create_detached(1, 0, 64, ctypes.byref(h))) == "BadArgument"   # < 2 ranks
    assert _status(L.qmm_tp_comm_create_detached(9, 0, 64, ctypes.byref(h))) == "BadArgument"   # > 8 ranks
    assert _status(L.qmm_tp_comm_create_detached(2, 2, 64, ctypes.byref(h))) == "BadArgument"   # rank out of range
    assert _status(L.qmm_tp_comm_create_detached(2, 0, 0, ctypes.byref(h))) == "BadArgument"    # no capacity
    assert _status(L.qmm_tp_comm_create_detached(2, 0, 64, None)) == "BadArgument"
    assert not h.value
