"""Spec inference and argument resolution through the C ABI (no GPU).

Known answers come from the reference's own test (src/weights.zig:493-541,
committed in tests/golden/golden.json) plus the remaining branches of
inferQuantSpec (src/weights.zig:132-185).
"""
import pytest

import qmm


def _infer(tensors):
    return qmm.infer_quant_spec([(t["name"], t["dtype"], t["shape"]) for t in tensors])


def test_reference_spec_cases(golden):
    for case in golden["spec_cases"]:
        exp = case["expect"]
        if "error" in exp:
            with pytest.raises(qmm.QmmError) as ei:
                _infer(case["tensors"])
            assert ei.value.name == exp["error"], case["ref"]
        else:
            assert _infer(case["tensors"]) == (exp["mode"], exp["group_size"], exp["bits"]), case["ref"]


def _err(tensors):
    with pytest.raises(qmm.QmmError) as ei:
        qmm.infer_quant_spec(tensors)
    return ei.value.name


def test_config_shapes():
    # benchmark configs: mxfp8 [17408, 5120] and nvfp4 [5120, 17408].
    assert qmm.infer_quant_spec([("a.weight", "U32", [17408, 1280]), ("a.scales", "U8", [17408, 160])]) == \
        ("mxfp8", 32, 8)
    assert qmm.infer_quant_spec([("a.weight", "U32", [5120, 2176]), ("a.scales", "U8", [5120, 1088])]) == \
        ("nvfp4", 16, 4)


def test_error_branches():
    # ratio neither 8 nor 2
    assert _err([("a.weight", "U32", [8, 12]), ("a.scales", "U8", [8, 4])]) == "NonstandardQuant"
    # packed cols not a multiple of scale cols
    assert _err([("a.weight", "U32", [8, 10]), ("a.scales", "U8", [8, 4])]) == "NonstandardQuant"
    # scales not 2-D
    assert _err([("a.weight", "U32", [8, 8]), ("a.scales", "U8", [32])]) == "NonstandardQuant"
    # scales without packed weight
    assert _err([("a.scales", "U8", [8, 4])]) == "NonstandardQuant"
    # packed weight of the wrong dtype
    assert _err([("a.weight", "BF16", [8, 8]), ("a.scales", "U8", [8, 4])]) == "NonstandardQuant"
    # second scales disagrees with the first ratio
    assert _err([("a.weight", "U32", [8, 8]), ("a.scales", "U8", [8, 4]),
                 ("b.weight", "U32", [8, 32]), ("b.scales", "U8", [8, 4])]) == "InconsistentQuant"
    # second scales of the wrong dtype
    assert _err([("a.weight", "U32", [8, 8]), ("a.scales", "U8", [8, 4]),
                 ("b.weight", "U32", [8, 8]), ("b.scales", "BF16", [8, 4])]) == "InconsistentQuant"
    # orphan packed weight next to a valid pair
    assert _err([("a.weight", "U32", [8, 8]), ("a.scales", "U8", [8, 4]),
                 ("b.weight", "U32", [8, 8])]) == "InconsistentQuant"
    # U8 tensor with no scales anywhere
    assert _err([("a.bias", "U8", [8])]) == "NonstandardQuant"
    # empty prefix
    assert _err([(".scales", "U8", [8, 4]), (".weight", "U32", [8, 8])]) == "NonstandardQuant"


def test_name_buffer_limit():
    # src/weights.zig:151: "<prefix>.weight" must fit the 1024-byte buffer.
    ok = "p" * 1017
    assert qmm.infer_quant_spec([(ok + ".weight", "U32", [8, 8]), (ok + ".scales", "U8", [8, 4])])[0] == "nvfp4"
    bad = "p" * 1018
    assert _err([(bad + ".weight", "U32", [8, 8]), (bad + ".scales", "U8", [8, 4])]) == "NonstandardQuant"


def test_dense_checkpoint_is_none():
    assert qmm.infer_quant_spec([("n.weight", "BF16", [16]), ("e.weight", "F32", [4, 4])]) == ("none", 0, 0)
    assert qmm.infer_quant_spec([]) == ("none", 0, 0)


def test_spec_from_args():
    s = qmm.spec_from_args(None, None, "mxfp8")
    assert s.astuple() == ("mxfp8", 32, 8)
    assert qmm.spec_from_args(16, 4, "nvfp4").astuple() == ("nvfp4", 16, 4)
    for g, b, m in [(64, None, "mxfp8"), (None, 4, "mxfp8"), (32, None, "nvfp4")]:
        with pytest.raises(qmm.QmmError) as ei:
            qmm.spec_from_args(g, b, m)
        assert ei.value.name == "BadMode"
    for m in ("affine", "mxfp4", ""):
        with pytest.raises(qmm.QmmError) as ei:
            qmm.spec_from_args(None, None, m)
        assert ei.value.name == "BadMode"


def test_mode_str():
    L = qmm.lib()
    assert L.qmm_mode_str(qmm.make_spec("nvfp4")) == b"nvfp4"
    assert L.qmm_mode_str(qmm.make_spec("mxfp8")) == b"mxfp8"
    assert L.qmm_mode_str(qmm.QuantSpec(0, 0, 0)) == b"mxfp8"   # weights.zig:52


@pytest.mark.parametrize("mode", ["mxfp8", "nvfp4"])
def test_shard_ranges(mode):
    # Column-parallel: contiguous row blocks covering N exactly once.
    n, k = 34816, 5120
    rows = [qmm.shard_range(n, k, mode, 0, r, 8) for r in range(8)]
    assert rows[0][0] == 0 and sum(r[1] for r in rows) == n
    assert all(rows[i][0] + rows[i][1] == rows[i + 1][0] for i in range(7))
    # Row-parallel: K / P slices on group and word boundaries.
    n, k = 5120, 17408
    for p in (2, 4, 8):
        shards = [qmm.shard_range(n, k, mode, 1, r, p) for r in range(p)]
        for r, (row0, rows, col0, cols) in enumerate(shards):
            assert (row0, rows) == (0, n)
            assert cols == k // p and col0 == r * cols
            assert col0 % 32 == 0 and cols % 32 == 0
    k_bad, p_bad = (48, 2) if mode == "nvfp4" else (64, 4)   # K/P not whole groups
    with pytest.raises(qmm.QmmError) as ei:
        qmm.shard_range(16, k_bad, mode, 1, 0, p_bad)
    assert ei.value.name == "BadShape"
