"""Checkpoint loader rules on the CPU (no kernel runs): sharded safetensors
headers and index as src/weights.zig reads them (WeightMap.load :258-352,
checkShardFile :241-255, parseHeaderJson :72-121, inferQuantSpec), and a
byte-exact round trip of tensor data.

The header cases are the reference's own (weights.zig "header parse
validates dtype and conv layout"; mlx_test.zig:47-113 "weights sharded
fixture roundtrips shapes and values"), written to files here.
"""
import json
import os
import struct

import numpy as np
import pytest

import qmm


def write_shard(path, header_json: str, data: bytes = b""):
    raw = header_json.encode()
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(raw)))
        f.write(raw)
        f.write(data)


def write_tensors(path, tensors: dict):
    """name -> numpy array (float32 -> F32, uint32 -> U32, uint8 -> U8, uint16 -> BF16 bits)."""
    dt = {np.float32: "F32", np.uint32: "U32", np.uint8: "U8", np.uint16: "BF16"}
    hdr, blobs, off = {"__metadata__": {}}, [], 0
    for name, a in tensors.items():
        a = np.ascontiguousarray(a)
        hdr[name] = {"dtype": dt[a.dtype.type], "shape": list(a.shape), "data_offsets": [off, off + a.nbytes]}
        blobs.append(a.tobytes())
        off += a.nbytes
    write_shard(path, json.dumps(hdr), b"".join(blobs))


def write_index(d, weight_map: dict):
    with open(os.path.join(d, "model.safetensors.index.json"), "w") as f:
        json.dump({"metadata": {}, "weight_map": weight_map}, f)


def status(exc_info):
    return exc_info.value.name


def test_header_rules_from_the_reference(tmp_path):
    d = str(tmp_path)
    good = ('{"__metadata__": {}, "a": {"dtype": "F32", "shape": [2], "data_offsets": [0, 8]},'
            ' "w": {"dtype": "BF16", "shape": [4, 2], "data_offsets": [8, 24]},'
            ' "c": {"dtype": "BF16", "shape": [10240, 4, 1], "data_offsets": [24, 40]}}')
    write_shard(os.path.join(d, "t.safetensors"), good, bytes(40))
    write_index(d, {"a": "t.safetensors", "w": "t.safetensors", "c": "t.safetensors"})
    ck = qmm.Checkpoint(d)
    assert ck.tensors() == {"a": ("F32", (2,)), "w": ("BF16", (4, 2)), "c": ("BF16", (10240, 4, 1))}
    ck.close()
    cases = [
        ('{"q": {"dtype": "F16", "shape": [2], "data_offsets": [0, 4]}}', "UnsupportedDtype"),
        ('{"m.conv1d.weight": {"dtype": "BF16", "shape": [8, 4, 2], "data_offsets": [0, 128]}}', "UnsupportedLayout"),
        (good[:-20], "BadHeader"),
        ("not json", "BadHeader"),
        ('{"q": {"dtype": "F32", "shape": [2.5], "data_offsets": [0, 4]}}', "BadHeader"),
        ('{"q": {"shape": [2], "data_offsets": [0, 4]}}', "BadHeader"),
        ('{"q": 3}', "BadHeader"),
        ('[1, 2]', "BadHeader"),
    ]
    for hdr, want in cases:
        write_shard(os.path.join(d, "t.safetensors"), hdr, bytes(128))
        with pytest.raises(qmm.QmmError) as ei:
            qmm.Checkpoint(d)
        assert status(ei) == want, (hdr, ei.value)


def test_header_length_cap(tmp_path):
    d = str(tmp_path)
    write_index(d, {"a": "t.safetensors"})
    p = os.path.join(d, "t.safetensors")
    for n in (0, 256 * 1024 * 1024 + 1):
        with open(p, "wb") as f:
            f.write(struct.pack("<Q", n))
        with pytest.raises(qmm.QmmError) as ei:
            qmm.Checkpoint(d)
        assert status(ei) == "BadHeader"
    with open(p, "wb") as f:
        f.write(b"\x01\x02")                          # shorter than the length field
    with pytest.raises(qmm.QmmError) as ei:
        qmm.Checkpoint(d)
    assert status(ei) == "BadHeader"


def test_index_rules(tmp_path):
    d = str(tmp_path)
    with pytest.raises(qmm.QmmError) as ei:
        qmm.Checkpoint(os.path.join(d, "no-such-dir"))
    assert status(ei) == "IoError"
    idx = os.path.join(d, "model.safetensors.index.json")
    for body in ("not json", '{"metadata": {}}', '{"weight_map": []}', '{"weight_map": {"a": 3}}', "[]"):
        with open(idx, "w") as f:
            f.write(body)
        with pytest.raises(qmm.QmmError) as ei:
            qmm.Checkpoint(d)
        assert status(ei) == "BadIndexJson", body
    write_index(d, {"a": "missing.safetensors"})
    with pytest.raises(qmm.QmmError) as ei:
        qmm.Checkpoint(d)
    assert status(ei) == "IoError"


def test_fixture_round_trip(tmp_path):
    """mlx_test.zig:47-113: three F32 tensors and a vision tensor in one shard;
    values come back exactly (names are kept as stored here)."""
    d = str(tmp_path)
    vals = np.array([1.5, -2.0, 1, 2, 3, 4, 7.0, 9.0], np.float32)
    hdr = ('{"__metadata__":{},'
           '"a":{"dtype":"F32","shape":[2],"data_offsets":[0,8]},'
           '"b":{"dtype":"F32","shape":[2,2],"data_offsets":[8,24]},'
           '"c":{"dtype":"F32","shape":[1],"data_offsets":[24,28]},'
           '"vision_tower.q":{"dtype":"F32","shape":[1],"data_offsets":[28,32]}}')
    write_shard(os.path.join(d, "t.safetensors"), hdr, vals.tobytes())
    write_index(d, {"a": "t.safetensors", "b": "t.safetensors", "c": "t.safetensors",
                    "vision_tower.q": "t.safetensors"})
    ck = qmm.Checkpoint(d)
    np.testing.assert_array_equal(ck.read("a"), [1.5, -2.0])
    np.testing.assert_array_equal(ck.read("b"), [[1, 2], [3, 4]])
    np.testing.assert_array_equal(ck.read("c"), [7.0])
    np.testing.assert_array_equal(ck.read("vision_tower.q"), [9.0])
    assert ck.spec.mode_str == "none"
    with pytest.raises(qmm.QmmError) as ei:
        ck.read("d")
    assert status(ei) == "MissingTensor"


def test_shards_duplicates_and_spans(tmp_path):
    d = str(tmp_path)
    rng = np.random.default_rng(0)
    a = rng.integers(0, 2**32, (8, 8), dtype=np.uint32)
    write_tensors(os.path.join(d, "s1.safetensors"), {"l.q_proj.weight": a,
                                                      "l.q_proj.scales": np.full((8, 4), 120, np.uint8)})
    write_tensors(os.path.join(d, "s2.safetensors"), {"l.norm.weight": np.zeros(16, np.uint16)})
    write_index(d, {"l.norm.weight": "s2.safetensors", "l.q_proj.weight": "s1.safetensors",
                    "l.q_proj.scales": "s1.safetensors"})
    ck = qmm.Checkpoint(d)
    # inferQuantSpec test shapes (weights.zig): packed [8, 8] U32, scales [8, 4] -> nvfp4.
    assert ck.spec.astuple() == ("nvfp4", 16, 4)
    assert list(ck.tensors()) == ["l.norm.weight", "l.q_proj.weight", "l.q_proj.scales"]   # shard order
    np.testing.assert_array_equal(ck.read("l.q_proj.weight"), a)
    ck.close()
    # The same name in two shards.
    write_tensors(os.path.join(d, "s2.safetensors"), {"l.norm.weight": np.zeros(16, np.uint16),
                                                      "l.q_proj.scales": np.zeros((8, 4), np.uint8)})
    with pytest.raises(qmm.QmmError) as ei:
        qmm.Checkpoint(d)
    assert status(ei) == "DuplicateTensor"
    # data_offsets that do not match the shape fail when read.
    write_shard(os.path.join(d, "s2.safetensors"),
                '{"l.norm.weight": {"dtype": "BF16", "shape": [16], "data_offsets": [0, 30]}}', bytes(32))
    ck = qmm.Checkpoint(d)
    with pytest.raises(qmm.QmmError) as ei:
        ck.read("l.norm.weight")
    assert status(ei) == "BadHeader"


def test_inconsistent_quant_is_rejected_at_open(tmp_path):
    d = str(tmp_path)
    write_tensors(os.path.join(d, "s.safetensors"), {
        "a.weight": np.zeros((8, 8), np.uint32), "a.scales": np.zeros((8, 4), np.uint8),     # r = 2 (nvfp4)
        "b.weight": np.zeros((8, 8), np.uint32), "b.scales": np.zeros((8, 1), np.uint8)})    # r = 8 (mxfp8)
    write_index(d, {k: "s.safetensors" for k in ("a.weight", "a.scales", "b.weight", "b.scales")})
    with pytest.raises(qmm.QmmError) as ei:
        qmm.Checkpoint(d)
    assert status(ei) == "InconsistentQuant"


def test_hostile_linear_shapes_fail_before_any_upload(tmp_path):
    """A header whose linear is absurdly large (2^60 packed columns) parses, and
    loading it fails with BadHeader on the host - the shape arithmetic is
    checked before it runs and nothing reaches the device."""
    d = str(tmp_path)
    hdr = {"big.weight": {"dtype": "U32", "shape": [1, 2 ** 60], "data_offsets": [0, 8]},
           "big.scales": {"dtype": "U8", "shape": [1, 2 ** 59], "data_offsets": [8, 16]}}
    write_shard(os.path.join(d, "s.safetensors"), json.dumps(hdr), bytes(16))
    write_index(d, {"big.weight": "s.safetensors", "big.scales": "s.safetensors"})
    ck = qmm.Checkpoint(d)
    assert ck.spec.astuple() == ("nvfp4", 16, 4)          # r = 2^60 / 2^59 = 2
    import ctypes
    h = ctypes.c_void_p()
    rc = qmm.lib().qmm_checkpoint_load_linear(ck._h, b"big", None, ctypes.byref(h))
    assert qmm.STATUS_NAMES.get(rc) == "BadHeader" and not h.value
    qmm.take_error()
    ck.close()
