"""Checkpoint -> resident weights on the B200: a two-shard safetensors
checkpoint written here (packed U32 codes + U8 scales from the oracle's
quantiser) loads through qmm_checkpoint_load_linear / _load_swiglu and
the weights compute what the oracle computes from the same tensors."""
import json
import os
import struct

import numpy as np
import pytest

import oracle
import qmm

pytestmark = pytest.mark.gpu


def write_tensors(path, tensors: dict):
    dt = {np.float32: "F32", np.uint32: "U32", np.uint8: "U8", np.uint16: "BF16"}
    hdr, blobs, off = {"__metadata__": {"format": "mlx"}}, [], 0
    for name, a in tensors.items():
        a = np.ascontiguousarray(a)
        hdr[name] = {"dtype": dt[a.dtype.type], "shape": list(a.shape), "data_offsets": [off, off + a.nbytes]}
        blobs.append(a.tobytes())
        off += a.nbytes
    raw = json.dumps(hdr).encode()
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(raw)))
        f.write(raw)
        f.write(b"".join(blobs))


def quant(n, k, mode, seed):
    rng = np.random.default_rng(seed)
    return oracle.quantize((rng.standard_normal((n, k), dtype=np.float32) * 0.02).astype(np.float32), mode)


def bits(t):
    import torch
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


@pytest.mark.parametrize("mode", ["mxfp8", "nvfp4"])
def test_checkpoint_linears_match_the_oracle(cuda_device, tmp_path, mode):
    import torch
    d = str(tmp_path)
    k = 512
    q = quant(320, k, mode, 1)
    g = quant(200, k, mode, 2)
    u = quant(200, k, mode, 3)
    pre = "language_model.model.layers.0"
    write_tensors(os.path.join(d, "model-00001-of-00002.safetensors"), {
        f"{pre}.self_attn.q_proj.weight": q[0], f"{pre}.self_attn.q_proj.scales": q[1],
        f"{pre}.input_layernorm.weight": np.zeros(k, np.uint16)})
    write_tensors(os.path.join(d, "model-00002-of-00002.safetensors"), {
        f"{pre}.mlp.gate_proj.weight": g[0], f"{pre}.mlp.gate_proj.scales": g[1],
        f"{pre}.mlp.up_proj.weight": u[0], f"{pre}.mlp.up_proj.scales": u[1]})
    wm = {}
    for name in (f"{pre}.self_attn.q_proj.weight", f"{pre}.self_attn.q_proj.scales", f"{pre}.input_layernorm.weight"):
        wm[name] = "model-00001-of-00002.safetensors"
    for name in (f"{pre}.mlp.gate_proj.weight", f"{pre}.mlp.gate_proj.scales", f"{pre}.mlp.up_proj.weight",
                 f"{pre}.mlp.up_proj.scales"):
        wm[name] = "model-00002-of-00002.safetensors"
    with open(os.path.join(d, "model.safetensors.index.json"), "w") as f:
        json.dump({"metadata": {}, "weight_map": wm}, f)

    ck = qmm.Checkpoint(d)
    assert ck.spec.mode_str == mode
    wq = ck.linear(f"{pre}.self_attn.q_proj")
    assert (wq.n, wq.k) == (320, k)
    gen = torch.Generator().manual_seed(5)
    x = torch.randn((3, k), generator=gen).to(torch.bfloat16)
    xd = x.to(cuda_device)
    y = bits(wq(xd))
    xb = bits(x)
    ref = oracle.qmm_f64(xb, *q, mode)
    assert oracle.parity_violations(oracle.bf16_bits_to_f32(y), ref, oracle.abs_qmm_f64(xb, *q, mode)) == 0
    # Same codes bit for bit as a weight created from the arrays directly.
    np.testing.assert_array_equal(y, bits(qmm.QuantizedWeight(*q, mode)(xd)))

    sw = ck.swiglu(f"{pre}.mlp.gate_proj", f"{pre}.mlp.up_proj")
    h = bits(sw(xd))
    gr, ur = oracle.qmm_f64(xb, *g, mode), oracle.qmm_f64(xb, *u, mode)
    ag, au = oracle.abs_qmm_f64(xb, *g, mode), oracle.abs_qmm_f64(xb, *u, mode)
    assert oracle.swiglu_violations(h, gr, ur, ag, au) == 0

    with pytest.raises(qmm.QmmError) as ei:
        ck.linear(f"{pre}.self_attn.k_proj")
    assert ei.value.name == "MissingTensor"
    ck.close()
