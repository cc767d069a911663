"""Tensor-parallel host logic on CPU ranks (world size 2, gloo).

The GPU path shards a weight with qmm_shard_range and either concatenates
row shards (N-shard, column-parallel: no collective) or sums K-shard partials
with one all-reduce (row-parallel; fp32 partials, one rounding to bf16 at the
end).  Here each gloo rank slices the packed checkpoint tensors with the same
ranges, computes its shard with the oracle, and the ranks combine results
through torch.distributed exactly as the GPU ranks do through NCCL:
  - N-shard: all-gather of row blocks == the unsharded result, bit for bit;
  - K-shard: all-reduce of fp64 partials == the unsharded fp64 result (to
    summation order), and all-reduce of fp32 partials rounded once to bf16
    meets the parity bar against the fp64 reference.
"""
import os
import socket
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _case(mode, n=256, k=1024, m=3, seed=5):
    import oracle
    rng = np.random.default_rng(seed)
    w = (rng.standard_normal((n, k), dtype=np.float32) * 0.02).astype(np.float32)
    codes, scales = oracle.quantize(w, mode)
    x = oracle.f32_to_bf16_bits(rng.standard_normal((m, k), dtype=np.float32))
    return codes, scales, x


def _worker(rank: int, world: int, port: int, mode: str, q):
    try:
        for p in (os.path.join(ROOT, "mlx-runner_b200"), os.path.join(ROOT, "oracle")):
            sys.path.insert(0, p)
        import torch
        import torch.distributed as dist
        import oracle
        import qmm
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
        codes, scales, x = _case(mode)
        n, words = codes.shape
        k = words * 32 // qmm.make_spec(mode).bits
        bits = qmm.make_spec(mode).bits
        group = qmm.make_spec(mode).group_size

        # N-shard: rows [row0, row0 + rows), every column.
        r0, rows, c0, cols = qmm.shard_range(n, k, mode, 0, rank, world)
        assert (c0, cols) == (0, k)
        y_part = oracle.qmm_f64(x, codes[r0:r0 + rows], scales[r0:r0 + rows], mode)
        gathered = [torch.zeros((x.shape[0], n * (i + 1) // world - n * i // world), dtype=torch.float64)
                    for i in range(world)]
        dist.all_gather(gathered, torch.from_numpy(np.ascontiguousarray(y_part)))
        y_n = torch.cat(gathered, dim=1).numpy()

        # K-shard: columns [col0, col0 + cols) on group and word boundaries.
        r0, rows, c0, cols = qmm.shard_range(n, k, mode, 1, rank, world)
        assert (r0, rows) == (0, n) and cols == k // world and c0 == rank * cols
        assert c0 % group == 0 and (c0 * bits) % 32 == 0
        cs = codes[:, c0 * bits // 32:(c0 + cols) * bits // 32]
        ss = scales[:, c0 // group:(c0 + cols) // group]
        xs = np.ascontiguousarray(x[:, c0:c0 + cols])
        p64 = torch.from_numpy(np.ascontiguousarray(oracle.qmm_f64(xs, cs, ss, mode)))
        dist.all_reduce(p64)
        # fp32 partial: exact fp32 dequantisation, fp32 products and sums.
        w32 = oracle.dequantize(cs, ss, mode).astype(np.float32)
        p32 = torch.from_numpy(np.ascontiguousarray(oracle.bf16_bits_to_f32(xs).astype(np.float32) @ w32.T))
        dist.all_reduce(p32)
        q.put((rank, y_n, p64.numpy(), p32.numpy()))
        dist.barrier()
        dist.destroy_process_group()
    except Exception as exc:  # surface the failure to the parent
        q.put((rank, repr(exc), None, None))


@pytest.mark.parametrize("mode", ["nvfp4", "mxfp8"])
def test_tp_world2_gloo(mode):
    import multiprocessing as mp
    import oracle
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, mode, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    for _ in range(world):
        rank, a, b, c = q.get(timeout=240)
        results[rank] = (a, b, c)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, (a, b, c) in results.items():
        assert not isinstance(a, str), f"rank {rank}: {a}"

    codes, scales, x = _case(mode)
    ref = oracle.qmm_f64(x, codes, scales, mode)
    absref = oracle.abs_qmm_f64(x, codes, scales, mode)
    for rank in range(world):
        y_n, p64, p32 = results[rank]
        np.testing.assert_array_equal(y_n, ref)                 # N-shard: concatenation is exact
        np.testing.assert_allclose(p64, ref, rtol=1e-12, atol=1e-12 * np.abs(ref).max())
        y = oracle.bf16_bits_to_f32(oracle.f32_to_bf16_bits(p32))
        assert oracle.parity_violations(y, ref, absref) == 0   # fp32 partials, one rounding


def test_shard_range_rules():
    import qmm
    # K shards: equal, whole groups and whole U32 words; N shards differ by <= 1 row.
    for mode, k in (("nvfp4", 17408), ("mxfp8", 5120)):
        for world in (2, 4, 8):
            spans = [qmm.shard_range(5120, k, mode, 1, r, world) for r in range(world)]
            assert [s[2] for s in spans] == [r * k // world for r in range(world)]
            assert all(s[3] == k // world for s in spans)
            rows = [qmm.shard_range(17408, k, mode, 0, r, world)[1] for r in range(world)]
            assert sum(rows) == 17408 and max(rows) - min(rows) <= 1
    with pytest.raises(qmm.QmmError):
        qmm.shard_range(5120, 17408 + 16, "nvfp4", 1, 0, 8)     # 17424 / 8 is not a whole group


# ---- the decoder layer's placement (mlx-runner_b200/tp_plan.py) ------------

SMALL_LAYER = {"in_proj_qkv": (160, 256), "in_proj_z": (96, 256), "in_proj_b": (8, 256), "in_proj_a": (8, 256),
               "out_proj": (256, 192), "gate_proj": (512, 256), "up_proj": (512, 256), "down_proj": (256, 512)}


def _layer(mode, seed=9):
    import oracle
    rng = np.random.default_rng(seed)
    w = {nm: oracle.quantize((rng.standard_normal(shape, dtype=np.float32) * 0.02).astype(np.float32), mode)
         for nm, shape in SMALL_LAYER.items()}
    x = oracle.f32_to_bf16_bits(rng.standard_normal((3, 256), dtype=np.float32))
    x6 = oracle.f32_to_bf16_bits(rng.standard_normal((3, 192), dtype=np.float32))
    return w, x, x6


def _silu_mul(g, u):
    return g / (1.0 + np.exp(-g)) * u


def _layer_worker(rank: int, world: int, port: int, mode: str, q):
    try:
        for p in (os.path.join(ROOT, "mlx-runner_b200"), os.path.join(ROOT, "oracle")):
            sys.path.insert(0, p)
        import torch
        import torch.distributed as dist
        import oracle
        import qmm
        import tp_plan
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
        w, x, x6 = _layer(mode)
        # in_proj: this rank's rows of qkv | z | b | a, concatenated (one launch
        # on the GPU); the gathered blocks are reassembled per projection.
        names = ("in_proj_qkv", "in_proj_z", "in_proj_b", "in_proj_a")
        parts = [tp_plan.take(*w[nm], mode, nm, rank, world) for nm in names]
        y_in = oracle.qmm_f64(x, np.concatenate([c for c, _ in parts]), np.concatenate([s for _, s in parts]), mode)
        blocks = [None] * world
        dist.all_gather_object(blocks, (y_in, [c.shape[0] for c, _ in parts]))
        # MLP: gate / up rows of this rank -> SwiGLU -> down's K-slice -> sum.
        s0, s1 = tp_plan.mlp_slices(512, 256, mode, rank, world)
        g_c, g_s = tp_plan.take(*w["gate_proj"], mode, "gate_proj", rank, world)
        u_c, u_s = tp_plan.take(*w["up_proj"], mode, "up_proj", rank, world)
        assert g_c.shape[0] == s1 - s0 == u_c.shape[0]
        h = _silu_mul(oracle.qmm_f64(x, g_c, g_s, mode), oracle.qmm_f64(x, u_c, u_s, mode))
        d_c, d_s = tp_plan.take(*w["down_proj"], mode, "down_proj", rank, world)
        part = torch.from_numpy(np.ascontiguousarray(h @ oracle.dequantize(d_c, d_s, mode).astype(np.float64).T))
        dist.all_reduce(part)
        # out_proj: this rank's K-slice of its input.
        o_c, o_s = tp_plan.take(*w["out_proj"], mode, "out_proj", rank, world)
        _, _, c0, cols = qmm.shard_range(256, 192, mode, 1, rank, world)
        po = torch.from_numpy(np.ascontiguousarray(oracle.qmm_f64(np.ascontiguousarray(x6[:, c0:c0 + cols]),
                                                                   o_c, o_s, mode)))
        dist.all_reduce(po)
        q.put((rank, blocks, h, part.numpy(), po.numpy(), (s0, s1)))
        dist.barrier()
        dist.destroy_process_group()
    except Exception as exc:
        q.put((rank, repr(exc), None, None, None, None))


@pytest.mark.parametrize("mode", ["nvfp4", "mxfp8"])
def test_tp_layer_plan_world2_gloo(mode):
    """A decoder layer placed by tp_plan on two CPU ranks equals the unsharded
    layer: column-parallel in_proj (concatenated per rank) reassembles exactly,
    the SwiGLU rows of a rank are down_proj's K-slice there, and the
    row-parallel sums (down, out_proj) match to fp64 summation order."""
    import multiprocessing as mp
    import oracle
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_layer_worker, args=(r, world, port, mode, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(world):
        item = q.get(timeout=240)
        res[item[0]] = item[1:]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, item in res.items():
        assert not isinstance(item[0], str), f"rank {rank}: {item[0]}"

    w, x, x6 = _layer(mode)
    names = ("in_proj_qkv", "in_proj_z", "in_proj_b", "in_proj_a")
    full = {nm: oracle.qmm_f64(x, *w[nm], mode) for nm in names}
    g = oracle.qmm_f64(x, *w["gate_proj"], mode)
    u = oracle.qmm_f64(x, *w["up_proj"], mode)
    h_full = _silu_mul(g, u)
    y_down = h_full @ oracle.dequantize(*w["down_proj"], mode).astype(np.float64).T
    y_out = oracle.qmm_f64(x6, *w["out_proj"], mode)
    for rank in range(world):
        blocks, h, part, po, (s0, s1) = res[rank]
        # Reassemble each projection from every rank's block of the concatenation.
        for j, nm in enumerate(names):
            pieces = []
            for y_r, sizes in blocks:
                off = sum(sizes[:j])
                pieces.append(y_r[:, off:off + sizes[j]])
            np.testing.assert_array_equal(np.concatenate(pieces, axis=1), full[nm])
        np.testing.assert_array_equal(h, h_full[:, s0:s1])
        np.testing.assert_allclose(part, y_down, rtol=1e-12, atol=1e-12 * np.abs(y_down).max())
        np.testing.assert_allclose(po, y_out, rtol=1e-12, atol=1e-12 * np.abs(y_out).max())


def test_tp_plan_placements():
    import tp_plan
    assert tp_plan.placement("in_proj_qkv", 2) == "column"
    assert tp_plan.placement("down_proj", 8) == "row"
    assert tp_plan.placement("k_proj", 4) == "column"      # 4 KV heads: one per rank
    assert tp_plan.placement("k_proj", 8) == "replicated"  # more ranks than KV heads
    assert tp_plan.placement("lm_head", 1) == "replicated"
    with pytest.raises(KeyError):
        tp_plan.placement("conv1d", 2)
    for world in (2, 4, 8):                                 # config 5's FFN splits evenly
        spans = [tp_plan.mlp_slices(17408, 5120, "nvfp4", r, world) for r in range(world)]
        assert spans[0][0] == 0 and spans[-1][1] == 17408
        assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
