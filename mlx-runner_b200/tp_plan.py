"""Tensor-parallel placement of the decoder's quantized projections over P
ranks - pure host logic over qmm_shard_range, used by bench.py's config 5
stack and checked on CPU ranks by tests/test_tp_gloo.py.

Column-parallel (axis 0: each rank holds a contiguous block of rows, its
outputs stay sharded, no collective): the projections whose outputs split by
heads or by FFN rows - GDN in_proj_qkv / in_proj_z / in_proj_b / in_proj_a
(src/model.zig:1066-1075), attention q_proj / k_proj / v_proj (:929-979),
the MLP gate_proj / up_proj (:905-915) and lm_head (:1309).
Row-parallel (axis 1: each rank holds a K-slice and the partial sums are
added across ranks): out_proj (:1230), o_proj and down_proj, whose inputs
are shards of column-parallel outputs.  k_proj / v_proj are replicated when
the ranks outnumber the KV heads.

For the MLP the two must meet: a rank's SwiGLU output rows (its gate / up
row block) are exactly down_proj's K-slice on that rank, which holds when
the FFN width divides evenly (checked by `mlp_slices`).
"""
from __future__ import annotations

import qmm

COLUMN = frozenset({"in_proj_qkv", "in_proj_z", "in_proj_b", "in_proj_a", "q_proj", "k_proj", "v_proj",
                    "gate_proj", "up_proj", "lm_head"})
ROW = frozenset({"out_proj", "o_proj", "down_proj"})
KV = frozenset({"k_proj", "v_proj"})


def placement(name: str, world: int, kv_heads: int = 4) -> str:
    """"column", "row" or "replicated" for projection `name` over `world` ranks."""
    if world == 1:
        return "replicated"
    if name in KV and world > kv_heads:
        return "replicated"
    if name in COLUMN:
        return "column"
    if name in ROW:
        return "row"
    raise KeyError(f"no tensor-parallel placement for {name!r}")


def take(codes, scales, mode: str, name: str, rank: int, world: int, kv_heads: int = 4):
    """This rank's (codes, scales) of the packed [N, K] tensors of `name`
    (numpy arrays or torch tensors; slices, not copies)."""
    spec = qmm.make_spec(mode)
    n = codes.shape[0]
    k = codes.shape[1] * 32 // spec.bits
    where = placement(name, world, kv_heads)
    if where == "replicated":
        return codes, scales
    axis = 0 if where == "column" else 1
    r0, rows, c0, cols = qmm.shard_range(n, k, mode, axis, rank, world)
    w0, w1 = c0 * spec.bits // 32, (c0 + cols) * spec.bits // 32
    g0, g1 = c0 // spec.group_size, (c0 + cols) // spec.group_size
    return codes[r0:r0 + rows, w0:w1], scales[r0:r0 + rows, g0:g1]


def mlp_slices(ffn: int, hidden: int, mode: str, rank: int, world: int) -> tuple[int, int]:
    """[start, stop) of this rank's FFN rows: its gate / up row block, which
    must equal down_proj's K-slice on the same rank."""
    r0, rows, _, _ = qmm.shard_range(ffn, hidden, mode, 0, rank, world)
    _, _, c0, cols = qmm.shard_range(hidden, ffn, mode, 1, rank, world)
    if (r0, rows) != (c0, cols):
        raise ValueError(f"FFN {ffn} does not split evenly over {world} ranks")
    return r0, r0 + rows
