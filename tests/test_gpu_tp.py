"""Tensor parallelism on 2, 4 and 8 GPUs (one process per GPU): K-sharded
row-parallel GEMM with the cross-rank sum, and N-sharded column-parallel
shards (no collective), both checked against the CPU oracle; each world
size is skipped where fewer GPUs are visible.  On one GPU: the exchange's
bounded wait running out.
"""
import os
import sys

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _case(mode, n, k, m, seed):
    import oracle
    rng = np.random.default_rng(seed)
    w = (rng.standard_normal((n, k), dtype=np.float32) * 0.02).astype(np.float32)
    codes, scales = oracle.quantize(w, mode)
    x = oracle.f32_to_bf16_bits(rng.standard_normal((m, k), dtype=np.float32))
    return codes, scales, x


def _rank(rank, world, uid, mode, n, k, m, q):
    try:
        for p in (os.path.join(ROOT, "mlx-runner_b200"), os.path.join(ROOT, "oracle")):
            sys.path.insert(0, p)
        import torch
        import qmm
        torch.cuda.set_device(rank)
        codes, scales, x = _case(mode, n, k, m, seed=9)
        xt = torch.from_numpy(x.view(np.int16)).view(torch.bfloat16)
        # Row-parallel: this rank's K slice, fp32 partials, one all-reduce.
        comm = qmm.TPComm(uid, world, rank, m * n)
        wk = qmm.QuantizedWeight(codes, scales, mode, shard=(1, rank, world))
        c0 = rank * (k // world)
        xs = xt[:, c0:c0 + k // world].contiguous().cuda()
        y_k = comm.run_rowparallel(wk, xs)
        # Column-parallel: this rank's rows, no collective.
        wn = qmm.QuantizedWeight(codes, scales, mode, shard=(0, rank, world))
        y_n = wn.run(xt.cuda())
        torch.cuda.synchronize()
        qmm.device_status()
        q.put((rank, y_k.cpu().view(torch.int16).numpy().view(np.uint16),
               y_n.cpu().view(torch.int16).numpy().view(np.uint16)))
        wk.close()
        wn.close()
        comm.close()
    except Exception as exc:
        q.put((rank, repr(exc), None))


@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("mode,n,k,m", [("nvfp4", 1024, 4096, 3), ("mxfp8", 768, 2048, 1),
                                        ("nvfp4", 5120, 17408, 4)])
def test_tp_gpus(world, mode, n, k, m):
    """K = 17408 / N = 5120 is benchmark config 2 (K slices of 8704 / 4352 /
    2176 codes); the smaller cases put few row blocks on each rank."""
    import torch
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import multiprocessing as mp
    import oracle
    import qmm
    uid = qmm.TPComm.unique_id()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, world, uid, mode, n, k, m, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = {}
    for _ in range(world):
        rank, a, b = q.get(timeout=600)
        out[rank] = (a, b)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for rank, (a, _) in out.items():
        assert not isinstance(a, str), f"rank {rank}: {a}"

    codes, scales, x = _case(mode, n, k, m, seed=9)
    ref, absref = oracle.qmm_f64_abs(x, codes, scales, mode)
    for rank in range(world):
        y = oracle.bf16_bits_to_f32(out[rank][0])
        assert oracle.parity_violations(y, ref, absref) == 0
    y_n = np.concatenate([oracle.bf16_bits_to_f32(out[r][1]) for r in range(world)], axis=1)
    assert oracle.parity_violations(y_n, ref, absref) == 0


def test_exchange_wait_times_out_and_reports(cuda_device):
    """The fused row-parallel exchange waiting for ranks that never run (a
    detached communicator: their flags are local memory nothing writes) gives
    up after its bounded 2 s wait; qmm_device_status reports Timeout once, and
    the device stays usable - a plain decode afterwards meets the parity bar.
    One GPU; no fault, no hang."""
    import time
    import torch
    import oracle
    import qmm
    n, k, m = 256, 2048, 2
    codes, scales, x = _case("nvfp4", n, k, m, seed=4)
    xt = torch.from_numpy(x.view(np.int16)).view(torch.bfloat16)
    comm = qmm.TPComm.detached(2, 0, m * n)
    w = qmm.QuantizedWeight(codes, scales, "nvfp4", shard=(1, 0, 2))
    xs = xt[:, :k // 2].contiguous().to(cuda_device)
    t0 = time.monotonic()
    comm.run_rowparallel(w, xs)
    with pytest.raises(qmm.QmmError) as ei:
        qmm.device_status()
    assert ei.value.name == "Timeout"
    assert time.monotonic() - t0 < 60
    qmm.device_status()                       # the word was cleared
    w.close()
    comm.close()
    w2 = qmm.QuantizedWeight(codes, scales, "nvfp4")
    y = w2(xt.to(cuda_device)).cpu().view(torch.int16).numpy().view(np.uint16)
    w2.close()
    got = oracle.bf16_bits_to_f32(y)
    assert oracle.parity_violations(got, oracle.qmm_f64(x, codes, scales, "nvfp4"),
                                    oracle.abs_qmm_f64(x, codes, scales, "nvfp4")) == 0
