"""Benchmark of the quantized-matmul hot path (one JSON line on rank 0).

Headline workload (the config the metric is quoted on):
nvfp4 small-batch GEMM for decode + MTP verify, x bf16 [M, 17408] with
M = 1, 2, 3, 4, W [5120, 17408] nvfp4 (E2M1 codes, group 16, UE4M3 scales).
On N GPUs the weight is K-sharded (row-parallel): every rank multiplies its
K/N slice and the fp32 partials are summed with one NCCL all-reduce.

A step is one pass of the hot path over one batch of synthetic input: the
four GEMMs (M = 1..4) against each of C resident weight copies, where the
copies together exceed the 126 MB L2 several times, so every step streams
its weights from HBM (no L2 flush needed).

  value  whole-job algorithmic GB/s (codes + scales + x + y of the full
         problem, every GEMM) / device time of the K timed steps, max over
         ranks, inputs resident in HBM;
  e2e    the same metric through the C-ABI call with host buffers: each GEMM
         copies its x from pinned host memory, runs, and copies y back;
  roofline  the GEMV kernel alone: per-launch algorithmic bytes / per-launch
         CUDA-event time against the measured HBM copy bandwidth;
  cpu_baseline  the CPU restatement (oracle, fp32 accumulate, OpenMP) on the
         host cores, one bounded sample of the same workload.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
"""
from __future__ import annotations

import argparse
import importlib.util
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "mlx-runner_b200")

N_OUT, K_IN, MODE = 5120, 17408, "nvfp4"
M_SET = (1, 2, 3, 4)
GROUP, BITS = 16, 4
L2_BYTES = 126 * 1024 * 1024
FALLBACK_HBM_GBS = 6650.0
# Per-launch DRAM traffic of the decode kernel (dram__bytes_read.sum +
# dram__bytes_write.sum) from an ncu --set full capture of two launches of
# this bench's decode run (50.22 MB read + 0.06 MB written per launch).
GEMV_TRAFFIC_BYTES = 50.28e6


def _load(name, path):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def algo_bytes(m: int, n: int = N_OUT, k: int = K_IN) -> int:
    """Compulsory bytes of one y[m, n] = x[m, k] . W^T: codes + scales + x + y."""
    return n * k * BITS // 8 + n * (k // GROUP) + m * k * 2 + m * n * 2


def step_bytes(copies: int) -> int:
    return copies * sum(algo_bytes(m) for m in M_SET)


def step_flops(copies: int) -> float:
    return copies * sum(2.0 * m * N_OUT * K_IN for m in M_SET)


def peaks() -> tuple[float, str]:
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


class ClockSampler:
    """nvidia-smi clocks + throttle reasons sampled while work runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines: list[str] = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            threading.Thread(target=self._read, daemon=True).start()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self) -> dict:
        sm, mx, reasons = [], [], set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx.append(float(f[2]))
            except ValueError:
                continue
            for nm, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(sm)}


def run_reference(args, rank: int) -> None:
    """The CPU restatement on the host cores, same metric and config."""
    if rank != 0:
        return
    oracle = _load("oracle", os.path.join(ROOT, "oracle", "oracle.py"))
    oracle.build()
    rng = np.random.default_rng(0)
    w = (rng.standard_normal((N_OUT, K_IN), dtype=np.float32) * 0.02).astype(np.float32)
    codes, scales = oracle.quantize(w, MODE)
    xs = {m: oracle.f32_to_bf16_bits(rng.standard_normal((m, K_IN), dtype=np.float32)) for m in M_SET}
    threads = oracle.max_threads()

    def one_step():
        for m in M_SET:
            oracle.qmm_f32(xs[m], codes, scales, MODE, threads)

    for _ in range(args.warmup):
        one_step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        one_step()
    dt = time.perf_counter() - t0
    gbs = step_bytes(1) * args.steps / dt / 1e9
    line = {
        "impl": "reference", "metric": METRIC, "value": gbs, "unit": "GB/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt * 1e3 / args.steps,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "nvfp4xbf16->f32acc",
        "data": "synthetic (seeded N(0,1) x, N(0,0.02^2) W quantized by the oracle)",
        "config": dict(CONFIG, copies=1, l2="CPU run, no L2 policy"),
        "cpu_baseline": {"value": gbs, "unit": "GB/s", "cores": threads, "kind": "port",
                         "sample": f"{args.steps} full steps (M=1..4, one weight copy), fp32 accumulate, "
                                   f"{threads} OpenMP threads"},
        "e2e": {"value": gbs, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


METRIC = "qmm HBM GB/s, nvfp4 M=1..4 decode/MTP GEMM (K=17408, N=5120)"
CONFIG = {"workload": "cfg2: nvfp4 small-batch GEMM, x bf16 [M in 1..4, 17408], W [5120, 17408], "
                      "K-sharded over the GPUs with an fp32 all-reduce",
          "mode": MODE, "m": list(M_SET), "n": N_OUT, "k": K_IN}


PREFILL = {"m": 32768, "n": 34816, "k": 5120, "mode": "nvfp4"}


def prefill_measure(args, qmm, oracle, dev, world: int, rank: int, barrier, max_over_ranks) -> dict:
    """BASELINE config 3 (32k-token nvfp4 gate/up GEMM) on the tcgen05 kernel;
    N-sharded (column-parallel, no collective) over the GPUs."""
    import torch
    m, n, k, mode = args.prefill_m, PREFILL["n"], PREFILL["k"], PREFILL["mode"]
    rng = np.random.default_rng(2)
    w = (rng.standard_normal((n, k), dtype=np.float32) * 0.02).astype(np.float32)
    codes, scales = oracle.quantize(w, mode)
    del w
    wt = qmm.QuantizedWeight(codes, scales, mode, shard=(0, rank, world))
    g = torch.Generator(device=dev).manual_seed(3)
    x = torch.randn((m, k), generator=g, device=dev, dtype=torch.float32).to(torch.bfloat16)
    y = torch.empty((m, wt.n), dtype=torch.bfloat16, device=dev)
    stream = torch.cuda.current_stream()
    for _ in range(max(1, args.prefill_warmup)):
        wt.run(x, out=y, stream=stream)
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.prefill_steps):
        wt.run(x, out=y, stream=stream)
    e1.record(stream)
    barrier()
    ms = max_over_ranks(e0.elapsed_time(e1)) / args.prefill_steps
    qmm.device_status(stream)
    flops = 2.0 * m * n * k
    tflops = flops / (ms * 1e-3) / 1e12
    peak, kind = bf16_peak()
    per_gpu = 2.0 * m * wt.n * k / (ms * 1e-3) / 1e12
    wt.close()
    return {"workload": f"cfg3: nvfp4 prefill GEMM x [{m}, {k}] . W[{n}, {k}]^T, N-sharded over {world} GPU(s)",
            "metric": "TFLOP/s", "value": tflops, "ms_per_gemm": ms, "steps": args.prefill_steps,
            "l2": f"x {m * k * 2 / 1e6:.0f} MB + W {wt.n * k * 9 / 16 / 1e6:.0f} MB streamed per GEMM "
                  f"({'larger' if m * k * 2 > L2_BYTES else 'not larger'} than L2)",
            "roofline": {"bound": "tensor", "achieved": per_gpu, "peak": peak, "unit": "TFLOP/s",
                         "frac": per_gpu / peak, "peak_kind": kind, "kernel": "qmm_gemm_kernel<nvfp4>",
                         "note": "dense bf16 MMA peak: W is dequantised exactly to bf16 (parity); "
                                 "the block-scaled FP4 peak (~9 PF nominal) needs x quantised to FP4"}}


def bf16_peak() -> tuple[float, str]:
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            return float(json.load(f)["bf16_tflops"]), "measured burst"
    except Exception:
        return 1590.0, "fallback"


def cpu_baseline_sample(budget_s: float = 10.0) -> dict:
    oracle = _load("oracle", os.path.join(ROOT, "oracle", "oracle.py"))
    oracle.build()
    rng = np.random.default_rng(0)
    w = (rng.standard_normal((N_OUT, K_IN), dtype=np.float32) * 0.02).astype(np.float32)
    codes, scales = oracle.quantize(w, MODE)
    xs = {m: oracle.f32_to_bf16_bits(rng.standard_normal((m, K_IN), dtype=np.float32)) for m in M_SET}
    threads = oracle.max_threads()
    for m in M_SET:
        oracle.qmm_f32(xs[m], codes, scales, MODE, threads)
    reps, t0 = 0, time.perf_counter()
    while True:
        for m in M_SET:
            oracle.qmm_f32(xs[m], codes, scales, MODE, threads)
        reps += 1
        if time.perf_counter() - t0 >= budget_s:
            break
    dt = time.perf_counter() - t0
    return {"value": step_bytes(1) * reps / dt / 1e9, "unit": "GB/s", "cores": threads, "kind": "port",
            "sample": f"{reps} full steps of one weight copy (M=1..4) in {dt:.1f} s, fp32 accumulate"}


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true", help="skip the host-buffer pass (profiling runs)")
    ap.add_argument("--soak", type=float, default=1.0, help="seconds of load before warm-up (clock samples)")
    ap.add_argument("--no-prefill", action="store_true", help="skip the config-3 prefill GEMM measurement")
    ap.add_argument("--eager", action="store_true", help="time eager launches instead of CUDA-graph replays")
    ap.add_argument("--prefill-only", action="store_true", help="only the prefill GEMM (profiling runs)")
    ap.add_argument("--prefill-m", type=int, default=PREFILL["m"])
    ap.add_argument("--prefill-steps", type=int, default=5)
    ap.add_argument("--prefill-warmup", type=int, default=2)
    args = ap.parse_args()

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank)
        return

    import torch
    import torch.distributed as dist
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=120))
    qmm = _load("qmm", os.path.join(PKG, "qmm.py"))
    oracle = _load("oracle", os.path.join(ROOT, "oracle", "oracle.py"))

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(v: float) -> float:
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    if args.prefill_only:
        pf = prefill_measure(args, qmm, oracle, dev, world, rank, barrier, max_over_ranks)
        if rank == 0:
            print(json.dumps({"prefill": pf}), flush=True)
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()
        return

    # Weights: identical on every rank (seed 0), K-sharded by rank.
    rng = np.random.default_rng(0)
    w_full = (rng.standard_normal((N_OUT, K_IN), dtype=np.float32) * 0.02).astype(np.float32)
    codes, scales = oracle.quantize(w_full, MODE)
    del w_full
    k_shard = K_IN // world
    shard_bytes = algo_bytes(0, N_OUT, k_shard)
    copies = max(4, -(-4 * L2_BYTES // shard_bytes))
    weights = [qmm.QuantizedWeight(codes, scales, MODE, shard=(1, rank, world)) for _ in range(copies)]
    comm = None
    if world > 1:
        uid = [qmm.TPComm.unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        comm = qmm.TPComm(uid[0], world, rank, max(M_SET) * N_OUT)

    gx = torch.Generator(device="cpu").manual_seed(1)
    x_full = {m: torch.randn((m, K_IN), generator=gx, dtype=torch.float32).to(torch.bfloat16) for m in M_SET}
    x_dev = {m: x_full[m][:, rank * k_shard:(rank + 1) * k_shard].contiguous().to(dev) for m in M_SET}
    y_dev = {m: torch.empty((m, N_OUT), dtype=torch.bfloat16, device=dev) for m in M_SET}
    stream = torch.cuda.current_stream()

    def gemm(wt, m):
        cur = torch.cuda.current_stream()     # the capture stream inside a graph capture
        if comm is None:
            wt.run(x_dev[m], out=y_dev[m], stream=cur)
        else:
            comm.run_rowparallel(wt, x_dev[m], out=y_dev[m], stream=cur)

    def step():
        for wt in weights:
            for m in M_SET:
                gemm(wt, m)

    launches_per_gemm = 1 if comm is None else 2   # GEMV (+ fp32->bf16 after the all-reduce)

    # One step (and, for the kernel-alone timing, one pass per M) is replayed
    # as a CUDA graph, as a decode loop runs it: the device time then excludes
    # host launch gaps.  With world > 1 the graphs hold the NCCL all-reduces;
    # every rank uses graphs only if every rank captured them.
    def capture() -> dict:
        # Graphs live only in the returned dict (no other references), so
        # clearing it releases them - graphs holding NCCL calls must be gone
        # before the communicators are destroyed.
        out = {}
        cap = torch.cuda.Stream()
        cap.wait_stream(stream)
        with torch.cuda.stream(cap):
            step()                              # settles per-weight launch state outside capture
        torch.cuda.synchronize()
        out["step"] = torch.cuda.CUDAGraph()
        with torch.cuda.graph(out["step"], stream=cap):
            step()
        for m in M_SET:
            out[m] = torch.cuda.CUDAGraph()
            with torch.cuda.graph(out[m], stream=cap):
                for wt in weights:
                    gemm(wt, m)
        torch.cuda.synchronize()
        return out

    graphs = {}
    launch_mode = "eager"
    if not args.eager:
        try:
            graphs = capture()
            launch_mode = "cuda_graph"
        except Exception as exc:  # capture unsupported here: time eager launches
            graphs = {}
            print(f"bench: graph capture failed ({exc}); timing eager launches", file=sys.stderr)
        if world > 1:
            ok = torch.tensor([1.0 if graphs else 0.0], device=dev)
            dist.all_reduce(ok, op=dist.ReduceOp.MIN)
            if ok.item() < 1.0:
                graphs = {}
                launch_mode = "eager"

    def run_step():
        if graphs:
            graphs["step"].replay()
        else:
            step()

    sampler = ClockSampler(local)
    with sampler:
        # Sustained load so the clock samples see the same work as the timed region.
        barrier()
        t_soak = time.perf_counter()
        while time.perf_counter() - t_soak < args.soak:
            run_step()
            torch.cuda.synchronize()
        for _ in range(args.warmup):
            run_step()
        barrier()
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ev0.record(stream)
        for _ in range(args.steps):
            run_step()
        ev1.record(stream)
        barrier()
        ms = max_over_ranks(ev0.elapsed_time(ev1))

        # Kernel-alone timing of the dominant kernel (events on its stream):
        # one pass of `copies` launches per M, averaged per launch.
        k_ms = []
        for m in M_SET:
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            if graphs:
                graphs[m].replay()
            else:
                for wt in weights:
                    gemm(wt, m)
            b.record(stream)
            torch.cuda.synchronize()
            k_ms.extend([(m, a.elapsed_time(b) / copies)] * copies)

    # e2e: host buffers through the C ABI, copies inside the timed region.
    x_host = {m: x_full[m][:, rank * k_shard:(rank + 1) * k_shard].contiguous().pin_memory() for m in M_SET}
    y_host = {m: torch.empty((m, N_OUT), dtype=torch.bfloat16).pin_memory() for m in M_SET}

    def e2e_step():
        for wt in weights:
            for m in M_SET:
                x_dev[m].copy_(x_host[m], non_blocking=True)
                gemm(wt, m)
                y_host[m].copy_(y_dev[m], non_blocking=True)

    e_steps, e_ms = 0, float("nan")
    if not args.no_e2e:
        for _ in range(max(1, args.warmup)):
            e2e_step()
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e_steps = max(1, min(args.steps, 50))
        e0.record(stream)
        for _ in range(e_steps):
            e2e_step()
        e1.record(stream)
        barrier()
        e_ms = max_over_ranks(e0.elapsed_time(e1))

    total_bytes = step_bytes(copies) * args.steps
    value = total_bytes / (ms * 1e-3) / 1e9
    e2e_value = step_bytes(copies) * e_steps / (e_ms * 1e-3) / 1e9 if e_steps else None
    h2d = copies * sum(m * k_shard * 2 for m in M_SET)
    d2h = copies * sum(m * N_OUT * 2 for m in M_SET)

    # Roofline of the GEMV: per-launch algorithmic bytes of this rank's shard.
    per_launch_bytes = sum(algo_bytes(m, N_OUT, k_shard) for m, _ in k_ms)
    per_launch_ms = sum(t for _, t in k_ms)
    achieved = per_launch_bytes / (per_launch_ms * 1e-3) / 1e9
    peak, peak_kind = peaks()
    clocks = sampler.summary()

    torch.cuda.synchronize()
    graphs.clear()
    for wt in weights:
        wt.close()
    weights = []
    prefill = None
    if not args.no_prefill:
        prefill = prefill_measure(args, qmm, oracle, dev, world, rank, barrier, max_over_ranks)

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "nvfp4xbf16->f32acc",
            "data": "synthetic (seeded N(0,1) x, N(0,0.02^2) W quantized by the oracle's NVFP4 rule)",
            "config": dict(CONFIG, copies=copies, parallelism=f"tp{world} (K-shard)" if world > 1 else "none",
                           launch=launch_mode,
                           l2=f"inputs larger than L2: {copies} weight copies x {shard_bytes / 1e6:.1f} MB rotate"),
            "tflops": step_flops(copies) * args.steps / (ms * 1e-3) / 1e12,
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "peak_kind": peak_kind,
                         "traffic": GEMV_TRAFFIC_BYTES,
                         "kernel": "qmm_gemv_tc_kernel<nvfp4>", "per_m_us": {
                             str(m): 1e3 * statistics.mean(t for mm, t in k_ms if mm == m) for m in M_SET}},
            "e2e": {"value": e2e_value, "unit": "GB/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "steps": e_steps},
            "gpu_launches": args.steps * copies * len(M_SET) * launches_per_gemm,
            "clocks": clocks,
            "prefill": prefill,
        }
        if not args.no_cpu_baseline and world == 1:
            line["cpu_baseline"] = cpu_baseline_sample()
        print(json.dumps(line), flush=True)

    if comm is not None:
        comm.close()
    for wt in weights:
        wt.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
