"""bench.py on the CPU: the algorithmic bytes and FLOPs its roofline fractions
divide by are the workload's own figures (benchmark configs 1-5: codes +
scales + x + y per call, 2*M*N*K per call, the config 5 stack's 25.6 G
weight elements), and the reference arm prints the contract's JSON line.
No GPU is used: the reference arm times the CPU restatement."""
import importlib.util
import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def bench():
    spec = importlib.util.spec_from_file_location("bench_under_test", os.path.join(ROOT, "bench.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_config2_bytes_and_flops(bench):
    # codes N*K/2 + scales N*K/16 = 50,135,040; x 2*M*K + y 2*M*N = 45,056 per row.
    for m in (1, 2, 3, 4):
        assert bench.algo_bytes(m) == 50_135_040 + 45_056 * m
    assert bench.step_bytes(1) == sum(50_135_040 + 45_056 * m for m in (1, 2, 3, 4))
    assert bench.step_flops(1) == pytest.approx(1.7826e8 * 10, rel=1e-4)


def test_config1_bytes():
    n, k = 17408, 5120
    assert n * k + n * k // 32 + 2 * k + 2 * n == 91_959_296


def test_config4_flops(bench):
    t = 32768
    flops = {name: 2.0 * t * n * k for name, n, k in bench.GDN_PREFILL}
    assert flops["in_proj_qkvz"] == pytest.approx(5.4976e12, rel=1e-4)
    assert flops["in_proj_ba"] == pytest.approx(3.2212e10, rel=1e-4)
    assert flops["out_proj"] == pytest.approx(2.0616e12, rel=1e-4)
    assert flops["gate_up"] == pytest.approx(1.16823e13, rel=1e-4)
    assert flops["down"] == pytest.approx(5.8412e12, rel=1e-4)
    assert sum(flops.values()) == pytest.approx(2.51148e13, rel=1e-4)


def test_config5_stack_elements(bench):
    gdn = sum(n * k for _, n, k in bench.GDN_LINEARS)
    attn = sum(n * k for _, n, k in bench.ATTN_LINEARS)
    mlp = 3 * bench.MLP_FFN * bench.HIDDEN
    elems = 48 * (gdn + mlp) + 16 * (attn + mlp) + bench.VOCAB * bench.HIDDEN
    assert elems == 25_621_954_560
    assert elems * 9 // 16 == 14_412_349_440


def test_reference_arm_prints_the_contract_line():
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--steps", "1",
                        "--warmup", "0"], capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    line = json.loads(r.stdout.strip().splitlines()[-1])
    for key in ("impl", "metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in line, key
    assert line["impl"] == "reference" and line["unit"] == "GB/s" and line["value"] > 0
    assert line["cpu_baseline"]["kind"] == "port" and line["cpu_baseline"]["cores"] >= 1
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["e2e"]["value"] == line["value"]
    assert line["config"]["workload"].startswith("cfg2")


def test_both_arms_print_one_config(bench):
    """The GPU arm and the reference arm print the same `config` for the same
    world size (run details live in `setup`), so the driver's comparison of
    the two lines sees one workload."""
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--steps", "1",
                        "--warmup", "0", "--gpus", "2"], capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    line = json.loads(r.stdout.strip().splitlines()[-1])
    assert line["config"] == bench.config_for(2)
    assert bench.config_for(1)["parallelism"] == "none"
    assert "copies" not in line["config"] and "launch" not in line["config"]
