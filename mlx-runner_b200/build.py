"""Build libqmm_b200.so (the C-ABI library) in-tree with nvcc for sm_100a.

    python mlx-runner_b200/build.py [--force]

Every .cu / .cpp under csrc/ is compiled with
``-gencode arch=compute_100a,code=sm_100a -O3 -lineinfo`` into _build/ and
linked into _build/libqmm_b200.so (CUDA runtime linked statically, NCCL
loaded at run time).  Objects are rebuilt when their source, or any header,
is newer than the object.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(BUILD, "libqmm_b200.so")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def nccl_include() -> list[str]:
    dirs = []
    try:
        import nvidia.nccl  # type: ignore
        dirs.append(os.path.join(list(nvidia.nccl.__path__)[0], "include"))
    except Exception:
        pass
    dirs.append("/usr/include")
    return [f"-I{d}" for d in dirs if os.path.exists(os.path.join(d, "nccl.h"))][:1]


def flags() -> list[str]:
    return ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-O3,-Wall",
                   "--expt-relaxed-constexpr", f"-I{os.path.join(ROOT, 'include')}", f"-I{CSRC}"] + nccl_include()


def build(force: bool = False, verbose: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cpp")))
    headers = glob.glob(os.path.join(CSRC, "*.h")) + glob.glob(os.path.join(CSRC, "*.cuh")) + \
        glob.glob(os.path.join(ROOT, "include", "*.h"))
    newest_header = max((os.path.getmtime(h) for h in headers), default=0)
    nv = nvcc()
    jobs = []
    objs = []
    for s in srcs:
        o = os.path.join(BUILD, os.path.basename(s) + ".o")
        objs.append(o)
        if force or not os.path.exists(o) or os.path.getmtime(o) < max(os.path.getmtime(s), newest_header):
            cmd = [nv, "-c", s, "-o", o] + flags()
            if s.endswith(".cpp"):
                cmd = [nv, "-x", "cu", "-c", s, "-o", o] + flags()
            jobs.append(cmd)

    def run(cmd):
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed:\n{' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
        if verbose and (r.stdout or r.stderr):
            print(r.stdout, r.stderr, flush=True)

    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 2)) as ex:
        list(ex.map(run, jobs))
    if jobs or force or not os.path.exists(LIB):
        tmp = LIB + f".tmp{os.getpid()}"
        run([nv, "-shared", "-o", tmp] + objs + ARCH + ["-ldl"])
        os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force, verbose=a.verbose))
    sys.exit(0)
