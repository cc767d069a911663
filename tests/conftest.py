"""Shared test setup.

* Registers the ``gpu`` marker: tests that need a B200 are marked
  ``@pytest.mark.gpu``; everything else runs on the CPU.
* Puts the package directory (``mlx-runner_b200/``, which holds the ctypes
  binding ``qmm``) and ``oracle/`` (the CPU checker) on sys.path.
* Builds the oracle (gcc) and, where nvcc exists, the CUDA library, if they
  are missing.  On the GPU box both arrive prebuilt.
"""
from __future__ import annotations

import os
import shutil
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "mlx-runner_b200")
for p in (PKG, os.path.join(ROOT, "oracle")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


def _ensure_built():
    import oracle  # noqa: E402
    if not os.path.exists(oracle.LIB_PATH):
        oracle.build()
    lib_path = os.path.join(PKG, "_build", "libqmm_b200.so")
    if not os.path.exists(lib_path) and (shutil.which("nvcc") or os.path.exists("/usr/local/cuda/bin/nvcc")):
        import importlib.util
        spec = importlib.util.spec_from_file_location("qmm_build", os.path.join(PKG, "build.py"))
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
        mod.build()


_ensure_built()


@pytest.fixture(scope="session")
def golden():
    import json
    with open(os.path.join(ROOT, "tests", "golden", "golden.json")) as f:
        return json.load(f)


@pytest.fixture(scope="session")
def cuda_device():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("GPU test selected but no CUDA device is visible")
    return torch.device("cuda:0")
