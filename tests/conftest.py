"""Shared fixtures.  GPU tests carry @pytest.mark.gpu and run on a B200;
everything else runs on the CPU (the oracle, host logic, the C ABI's
host-side checks, gloo multi-process tests)."""
from __future__ import annotations

import importlib
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (ROOT, os.path.join(ROOT, "oracle"), os.path.join(ROOT, "tests", "golden")):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = os.path.join(ROOT, "tests", "golden", "ref_int8kv.npz")


def _ensure_built() -> None:
    """Builds the oracle and the native library in-tree when they are absent
    (a fresh checkout); on the GPU box the prebuilt files travel with the tree."""
    if not os.path.exists(os.path.join(ROOT, "oracle", "liboracle_int8kv.so")):
        subprocess.run(["make", "-C", os.path.join(ROOT, "oracle"), os.path.join(ROOT, "oracle", "liboracle_int8kv.so")],
                       check=True, capture_output=True)
    if not os.path.exists(os.path.join(ROOT, "pop2-bezier_b200", "libpp_b200.so")):
        subprocess.run([sys.executable, os.path.join(ROOT, "pop2-bezier_b200", "build_native.py")], check=True,
                       capture_output=True)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an NVIDIA B200 (sm_100a)")
    _ensure_built()


@pytest.fixture(scope="session")
def pp():
    return importlib.import_module("pop2-bezier_b200")


@pytest.fixture(scope="session")
def oracle():
    import oracle as o  # oracle/oracle.py

    return o


@pytest.fixture(scope="session")
def golden():
    import numpy as np

    return np.load(GOLDEN)


@pytest.fixture(scope="session")
def cuda():
    import torch

    if not torch.cuda.is_available():
        raise RuntimeError("GPU test collected without a CUDA device")
    major, minor = torch.cuda.get_device_capability(0)
    if (major, minor) != (10, 0):
        raise RuntimeError(f"GPU tests target sm_100 (B200); device is sm_{major}{minor}")
    return torch.device("cuda", 0)
