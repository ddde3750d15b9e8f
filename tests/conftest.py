"""Shared test set-up.

Markers: `gpu` tests need a B200 (sm_100a) and run the CUDA library through its
C ABI; everything else runs on the CPU. The repository root and the package
directory are put on sys.path so tests import `gemm_b200` (the ctypes binding)
and `oracle.oracle` (the CPU checker).
"""
import os
import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent
PKG = REPO / "gemm-project_b200"
for p in (str(REPO), str(PKG)):
    if p not in sys.path:
        sys.path.insert(0, p)

# The launch log is the reference's stdout line; keep test output readable.
os.environ.setdefault("GEMM_LAUNCH_LOG", "0")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 GPU (sm_100a)")
    config.addinivalue_line("markers", "multigpu: needs two or more B200 GPUs (run on its own)")


@pytest.fixture(scope="session")
def lib():
    """The built library (built on demand; GPU tests never fall back to CPU)."""
    sys.path.insert(0, str(PKG))
    import build as pkg_build  # gemm-project_b200/build.py
    pkg_build.build()
    import gemm_b200
    return gemm_b200.load()


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("GPU test collected on a machine without CUDA: run with -m 'not gpu'")
    major, minor = torch.cuda.get_device_capability()
    if (major, minor) != (10, 0):
        pytest.fail(f"this library targets sm_100a (B200); found sm_{major}{minor}")
    torch.backends.cuda.matmul.allow_tf32 = False
    return torch.device("cuda:0")
