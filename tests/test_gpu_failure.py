"""Failure detection on the GPU without a GPU fault.

Every spin-wait in the library's kernels is bounded. The self-test kernel
waits on an mbarrier that nothing completes; with a 1 ms bound it must record
code 5 in the device error word and return (status 1005), leaving the context
usable for the next GEMM. No trap, assert, bad address or endless loop is used.
"""
import pytest

from gpu_harness import run, verify

pytestmark = pytest.mark.gpu


def test_bounded_wait_reports_instead_of_hanging(lib, cuda):
    assert lib.gemm_launcher_status() == 0
    assert lib.gemm_selftest_wait_timeout(1000, None) == 1005
    # status is cleared by the read
    assert lib.gemm_launcher_status() == 0
    # the context is still healthy: a normal GEMM runs and is correct
    c, a, b, c0 = run(lib, cuda, 256, 512, 192, 1.0, 0.5, fn="launcher")
    assert verify(c, a, b, c0, 1.0, 0.5).passed


def test_normal_work_reports_no_timeout(lib, cuda):
    for shape in [(1024, 1024, 1024), (1, 4096, 4096), (4096, 1, 4096)]:
        run(lib, cuda, *shape, fn="launcher")
    assert lib.gemm_launcher_status() == 0
