"""Failure detection on the GPU without a GPU fault.

Every spin-wait in the library's kernels is bounded. The self-test kernel
waits on an mbarrier that nothing completes; with a 1 ms bound it must record
code 5 in the device error word and return (status 1005), leaving the context
usable for the next GEMM. The real tile kernels are run with their operand
feed switched off, so that their own waits run out the same way, and the
multi-GPU ring's flag kernel waits on a flag word nothing sets. No trap,
assert, bad address or endless loop is used.
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


# The real tile kernel with its operand feed switched off (gemm_selftest_stall):
# no A or B load is ever issued, so its UMMA issuer and epilogue waits run out
# after 1 ms; the kernel must record its code (1001-1003), unwind, free its
# TMEM and return, leave C untouched, and the next GEMM must be correct. beta is
# 0 inside the self test, so no C box is ever requested either.
@pytest.mark.parametrize("path,tile_n,shape", [
    (1, 128, (300, 520, 200)),       # 128 x 128 tile, TMA feed
    (1, 4, (512, 1024, 640)),        # 256 x 512 CTA-pair tile (the 8192^3 kernel)
    (1, 5, (300, 1000, 4104)),       # 128 x 256 tiles, K split over a cluster
    (7, 128, (300, 520, 200)),       # per-thread operand loads
], ids=["128x128", "pair256x512", "split-k", "lsu"])
def test_tile_kernel_bounded_waits_unwind(lib, cuda, path, tile_n, shape):
    import ctypes
    import torch
    from gpu_harness import Guarded
    m, n, k = shape
    ga = Guarded((m, k), cuda, fill=1.0)
    gb = Guarded((k, n), cuda, fill=1.0)
    gc = Guarded((m, n), cuda, fill=7.0)
    assert lib.gemm_launcher_status() == 0
    st = lib.gemm_selftest_stall(ga.tensor.data_ptr(), gb.tensor.data_ptr(), gc.tensor.data_ptr(),
                                 m, n, k, path, tile_n, 1000, None)
    assert st in (1001, 1002, 1003), st
    assert lib.gemm_launcher_status() == 0
    torch.cuda.synchronize()
    assert bool((gc.tensor == 7.0).all()) and gc.canaries_ok(), "C written by a stalled kernel"
    c, a, b, c0 = run(lib, cuda, m, n, k, 0.75, 0.5, path=path, tile_n=tile_n)
    assert verify(c, a, b, c0, 0.75, 0.5).passed


def test_peer_flag_wait_bounded(lib, cuda):
    """The copy-engine ring's flag kernel (gemm_peer_flags) on one GPU with a
    flag word that nothing sets: the bounded wait must record code 6 (status
    1006) and return; a second wait issued before the status is read must skip
    its wait (so a failed ring drains fast) instead of sitting out its own 5 s
    bound; after the read, a signal followed by a satisfied wait reports
    nothing. Only this process's own flag words are touched."""
    import time
    import torch

    flags = torch.zeros(2, dtype=torch.int32, device=cuda)
    stream = torch.cuda.current_stream().cuda_stream
    p0, p1 = flags.data_ptr(), flags.data_ptr() + 4
    assert lib.gemm_launcher_status() == 0
    t0 = time.monotonic()
    assert lib.gemm_peer_flags(None, 0, None, 0, p0, 1, None, 0, 1000, stream) == 0
    assert lib.gemm_peer_flags(None, 0, None, 0, p0, 1, None, 0, 5_000_000, stream) == 0
    torch.cuda.synchronize()
    assert time.monotonic() - t0 < 2.5
    assert lib.gemm_launcher_status() == 1006
    assert lib.gemm_launcher_status() == 0
    # signal word 1 to 7, then wait for word 1 >= 7 and word 0 >= 0: satisfied
    assert lib.gemm_peer_flags(p1, 7, None, 0, p1, 7, p0, 0, 1_000_000, stream) == 0
    torch.cuda.synchronize()
    assert lib.gemm_launcher_status() == 0
    assert flags.tolist() == [0, 7]
    c, a, b, c0 = run(lib, cuda, 256, 512, 192, 1.0, 0.5, fn="launcher")
    assert verify(c, a, b, c0, 1.0, 0.5).passed
