"""gemm_launcher_noalloc against gemm_launcher_stream (needs a B200).

Some callers cannot let a library allocate device memory: serving processes
that reserve nearly all HBM for their own pools up front, and frameworks whose
allocator must account for every device byte. gemm_launcher_noalloc serves
them: where the tensor-core path has to repack a misaligned or odd-pitched A
or B, it uses a fixed 32 MiB device buffer compiled into the library instead
of cudaMallocAsync. These tests call it through the C ABI on the shapes that
need that repack (and on ones that do not), twice in a row on the same
inputs, and compare each result with the allocating entry point's result
under the same tolerance rules as every other parity test. A shape whose
repack exceeds 32 MiB must be refused before anything is launched.

The file is named so that pytest collects it last.
"""
import ctypes

import pytest
import torch

from gpu_harness import Guarded
from oracle import oracle

pytestmark = pytest.mark.gpu

CASES = [
    # (M, N, K, alpha, beta, offset of A/B/C in halves)
    (1023, 2049, 777, 0.75, -0.25, 1),   # both A and B repacked (odd K, odd N, misaligned)
    (129, 257, 65, 1.0, 0.5, 1),         # repack with tile edges on M, N and K
    (300, 1024, 544, 0.7, -0.3, 1),      # aligned pitches, misaligned bases
    (512, 1000, 1001, 1.0, 0.0, 0),      # odd K only: A repacked
    (256, 1024, 1024, 1.0, 0.5, 0),      # no repack needed
    (3, 5000, 4097, 0.75, -0.25, 1),     # skinny kernel (no scratch)
]


def _setup(cuda, m, n, k, beta, off, seed):
    a, b, c0 = oracle.make_inputs(m, n, k, "uniform", seed=seed)
    ga = Guarded((m, k), cuda, offset=64 + off)
    gb = Guarded((k, n), cuda, offset=64 + off)
    ga.tensor.copy_(a)
    gb.tensor.copy_(b)
    return a, b, c0, ga, gb


def _run(lib, fn, ga, gb, c0, m, n, k, alpha, beta, off, cuda):
    gc = Guarded((m, n), cuda, fill=float("nan") if beta == 0 else 0.0, offset=64 + off)
    if beta != 0:
        gc.tensor.copy_(c0)
    torch.cuda.synchronize()
    rc = fn(ga.tensor.data_ptr(), gb.tensor.data_ptr(), gc.tensor.data_ptr(), m, n, k,
            ctypes.c_float(alpha), ctypes.c_float(beta), None)
    torch.cuda.synchronize()
    assert lib.gemm_launcher_status() == 0
    assert gc.canaries_ok()
    return rc, gc.tensor.cpu()


@pytest.mark.parametrize("case", CASES, ids=str)
def test_noalloc_matches_allocating_entry_point(lib, cuda, case):
    m, n, k, alpha, beta, off = case
    a, b, c0, ga, gb = _setup(cuda, m, n, k, beta, off, seed=m + n + k)
    rc_ref, expected = _run(lib, lambda *x: lib.gemm_launcher_stream(*x) or 0, ga, gb, c0, m, n, k,
                            alpha, beta, off, cuda)
    ref32 = oracle.reference_fp32(a, b, c0, alpha, beta)
    assert oracle.check(expected, ref32).passed
    for _ in range(2):  # two calls in a row share (and reuse) the static buffer
        rc, got = _run(lib, lib.gemm_launcher_noalloc, ga, gb, c0, m, n, k, alpha, beta, off, cuda)
        assert rc == 0
        chk = oracle.check(got, expected.float())
        assert chk.passed, f"noalloc vs allocating entry point {case}: {chk}"
        assert oracle.check(got, ref32).passed
    assert torch.equal(ga.tensor.cpu(), a) and torch.equal(gb.tensor.cpu(), b)


def test_noalloc_refuses_repack_beyond_its_buffer(lib, cuda, capfd):
    # odd K: A would be repacked to 4200 x 4104 halves = 34.5 MB > 32 MiB
    m, n, k = 4200, 256, 4097
    ga = Guarded((m, k), cuda, fill=1.0)
    gb = Guarded((k, n), cuda, fill=1.0)
    gc = Guarded((m, n), cuda, fill=5.0)
    torch.cuda.synchronize()
    rc = lib.gemm_launcher_noalloc(ga.tensor.data_ptr(), gb.tensor.data_ptr(), gc.tensor.data_ptr(),
                                   m, n, k, ctypes.c_float(1.0), ctypes.c_float(0.0), None)
    torch.cuda.synchronize()
    assert rc == -2
    assert "repack scratch" in capfd.readouterr().err
    assert bool((gc.tensor == 5.0).all()) and gc.canaries_ok()
    assert lib.gemm_launcher_status() == 0
