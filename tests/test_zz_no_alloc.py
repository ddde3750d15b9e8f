"""gemm_launcher_noalloc against gemm_launcher_stream (needs a B200).

Some callers cannot let a library allocate device memory: serving processes
that reserve nearly all HBM for their own pools up front, and frameworks whose
allocator must account for every device byte. gemm_launcher_noalloc serves
them: where gemm_launcher_stream's plan for a call would take repack scratch
(a misaligned or odd-pitched A or B on a problem large enough for the
tensor-core path to repack it), it uses a fixed 32 MiB device buffer compiled
into the library instead of cudaMallocAsync; every other call runs exactly as
gemm_launcher_stream, whose other kernels allocate nothing.

The comparison tests call it through the C ABI twice in a row on the same
inputs, with the repack feed forced (GEMM_LSU=-1, so that the fixed buffer is
used on every misaligned shape) and with the default feed, and compare each
result with the allocating entry point's under the same tolerance rules as
every other parity test. A separate test runs in a fresh process, checks from
the launch log that the repack kernels wrote into the fixed buffer, and checks
that free device memory does not move across calls on shapes that process has
never run. A shape whose repack exceeds 32 MiB must be refused before anything
is launched.

The file is named so that pytest collects it last.
"""
import ctypes
import os
import subprocess
import sys
from pathlib import Path

import pytest
import torch

from gpu_harness import Guarded
from oracle import oracle

pytestmark = pytest.mark.gpu

REPO = Path(__file__).resolve().parent.parent

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


@pytest.mark.parametrize("feed", ["-1", "0"], ids=["repack-feed", "default-feed"])
@pytest.mark.parametrize("case", CASES, ids=str)
def test_noalloc_matches_allocating_entry_point(lib, cuda, monkeypatch, case, feed):
    monkeypatch.setenv("GEMM_LSU", feed)
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
        # the same plan (tile, K split) as the allocating entry point: identical bits
        assert torch.equal(got, expected), f"noalloc differs in bits from the allocating path {case}"
        assert oracle.check(got, ref32).passed
    assert torch.equal(ga.tensor.cpu(), a) and torch.equal(gb.tensor.cpu(), b)


_FRESH_PROCESS = r"""
import ctypes, sys
sys.path[:0] = [sys.argv[1], sys.argv[1] + "/gemm-project_b200"]
import torch
import gemm_b200
lib = gemm_b200.load()
dev = torch.device("cuda:0")
f = ctypes.c_float

def make(m, n, k):
    # one half past each allocation's base: not 16-byte aligned
    return [torch.full((r * c + 1,), 0.5, dtype=torch.float16, device=dev)[1:]
            for r, c in ((m, k), (k, n), (m, n))]

def call(m, n, k, bufs):
    a, b, c = bufs
    rc = lib.gemm_launcher_noalloc(a.data_ptr(), b.data_ptr(), c.data_ptr(), m, n, k,
                                   f(1.0), f(0.0), None)
    torch.cuda.synchronize()
    assert rc == 0 and lib.gemm_launcher_status() == 0, rc

shapes = [(300, 520, 1001), (2000, 2056, 3001), (1500, 3000, 2049)]
bufs = [make(*s) for s in shapes]         # every input allocated before the measurement
torch.cuda.synchronize()
call(*shapes[0], bufs[0])                 # first call: library set-up on this device
free0 = torch.cuda.mem_get_info()[0]
for s, bb in zip(shapes[1:], bufs[1:]):   # shapes this process has never run
    call(*s, bb)
    call(*s, bb)
free1 = torch.cuda.mem_get_info()[0]
print(f"FREE_DELTA {free0 - free1}", flush=True)
"""


def test_noalloc_uses_fixed_buffer_in_fresh_process(lib, cuda):
    """Repack shapes never seen by the process: the launch log shows the repack
    kernels writing into the fixed buffer, and free device memory does not move
    across the calls (modules load eagerly in that process, so a kernel's first
    launch takes no memory either)."""
    env = dict(os.environ, GEMM_LSU="-1", GEMM_LAUNCH_LOG="1", CUDA_MODULE_LOADING="EAGER")
    proc = subprocess.run([sys.executable, "-c", _FRESH_PROCESS, str(REPO)], capture_output=True,
                          text=True, env=env, timeout=300)
    assert proc.returncode == 0, proc.stdout[-3000:] + proc.stderr[-3000:]
    out = proc.stdout
    assert "pack_rows_kernel<A,B,static>: M=2000 N=2056 K=3001" in out, out[-3000:]
    assert "pack_rows_kernel<A,B,static>: M=1500 N=3000 K=2049" in out, out[-3000:]
    assert "pack_rows_kernel<A,B>:" not in out and "pack_rows_kernel<A>:" not in out
    delta = [int(ln.split()[1]) for ln in out.splitlines() if ln.startswith("FREE_DELTA")]
    assert delta == [0], out[-2000:]


def test_noalloc_refuses_repack_beyond_its_buffer(lib, cuda, monkeypatch, capfd):
    monkeypatch.setenv("GEMM_LSU", "-1")
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
