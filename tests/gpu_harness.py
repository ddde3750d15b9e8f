"""GPU-side harness shared by the `gpu` tests.

Mirrors the reference's correctness harness (tests/test_gemm.py:26-45):
guarded device buffers with 64 halves of canary 123.0 on each side, a
NaN-filled C when beta == 0 (proves C is not read), synchronize / call /
synchronize around the C-ABI call, inputs checked bit-unchanged. Pointers can
be offset by whole halves inside the guarded allocation to produce the
reference's misaligned cases (tests/test_gemm.py:140-162).

Results are compared with the CPU oracle (oracle/oracle.py). For outputs too
large to evaluate on the CPU in seconds, a seeded sample of rows is checked
against the CPU oracle and the whole matrix against torch's FP32 CUDA matmul
with TF32 off, which is the reference's own check (tests/test_gemm.py:91,
191-193).
"""
from __future__ import annotations

import ctypes

import torch

from oracle import oracle

GUARD = 64
CANARY = 123.0
FULL_CPU_LIMIT = 4e9  # M*N*K up to which the whole result is checked on the CPU


class Guarded:
    """A tensor of `shape` placed at element `offset` inside a canary-filled buffer."""

    def __init__(self, shape, device, fill=float("nan"), offset=GUARD):
        numel = 1
        for d in shape:
            numel *= d
        self.offset = offset
        self.buffer = torch.full((numel + offset + GUARD,), CANARY, device=device, dtype=torch.float16)
        self.tensor = self.buffer[offset:offset + numel].view(shape)
        if numel:
            self.tensor.fill_(fill)

    def canaries_ok(self) -> bool:
        b = self.buffer
        return bool((b[:self.offset] == CANARY).all() and (b[b.numel() - GUARD:] == CANARY).all())


def call(lib, fn_name, a, b, c, m, n, k, alpha, beta, *extra):
    torch.cuda.synchronize()
    fn = getattr(lib, fn_name)
    rc = fn(a.data_ptr(), b.data_ptr(), c.data_ptr(), m, n, k, ctypes.c_float(alpha),
            ctypes.c_float(beta), *extra)
    torch.cuda.synchronize()
    return rc


def run(lib, device, m, n, k, alpha=1.0, beta=0.0, dist="uniform", seed=0, path=0, tile_n=0,
        offsets=(0, 0, 0), c_init=None, fn="ex"):
    """Run one GEMM through the C ABI on guarded buffers; return (c_out, a, b, c0, guards).
    offsets: extra half-element offsets of A, B, C (1 = the reference's 2-byte misalignment)."""
    a_cpu, b_cpu, c_cpu = oracle.make_inputs(m, n, k, dist, seed)
    if c_init is not None:
        c_cpu = torch.full((m, n), c_init, dtype=torch.float16)
    ga = Guarded((m, k), device, offset=GUARD + offsets[0])
    gb = Guarded((k, n), device, offset=GUARD + offsets[1])
    c_fill = float("nan") if beta == 0.0 else 0.0
    gc = Guarded((m, n), device, fill=c_fill, offset=GUARD + offsets[2])
    if m * k:
        ga.tensor.copy_(a_cpu)
    if k * n:
        gb.tensor.copy_(b_cpu)
    if beta != 0.0 and m * n:
        gc.tensor.copy_(c_cpu)
    if fn == "launcher":
        call(lib, "gemm_launcher", ga.tensor, gb.tensor, gc.tensor, m, n, k, alpha, beta)
    elif fn == "cublas":
        call(lib, "gemm_cublas", ga.tensor, gb.tensor, gc.tensor, m, n, k, alpha, beta)
    else:
        rc = call(lib, "gemm_launcher_ex", ga.tensor, gb.tensor, gc.tensor, m, n, k, alpha, beta,
                  None, path, tile_n)
        assert rc == 0, f"gemm_launcher_ex refused path={path} tile_n={tile_n} for {(m, n, k)}"
    status = lib.gemm_launcher_status()
    assert status == 0, f"library status {status} after {(m, n, k)}"
    assert ga.canaries_ok() and gb.canaries_ok() and gc.canaries_ok(), "guard canary overwritten"
    if m * k:
        assert torch.equal(ga.tensor.cpu(), a_cpu), "A modified"
    if k * n:
        assert torch.equal(gb.tensor.cpu(), b_cpu), "B modified"
    return gc.tensor, a_cpu, b_cpu, c_cpu


def verify(c_dev, a, b, c0, alpha, beta, seed=0, sample_rows=256):
    """Check a GPU result against the CPU oracle (whole matrix when cheap,
    otherwise a seeded row sample plus the whole matrix against torch FP32 CUDA)."""
    m, k = a.shape
    n = b.shape[1]
    if m * n * k <= FULL_CPU_LIMIT or m <= sample_rows:
        ref = oracle.reference_fp32(a, b, c0, alpha, beta)
        return oracle.check(c_dev, ref)
    g = torch.Generator().manual_seed(seed + 7)
    rows = torch.randperm(m, generator=g)[:sample_rows].sort().values
    ref_rows = oracle.reference_fp32(a[rows], b, c0[rows], alpha, beta)
    chk_rows = oracle.check(c_dev[rows.to(c_dev.device)], ref_rows)
    if not chk_rows.passed:
        return chk_rows
    ref_full = alpha * (a.to(c_dev.device).float() @ b.to(c_dev.device).float())
    if beta != 0.0:
        ref_full += beta * c0.to(c_dev.device).float()
    return oracle.check(c_dev, ref_full)
