"""CPU oracle and checkers for the FP16 GEMM path.

TEST INFRASTRUCTURE ONLY. Only tests/, __graft_entry__.smoke() and bench.py's
CPU-baseline leg may import this module, and only as the checker (or, in the
baseline leg, as the timed CPU reference). The shipped library never calls it.

Two restatements of the reference's arithmetic (FP16 operands, FP32
accumulation, epilogue alpha*acc + beta*C, C not read when beta == 0):

* `reference_fp32` evaluates exactly the formula the reference's tests use,
  `alpha*(a.float()@b.float()) + beta*c.float()` (tests/test_gemm.py:91,130,156),
  with torch on the CPU in FP32, unrounded. Fast enough for the full configs
  (multi-threaded BLAS sgemm).
* `gemm_oracle.c` (loaded through ctypes, `c_gemm` / `c_unrounded`) is a
  plain-C k-ordered fmaf loop with its own binary16 conversions, for small
  cases and for pinning the torch path.

Checkers implement both tolerances: the reference's own pass rule
(|c-ref| <= 0.002 + 0.002|ref|, all finite; tests/test_gemm.py:11,48-61) and the
north-star rule (max |c-ref| <= 1e-2 (1+|ref|) and relative Frobenius error
<= 1e-3).

Input generators follow one convention for every config: a CPU
torch.Generator seeded with the config's seed draws A, then B, then C, in FP32,
rounded to half. Uniform[-1,1) is rand*2-1; Normal(0, 1/sqrt(K)) is randn/sqrt(K).
"""
from __future__ import annotations

import ctypes
import math
import os
import subprocess
from dataclasses import dataclass
from pathlib import Path

import numpy as np
import torch

ORACLE_DIR = Path(__file__).resolve().parent
C_LIB_PATH = ORACLE_DIR / "_build" / "liboracle.so"
REF_LIB_PATH = ORACLE_DIR / "_ref" / "libgemm_ref.so"

REF_ATOL = REF_RTOL = 0.002          # tests/test_gemm.py:11
NS_ABS = 1e-2                        # north star: max |C-ref| <= 1e-2 (1 + |ref|)
NS_FROB = 1e-3                       # north star: relative Frobenius error <= 1e-3

_clib = None


def build_c(force: bool = False) -> Path:
    if force or not C_LIB_PATH.exists() or (
            C_LIB_PATH.stat().st_mtime < (ORACLE_DIR / "gemm_oracle.c").stat().st_mtime):
        subprocess.run(["make", "-s", "-C", str(ORACLE_DIR), "all"], check=True)
    return C_LIB_PATH


def clib() -> ctypes.CDLL:
    global _clib
    if _clib is None:
        lib = ctypes.CDLL(str(build_c()))
        P = ctypes.c_void_p
        lib.oracle_gemm_f32.argtypes = [P, ctypes.c_long, P, ctypes.c_long, P, ctypes.c_long,
                                        ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_float,
                                        ctypes.c_float]
        lib.oracle_gemm_f32_unrounded.argtypes = [P, P, P, P, ctypes.c_int, ctypes.c_int,
                                                  ctypes.c_int, ctypes.c_float, ctypes.c_float]
        lib.oracle_audit_f64.argtypes = [P, P, P, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                         ctypes.c_double, ctypes.c_double, P, P, ctypes.c_int, P]
        lib.oracle_half_to_float.argtypes = [ctypes.c_uint16]
        lib.oracle_half_to_float.restype = ctypes.c_float
        lib.oracle_float_to_half.argtypes = [ctypes.c_float]
        lib.oracle_float_to_half.restype = ctypes.c_uint16
        lib.oracle_halves_to_floats.argtypes = [P, P, ctypes.c_long]
        lib.oracle_floats_to_halves.argtypes = [P, P, ctypes.c_long]
        _clib = lib
    return _clib


def _u16(t: torch.Tensor) -> np.ndarray:
    return np.ascontiguousarray(t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16))


# ---------------------------------------------------------------------------
# References
# ---------------------------------------------------------------------------
def reference_fp32(a: torch.Tensor, b: torch.Tensor, c: torch.Tensor | None, alpha: float,
                   beta: float) -> torch.Tensor:
    """Unrounded FP32 alpha*(A@B) + beta*C on the CPU (C ignored when beta == 0)."""
    a32 = a.detach().cpu().float()
    b32 = b.detach().cpu().float()
    out = alpha * (a32 @ b32)
    if beta != 0.0 and c is not None:
        out = out + beta * c.detach().cpu().float()
    return out


def c_gemm(a: torch.Tensor, b: torch.Tensor, c: torch.Tensor, alpha: float, beta: float) -> torch.Tensor:
    """The C restatement: returns the rounded FP16 result as a CPU tensor."""
    m, k = a.shape
    n = b.shape[1]
    A, B = _u16(a), _u16(b)
    C = _u16(c).copy()
    clib().oracle_gemm_f32(A.ctypes.data, k, B.ctypes.data, n, C.ctypes.data, n, m, n, k,
                           float(alpha), float(beta))
    return torch.from_numpy(C.view(np.int16).copy()).view(torch.float16).reshape(m, n)


def c_unrounded(a, b, c, alpha, beta) -> torch.Tensor:
    m, k = a.shape
    n = b.shape[1]
    A, B, C = _u16(a), _u16(b), _u16(c)
    out = np.empty((m, n), dtype=np.float32)
    clib().oracle_gemm_f32_unrounded(A.ctypes.data, B.ctypes.data, C.ctypes.data, out.ctypes.data,
                                     m, n, k, float(alpha), float(beta))
    return torch.from_numpy(out)


def audit_f64(a, b, c0, alpha, beta, rows, cols) -> np.ndarray:
    m, k = a.shape
    n = b.shape[1]
    A, B, C = _u16(a), _u16(b), _u16(c0)
    r = np.ascontiguousarray(rows, dtype=np.int32)
    cc = np.ascontiguousarray(cols, dtype=np.int32)
    out = np.empty(len(r), dtype=np.float64)
    clib().oracle_audit_f64(A.ctypes.data, B.ctypes.data, C.ctypes.data, m, n, k, float(alpha),
                            float(beta), r.ctypes.data, cc.ctypes.data, len(r), out.ctypes.data)
    return out


# ---------------------------------------------------------------------------
# Checkers
# ---------------------------------------------------------------------------
@dataclass
class Check:
    passed: bool
    ref_pass: bool          # reference rule: finite and |c-ref| <= 0.002 + 0.002|ref|
    ns_pass: bool           # north-star rule
    finite: bool
    violations: int
    max_abs_error: float
    max_scaled_error: float  # max |c-ref| / (1+|ref|)
    rel_frobenius: float

    def __str__(self) -> str:
        return (f"pass={self.passed} ref_rule={self.ref_pass} ns_rule={self.ns_pass} "
                f"finite={self.finite} violations={self.violations} max_abs={self.max_abs_error:.3g} "
                f"max_scaled={self.max_scaled_error:.3g} rel_frob={self.rel_frobenius:.3g}")


def check(c: torch.Tensor, ref: torch.Tensor, rule: str = "both") -> Check:
    """Compare an FP16 result with the unrounded FP32 reference."""
    c32 = c.detach().cpu().float()
    ref = ref.detach().cpu().float()
    if c32.numel() == 0:
        return Check(True, True, True, True, 0, 0.0, 0.0, 0.0)
    finite = bool(torch.isfinite(c32).all())
    diff = (c32 - ref).abs()
    violations = int((diff > REF_ATOL + REF_RTOL * ref.abs()).sum())
    max_abs = float(diff.max())
    max_scaled = float((diff / (1.0 + ref.abs())).max())
    denom = float(ref.double().square().sum().sqrt())
    rel = float(diff.double().square().sum().sqrt()) / max(denom, 1e-30)
    ref_pass = finite and violations == 0
    ns_pass = finite and max_scaled <= NS_ABS and rel <= NS_FROB
    passed = {"both": ref_pass and ns_pass, "ref": ref_pass, "ns": ns_pass}[rule]
    return Check(passed, ref_pass, ns_pass, finite, violations, max_abs, max_scaled, rel)


# ---------------------------------------------------------------------------
# Input generators for the BASELINE configs
# ---------------------------------------------------------------------------
def uniform(g: torch.Generator, shape) -> torch.Tensor:
    return (torch.rand(shape, generator=g) * 2 - 1).half()


def normal(g: torch.Generator, shape, k: int) -> torch.Tensor:
    return (torch.randn(shape, generator=g) / math.sqrt(k)).half()


def make_inputs(m: int, n: int, k: int, dist: str, seed: int = 0, c_dist: str = "uniform"):
    """A, B, C as CPU half tensors drawn in that order from one seeded generator.
    dist: 'uniform' (U[-1,1)) or 'normal' (N(0, 1/sqrt(K))) for A and B;
    c_dist: 'uniform' or 'zero'."""
    g = torch.Generator("cpu").manual_seed(seed)
    if dist == "uniform":
        a, b = uniform(g, (m, k)), uniform(g, (k, n))
    elif dist == "normal":
        a, b = normal(g, (m, k), max(k, 1)), normal(g, (k, n), max(k, 1))
    else:
        raise ValueError(dist)
    c = uniform(g, (m, n)) if c_dist == "uniform" else torch.zeros((m, n), dtype=torch.float16)
    return a, b, c


# The BASELINE.json configs (the bench workload and the parity cases).
CONFIGS = {
    "square1024": dict(m=1024, n=1024, k=1024, dist="uniform", c_dist="uniform", alpha=1.0, beta=0.0),
    "square4096": dict(m=4096, n=4096, k=4096, dist="normal", c_dist="uniform", alpha=1.0, beta=0.5),
    "square8192": dict(m=8192, n=8192, k=8192, dist="normal", c_dist="uniform", alpha=1.0, beta=0.5),
    "gemv_m1": dict(m=1, n=28672, k=8192, dist="uniform", c_dist="uniform", alpha=1.0, beta=0.0),
    "gemv_n1": dict(m=28672, n=1, k=8192, dist="uniform", c_dist="uniform", alpha=1.0, beta=0.0),
    "odd_1023": dict(m=1023, n=2049, k=777, dist="uniform", c_dist="uniform", alpha=0.75, beta=-0.25,
                     offset=1),
    "odd_3": dict(m=3, n=5000, k=4097, dist="uniform", c_dist="uniform", alpha=0.75, beta=-0.25,
                  offset=1),
    "sharded32768": dict(m=32768, n=32768, k=16384, dist="normal", c_dist="zero", alpha=1.0, beta=0.0),
}


def cpu_threads() -> int:
    return len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)
