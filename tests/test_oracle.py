"""Pin the CPU oracle before trusting it (no GPU needed).

* binary16 conversions of the C restatement against numpy's IEEE float16,
  exhaustively for half -> float and on edge/random values for float -> half;
* both oracles (torch FP32 formula of the reference's tests and the C k-ordered
  loop) against the committed FP64 golden fixtures (tests/golden/);
* the reference's own known-answer cases (tests/test_gemm.py:166-184): sums
  that are exact in FP32 give exactly 32.0 and K * 2^-26;
* the checker's two tolerance rules, including that it catches planted errors.
"""
import math

import numpy as np
import pytest
import torch

from oracle import oracle

GOLDEN = oracle.ORACLE_DIR.parent / "tests" / "golden" / "golden_gemm.npz"


def test_half_to_float_exhaustive():
    lib = oracle.clib()
    bits = np.arange(65536, dtype=np.uint16)
    out = np.empty(65536, dtype=np.float32)
    lib.oracle_halves_to_floats(bits.ctypes.data, out.ctypes.data, 65536)
    expect = bits.view(np.float16).astype(np.float32)
    nan = np.isnan(expect)
    assert np.array_equal(np.isnan(out), nan)
    assert np.array_equal(out[~nan].view(np.uint32), expect[~nan].view(np.uint32))


def test_float_to_half_matches_ieee():
    lib = oracle.clib()
    rng = np.random.default_rng(0)
    vals = np.concatenate([
        rng.standard_normal(200000).astype(np.float32) * np.float32(8.0),
        rng.uniform(-70000, 70000, 50000).astype(np.float32),
        (rng.uniform(-1, 1, 50000) * 2.0 ** -14).astype(np.float32),  # subnormal range
        np.array([0.0, -0.0, 65504.0, 65519.996, 65520.0, -65520.0, 2 ** -24, 2 ** -25,
                  2 ** -25 * 1.0000001, 3 * 2 ** -26, np.inf, -np.inf, 6.103515625e-05,
                  6.1e-05, 1.0009765625, 1.00048828125, 1.00146484375], dtype=np.float32),
    ])
    # every half value and every midpoint between neighbours (ties to even)
    h = np.arange(0, 0x7C00, dtype=np.uint16).view(np.float16).astype(np.float64)
    mids = ((h[:-1] + h[1:]) / 2).astype(np.float32)
    vals = np.concatenate([vals, mids, -mids])
    out = np.empty(len(vals), dtype=np.uint16)
    lib.oracle_floats_to_halves(vals.ctypes.data, out.ctypes.data, len(vals))
    expect = vals.astype(np.float16).view(np.uint16)
    assert np.array_equal(out, expect)


def _golden_cases():
    d = np.load(GOLDEN)
    for name in d["names"]:
        m, n, k, alpha, beta = d[f"{name}/meta"]
        yield (str(name), int(m), int(n), int(k), float(alpha), float(beta),
               torch.from_numpy(d[f"{name}/A"].view(np.int16).copy()).view(torch.float16).reshape(int(m), int(k)),
               torch.from_numpy(d[f"{name}/B"].view(np.int16).copy()).view(torch.float16).reshape(int(k), int(n)),
               torch.from_numpy(d[f"{name}/C"].view(np.int16).copy()).view(torch.float16).reshape(int(m), int(n)),
               torch.from_numpy(d[f"{name}/expect64"].astype(np.float32)).reshape(int(m), int(n)))


@pytest.mark.parametrize("case", list(_golden_cases()), ids=lambda c: c[0])
def test_oracles_against_golden(case):
    name, m, n, k, alpha, beta, a, b, c, expect = case
    ref32 = oracle.reference_fp32(a, b, c, alpha, beta)
    assert torch.allclose(ref32, expect, atol=1e-5, rtol=1e-5), name
    unr = oracle.c_unrounded(a, b, c, alpha, beta)
    assert torch.allclose(unr, expect, atol=1e-5, rtol=1e-5), name
    rounded = oracle.c_gemm(a, b, c, alpha, beta)
    chk = oracle.check(rounded, expect)
    assert chk.passed, f"{name}: {chk}"
    # the rounded C result is the FP16 rounding of the unrounded one
    assert torch.equal(rounded, unr.half()) or oracle.check(rounded, unr).passed


def test_hand_checked_tiny_product():
    a = torch.tensor([[1, -2, 3], [0, 4, -1]], dtype=torch.float16)
    b = torch.tensor([[2, 1], [1, 0], [-1, 5]], dtype=torch.float16)
    c = torch.full((2, 2), float("nan"), dtype=torch.float16)
    out = oracle.c_gemm(a, b, c, 1.0, 0.0)  # beta == 0: C (NaN) is not read
    assert out.tolist() == [[-3.0, 16.0], [5.0, -5.0]]


@pytest.mark.parametrize("m,n,k", [(1, 4096, 18944), (8, 1024, 18944), (256, 6144, 4096),
                                   (256, 2048, 18944)])
def test_reference_cancellation_kat(m, n, k):
    """A = 256, B = +1 for the first half of K, -1 after, -0.875 in the last row:
    exact FP32 partial sums give exactly 32.0 (tests/test_gemm.py:166-184)."""
    a = torch.full((m, k), 256.0, dtype=torch.float16)
    b = torch.ones((k, n), dtype=torch.float16)
    b[k // 2:] = -1.0
    b[-1] = -0.875
    ref = oracle.reference_fp32(a, b, None, 1.0, 0.0)
    assert bool((ref == 32.0).all())
    if m * n * k <= 2e8:
        c = torch.zeros((m, n), dtype=torch.float16)
        assert bool((oracle.c_gemm(a, b, c, 1.0, 0.0) == 32.0).all())


def test_reference_tiny_kat():
    """A = B = 2^-13 at (32, 1024, 4096): exactly K * 2^-26 = 2^-14 (tests/test_gemm.py:176-178)."""
    m, n, k = 32, 1024, 4096
    a = torch.full((m, k), 2.0 ** -13, dtype=torch.float16)
    b = torch.full((k, n), 2.0 ** -13, dtype=torch.float16)
    c = torch.zeros((m, n), dtype=torch.float16)
    assert bool((oracle.reference_fp32(a, b, None, 1.0, 0.0) == k * 2.0 ** -26).all())
    assert bool((oracle.c_gemm(a, b, c, 1.0, 0.0) == k * 2.0 ** -26).all())


def test_fp64_audit_matches_fp32_reference():
    a, b, c = oracle.make_inputs(64, 96, 200, "uniform", seed=3)
    ref = oracle.reference_fp32(a, b, c, 0.75, -0.25)
    rows = np.arange(64) % 64
    cols = (np.arange(64) * 7) % 96
    audit = oracle.audit_f64(a, b, c, 0.75, -0.25, rows, cols)
    assert np.allclose(audit, ref[rows, cols].double().numpy(), atol=1e-5)


def test_checker_catches_planted_errors():
    a, b, c = oracle.make_inputs(32, 48, 64, "uniform", seed=1)
    ref = oracle.reference_fp32(a, b, c, 1.0, 0.5)
    good = oracle.c_gemm(a, b, c, 1.0, 0.5)
    assert oracle.check(good, ref).passed
    bad = good.clone()
    bad[3, 5] = bad[3, 5] + 0.25  # one wrong element
    chk = oracle.check(bad, ref)
    assert not chk.passed and chk.violations == 1
    nan = good.clone()
    nan[0, 0] = float("nan")
    assert not oracle.check(nan, ref).finite
    # an FP16 accumulator would fail the reference's cancellation case
    k = 4096
    a1 = torch.full((1, k), 256.0, dtype=torch.float16)
    b1 = torch.ones((k, 8), dtype=torch.float16)
    b1[k // 2:] = -1.0
    b1[-1] = -0.875
    acc = torch.zeros(8, dtype=torch.float16)
    for i in range(k):
        acc = (acc.float() + a1[0, i].float() * b1[i].float()).half()
    assert not bool((acc == 32.0).all())


def test_generators_are_seeded_and_ordered():
    a1, b1, c1 = oracle.make_inputs(16, 24, 40, "normal", seed=0)
    a2, b2, c2 = oracle.make_inputs(16, 24, 40, "normal", seed=0)
    assert torch.equal(a1, a2) and torch.equal(b1, b2) and torch.equal(c1, c2)
    assert abs(float(a1.float().std()) - 1 / math.sqrt(40)) < 0.05
    _, _, z = oracle.make_inputs(4, 4, 4, "normal", seed=0, c_dist="zero")
    assert bool((z == 0).all())
