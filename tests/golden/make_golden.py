"""Generate the golden GEMM fixtures in this folder (golden_gemm.npz).

Each case stores seeded FP16 inputs (A, B, C as uint16 bit patterns), alpha,
beta, and the expected outputs computed in FP64 from the half inputs
(`expect64` = alpha * sum_k A*B + beta * C evaluated in FP64, stored as FP32). Expected values are
independent of accumulation order, so they pin both oracles (the torch FP32
formula of the reference's tests, tests/test_gemm.py:91,130,156, and the C
restatement) and the GPU kernels to within FP32-accumulation error.

The cases are written for this repository; they are not the reference's
bundled third-party cases (tests/test_gemm.py:69-104, CC BY-NC-ND), which are
not reproduced. They cover the reference's edge classes: hand-checkable tiny
products, odd M/N/K, K = 0, beta != 0 with alpha = 0, and shapes that cross
the 128 x 256 tile and 64-wide K-block boundaries.

Run: python tests/golden/make_golden.py
"""
from __future__ import annotations

from pathlib import Path

import numpy as np

OUT = Path(__file__).resolve().parent / "golden_gemm.npz"

CASES = [
    # name, M, N, K, alpha, beta, seed
    ("tiny_2x2x3", 2, 2, 3, 1.0, 0.0, 1),
    ("unit_alpha_beta", 4, 4, 4, 0.5, 2.0, 2),
    ("alpha_zero", 8, 8, 8, 0.0, 1.0, 3),
    ("k_zero", 5, 7, 0, 1.0, -0.5, 4),
    ("odd_small", 17, 19, 23, 0.7, -0.3, 5),
    ("gemv_row", 1, 300, 129, 1.0, 0.0, 6),
    ("gemv_col", 300, 1, 129, 1.0, 0.25, 7),
    ("rows3", 3, 520, 257, 0.75, -0.25, 8),
    ("tile_edges", 129, 257, 65, 1.0, 0.5, 9),
    ("kblock_edges", 130, 70, 200, -1.25, 0.0, 10),
]


def half_bits(x: np.ndarray) -> np.ndarray:
    return x.astype(np.float16).view(np.uint16)


def make_case(m, n, k, alpha, beta, seed):
    rng = np.random.default_rng(seed)
    a = rng.uniform(-1, 1, size=(m, k)).astype(np.float16)
    b = rng.uniform(-1, 1, size=(k, n)).astype(np.float16)
    c = rng.uniform(-1, 1, size=(m, n)).astype(np.float16)
    if m == 2 and n == 2 and k == 3:  # hand-checkable: small integers
        a = np.array([[1, -2, 3], [0, 4, -1]], dtype=np.float16)
        b = np.array([[2, 1], [1, 0], [-1, 5]], dtype=np.float16)
    expect = alpha * (a.astype(np.float64) @ b.astype(np.float64))
    if beta != 0.0:
        expect = expect + beta * c.astype(np.float64)
    return a.view(np.uint16), b.view(np.uint16), c.view(np.uint16), expect


def main():
    data = {}
    names = []
    for name, m, n, k, alpha, beta, seed in CASES:
        a, b, c, e = make_case(m, n, k, alpha, beta, seed)
        data[f"{name}/A"] = a
        data[f"{name}/B"] = b
        data[f"{name}/C"] = c
        data[f"{name}/expect64"] = e.astype(np.float32)  # FP64 result, stored at FP32 precision
        data[f"{name}/meta"] = np.array([m, n, k, alpha, beta], dtype=np.float64)
        names.append(name)
    data["names"] = np.array(names)
    np.savez_compressed(OUT, **data)
    print(f"wrote {OUT} ({len(names)} cases)")


if __name__ == "__main__":
    main()
