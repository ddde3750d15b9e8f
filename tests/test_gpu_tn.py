"""gemm_launcher_tn: C = alpha * A @ Bt^T + beta * C with Bt[N,K] (needs a B200).

Same tcgen05 kernels with B read K-major; checked against the CPU oracle on
every tile shape, across tile and K-block edges, with misaligned pointers
(read in place by per-thread loads, or repacked) and with beta = 0 on a
NaN-filled C.
"""
import ctypes

import pytest
import torch

from gpu_harness import Guarded
from oracle import oracle

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("tile", [0, 64, 128, 256, 2, 3, 4])
@pytest.mark.parametrize("shape", [(128, 256, 64), (129, 257, 65), (300, 1000, 72), (1, 8, 8),
                                   (1024, 1024, 1024), (640, 384, 4104), (17, 19, 23)], ids=str)
@pytest.mark.parametrize("offset,beta,feed", [(0, 0.0, "0"), (1, 0.5, "1"), (1, 0.5, "-1")],
                         ids=["aligned", "misaligned-lsu", "misaligned-repack"])
def test_tn_matches_oracle(lib, cuda, monkeypatch, shape, tile, offset, beta, feed):
    monkeypatch.setenv("GEMM_LSU", feed)  # misaligned Bt/A: read in place, or repacked
    m, n, k = shape
    a, b, c0 = oracle.make_inputs(m, n, k, "normal", seed=m + 3 * n + k)
    bt = b.t().contiguous()
    ga = Guarded((m, k), cuda, offset=64 + offset)
    gb = Guarded((n, k), cuda, offset=64 + offset)
    gc = Guarded((m, n), cuda, fill=float("nan") if beta == 0 else 0.0, offset=64 + offset)
    ga.tensor.copy_(a)
    gb.tensor.copy_(bt)
    if beta != 0:
        gc.tensor.copy_(c0)
    torch.cuda.synchronize()
    rc = lib.gemm_launcher_tn(ga.tensor.data_ptr(), gb.tensor.data_ptr(), gc.tensor.data_ptr(), m,
                              n, k, ctypes.c_float(0.75), ctypes.c_float(beta), None, tile)
    torch.cuda.synchronize()
    assert rc == 0 and lib.gemm_launcher_status() == 0
    assert ga.canaries_ok() and gb.canaries_ok() and gc.canaries_ok()
    chk = oracle.check(gc.tensor, oracle.reference_fp32(a, b, c0, 0.75, beta))
    assert chk.passed, f"{shape} tile={tile}: {chk}"
    assert torch.equal(gb.tensor.cpu(), bt)
