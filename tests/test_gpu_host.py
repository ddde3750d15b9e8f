"""gemm_host: GEMM on host-resident operands with slab-pipelined transfers.

CPU tests: argument checks (no device work). GPU tests: parity with the CPU
oracle on the same seeded inputs, for one and several slabs, ragged slab
counts, beta == 0 (C not sent) and beta != 0, out != c, and B already on the
device.
"""
import pytest
import torch

import gemm_b200
from oracle import oracle


def test_rejects_device_and_wrong_dtype_tensors():
    a = torch.zeros(4, 8, dtype=torch.float16)
    b = torch.zeros(8, 4, dtype=torch.float16)
    c = torch.zeros(4, 4, dtype=torch.float16)
    with pytest.raises(gemm_b200.GemmError):
        gemm_b200.gemm_host(a.float(), b, c)
    with pytest.raises(gemm_b200.GemmError):
        gemm_b200.gemm_host(a, b.t(), c)  # not contiguous
    with pytest.raises(gemm_b200.GemmError):
        gemm_b200.gemm_host(a, b, torch.zeros(5, 4, dtype=torch.float16))


@pytest.mark.gpu
@pytest.mark.parametrize("m,n,k,slabs", [(1024, 768, 512, 8), (1000, 520, 777, 3), (300, 4096, 1024, 8),
                                         (100, 256, 64, 8), (2048, 1024, 2048, 1)], ids=str)
@pytest.mark.parametrize("beta", [0.0, 0.5])
def test_matches_oracle(lib, cuda, m, n, k, slabs, beta):
    a, b, c = oracle.make_inputs(m, n, k, "normal", m + n + k)
    a_h, b_h, c_h = a.pin_memory(), b.pin_memory(), c.pin_memory()
    out = torch.empty_like(c_h).pin_memory()
    gemm_b200.gemm_host(a_h, b_h, c_h, 0.75, beta, out=out, slabs=slabs)
    torch.cuda.current_stream().synchronize()
    assert lib.gemm_launcher_status() == 0
    assert torch.equal(c_h, c), "c must not be modified when out is given"
    chk = oracle.check(out, oracle.reference_fp32(a, b, c, 0.75, beta))
    assert chk.passed, f"{(m, n, k, slabs, beta)}: {chk}"


@pytest.mark.gpu
def test_in_place_and_repeated(lib, cuda):
    """out defaults to c; two calls in a row on the same buffers."""
    m, n, k = 640, 1024, 512
    a, b, c = oracle.make_inputs(m, n, k, "uniform", 7)
    a_h, b_h, c_h = a.pin_memory(), b.pin_memory(), c.clone().pin_memory()
    gemm_b200.gemm_host(a_h, b_h, c_h, 1.0, 1.0, slabs=4)
    gemm_b200.gemm_host(a_h, b_h, c_h, 1.0, 1.0, slabs=4)
    torch.cuda.current_stream().synchronize()
    once = oracle.reference_fp32(a, b, c, 1.0, 1.0).half()
    chk = oracle.check(c_h, oracle.reference_fp32(a, b, once, 1.0, 1.0))
    assert chk.passed, str(chk)


@pytest.mark.gpu
@pytest.mark.parametrize("beta", [0.0, -0.25])
def test_device_resident_b(lib, cuda, beta):
    """B already on the device (a resident weight, or a replica a multi-GPU job
    broadcast once): only A (and C when beta != 0) cross PCIe; B is not modified."""
    m, n, k = 1500, 1032, 776
    a, b, c = oracle.make_inputs(m, n, k, "normal", 11)
    b_d = b.to(cuda)
    a_h, c_h = a.pin_memory(), c.pin_memory()
    out = torch.empty_like(c_h).pin_memory()
    gemm_b200.gemm_host(a_h, b_d, c_h, 0.75, beta, out=out, slabs=4)
    torch.cuda.current_stream().synchronize()
    assert lib.gemm_launcher_status() == 0
    assert torch.equal(b_d.cpu(), b)
    chk = oracle.check(out, oracle.reference_fp32(a, b, c, 0.75, beta))
    assert chk.passed, str(chk)
