"""gemm_launcher_sub: dense GEMM on row-strided sub-matrices and part of the GPU,
the building block of the overlapped multi-GPU broadcast (needs a B200).

C is a column block of a wider matrix (row pitch = the wide width). Columns
outside the block must stay untouched. An SM cap must not change the result.
A and B that TMA cannot address are refused, not repacked.
"""
import ctypes

import pytest
import torch

import gemm_b200
from oracle import oracle

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("c0,c1", [(512, 2560), (3, 1003), (2048, 3000)], ids=str)
@pytest.mark.parametrize("max_sms", [0, 132, 7])
def test_column_block_of_c(lib, cuda, c0, c1, max_sms):
    m, n, k = 1000, 3000, 520
    a, b, c = oracle.make_inputs(m, n, k, "normal", c0 + max_sms)
    ad, cd = a.to(cuda), c.to(cuda)
    b_blk = b[:, c0:c1].contiguous()
    before = cd.clone()
    gemm_b200.gemm_sub(ad, b_blk.to(cuda), cd[:, c0:c1], 0.75, 0.5, max_sms=max_sms)
    torch.cuda.synchronize()
    assert lib.gemm_launcher_status() == 0
    ref = oracle.reference_fp32(a, b_blk, c[:, c0:c1].contiguous(), 0.75, 0.5)
    chk = oracle.check(cd[:, c0:c1], ref)
    assert chk.passed, str(chk)
    assert torch.equal(cd[:, :c0], before[:, :c0]) and torch.equal(cd[:, c1:], before[:, c1:])


def test_sm_cap_does_not_change_the_result(lib, cuda):
    m, n, k = 2048, 4096, 1024
    a, b, _ = oracle.make_inputs(m, n, k, "normal", 3)
    ad, bd = a.to(cuda), b.to(cuda)
    outs = []
    for cap in (0, 100, 16):
        c = torch.zeros(m, n, dtype=torch.float16, device=cuda)
        gemm_b200.gemm_sub(ad, bd, c, 1.0, 0.0, max_sms=cap)
        torch.cuda.synchronize()
        outs.append(c)
    assert torch.equal(outs[0], outs[1]) and torch.equal(outs[0], outs[2])


def test_refuses_operands_tma_cannot_address(lib, cuda):
    h = dict(dtype=torch.float16, device=cuda)
    a, b, c = torch.zeros(64, 100, **h), torch.zeros(100, 64, **h), torch.zeros(64, 64, **h)
    f = ctypes.c_float
    # lda = 100 is not a multiple of 8 halves (16 bytes)
    assert lib.gemm_launcher_sub(a.data_ptr(), 100, b.data_ptr(), 64, c.data_ptr(), 64, 64, 64, 100,
                                 f(1.0), f(0.0), None, 0) == -1
    # K = 0 and pitches narrower than the widths
    assert lib.gemm_launcher_sub(a.data_ptr(), 104, b.data_ptr(), 64, c.data_ptr(), 64, 64, 64, 0,
                                 f(1.0), f(0.0), None, 0) == -1
    assert lib.gemm_launcher_sub(a.data_ptr(), 96, b.data_ptr(), 64, c.data_ptr(), 64, 64, 64, 100,
                                 f(1.0), f(0.0), None, 0) == -1
    assert lib.gemm_launcher_status() == 0
