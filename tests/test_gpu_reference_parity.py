"""Pin the oracle against the reference itself, run on the B200.

oracle/_ref/libgemm_ref.so is the reference's unmodified src/gemm.cu compiled
for sm_100a by `make -C oracle ref` (test-only checker; built where the
reference checkout exists and carried to the GPU box as a file). For shapes
that reach each of the reference's kernel families (its GEMV, small-M
mma.sync, large-M mma.sync, 64x64 swizzle and WMMA fallbacks), the reference
library, this library and the CPU oracle see identical inputs; the reference's
outputs must pass the oracle's checks (pinning the oracle) and this library's
outputs must agree with the reference's to within FP32-accumulation noise.
"""
import ctypes

import pytest
import torch

from gpu_harness import Guarded
from oracle import oracle

pytestmark = pytest.mark.gpu

SHAPES = [
    # (M, N, K, alpha, beta): reference kernel reached (src/gemm.cu dispatch)
    (1, 4096, 1024, 1.0, 0.0),       # gemm_gemv_kernel<8,16,4>
    (1, 1088, 640, 1.0, 0.0),        # gemm_gemv_kernel<2,16,4>
    (8, 6144, 512, 1.0, 0.0),        # gemm_mma_llm_kernel<16,128,3>
    (32, 1024, 1024, 0.7, -0.3),     # gemm_mma_llm_kernel<32,128,3>
    (256, 8192, 4096, 1.0, 0.0),     # gemm_mma_llm_kernel<64,128,3,32>
    (256, 4096, 8192, 1.0, 0.0),     # gemm_mma_llm_kernel<128,64,4,4>
    (1024, 1024, 1024, 1.0, 0.0),    # gemm_wmma_swizzle_kernel<3>
    (48, 80, 96, 1.0, 0.5),          # gemm_wmma_gmem_kernel
    (17, 19, 23, 0.75, -0.25),       # gemm_wmma_smem_kernel
    (300, 1, 777, 1.0, 0.25),        # gemm_wmma_smem_kernel (N = 1)
]


@pytest.fixture(scope="module")
def ref_lib():
    if not oracle.REF_LIB_PATH.exists():
        pytest.skip("oracle/_ref/libgemm_ref.so not built (needs the reference checkout)")
    lib = ctypes.CDLL(str(oracle.REF_LIB_PATH))
    lib.gemm_launcher.argtypes = [ctypes.c_void_p] * 3 + [ctypes.c_int] * 3 + [ctypes.c_float] * 2
    lib.gemm_launcher.restype = None
    return lib


@pytest.mark.parametrize("shape", SHAPES, ids=str)
def test_reference_library_and_ours_agree_with_oracle(lib, ref_lib, cuda, shape, capfd):
    m, n, k, alpha, beta = shape
    a, b, c0 = oracle.make_inputs(m, n, k, "normal", seed=m * 7 + n)
    ga, gb = Guarded((m, k), cuda), Guarded((k, n), cuda)
    ga.tensor.copy_(a)
    gb.tensor.copy_(b)
    outs = {}
    for name, which in (("reference", ref_lib), ("ours", lib)):
        gc = Guarded((m, n), cuda, fill=float("nan") if beta == 0 else 0.0)
        if beta != 0:
            gc.tensor.copy_(c0)
        torch.cuda.synchronize()
        which.gemm_launcher(ga.tensor.data_ptr(), gb.tensor.data_ptr(), gc.tensor.data_ptr(), m, n,
                            k, ctypes.c_float(alpha), ctypes.c_float(beta))
        torch.cuda.synchronize()
        assert gc.canaries_ok(), name
        outs[name] = gc.tensor.cpu()
    capfd.readouterr()  # the reference prints its launch line
    ref = oracle.reference_fp32(a, b, c0, alpha, beta)
    chk_ref = oracle.check(outs["reference"], ref)
    chk_ours = oracle.check(outs["ours"], ref)
    assert chk_ref.passed, f"reference library vs oracle: {chk_ref}"
    assert chk_ours.passed, f"this library vs oracle: {chk_ours}"
    # ours vs the reference's own output: both FP32-accumulated, so they differ
    # by at most a couple of FP16 ulps of the result
    diff = (outs["ours"].float() - outs["reference"].float()).abs()
    scale = outs["reference"].float().abs() + 1.0
    assert float((diff / scale).max()) <= 4e-3
