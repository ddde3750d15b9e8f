"""PyTorch operators over the C ABI (gemm-project_b200/csrc/torch_op.cpp).

trtllm_gemm_sample::gemm mirrors the reference's TRT-LLM sample operator
(samples/trtllm_gemm/binding.cpp:17-60) and its launcher's acceptance rule
(samples/trtllm_gemm/launcher.cu:6-11); the tests follow what the reference's
adapter relies on (samples/trtllm_gemm/adapter.py:61-75): the schema, the Meta
kernel, results on PyTorch's current stream, the rejections it expects, and
replay inside a CUDA graph (the adapter installs before graph capture).
gemm_b200::gemm / gemm_b200::linear are the general operators (any shape;
linear takes the weight in its stored [N, K] layout).

CPU tests: library loads, schemas, Meta shapes. GPU tests: parity with the CPU
oracle on the same seeded inputs.
"""
import ctypes

import pytest
import torch

import gemm_b200
from oracle import oracle


@pytest.fixture(scope="module")
def ops(lib):
    import build as pkg_build
    pkg_build.build_torch_op()
    return gemm_b200.load_torch_ops()


# ---------------------------------------------------------------------------
# CPU: registration and Meta kernels
# ---------------------------------------------------------------------------
def test_schemas(ops):
    assert str(ops.trtllm_gemm_sample.gemm.default._schema) == \
        "trtllm_gemm_sample::gemm(Tensor a, Tensor b) -> Tensor"
    assert str(ops.gemm_b200.linear.default._schema) == "gemm_b200::linear(Tensor x, Tensor w) -> Tensor"
    assert "Tensor? c=None" in str(ops.gemm_b200.gemm.default._schema)


def test_meta_shapes(ops):
    meta = dict(dtype=torch.float16, device="meta")
    a, b = torch.empty(8, 1024, **meta), torch.empty(1024, 4096, **meta)
    assert ops.trtllm_gemm_sample.gemm(a, b).shape == (8, 4096)
    assert ops.gemm_b200.gemm(a, b).shape == (8, 4096)
    x, w = torch.empty(2, 3, 1024, **meta), torch.empty(512, 1024, **meta)
    assert ops.gemm_b200.linear(x, w).shape == (2, 3, 512)


def test_no_cpu_kernel(ops):
    """The operators are CUDA-only: there is no CPU fallback to land on."""
    a, b = torch.zeros(8, 1024, dtype=torch.float16), torch.zeros(1024, 4096, dtype=torch.float16)
    with pytest.raises(NotImplementedError):
        ops.trtllm_gemm_sample.gemm(a, b)


def test_sample_launcher_rejects_without_gpu(lib):
    """launchGemmSample's acceptance rule is checked before any device work."""
    for m, n, k in [(0, 512, 512), (17, 512, 512), (1, 500, 512), (1, 576, 512), (1, 512, 520),
                    (1, 512, 256)]:
        if (m, n, k) == (1, 576, 512):
            continue  # inside the rule (n % 64 == 0): needs a GPU
        assert not lib.launchGemmSample(16, 16, 16, m, n, k, None), (m, n, k)
    assert not lib.launchGemmSample(18, 16, 16, 8, 512, 512, None)  # a not 16-byte aligned
    assert lib.gemm_launch_error() == 0


# ---------------------------------------------------------------------------
# GPU: parity with the oracle
# ---------------------------------------------------------------------------
def _inputs(m, n, k, seed, dev):
    a, b, c = oracle.make_inputs(m, n, k, "uniform", seed)
    return a, b, c, a.to(dev), b.to(dev), c.to(dev)


@pytest.mark.gpu
@pytest.mark.parametrize("m,n,k", [(1, 4096, 4096), (3, 512, 512), (8, 14336, 4096),
                                   (16, 4096, 14336), (13, 576, 1056)])
def test_sample_gemm_matches_oracle_on_current_stream(ops, cuda, m, n, k):
    a, b, _, ad, bd, _ = _inputs(m, n, k, m + n + k, cuda)
    side = torch.cuda.Stream()
    with torch.cuda.stream(side):
        out = ops.trtllm_gemm_sample.gemm(ad, bd)
    side.synchronize()
    chk = oracle.check(out, oracle.reference_fp32(a, b, None, 1.0, 0.0))
    assert chk.passed, f"{(m, n, k)}: {chk}"


@pytest.mark.gpu
def test_sample_gemm_rejections(ops, cuda):
    dev = cuda
    h = dict(dtype=torch.float16, device=dev)
    cases = [
        (torch.zeros(17, 512, **h), torch.zeros(512, 512, **h), "Shape outside sample dispatch"),
        (torch.zeros(4, 520, **h), torch.zeros(520, 512, **h), "Shape outside sample dispatch"),
        (torch.zeros(4, 512, **h), torch.zeros(512, 500, **h), "Shape outside sample dispatch"),
        (torch.zeros(4, 512, dtype=torch.float32, device=dev), torch.zeros(512, 512, **h),
         "FP16 required"),
        (torch.zeros(4, 512, **h), torch.zeros(256, 512, **h), "Invalid GEMM dimensions"),
        (torch.zeros(512, 4, **h).t(), torch.zeros(512, 512, **h), "Contiguous operands required"),
        (torch.zeros(4 * 512 + 1, **h)[1:].view(4, 512), torch.zeros(512, 512, **h),
         "16-byte alignment required"),
    ]
    for a, b, msg in cases:
        with pytest.raises(RuntimeError, match=msg):
            ops.trtllm_gemm_sample.gemm(a, b)


@pytest.mark.gpu
def test_sample_gemm_in_cuda_graph(ops, cuda):
    m, n, k = 8, 4096, 4096
    a, b, _, ad, bd, _ = _inputs(m, n, k, 7, cuda)
    ops.trtllm_gemm_sample.gemm(ad, bd)  # first call outside capture (one-time device set-up)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        out = ops.trtllm_gemm_sample.gemm(ad, bd)
    a2, b2, _ = oracle.make_inputs(m, n, k, "uniform", 8)
    ad.copy_(a2)
    bd.copy_(b2)
    g.replay()
    torch.cuda.synchronize()
    chk = oracle.check(out, oracle.reference_fp32(a2, b2, None, 1.0, 0.0))
    assert chk.passed, str(chk)
    del g


@pytest.mark.gpu
@pytest.mark.parametrize("m,n,k,alpha,beta", [(300, 520, 200, 0.75, 0.5), (1, 28672, 1024, 1.0, 0.0),
                                              (1023, 2049, 777, 0.75, -0.25), (64, 4096, 4096, 1.0, 1.0)])
def test_general_gemm(ops, cuda, m, n, k, alpha, beta):
    a, b, c, ad, bd, cd = _inputs(m, n, k, m + 3 * n + k, cuda)
    c_before = cd.clone()
    out = ops.gemm_b200.gemm(ad, bd, cd if beta != 0 else None, alpha, beta)
    torch.cuda.synchronize()
    assert torch.equal(cd, c_before), "c must not be modified"
    chk = oracle.check(out, oracle.reference_fp32(a, b, c, alpha, beta))
    assert chk.passed, f"{(m, n, k)}: {chk}"


@pytest.mark.gpu
@pytest.mark.parametrize("lead,n,k", [((5,), 4096, 1024), ((2, 3), 1000, 777), ((1,), 14336, 4096),
                                      ((512,), 512, 4104)])
def test_linear_weight_layout(ops, cuda, lead, n, k):
    m = 1
    for d in lead:
        m *= d
    x, w, _ = oracle.make_inputs(m, n, k, "uniform", m + n)  # x[M,K]; w drawn as [K,N]
    wt = w.t().contiguous()                                  # the stored weight W[N,K]
    out = ops.gemm_b200.linear(x.view(*lead, k).to(cuda), wt.to(cuda))
    torch.cuda.synchronize()
    assert out.shape == (*lead, n)
    chk = oracle.check(out.view(m, n), oracle.reference_fp32(x, w, None, 1.0, 0.0))
    assert chk.passed, f"{(lead, n, k)}: {chk}"


@pytest.mark.gpu
def test_opcheck(ops, cuda):
    """PyTorch's operator consistency checks (schema, fake/Meta vs real)."""
    h = dict(dtype=torch.float16, device=cuda)
    a, b = torch.randn(8, 1024, **h), torch.randn(1024, 4096, **h)
    utils = ("test_schema", "test_faketensor")
    torch.library.opcheck(ops.trtllm_gemm_sample.gemm.default, (a, b), test_utils=utils)
    torch.library.opcheck(ops.gemm_b200.gemm.default, (a, b), test_utils=utils)
    torch.library.opcheck(ops.gemm_b200.linear.default, (a, b.t().contiguous()), test_utils=utils)
