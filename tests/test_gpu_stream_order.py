"""Stream order under programmatic dependent launch (needs a B200).

The tcgen05 GEMM kernels are launched as programmatic dependents: a kernel may
start its set-up while the previous kernel in the stream is still running, and
it waits for that kernel (griddepcontrol.wait) before it reads A, B or C. These
tests chain launches whose inputs the kernel just before has written: a PyTorch
elementwise kernel writes A, then a GEMM reads that A and the C written by the
previous GEMM (beta != 0), and a PyTorch kernel reads the last C. The chain runs
in a plain stream and replayed from a CUDA graph, and its end is compared with
the same chain on the CPU (each step rounded to half, as on the device).
"""
import pytest
import torch

import gemm_b200
from oracle import oracle

pytestmark = pytest.mark.gpu

STEPS = 4
ALPHAS = [1.0, -0.75, 0.5, 1.25]
BETA = 0.5


def _cpu_chain(a_list, b, c0):
    """Rounded C after STEPS-1 steps, and the unrounded last step."""
    c = c0
    for i in range(STEPS - 1):
        c = oracle.reference_fp32(a_list[i], b, c, ALPHAS[i], BETA).half()
    return oracle.reference_fp32(a_list[STEPS - 1], b, c, ALPHAS[STEPS - 1], BETA)


@pytest.mark.parametrize("m,n,k,tile", [(1024, 1024, 1024, 0), (512, 2048, 4096, 0), (256, 4096, 4096, 5),
                                        (640, 384, 4104, 2), (2048, 2048, 512, 4), (300, 1000, 72, 128)],
                         ids=str)
@pytest.mark.parametrize("graph", [False, True], ids=["stream", "graph"])
def test_chain_reads_what_the_previous_kernel_wrote(lib, cuda, m, n, k, tile, graph):
    a_list = [oracle.make_inputs(m, n, k, "normal", seed=s)[0] for s in range(STEPS)]
    _, b, c0 = oracle.make_inputs(m, n, k, "normal", seed=99)
    ref = _cpu_chain(a_list, b, c0)

    neg_a = [(-a).to(cuda) for a in a_list]  # -A: a negation kernel writes A
    a_dev = torch.empty(m, k, dtype=torch.float16, device=cuda)
    b_dev, c0_dev = b.to(cuda), c0.to(cuda)
    c_dev = torch.empty(m, n, dtype=torch.float16, device=cuda)

    def chain():
        c_dev.copy_(c0_dev)
        for i in range(STEPS):
            torch.neg(neg_a[i], out=a_dev)
            if tile:
                gemm_b200.gemm(a_dev, b_dev, c_dev, ALPHAS[i], BETA, path=1, tile_n=tile)
            else:
                gemm_b200.gemm(a_dev, b_dev, c_dev, ALPHAS[i], BETA)
        return c_dev * 1.0  # a PyTorch kernel reading the last C

    if graph:
        side = torch.cuda.Stream()
        with torch.cuda.stream(side):
            chain()  # one-time device set-up outside capture
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=side):
            out = chain()
        for _ in range(2):
            g.replay()
        torch.cuda.synchronize()
        del g
    else:
        out = chain()
        torch.cuda.synchronize()
    assert lib.gemm_launcher_status() == 0
    chk = oracle.check(out, ref)
    assert chk.passed, f"{(m, n, k, tile, graph)}: {chk}"
