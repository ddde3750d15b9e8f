"""Parity of the CUDA library with the CPU oracle, through the C ABI (needs a B200).

Coverage follows the reference's suite (tests/test_gemm.py): its launcher
cases by class (LLM projection shapes at decode/prefill token counts, odd M,
K = 1025, K = 0, M = 0, N = 0), its misaligned A/B/C cases, its exact
known-answer cases, canaries and NaN-filled C, plus every BASELINE config and
every kernel path forced on shapes that cross its tile edges.
"""
import ctypes

import pytest
import torch

from gpu_harness import Guarded, run, verify
from oracle import oracle

pytestmark = pytest.mark.gpu

PATH_TC, PATH_ROWS, PATH_COL, PATH_ROWS_LSU, PATH_COL_LSU, PATH_DEC, PATH_TC_LSU = 1, 2, 3, 4, 5, 6, 7


def _go(lib, cuda, m, n, k, alpha=1.0, beta=0.0, **kw):
    c, a, b, c0 = run(lib, cuda, m, n, k, alpha, beta, **kw)
    chk = verify(c, a, b, c0, alpha, beta, seed=kw.get("seed", 0))
    assert chk.passed, f"{(m, n, k)} alpha={alpha} beta={beta} {kw}: {chk}"
    return chk


# ---------------------------------------------------------------------------
# BASELINE.json configs
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("name", ["square1024", "square4096", "square8192", "gemv_m1", "gemv_n1",
                                  "odd_1023", "odd_3"])
def test_baseline_config(lib, cuda, name):
    cfg = oracle.CONFIGS[name]
    off = cfg.get("offset", 0)
    _go(lib, cuda, cfg["m"], cfg["n"], cfg["k"], cfg["alpha"], cfg["beta"], dist=cfg["dist"],
        offsets=(off, off, off), fn="launcher")


def test_sharded_config_one_slab(lib, cuda):
    """One 4096-row slab of the 32768x32768x16384 config (what each of 8 ranks runs)."""
    _go(lib, cuda, 4096, 32768, 16384, 1.0, 0.0, dist="normal", fn="launcher")


# ---------------------------------------------------------------------------
# Every path, forced, across tile and K-block edges
# ---------------------------------------------------------------------------
TC_SHAPES = [(128, 256, 64), (256, 512, 128), (129, 257, 65), (1, 8, 8), (127, 200, 1000),
             (300, 1000, 72), (1024, 1024, 1024), (640, 384, 4104), (2048, 2048, 64),
             (513, 264, 200), (1000, 2056, 136)]


@pytest.mark.parametrize("tile_n", [64, 128, 256, 2, 3, 4],
                         ids=["128x64", "128x128", "128x256", "pair256x256", "pair512x256",
                              "pair256x512"])
@pytest.mark.parametrize("shape", TC_SHAPES, ids=str)
def test_tc_path(lib, cuda, shape, tile_n):
    m, n, k = shape
    _go(lib, cuda, m, n, k, 0.75, 0.5, dist="normal", path=PATH_TC, tile_n=tile_n, seed=m + n + k)


# The tile kernel with per-thread operand loads (path 7: A and B read in place at
# any alignment and pitch, no repack): both of its tiles, ragged M/N/K, each
# pointer at half offsets 0, 1 and 3 (phases of the 16-byte lines), K and N that
# are not multiples of 8 (rows of alternating phase), beta = 0 over NaN C.
LSU_SHAPES = [(128, 256, 64), (129, 257, 65), (1023, 2049, 777), (300, 1000, 72), (17, 19, 23),
              (513, 264, 200), (640, 384, 4104), (1000, 2056, 136), (256, 130, 1031)]


@pytest.mark.parametrize("tile_n", [64, 128], ids=["128x64", "128x128"])
@pytest.mark.parametrize("shape", LSU_SHAPES, ids=str)
@pytest.mark.parametrize("offsets", [(0, 0, 0), (1, 1, 1), (3, 1, 0), (0, 3, 1)], ids=str)
def test_tc_lsu_path(lib, cuda, shape, tile_n, offsets):
    m, n, k = shape
    beta = 0.0 if offsets[0] == 3 else -0.25
    _go(lib, cuda, m, n, k, 0.75, beta, dist="normal", path=PATH_TC_LSU, tile_n=tile_n,
        offsets=offsets, seed=m + n + k + sum(offsets))


@pytest.mark.parametrize("tile,ks", [(64, 4), (64, 8), (128, 2), (128, 4), (128, 8)], ids=str)
def test_tc_lsu_split_k(lib, cuda, monkeypatch, tile, ks):
    monkeypatch.setenv("GEMM_SPLITK_TILE", str(tile))
    monkeypatch.setenv("GEMM_SPLITK_KS", str(ks))
    _go(lib, cuda, 300, 1001, 4097, 0.75, -0.5, dist="normal", path=PATH_TC_LSU,
        offsets=(1, 1, 1), seed=tile + ks)


@pytest.mark.parametrize("lsu", ["1", "-1"], ids=["lsu", "repack"])
@pytest.mark.parametrize("shape", [(1023, 2049, 777), (129, 257, 65), (2048, 1024, 1001)], ids=str)
def test_misaligned_dense_both_feeds(lib, cuda, monkeypatch, lsu, shape):
    """The automatic dispatch on misaligned operands through either operand feed:
    in-place per-thread loads or the repack into scratch."""
    import gemm_b200
    monkeypatch.setenv("GEMM_LSU", lsu)
    m, n, k = shape
    _go(lib, cuda, m, n, k, 0.75, -0.25, offsets=(1, 1, 1), seed=m + k, fn="launcher")
    assert ("lsu" in gemm_b200.last_kernel()) == (lsu == "1"), gemm_b200.last_kernel()


def _misaligned_calls(lib, cuda, m, n, k, calls):
    """free device memory before the first and after the last of `calls`
    gemm_launcher calls on operands offset by one half (fresh buffers)."""
    ga = Guarded((m, k), cuda, fill=0.5, offset=65)
    gb = Guarded((k, n), cuda, fill=0.25, offset=65)
    gc = Guarded((m, n), cuda, fill=1.0, offset=65)
    f = ctypes.c_float
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    for _ in range(calls):
        lib.gemm_launcher(ga.tensor.data_ptr(), gb.tensor.data_ptr(), gc.tensor.data_ptr(), m, n, k,
                          f(0.75), f(-0.25))
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert lib.gemm_launcher_status() == 0 and gc.canaries_ok()
    return free0, free1


def test_tiny_misaligned_dense_allocates_nothing(lib, cuda):
    """Tiny misaligned problems are read in place by the tile kernel: not even
    the first call takes device memory."""
    import gemm_b200
    free0, free1 = _misaligned_calls(lib, cuda, 129, 257, 65, 100)
    assert "lsu" in gemm_b200.last_kernel()
    assert free1 == free0, f"free device memory moved by {free0 - free1} bytes"


def test_misaligned_dense_steady_state_allocates_nothing(lib, cuda):
    """The reference's misaligned dense config through gemm_launcher: the repack
    scratch comes from the library's pool, so after the first call 100 more take
    no further device memory."""
    import gemm_b200
    _misaligned_calls(lib, cuda, 1023, 2049, 777, 1)
    free0, free1 = _misaligned_calls(lib, cuda, 1023, 2049, 777, 100)
    assert gemm_b200.last_kernel() == "tc_gemm_kernel<128x128>"
    assert free1 == free0, f"free device memory moved by {free0 - free1} bytes"


# Cluster split-K on 128 x 256 tiles (tile code 5): ragged M, N and K, the
# automatic choice at 1024^3, a misaligned C (the reduction's scalar stores).
SPLIT_K_SHAPES = [(1024, 1024, 1024), (129, 257, 650), (300, 1000, 4104), (1000, 520, 8192),
                  (64, 4096, 4096), (513, 264, 200)]


@pytest.mark.parametrize("shape", SPLIT_K_SHAPES, ids=str)
@pytest.mark.parametrize("beta", [0.0, -0.5])
def test_split_k_cluster(lib, cuda, shape, beta):
    m, n, k = shape
    _go(lib, cuda, m, n, k, 0.75, beta, dist="normal", path=PATH_TC, tile_n=5, seed=m + 7 * k)


# Split-K on every single-CTA tile width, plans forced through the planner's
# override: ragged M, N and K, beta != 0, a misaligned C (scalar stores).
@pytest.mark.parametrize("tile,ks", [(64, 2), (64, 4), (128, 2), (128, 4), (128, 8), (256, 8)],
                         ids=str)
@pytest.mark.parametrize("shape,c_off", [((300, 1000, 4104), 0), ((256, 1024, 4096), 0),
                                         ((700, 900, 3000), 1), ((96, 4096, 1000), 0)], ids=str)
def test_split_k_tile_widths(lib, cuda, monkeypatch, tile, ks, shape, c_off):
    monkeypatch.setenv("GEMM_SPLITK_TILE", str(tile))
    monkeypatch.setenv("GEMM_SPLITK_KS", str(ks))
    m, n, k = shape
    _go(lib, cuda, m, n, k, 0.75, -0.5, dist="normal", path=PATH_TC, offsets=(0, 0, c_off),
        seed=tile + ks + m)


def test_split_k_misaligned_c(lib, cuda):
    _go(lib, cuda, 700, 900, 3000, 0.75, 0.25, path=PATH_TC, tile_n=5, offsets=(0, 0, 1), seed=3)


@pytest.mark.parametrize("group", [1, 3, 64, -1, -3, -64])
@pytest.mark.parametrize("tile_n", [128, 4], ids=["128x128", "pair256x512"])
def test_tc_raster_orders(lib, cuda, monkeypatch, group, tile_n):
    """Every tile is produced exactly once under row- and column-major raster groups,
    including partial last groups."""
    monkeypatch.setenv("GEMM_RASTER_GROUP", str(group))
    _go(lib, cuda, 1300, 2900, 136, 0.75, 0.5, dist="normal", path=PATH_TC, tile_n=tile_n,
        seed=group + 100)


@pytest.mark.parametrize("shape", [(1, 8, 8), (2, 264, 300), (3, 5000, 4097), (4, 1024, 1025),
                                   (5, 2048, 8192), (8, 6144, 4096), (1, 28672, 8192),
                                   (7, 131, 515), (1, 1, 9), (6, 24, 20000), (1, 4096, 1024),
                                   (3, 5000, 4096), (8, 264, 40)], ids=str)
@pytest.mark.parametrize("offset", [0, 1, 3])
@pytest.mark.parametrize("path", [PATH_ROWS, PATH_ROWS_LSU], ids=["auto", "lsu"])
def test_rows_path(lib, cuda, shape, offset, path):
    m, n, k = shape
    _go(lib, cuda, m, n, k, 0.7, -0.3, path=path, offsets=(offset, offset, offset),
        seed=m * 31 + offset)


@pytest.mark.parametrize("shape", [(28672, 1, 8192), (9, 1, 8), (1000, 1, 777), (4096, 1, 14336),
                                   (33, 1, 1), (100, 1, 264), (65, 1, 4096)], ids=str)
@pytest.mark.parametrize("offset", [0, 1])
@pytest.mark.parametrize("path", [PATH_COL, PATH_COL_LSU], ids=["auto", "lsu"])
def test_col_path(lib, cuda, shape, offset, path):
    m, n, k = shape
    _go(lib, cuda, m, n, k, 1.0, 0.25, path=path, offsets=(offset, offset, offset), seed=m)


@pytest.mark.parametrize("shape", [(2, 264, 296), (8, 6144, 4096), (16, 1024, 18944), (17, 640, 672),
                                   (32, 6144, 4096), (33, 2056, 1000), (64, 512, 64), (5, 8, 8),
                                   (3, 5000, 4096), (48, 4104, 2000), (64, 28672, 8192),
                                   (65, 4096, 4096), (128, 4096, 4096), (129, 1000, 520),
                                   (200, 2048, 8192), (256, 512, 64), (256, 28672, 1024),
                                   (97, 8, 8)], ids=str)
def test_small_m_tensor_core_path(lib, cuda, shape):
    m, n, k = shape
    _go(lib, cuda, m, n, k, 0.75, -0.5, dist="normal", path=PATH_DEC, seed=m + n)
    _go(lib, cuda, m, n, k, 1.0, 0.0, dist="normal", path=PATH_DEC, seed=m + n + 1)


# ---------------------------------------------------------------------------
# The reference's launcher cases by class (tests/test_gemm.py:12-23,107-163)
# ---------------------------------------------------------------------------
MODEL_DIMS = {"llama3_8b": (4096, 14336, 1024, 128256), "qwen25_7b": (3584, 18944, 512, 152064)}


def _llm_cases():
    cases = [(1024, 1024, 1024)]
    for hidden, ffn, kv, vocab in MODEL_DIMS.values():
        for n, k in [(hidden + 2 * kv, hidden), (hidden, hidden), (2 * ffn, hidden), (hidden, ffn)]:
            for m in [1, 8, 32, 64, 128, 512, 2048]:
                cases.append((m, n, k))
        for m in [1, 32, 128]:
            cases.append((m, vocab, hidden))
    return cases


@pytest.mark.parametrize("shape", _llm_cases(), ids=str)
def test_llm_projection_shapes(lib, cuda, shape):
    m, n, k = shape
    c, a, b, c0 = run(lib, cuda, m, n, k, 1.0, 0.0, dist="normal", seed=sum(shape), fn="launcher")
    chk = verify(c, a, b, c0, 1.0, 0.0, sample_rows=64)
    assert chk.passed, f"{shape}: {chk}"


REGRESSION = [(1, 4096, 1025), (1, 512, 1025), (1, 1024, 8192), (2, 512, 512), (3, 576, 640),
              (17, 640, 672), (31, 512, 1024), (47, 1024, 512), (63, 1024, 640), (65, 1024, 640),
              (96, 1024, 1024), (128, 576, 18944), (384, 2048, 14336), (1664, 2048, 14336),
              (832, 2048, 8256), (17, 19, 0)]


@pytest.mark.parametrize("shape", REGRESSION, ids=str)
def test_regression_shapes(lib, cuda, shape):
    m, n, k = shape
    c, a, b, c0 = run(lib, cuda, m, n, k, 0.7, -0.3, seed=m + k, c_init=2.0, fn="launcher")
    chk = verify(c, a, b, c0, 0.7, -0.3)
    assert chk.passed, f"{shape}: {chk}"


@pytest.mark.parametrize("m,n", [(0, 19), (19, 0), (0, 0)])
def test_empty_output_is_noop(lib, cuda, m, n):
    gc = Guarded((max(m, 1), max(n, 1)), cuda, fill=7.0)
    a = torch.ones(64, device=cuda, dtype=torch.float16)
    torch.cuda.synchronize()
    lib.gemm_launcher(a.data_ptr(), a.data_ptr(), gc.tensor.data_ptr(), m, n, 32,
                      ctypes.c_float(1.0), ctypes.c_float(1.0))
    torch.cuda.synchronize()
    assert lib.gemm_launcher_status() == 0
    assert bool((gc.tensor == 7.0).all()) and gc.canaries_ok()


@pytest.mark.parametrize("beta", [0.0, -0.5])
def test_k_zero_scales_c(lib, cuda, beta):
    c, a, b, c0 = run(lib, cuda, 17, 19, 0, 1.0, beta, fn="launcher")
    expect = torch.zeros(17, 19) if beta == 0.0 else (beta * c0.float())
    assert torch.equal(c.cpu(), expect.half())


@pytest.mark.parametrize("which", ["A", "B", "C"])
def test_single_pointer_misaligned(lib, cuda, which):
    """One pointer shifted by one half (tests/test_gemm.py:140-162)."""
    off = {"A": (1, 0, 0), "B": (0, 1, 0), "C": (0, 0, 1)}[which]
    c, a, b, c0 = run(lib, cuda, 17, 1024, 544, 0.7, -0.3, offsets=off, c_init=2.0, fn="launcher")
    assert verify(c, a, b, c0, 0.7, -0.3).passed
    c, a, b, c0 = run(lib, cuda, 300, 1024, 544, 0.7, -0.3, offsets=off, c_init=2.0, fn="launcher")
    assert verify(c, a, b, c0, 0.7, -0.3).passed


# ---------------------------------------------------------------------------
# Exact known-answer cases (tests/test_gemm.py:166-184)
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("m,n,k,tiny", [(1, 4096, 18944, False), (8, 1024, 18944, False),
                                        (32, 1024, 4096, True), (256, 6144, 4096, False),
                                        (256, 2048, 18944, False), (4096, 1, 18944, False)])
def test_exact_known_answers(lib, cuda, m, n, k, tiny):
    ga = Guarded((m, k), cuda, fill=2.0 ** -13 if tiny else 256.0)
    gb = Guarded((k, n), cuda, fill=2.0 ** -13 if tiny else 1.0)
    if not tiny:
        if n == 1:
            ga.tensor[:, k // 2:] = -256.0
            ga.tensor[:, -1] = -224.0
        else:
            gb.tensor[k // 2:] = -1.0
            gb.tensor[-1] = -0.875
    gc = Guarded((m, n), cuda)
    torch.cuda.synchronize()
    lib.gemm_launcher(ga.tensor.data_ptr(), gb.tensor.data_ptr(), gc.tensor.data_ptr(), m, n, k,
                      ctypes.c_float(1.0), ctypes.c_float(0.0))
    torch.cuda.synchronize()
    expected = k * 2.0 ** -26 if tiny else 32.0
    assert lib.gemm_launcher_status() == 0
    assert bool((gc.tensor == expected).all()), f"{(m, n, k)} not exact"
    assert gc.canaries_ok()


def test_cublas_comparator_agrees(lib, cuda):
    c, a, b, c0 = run(lib, cuda, 512, 768, 1024, 0.5, 0.5, fn="cublas")
    assert verify(c, a, b, c0, 0.5, 0.5).passed


def test_dispatch_choices(lib, cuda):
    """The automatic dispatch picks the sm_100a kernel family for each config class."""
    import gemm_b200
    names = {}
    for shape in [(1024, 1024, 1024), (1, 28672, 8192), (28672, 1, 8192), (3, 5000, 4097),
                  (8192, 8192, 64)]:
        run(lib, cuda, *shape, fn="launcher")
        names[shape] = gemm_b200.last_kernel()
    assert names[(1024, 1024, 1024)].startswith("tc_gemm_kernel")
    assert names[(8192, 8192, 64)].startswith("tc_gemm_kernel<2")  # a CTA-pair tile
    assert names[(1, 28672, 8192)].startswith("rows_tma_kernel<1>")
    assert names[(28672, 1, 8192)].startswith("col_tma_kernel")
    # K odd: A is not TMA-addressable, so the streaming kernel reads it directly
    assert names[(3, 5000, 4097)].startswith("rows_tma_kernel<4,a-direct>")
    run(lib, cuda, 8, 6144, 4096, fn="launcher")
    assert gemm_b200.last_kernel().startswith("skinny_tc_kernel<16>")
    # 32 < M <= 64: split-K dense tiles when the output tiles are few, else small-M
    run(lib, cuda, 48, 4096, 4096, fn="launcher")
    assert gemm_b200.last_kernel().startswith("tc_gemm_kernel<128x128>")
    run(lib, cuda, 48, 28672, 1024, fn="launcher")
    assert gemm_b200.last_kernel().startswith("skinny_tc_kernel<64>")
    # M > 64: the dense path, whose single-CTA tiles split K over a cluster when
    # they are too few to fill the GPU (128 x 128 tiles, 4 parts, here)
    run(lib, cuda, 96, 4096, 14336, fn="launcher")
    assert gemm_b200.last_kernel().startswith("tc_gemm_kernel")
    run(lib, cuda, 128, 4096, 4096, fn="launcher")
    assert gemm_b200.last_kernel().startswith("tc_gemm_kernel<128x128>")
    run(lib, cuda, 200, 4096, 8192, fn="launcher")
    assert gemm_b200.last_kernel().startswith("tc_gemm_kernel")
