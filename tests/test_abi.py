"""The C-ABI library loads and exports every entry point its header declares
(no compute calls: these run without a GPU). Mirrors the reference's build gate,
which requires `nm -D` to list `T gemm_launcher` (tools/project.py:137-138)."""
import ctypes
import re
import subprocess
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent
HEADER = REPO / "include" / "gemm_b200.h"


def declared_symbols():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"GEMM_API\s+[\w\s\*]+?\b(\w+)\s*\(", text)))


def test_header_declares_reference_entry_point():
    syms = declared_symbols()
    assert "gemm_launcher" in syms           # src/gemm.cu:104-105
    assert "launchGemmSample" in syms        # samples/trtllm_gemm/launcher.cu:4-5
    assert len(syms) >= 8


def test_library_exports_every_declared_symbol(lib):
    path = Path(lib._name)
    out = subprocess.run(["nm", "-D", "--defined-only", str(path)], capture_output=True, text=True,
                         check=True).stdout
    exported = {ln.split()[-1] for ln in out.splitlines() if " T " in ln}
    missing = [s for s in declared_symbols() if s not in exported]
    assert not missing, f"declared but not exported: {missing}"
    for s in declared_symbols():
        assert getattr(lib, s) is not None
    # internal kernels and helpers stay hidden: the header is the whole ABI
    assert exported == set(declared_symbols()), sorted(exported ^ set(declared_symbols()))


def test_reference_ctypes_binding_still_works(lib):
    """The reference's exact ctypes signature (tests/test_gemm.py:194-197)."""
    raw = ctypes.CDLL(lib._name)
    fn = raw.gemm_launcher
    fn.argtypes = [ctypes.c_void_p] * 3 + [ctypes.c_int] * 3 + [ctypes.c_float] * 2
    fn.restype = None
    # M <= 0 returns before touching CUDA, so this is safe without a GPU.
    fn(None, None, None, 0, 16, 16, 1.0, 0.0)
    fn(None, None, None, 16, -1, 16, 1.0, 0.0)


@pytest.mark.parametrize("m,world", [(32768, 1), (32768, 2), (32768, 8), (10, 4), (3, 8), (0, 2),
                                     (1023, 7)])
def test_slab_rows_partition(lib, m, world):
    import gemm_b200
    covered = []
    sizes = []
    for r in range(world):
        row0, rows = gemm_b200.slab_rows(m, world, r)
        covered.extend(range(row0, row0 + rows))
        sizes.append(rows)
    assert covered == list(range(m))              # contiguous, disjoint, complete
    assert max(sizes) - min(sizes) <= 1           # balanced
    assert sizes == sorted(sizes, reverse=True)   # remainder on the low ranks


@pytest.mark.parametrize("args", [(-1, 2, 0), (8, 0, 0), (8, 2, 2), (8, 2, -1)])
def test_slab_rows_rejects_bad_arguments(lib, args):
    row0 = ctypes.c_int(0)
    assert lib.gemm_slab_rows(*args, ctypes.byref(row0)) == -1
    assert lib.gemm_slab_rows(8, 2, 0, None) == -1


def test_load_raises_when_library_missing(tmp_path):
    import gemm_b200
    with pytest.raises(gemm_b200.GemmError):
        gemm_b200.load(tmp_path / "nope.so")
