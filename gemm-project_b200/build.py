"""Build libgemm.so (sm_100a) in-tree with nvcc.

Counterpart of the reference's build step (tools/project.py:126-139: `nvcc -O3
-std=c++17 -lineinfo -arch=$CUDA_ARCH --shared -fPIC -lcublas`, then `nm -D`
must show `T gemm_launcher`). Here the architecture is fixed to sm_100a, the
CUDA runtime is linked statically (so the library does not depend on which
libcudart torch loaded first), and only the C-ABI symbols are exported.

Usage: python gemm-project_b200/build.py [--force] [--torch-op]
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
REPO = PKG.parent
CSRC = PKG / "csrc"
LIB_DIR = PKG / "lib"
LIB = LIB_DIR / "libgemm.so"
SOURCES = [CSRC / "gemm_launcher.cu", CSRC / "cublas_ref.cu"]
DEPS = SOURCES + sorted(CSRC.glob("*.cuh")) + [REPO / "include" / "gemm_b200.h"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
EXPORTS = [
    "gemm_launcher", "gemm_launcher_stream", "gemm_launcher_ex", "gemm_launcher_status",
    "gemm_last_kernel", "gemm_cublas", "gemm_cublas_stream", "gemm_slab_rows",
    "gemm_selftest_wait_timeout", "gemm_launcher_noalloc", "gemm_launcher_tn",
    "launchGemmSample", "gemm_launch_error", "gemm_launcher_sub", "gemm_selftest_stall",
    "gemm_peer_export", "gemm_peer_open", "gemm_peer_close", "gemm_peer_copy2d", "gemm_peer_flags",
]


def nvcc() -> str:
    cuda_home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    cand = Path(cuda_home) / "bin" / "nvcc"
    if cand.exists():
        return str(cand)
    found = shutil.which("nvcc")
    if not found:
        raise RuntimeError("nvcc not found (set CUDA_HOME)")
    return found


def up_to_date() -> bool:
    if not LIB.exists():
        return False
    mtime = LIB.stat().st_mtime
    return all(p.stat().st_mtime <= mtime for p in DEPS)


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and up_to_date():
        return LIB
    LIB_DIR.mkdir(parents=True, exist_ok=True)
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [
        nvcc(), "-O3", "-std=c++17", *ARCH, "-lineinfo", "--shared",
        "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
        "-cudart", "static", f"-I{REPO / 'include'}",
        "-o", str(tmp), *map(str, SOURCES), "-lcublas",
        "-Xlinker", "-rpath=/usr/local/cuda/lib64",
    ]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"nvcc failed:\n{' '.join(cmd)}\n{proc.stdout}\n{proc.stderr}")
    if verbose:
        sys.stderr.write(proc.stderr)
    os.replace(tmp, LIB)
    check_exports(LIB)
    return LIB


TORCH_OP_SRC = CSRC / "torch_op.cpp"
TORCH_OP_LIB = LIB_DIR / "libgemm_torch_op.so"


def build_torch_op(force: bool = False) -> Path:
    """PyTorch operator library (trtllm_gemm_sample::gemm, gemm_b200::gemm,
    gemm_b200::linear) over libgemm.so, compiled with the host compiler against
    the installed torch headers; found next to libgemm.so through $ORIGIN."""
    lib = build(force=force)
    deps = [TORCH_OP_SRC, REPO / "include" / "gemm_b200.h", lib]
    if (not force and TORCH_OP_LIB.exists()
            and all(p.stat().st_mtime <= TORCH_OP_LIB.stat().st_mtime for p in deps)):
        return TORCH_OP_LIB
    import torch
    from torch.utils import cpp_extension

    cuda_home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    abi = 1 if torch.compiled_with_cxx11_abi() else 0
    torch_lib = cpp_extension.library_paths()[0]
    tmp = TORCH_OP_LIB.with_suffix(".so.tmp")
    cmd = [
        os.environ.get("CXX", "g++"), "-O2", "-std=c++17", "-fPIC", "-shared",
        f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
        *[f"-I{p}" for p in cpp_extension.include_paths()],
        f"-I{cuda_home}/include", f"-I{REPO / 'include'}",
        str(TORCH_OP_SRC), "-o", str(tmp),
        f"-L{LIB_DIR}", "-lgemm", "-Wl,-rpath,$ORIGIN",
        f"-L{torch_lib}", "-lc10", "-lc10_cuda", "-ltorch_cpu", "-ltorch", f"-Wl,-rpath,{torch_lib}",
    ]
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"torch op build failed:\n{' '.join(cmd)}\n{proc.stdout}\n{proc.stderr}")
    os.replace(tmp, TORCH_OP_LIB)
    return TORCH_OP_LIB


def check_exports(lib: Path) -> None:
    """The reference's build gate (tools/project.py:137-138), for every entry point."""
    out = subprocess.run(["nm", "-D", "--defined-only", str(lib)], capture_output=True, text=True,
                         check=True).stdout
    have = {line.split()[-1] for line in out.splitlines() if " T " in line}
    missing = [s for s in EXPORTS if s not in have]
    if missing:
        raise RuntimeError(f"{lib} does not export {missing}")


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    ap.add_argument("--torch-op", action="store_true", help="also build libgemm_torch_op.so")
    args = ap.parse_args()
    print(build(force=args.force, verbose=args.verbose))
    if args.torch_op:
        print(build_torch_op(force=args.force))
