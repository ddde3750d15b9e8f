"""Python host side of the B200 FP16 GEMM library.

The library is native: every computation runs in `lib/libgemm.so` (built from
`csrc/` for sm_100a). This module only binds its C ABI with ctypes, the way the
reference's own harness binds its `gemm_launcher` (tests/test_gemm.py:194-197:
`argtypes = [c_void_p]*3 + [c_int]*3 + [c_float]*2`, `restype = None`), and
adds torch-tensor conveniences on top. There is no fallback: if the shared
library is missing or fails to load, `load()` raises.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

PKG_ROOT = Path(__file__).resolve().parent.parent
LIB_PATH = PKG_ROOT / "lib" / "libgemm.so"

PATH_AUTO, PATH_TC, PATH_ROWS, PATH_COL = 0, 1, 2, 3

_lib: ctypes.CDLL | None = None


class GemmError(RuntimeError):
    pass


def _bind(lib: ctypes.CDLL) -> ctypes.CDLL:
    vp, i, f = ctypes.c_void_p, ctypes.c_int, ctypes.c_float
    gemm8 = [vp, vp, vp, i, i, i, f, f]
    lib.gemm_launcher.argtypes = gemm8
    lib.gemm_launcher.restype = None
    lib.gemm_launcher_stream.argtypes = gemm8 + [vp]
    lib.gemm_launcher_stream.restype = None
    lib.gemm_launcher_ex.argtypes = gemm8 + [vp, i, i]
    lib.gemm_launcher_ex.restype = i
    lib.gemm_launcher_status.argtypes = []
    lib.gemm_launcher_status.restype = i
    lib.gemm_last_kernel.argtypes = []
    lib.gemm_last_kernel.restype = ctypes.c_char_p
    lib.gemm_cublas.argtypes = gemm8
    lib.gemm_cublas.restype = None
    lib.gemm_cublas_stream.argtypes = gemm8 + [vp]
    lib.gemm_cublas_stream.restype = None
    lib.gemm_slab_rows.argtypes = [i, i, i, ctypes.POINTER(i)]
    lib.gemm_slab_rows.restype = i
    lib.gemm_selftest_wait_timeout.argtypes = [i, vp]
    lib.gemm_selftest_wait_timeout.restype = i
    lib.gemm_launcher_noalloc.argtypes = gemm8 + [vp]
    lib.gemm_launcher_noalloc.restype = i
    lib.gemm_launcher_tn.argtypes = gemm8 + [vp, i]
    lib.gemm_launcher_tn.restype = i
    lib.launchGemmSample.argtypes = [vp, vp, vp, i, i, i, vp]
    lib.launchGemmSample.restype = ctypes.c_bool
    lib.gemm_launch_error.argtypes = []
    lib.gemm_launch_error.restype = i
    lib.gemm_launcher_sub.argtypes = [vp, i, vp, i, vp, i, i, i, i, f, f, vp, i]
    lib.gemm_launcher_sub.restype = i
    lib.gemm_selftest_stall.argtypes = [vp, vp, vp, i, i, i, i, i, i, vp]
    lib.gemm_selftest_stall.restype = i
    sz = ctypes.c_size_t
    lib.gemm_peer_export.argtypes = [vp, vp, ctypes.POINTER(ctypes.c_ulonglong)]
    lib.gemm_peer_export.restype = i
    lib.gemm_peer_open.argtypes = [vp, ctypes.POINTER(vp)]
    lib.gemm_peer_open.restype = i
    lib.gemm_peer_close.argtypes = [vp]
    lib.gemm_peer_close.restype = i
    lib.gemm_peer_copy2d.argtypes = [vp, sz, vp, sz, sz, sz, vp]
    lib.gemm_peer_copy2d.restype = i
    lib.gemm_peer_flags.argtypes = [vp, i, vp, i, vp, i, vp, i, ctypes.c_longlong, vp]
    lib.gemm_peer_flags.restype = i
    return lib


def load(path: str | os.PathLike | None = None) -> ctypes.CDLL:
    """Load (once) and bind libgemm.so. Raises GemmError if it is absent."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    p = Path(path) if path is not None else LIB_PATH
    if not p.exists():
        raise GemmError(f"{p} is missing: build it with `python gemm-project_b200/build.py`")
    lib = _bind(ctypes.CDLL(str(p)))
    if path is None:
        _lib = lib
    return lib


TORCH_OP_PATH = PKG_ROOT / "lib" / "libgemm_torch_op.so"
_torch_ops_loaded = False


def load_torch_ops(path: str | os.PathLike | None = None):
    """Register the PyTorch operators (torch.ops.trtllm_gemm_sample.gemm,
    torch.ops.gemm_b200.gemm, torch.ops.gemm_b200.linear) from
    libgemm_torch_op.so and return torch.ops. Raises GemmError if the library
    is absent (build it with `python gemm-project_b200/build.py --torch-op`)."""
    global _torch_ops_loaded
    import torch
    p = Path(path) if path is not None else TORCH_OP_PATH
    if not _torch_ops_loaded:
        if not p.exists():
            raise GemmError(f"{p} is missing: build it with "
                            "`python gemm-project_b200/build.py --torch-op`")
        torch.ops.load_library(str(p))
        _torch_ops_loaded = True
    return torch.ops


def _stream_handle(stream) -> int:
    if stream is None:
        import torch
        stream = torch.cuda.current_stream()
    return int(getattr(stream, "cuda_stream", stream))


def _check(a, b, c):
    import torch
    for name, t in (("A", a), ("B", b), ("C", c)):
        if t.dtype != torch.float16 or not t.is_cuda:
            raise GemmError(f"{name} must be a CUDA float16 tensor")
        if not t.is_contiguous():
            raise GemmError(f"{name} must be contiguous row-major")
    m, k = a.shape
    k2, n = b.shape
    if k2 != k or tuple(c.shape) != (m, n):
        raise GemmError(f"shape mismatch A{tuple(a.shape)} B{tuple(b.shape)} C{tuple(c.shape)}")
    return m, n, k


def gemm(a, b, c, alpha: float = 1.0, beta: float = 0.0, stream=None, path: int = PATH_AUTO,
         tile_n: int = 0) -> None:
    """C = half(alpha * A@B (FP32 accumulate) + beta * C), in place, on `stream`
    (torch's current stream by default). Asynchronous like the C entry point."""
    lib = load()
    m, n, k = _check(a, b, c)
    s = _stream_handle(stream)
    if path == PATH_AUTO and tile_n == 0:
        lib.gemm_launcher_stream(a.data_ptr(), b.data_ptr(), c.data_ptr(), m, n, k, alpha, beta, s)
    else:
        rc = lib.gemm_launcher_ex(a.data_ptr(), b.data_ptr(), c.data_ptr(), m, n, k, alpha, beta, s,
                                  path, tile_n)
        if rc != 0:
            raise GemmError(f"path {path} / tile_n {tile_n} cannot serve M={m} N={n} K={k}")


def gemm_sub(a, b, c, alpha: float = 1.0, beta: float = 0.0, stream=None, max_sms: int = 0) -> None:
    """C = half(alpha * A@B + beta * C) in place, where A, B, C may be row-strided
    views (unit column stride, e.g. a column block of a wider C), on at most
    `max_sms` SMs (0 = all). The dense tcgen05 path of gemm_launcher_sub."""
    import torch
    lib = load()
    for name, t in (("A", a), ("B", b), ("C", c)):
        if t.dtype != torch.float16 or not t.is_cuda or t.dim() != 2 or t.stride(1) != 1:
            raise GemmError(f"{name} must be a 2-D CUDA float16 tensor with unit column stride")
    m, k = a.shape
    k2, n = b.shape
    if k2 != k or tuple(c.shape) != (m, n):
        raise GemmError(f"shape mismatch A{tuple(a.shape)} B{tuple(b.shape)} C{tuple(c.shape)}")
    rc = lib.gemm_launcher_sub(a.data_ptr(), a.stride(0), b.data_ptr(), b.stride(0), c.data_ptr(),
                               c.stride(0), m, n, k, alpha, beta, _stream_handle(stream), max_sms)
    if rc != 0:
        raise GemmError(f"gemm_launcher_sub refused M={m} N={n} K={k} "
                        f"(pitches {a.stride(0)}, {b.stride(0)}, {c.stride(0)})")


_host_streams: dict = {}


def gemm_host(a, b, c, alpha: float = 1.0, beta: float = 0.0, out=None, slabs: int = 8,
              stream=None):
    """C = half(alpha * A@B + beta * C) for operands in HOST memory, computed on
    the current CUDA device; the result goes to `out` (a host tensor, default c).

    The transfers are pipelined over row slabs on three streams: B crosses to
    the device first, then each slab's rows of A (and of C when beta != 0);
    each slab's GEMM starts as soon as its rows have landed, and its rows of C
    go back while later slabs still travel. PCIe carries both directions at
    once, so a call costs about its host-to-device bytes / PCIe bandwidth
    instead of the sum of all transfers and the GEMM. Pinned host tensors are
    needed for the copies to overlap (pageable ones work, synchronously).
    Asynchronous like the device entry points: `stream` (a torch.cuda.Stream;
    default: the current stream) is ordered after the last copy back;
    synchronize it before reading `out`.

    B may instead be a contiguous CUDA tensor on the current device (a weight
    that stays resident, or a replica of B that a multi-GPU job broadcast once):
    then only A (and C) cross PCIe.
    """
    import torch
    b_resident = b.is_cuda
    for name, t in (("A", a), ("B", b), ("C", c)) + ((("out", out),) if out is not None else ()):
        on_device_ok = name == "B" and b_resident
        if (t.dtype != torch.float16 or (t.is_cuda and not on_device_ok) or t.dim() != 2
                or not t.is_contiguous()):
            raise GemmError(f"{name} must be a contiguous 2-D float16 host tensor"
                            + (" (B may be a CUDA tensor)" if name == "B" else ""))
    if b_resident and b.device.index != torch.cuda.current_device():
        raise GemmError("a device-resident B must be on the current CUDA device")
    m, k = a.shape
    k2, n = b.shape
    if k2 != k or tuple(c.shape) != (m, n) or (out is not None and tuple(out.shape) != (m, n)):
        raise GemmError(f"shape mismatch A{tuple(a.shape)} B{tuple(b.shape)} C{tuple(c.shape)}")
    if out is None:
        out = c
    if m == 0 or n == 0:
        return out
    dev = torch.device("cuda", torch.cuda.current_device())
    caller = torch.cuda.current_stream(dev) if stream is None else stream
    if dev.index not in _host_streams:
        _host_streams[dev.index] = tuple(torch.cuda.Stream(dev) for _ in range(3))
    h2d, comp, d2h = _host_streams[dev.index]
    read_c = beta != 0.0
    # slabs of whole 128-row tiles (one slab for small M)
    if m < 256 or slabs <= 1:
        rows = m
    else:
        rows = max(128, (-(-m // slabs)) // 128 * 128)
    bounds = [(r, min(m, r + rows)) for r in range(0, m, rows)]
    a_d = torch.empty((m, k), dtype=torch.float16, device=dev)
    b_d = b if b_resident else torch.empty((k, n), dtype=torch.float16, device=dev)
    c_d = torch.empty((m, n), dtype=torch.float16, device=dev)
    for t in (a_d, b_d, c_d):  # used on the side streams: keep them alive until those finish
        for s in (h2d, comp, d2h):
            t.record_stream(s)
    h2d.wait_stream(caller)
    b_done = torch.cuda.Event()
    with torch.cuda.stream(h2d):
        if not b_resident:
            b_d.copy_(b, non_blocking=True)
        b_done.record(h2d)
    done = None
    for r0, r1 in bounds:
        landed, computed = torch.cuda.Event(), torch.cuda.Event()
        with torch.cuda.stream(h2d):
            a_d[r0:r1].copy_(a[r0:r1], non_blocking=True)
            if read_c:
                c_d[r0:r1].copy_(c[r0:r1], non_blocking=True)
            landed.record(h2d)
        comp.wait_event(b_done)
        comp.wait_event(landed)
        gemm(a_d[r0:r1], b_d, c_d[r0:r1], alpha, beta, stream=comp)
        computed.record(comp)
        d2h.wait_event(computed)
        with torch.cuda.stream(d2h):
            out[r0:r1].copy_(c_d[r0:r1], non_blocking=True)
        done = torch.cuda.Event()
        done.record(d2h)
    caller.wait_event(done)
    return out


def gemm_tn(a, bt, c, alpha: float = 1.0, beta: float = 0.0, stream=None, tile_n: int = 0) -> None:
    """C = half(alpha * A @ Bt.T + beta * C) with Bt[N,K] (a linear layer's weight layout)."""
    lib = load()
    import torch
    for name, t in (("A", a), ("Bt", bt), ("C", c)):
        if t.dtype != torch.float16 or not t.is_cuda or not t.is_contiguous():
            raise GemmError(f"{name} must be a contiguous CUDA float16 tensor")
    m, k = a.shape
    n, k2 = bt.shape
    if k2 != k or tuple(c.shape) != (m, n):
        raise GemmError(f"shape mismatch A{tuple(a.shape)} Bt{tuple(bt.shape)} C{tuple(c.shape)}")
    rc = lib.gemm_launcher_tn(a.data_ptr(), bt.data_ptr(), c.data_ptr(), m, n, k, alpha, beta,
                              _stream_handle(stream), tile_n)
    if rc != 0:
        raise GemmError(f"gemm_launcher_tn refused tile_n={tile_n}")


def cublas(a, b, c, alpha: float = 1.0, beta: float = 0.0, stream=None) -> None:
    """cuBLAS comparator with the same semantics (benchmarks only)."""
    lib = load()
    m, n, k = _check(a, b, c)
    lib.gemm_cublas_stream(a.data_ptr(), b.data_ptr(), c.data_ptr(), m, n, k, alpha, beta,
                           _stream_handle(stream))


def status() -> int:
    """Sticky library status (0 = ok); see include/gemm_b200.h."""
    return int(load().gemm_launcher_status())


def last_kernel() -> str:
    return load().gemm_last_kernel().decode()


def slab_rows(m: int, world: int, rank: int) -> tuple[int, int]:
    """(row0, rows) of the C row slab that `rank` of `world` owns."""
    row0 = ctypes.c_int(0)
    rows = load().gemm_slab_rows(m, world, rank, ctypes.byref(row0))
    if rows < 0:
        raise GemmError(f"invalid slab request M={m} world={world} rank={rank}")
    return row0.value, rows
