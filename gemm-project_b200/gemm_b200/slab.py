"""Multi-GPU launcher: C = alpha*A@B + beta*C sharded by C row slabs.

The reference is single-GPU (no NCCL, MPI or torch.distributed anywhere in it),
so this has no counterpart there. The partition is the natural one for a
row-major GEMM: rank r of R owns C rows [row0, row0 + rows) (remainder on the
low ranks, `gemm_slab_rows` in the C library), the matching contiguous A rows,
and a full replica of B. B is broadcast once from `src` over the process
group's backend (NCCL over NVLink/NVSwitch on B200s). Each rank then runs the
unchanged single-GPU `gemm_launcher_stream` on its slab: no reduction, no
collective inside a step, no kernel that reads another GPU's memory.

`broadcast_and_run` overlaps that broadcast with the GEMM. B travels as column
blocks, and each rank computes C[:, block] = A @ B[:, block] as soon as the block
has landed, while the next blocks are still in flight. Every output element
still takes its whole K range in one kernel, so the arithmetic is that of the
plain path. Splitting along K would instead round C to FP16 between blocks.

`PeerRing` does the same without NCCL: B's column chunks travel along a ring of
the ranks by copy-engine copies from the predecessor's IPC-mapped replica, so
the slab GEMM keeps every SM but one pair, where NCCL's kernels needed 16. The
ranks order the copies through flag words in each other's memory, set and
awaited by a one-thread kernel with a bounded wait (`ring_program` states the
protocol; the library's gemm_peer_* entry points carry it out).

One process per GPU; the group comes from `torch.distributed`. The compute steps
are injectable so the host logic (partition, broadcast, gather) is testable on
CPU ranks with the gloo backend.

Failure detection: the broadcasts take an optional host deadline. The host then
polls the collective's completion and the communicator's asynchronous error
state; when the deadline passes or an error appears, it aborts the group's
communicators (ncclCommAbort under NCCL, which also ends a collective still
waiting for a peer) and raises CommDeadlineExceeded, so that a rank that died
or stalled surfaces as an error within the deadline instead of a hang. The
group that carries broadcast_and_run's blocks uses non-blocking NCCL
communicators, whose calls never hold the host.
"""
from __future__ import annotations

import ctypes
import time
from typing import Callable, Optional

import torch
import torch.distributed as dist

from . import gemm as _gpu_gemm
from . import gemm_sub as _gpu_gemm_sub
from . import slab_rows


class CommDeadlineExceeded(RuntimeError):
    """A collective did not complete within its host deadline (or its
    communicator reported an asynchronous error); the group was aborted."""


def _gpu_compute_sub(a, b_block, c_view, alpha, beta, max_sms):
    """The dense kernel on strided views with an SM cap (gemm_launcher_sub).
    An A slab that the kernel cannot read in place (K % 8 != 0 or a base that
    is not 16-byte aligned) goes through the regular entry point on contiguous
    copies instead, without the SM cap."""
    k = a.shape[1]
    if k % 8 == 0 and a.data_ptr() % 16 == 0:
        _gpu_gemm_sub(a, b_block, c_view, alpha, beta, max_sms=max_sms)
        return
    c_tmp = c_view.contiguous()
    _gpu_gemm(a.contiguous(), b_block.contiguous(), c_tmp, alpha, beta)
    c_view.copy_(c_tmp)


class SlabGemm:
    def __init__(self, group: Optional[dist.ProcessGroup] = None,
                 compute: Optional[Callable] = None, compute_sub: Optional[Callable] = None,
                 bcast_group: Optional[dist.ProcessGroup] = None):
        self.group = group
        # group that carries broadcast_and_run's blocks (see broadcast_group())
        self.bcast_group = bcast_group if bcast_group is not None else group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        # compute(a_slab, b, c_slab, alpha, beta) -> None (in place on c_slab)
        self.compute = compute or (lambda a, b, c, alpha, beta: _gpu_gemm(a, b, c, alpha, beta))
        # compute_sub(a_slab, b_block, c_view, alpha, beta, max_sms) -> None, where
        # b_block may be a row-strided view and c_view is a column block of C
        # (row pitch = C's width)
        self.compute_sub = compute_sub or _gpu_compute_sub

    def partition(self, m: int) -> tuple[int, int]:
        """(row0, rows) of this rank's C slab."""
        return slab_rows(m, self.world, self.rank)

    def broadcast_b(self, b: torch.Tensor, src: int = 0,
                    deadline_s: Optional[float] = None) -> torch.Tensor:
        """Replicate B from `src` into `b` on every rank (in place), once.
        With `deadline_s`, the host waits at most that long for the broadcast
        to complete (see await_works)."""
        if deadline_s is None:
            dist.broadcast(b, src=src, group=self.group)
            return b
        work = dist.broadcast(b, src=src, group=self.group, async_op=True)
        self.await_works([work], deadline_s, self.group, "broadcast of B")
        return b

    @staticmethod
    def _comm_error(group) -> Optional[str]:
        """The asynchronous error state of the group's NCCL communicators
        (ncclCommGetAsyncError as torch reports it), or None."""
        pg = group if group is not None else dist.distributed_c10d._get_default_group()
        try:
            backend = pg._get_backend(torch.device("cuda"))
        except Exception:
            return None
        get_error = getattr(backend, "get_error", None)
        if get_error is None:
            return None
        err = str(get_error())
        return None if err.endswith("SUCCESS") else err

    @staticmethod
    def abort(group) -> None:
        """Abort the group's communicators (ncclCommAbort for NCCL). Backends
        without an abort (gloo) are left to their own process-group timeout."""
        pg = group if group is not None else dist.distributed_c10d._get_default_group()
        try:
            pg.abort()
        except Exception:
            pass

    def await_works(self, works, deadline_s: float, group, what: str) -> None:
        """Poll `works` (async collective handles) on the host until all have
        completed, for at most `deadline_s` seconds. If the deadline passes, or
        the communicator reports an asynchronous error first, abort the group
        and raise CommDeadlineExceeded; an error the backend raised itself is
        re-raised as CommDeadlineExceeded too, after the same abort."""
        t0 = time.monotonic()
        try:
            while True:
                if all(w.is_completed() for w in works):
                    for w in works:
                        w.wait()
                    return
                err = self._comm_error(group)
                if err is not None:
                    raise CommDeadlineExceeded(f"{what}: communicator error {err}")
                if time.monotonic() - t0 > deadline_s:
                    raise CommDeadlineExceeded(
                        f"{what}: not complete after {deadline_s:.3g} s (a peer stalled or died)")
                time.sleep(0.0005)
        except CommDeadlineExceeded:
            self.abort(group)
            raise
        except Exception as e:
            self.abort(group)
            raise CommDeadlineExceeded(f"{what}: {type(e).__name__}: {e}") from e

    @staticmethod
    def broadcast_group(ranks: list[int], max_ctas: int,
                        nonblocking: bool = True) -> dist.ProcessGroup:
        """A NCCL group for broadcast_and_run whose collectives use at most
        `max_ctas` CTAs, on a high-priority stream. With the GEMM leaving that
        many SMs free, every broadcast CTA finds an SM. Otherwise a ring
        channel whose CTA cannot be scheduled stalls its peers until the GEMM
        ends, and the overlap is lost. Its communicators are non-blocking
        (NCCL config `blocking = 0`), so a deadline can abort them. Collective:
        every rank calls it."""
        opts = dist.ProcessGroupNCCL.Options()
        opts.config.max_ctas = max_ctas
        opts.config.min_ctas = 1
        if nonblocking:
            opts.config.blocking = 0
        opts.is_high_priority_stream = True
        return dist.new_group(ranks=ranks, backend="nccl", pg_options=opts)

    # Rates for broadcast_and_run's SM reservation model (measured on B200s: NCCL
    # broadcast over NVLink 580-680 GB/s, the slab GEMM 1.2-1.5 PFLOP/s), and the
    # margin on the broadcast's modelled end. A block that takes every SM while
    # a broadcast kernel is still queued stalls the broadcast for a whole block
    # GEMM, while reserving SMs one block too long costs about a tenth of one,
    # so the margin errs on the long side.
    BCAST_BYTES_PER_S = 6.0e11
    GEMM_FLOP_PER_S = 1.3e15
    BCAST_MARGIN = 1.5

    @classmethod
    def reserve_schedule(cls, rows: int, k: int, widths: list[int], elem_bytes: int = 2) -> list[bool]:
        """For each column block of broadcast_and_run, whether its GEMM leaves
        SMs free for the broadcast: True while the block's modelled start
        (one block's broadcast plus the earlier blocks' GEMMs) falls before
        BCAST_MARGIN times the modelled end of the whole broadcast. The last
        block never reserves (nothing is left to broadcast after it lands)."""
        total = sum(widths)
        t_end = cls.BCAST_MARGIN * k * total * elem_bytes / cls.BCAST_BYTES_PER_S
        start = k * widths[0] * elem_bytes / cls.BCAST_BYTES_PER_S if widths else 0.0
        out = []
        for j, w in enumerate(widths):
            out.append(j + 1 < len(widths) and start < t_end)
            start += 2.0 * rows * w * k / cls.GEMM_FLOP_PER_S
        return out

    def broadcast_and_run(self, a_slab: torch.Tensor, b: torch.Tensor, c_slab: torch.Tensor,
                          alpha: float = 1.0, beta: float = 0.0, src: int = 0, chunks: int = 8,
                          reserve_sms: int = 16,
                          deadline_s: Optional[float] = None) -> list[torch.Tensor]:
        """broadcast_b(b, src) followed by run(...), overlapped.

        B[K, N] (filled on `src`; its contents elsewhere are ignored) is split
        into `chunks` column blocks (widths rounded up to multiples of 8; the
        last block takes the rest). On `src` each block is packed,
        and all blocks are broadcast asynchronously in order. Each rank's stream
        waits for block j, then computes C[:, block j] = alpha * A @ B[:, block j]
        + beta * C[:, block j] while blocks j+1.. are in flight. While blocks are
        still in flight the GEMM leaves `reserve_sms` SMs free, because the
        collective's kernels cannot start while a persistent GEMM holds every
        SM; the blocks computed after the broadcast has ended take every SM.
        Which blocks those are comes from reserve_schedule's model of the two
        rates. Returns the
        blocks, which hold this rank's replica of B in column-block layout.
        Ranks must call it collectively with the same chunks. With
        `deadline_s`, the host then waits at most that long for every block
        to arrive (await_works), so the call returns only after the broadcast."""
        k, n = b.shape
        # block widths are multiples of 8 columns (the last one takes the rest),
        # and every block is stored with a row pitch rounded up to 8 halves, so
        # each is a TMA-addressable operand of the dense kernel whatever N is
        width = -(-(-(-n // chunks)) // 8) * 8
        bounds = [(c0, min(n, c0 + width)) for c0 in range(0, n, width)]
        blocks, works = [], []
        for c0, c1 in bounds:
            pitch = -(-(c1 - c0) // 8) * 8
            store = torch.empty((k, pitch), dtype=b.dtype, device=b.device)
            blk = store[:, :c1 - c0]
            if self.rank == src:
                blk.copy_(b[:, c0:c1])
            works.append(dist.broadcast(store, src=src, group=self.bcast_group, async_op=True))
            blocks.append(blk)
        total_sms = (torch.cuda.get_device_properties(b.device).multi_processor_count
                     if b.is_cuda else 0)
        reserve = self.reserve_schedule(a_slab.shape[0], k, [c1 - c0 for c0, c1 in bounds],
                                        b.element_size())
        for (c0, c1), blk, work, pending in zip(bounds, blocks, works, reserve):
            work.wait()  # this stream waits for block j; the host does not block
            max_sms = max(2, total_sms - reserve_sms) if (pending and total_sms) else 0
            if a_slab.shape[0]:
                self.compute_sub(a_slab, blk, c_slab[:, c0:c1], alpha, beta, max_sms)
        if deadline_s is not None:
            self.await_works(works, deadline_s, self.bcast_group, "column-block broadcast of B")
        return blocks

    def run(self, a_slab: torch.Tensor, b: torch.Tensor, c_slab: torch.Tensor, alpha: float = 1.0,
            beta: float = 0.0) -> None:
        """This rank's share of the GEMM (no communication)."""
        if a_slab.shape[0]:
            self.compute(a_slab, b, c_slab, alpha, beta)

    def gather_c(self, c_slab: torch.Tensor, m: int) -> Optional[torch.Tensor]:
        """Assemble the full C on rank 0 (verification only; not part of a step).
        Slabs differ by at most one row, so each is padded to the largest."""
        n = c_slab.shape[1]
        max_rows = slab_rows(m, self.world, 0)[1]
        padded = torch.zeros((max_rows, n), dtype=c_slab.dtype, device=c_slab.device)
        padded[:c_slab.shape[0]] = c_slab
        parts = [torch.empty_like(padded) for _ in range(self.world)]
        dist.all_gather(parts, padded, group=self.group)
        if self.rank != 0:
            return None
        rows = [slab_rows(m, self.world, r)[1] for r in range(self.world)]
        return torch.cat([p[:r] for p, r in zip(parts, rows)], dim=0)


# ---------------------------------------------------------------------------
# Copy-engine ring (PeerRing)
# ---------------------------------------------------------------------------
def ring_layout(n: int, chunk_cols: int = 2048, block_cols: int = 4096, first_chunk_cols: int = 512,
                first_block_cols: int = 2048) -> tuple[list, list]:
    """Column chunks and GEMM blocks of PeerRing over N = n columns, as
    ([(c0, c1) per chunk], [end chunk index per block]).

    Chunk widths start at first_chunk_cols and double up to chunk_cols, so that
    the first columns cross the ring's hops quickly; the last chunk takes the
    rest. A GEMM block is a run of whole chunks: the first one ends at the first
    chunk boundary at or past first_block_cols, each later one at the first
    boundary at least block_cols further on; a remainder narrower than half a
    block joins the last full block. All widths are multiples of 8 columns."""
    for v in (chunk_cols, block_cols, first_chunk_cols, first_block_cols):
        if v < 8 or v % 8:
            raise ValueError("chunk and block widths must be positive multiples of 8")
    bounds, c0, w = [], 0, min(first_chunk_cols, chunk_cols)
    while c0 < n:
        bounds.append((c0, min(n, c0 + w)))
        c0 += w
        w = min(2 * w, chunk_cols)
    block_ends, target = [], first_block_cols
    for j, (_, c1) in enumerate(bounds):
        # a remainder under half a block joins this block instead of running alone
        if j == len(bounds) - 1 or (c1 >= target and n - c1 >= block_cols // 2):
            block_ends.append(j + 1)
            target = c1 + block_cols
    return bounds, block_ends


def ring_program(position: int, world: int, n_chunks: int, block_ends: list[int],
                 seq: int) -> tuple[list, list]:
    """The operations one rank issues in call `seq` (1, 2, ...) of PeerRing, as
    (copy_stream_ops, compute_stream_ops). `position` is the rank's place on the
    ring (0 = the source, which holds B; position p copies from p - 1). GEMM
    block g covers chunks [block_ends[g - 1], block_ends[g]).

    Each rank owns two flag words, both monotone counters over the calls:
    `ready`, set by its predecessor to the number of chunks it may copy so far,
    and `consumed`, set by its successor to the number of chunks the successor
    has copied. With n = n_chunks and base = (seq - 1) * n:

    copy stream (positions >= 1):
      ("join_compute",)           wait for this rank's earlier compute-stream work
                                  (the previous call's GEMMs read the replica)
      for chunk j:
        ("flags", signals, waits) signal ready_succ = base + j (chunk j - 1 is
                                  here), then wait until ready >= base + j + 1
        ("copy", j)               chunk j from the predecessor's replica
        ("block_ready", g)        after the last chunk of GEMM block g
      ("flags", signals, [])      ready_succ = consumed_pred = base + n
      ("block_ready", last)       the last block's only after that final signal,
                                  since its GEMM leaves no SM free
    compute stream:
      position 0 first signals ready_succ = base + n: all of B is there;
      ("gemm", g, reserve)        block g, after its block_ready on positions
                                  >= 1; `reserve` asks the GEMM to leave SMs
                                  free for the copy stream's flag kernels
      a rank with a successor ends with a wait until consumed >= base + n, so
      that neither the caller (on position 0) nor the next call overwrites
      chunks the successor is still copying.

    A signal is ("succ" | "pred", "ready" | "consumed", value); a wait is
    ("ready" | "consumed", value), satisfied once the word minus the value is
    >= 0."""
    if not (0 <= position < world and n_chunks >= 1 and seq >= 1 and block_ends
            and block_ends[-1] == n_chunks
            and all(a < b for a, b in zip([0] + block_ends, block_ends))):
        raise ValueError("bad ring program arguments")
    n_blocks = len(block_ends)
    ends = set(block_ends[:-1])
    base = (seq - 1) * n_chunks
    has_succ = position + 1 < world
    copy_ops, compute_ops = [], []
    if position == 0:
        if has_succ:
            compute_ops.append(("flags", [("succ", "ready", base + n_chunks)], []))
        compute_ops += [("gemm", g, False) for g in range(n_blocks)]
    else:
        copy_ops.append(("join_compute",))
        for j in range(n_chunks):
            signals = [("succ", "ready", base + j)] if (has_succ and j > 0) else []
            copy_ops.append(("flags", signals, [("ready", base + j + 1)]))
            copy_ops.append(("copy", j))
            if j + 1 in ends:
                copy_ops.append(("block_ready", block_ends.index(j + 1)))
        final = [("succ", "ready", base + n_chunks)] if has_succ else []
        copy_ops.append(("flags", final + [("pred", "consumed", base + n_chunks)], []))
        # the last block's GEMM takes every SM, so it starts only after the
        # final signal has gone out
        copy_ops.append(("block_ready", n_blocks - 1))
        compute_ops += [("gemm", g, g + 1 < n_blocks) for g in range(n_blocks)]
    if has_succ:
        compute_ops.append(("flags", [], [("consumed", base + n_chunks)]))
    return copy_ops, compute_ops


class PeerRing:
    """B replicated from `src` to every rank of `group` by copy engines along a
    ring, and the row-slab GEMM run block by block as B's column chunks land.

    `b` is this rank's [K, N] FP16 replica buffer, contiguous, on this rank's
    GPU. On `src` it holds B (the caller writes it, in stream order, before each
    call); elsewhere every call overwrites it with B, so it doubles as the
    resident replica afterwards. Construction is collective: the ranks exchange
    IPC handles of their replicas and flag words and map their ring neighbours'.
    Every rank must be on its own GPU (checked): the flag kernels of two ranks
    that wait on each other must never share one.

    Chunks and GEMM blocks follow ring_layout (chunk widths growing from
    first_chunk_cols to chunk_cols; blocks of first_block_cols, then block_cols).
    The chunks are the same on every rank; the GEMM blocks are this rank's own
    and may differ per call: with block_cols None they are 8192 columns wide for
    slabs of 6144 rows or more and 4096 below (measured on 4 B200s with K=16384:
    4096-row slabs 3.50 ms against 3.87 with 8192-column blocks, 8192-row slabs
    6.87 ms against 7.80 with 4096-column blocks). Chunks move by
    cudaMemcpy2DAsync on a high-priority stream. Every output element takes its
    whole K range in one kernel, so C is bit-identical to the plain path."""

    def __init__(self, b: torch.Tensor, group: Optional[dist.ProcessGroup] = None, src: int = 0,
                 chunk_cols: int = 2048, block_cols: Optional[int] = None,
                 first_chunk_cols: int = 512, first_block_cols: int = 2048, reserve_sms: int = 2,
                 timeout_s: float = 10.0, compute_sub: Optional[Callable] = None):
        if b.dtype != torch.float16 or not b.is_cuda or b.dim() != 2 or not b.is_contiguous():
            raise ValueError("b must be a contiguous 2-D CUDA float16 tensor")
        from . import load
        self.lib = load()
        self.group, self.b = group, b
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.src = src
        self.k, self.n = b.shape
        self.layout_args = (chunk_cols, block_cols, first_chunk_cols, first_block_cols)
        self.bounds, _ = ring_layout(self.n, chunk_cols, 4096, first_chunk_cols, first_block_cols)
        self.block_ends, self.blocks = self.block_layout(4096 if block_cols is None else 0)
        self.reserve_sms = reserve_sms
        self.timeout_us = int(timeout_s * 1e6)
        self.compute_sub = compute_sub or _gpu_compute_sub
        self.position = (self.rank - src) % self.world
        self.seq = 0
        self.flags = torch.zeros(2, dtype=torch.int32, device=b.device)  # [ready, consumed]
        self.copy_stream = torch.cuda.Stream(device=b.device, priority=-1)
        self.events = [torch.cuda.Event() for _ in self.bounds]
        self.total_sms = torch.cuda.get_device_properties(b.device).multi_processor_count
        self._mapped: dict[bytes, int] = {}
        torch.cuda.synchronize(b.device)

        mine = {"b": self._export(b), "flags": self._export(self.flags),
                "uuid": str(torch.cuda.get_device_properties(b.device).uuid),
                "shape": (self.k, self.n, tuple(self.bounds), src)}
        everyone = [None] * self.world
        dist.all_gather_object(everyone, mine, group=group)
        if len({e["uuid"] for e in everyone}) != self.world:
            raise RuntimeError("PeerRing needs one GPU per rank; two ranks share a GPU")
        if len({e["shape"] for e in everyone}) != 1:
            raise ValueError("ranks disagree on B's shape or the ring's chunking")
        ring = [(src + p) % self.world for p in range(self.world)]
        self.pred = ring[self.position - 1] if self.position > 0 else None
        self.succ = ring[self.position + 1] if self.position + 1 < self.world else None
        self.pred_b = self.pred_flags = self.succ_flags = None
        if self.pred is not None:
            self.pred_b = self._open(everyone[self.pred]["b"])
            self.pred_flags = self._open(everyone[self.pred]["flags"])
        if self.succ is not None:
            self.succ_flags = self._open(everyone[self.succ]["flags"])
        self.closed = False
        dist.barrier(group=group)

    def block_layout(self, rows: int) -> tuple[list, list]:
        """(block end chunk indices, [(c0, c1) per GEMM block]) for a slab of
        `rows` rows."""
        chunk_cols, block_cols, first_chunk_cols, first_block_cols = self.layout_args
        if block_cols is None:
            block_cols = 8192 if rows >= 6144 else 4096
        _, ends = ring_layout(self.n, chunk_cols, block_cols, first_chunk_cols, first_block_cols)
        return ends, [(self.bounds[j0][0], self.bounds[j1 - 1][1])
                      for j0, j1 in zip([0] + ends[:-1], ends)]

    def _export(self, t: torch.Tensor) -> tuple[bytes, int]:
        handle = ctypes.create_string_buffer(64)
        offset = ctypes.c_ulonglong()
        if self.lib.gemm_peer_export(t.data_ptr(), handle, ctypes.byref(offset)) != 0:
            raise RuntimeError(f"gemm_peer_export failed (CUDA error {self.lib.gemm_launch_error()})")
        return handle.raw, offset.value

    def _open(self, exported: tuple[bytes, int]) -> int:
        handle, offset = exported
        if handle not in self._mapped:
            base = ctypes.c_void_p()
            if self.lib.gemm_peer_open(handle, ctypes.byref(base)) != 0:
                raise RuntimeError(f"gemm_peer_open failed (CUDA error {self.lib.gemm_launch_error()})")
            self._mapped[handle] = base.value
        return self._mapped[handle] + offset

    def close(self) -> None:
        """Unmap the neighbours' memory (collective: after every rank's last
        call has completed on the device)."""
        torch.cuda.synchronize(self.b.device)
        dist.barrier(group=self.group)
        for base in self._mapped.values():
            self.lib.gemm_peer_close(base)
        self._mapped.clear()
        self.pred_b = self.pred_flags = self.succ_flags = None
        self.closed = True

    def _flags(self, signals, waits, stream) -> None:
        sig = [(None, 0), (None, 0)]
        for i, (who, which, value) in enumerate(signals):
            base = self.succ_flags if who == "succ" else self.pred_flags
            sig[i] = (base + (0 if which == "ready" else 4), value)
        wt = [(None, 0), (None, 0)]
        for i, (which, value) in enumerate(waits):
            wt[i] = (self.flags.data_ptr() + (0 if which == "ready" else 4), value)
        if self.lib.gemm_peer_flags(sig[0][0], sig[0][1], sig[1][0], sig[1][1], wt[0][0], wt[0][1],
                                    wt[1][0], wt[1][1], self.timeout_us, stream.cuda_stream) != 0:
            raise RuntimeError("gemm_peer_flags launch failed")

    def broadcast_and_run(self, a_slab: torch.Tensor, c_slab: torch.Tensor, alpha: float = 1.0,
                          beta: float = 0.0, deadline_s: Optional[float] = None) -> torch.Tensor:
        """One call (collective, every rank in the same order): B from `src`
        into every rank's replica, and this rank's C slab = alpha * A_slab @ B +
        beta * C_slab, block by block as B's chunks land. Asynchronous on the
        current stream; returns the replica. With `deadline_s`, the host waits
        for the call to finish on the device for at most that long and raises
        CommDeadlineExceeded if it did not, or if a flag wait ran out (library
        status 1006)."""
        if self.closed:
            raise RuntimeError("PeerRing is closed")
        self.seq += 1
        compute = torch.cuda.current_stream(self.b.device)
        self.block_ends, self.blocks = self.block_layout(a_slab.shape[0])
        copy_ops, compute_ops = ring_program(self.position, self.world, len(self.bounds),
                                             self.block_ends, self.seq)
        esz = self.b.element_size()
        row_bytes = self.n * esz
        for op in copy_ops:
            if op[0] == "join_compute":
                self.copy_stream.wait_stream(compute)
            elif op[0] == "flags":
                self._flags(op[1], op[2], self.copy_stream)
            elif op[0] == "copy":
                c0, c1 = self.bounds[op[1]]
                if self.lib.gemm_peer_copy2d(self.b.data_ptr() + c0 * esz, row_bytes,
                                             self.pred_b + c0 * esz, row_bytes, (c1 - c0) * esz,
                                             self.k, self.copy_stream.cuda_stream) != 0:
                    raise RuntimeError("gemm_peer_copy2d failed")
            elif op[0] == "block_ready":
                self.events[op[1]].record(self.copy_stream)
        for op in compute_ops:
            if op[0] == "flags":
                self._flags(op[1], op[2], compute)
            elif op[0] == "gemm":
                g, reserve = op[1], op[2]
                if self.position > 0:
                    compute.wait_event(self.events[g])
                c0, c1 = self.blocks[g]
                max_sms = max(2, self.total_sms - self.reserve_sms) if reserve else 0
                if a_slab.shape[0]:
                    self.compute_sub(a_slab, self.b[:, c0:c1], c_slab[:, c0:c1], alpha, beta, max_sms)
        if deadline_s is not None:
            done = torch.cuda.Event()
            done.record(compute)
            t0 = time.monotonic()
            while not done.query():
                if time.monotonic() - t0 > deadline_s:
                    raise CommDeadlineExceeded(
                        f"ring broadcast of B: not complete after {deadline_s:.3g} s")
                time.sleep(0.0005)
            from . import status
            st = status()
            if st == 1006:
                raise CommDeadlineExceeded("ring broadcast of B: a peer flag wait ran out")
            if st != 0:
                raise RuntimeError(f"ring broadcast of B: library status {st}")
        return self.b
