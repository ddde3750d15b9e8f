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
