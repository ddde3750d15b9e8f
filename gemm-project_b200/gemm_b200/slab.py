"""Multi-GPU launcher: C = alpha*A@B + beta*C sharded by C row slabs.

The reference is single-GPU (no NCCL, MPI or torch.distributed anywhere in it),
so this has no counterpart there. The partition is the natural one for a
row-major GEMM: rank r of R owns C rows [row0, row0 + rows) (remainder on the
low ranks, `gemm_slab_rows` in the C library), the matching contiguous A rows,
and a full replica of B. B is broadcast once from `src` over the process
group's backend (NCCL over NVLink/NVSwitch on B200s). Each rank then runs the
unchanged single-GPU `gemm_launcher_stream` on its slab: no reduction, no
collective inside a step, no kernel that reads another GPU's memory.

One process per GPU; the group comes from `torch.distributed`. The compute step
is injectable so the host logic (partition, broadcast, gather) is testable on
CPU ranks with the gloo backend.
"""
from __future__ import annotations

from typing import Callable, Optional

import torch
import torch.distributed as dist

from . import gemm as _gpu_gemm
from . import slab_rows


class SlabGemm:
    def __init__(self, group: Optional[dist.ProcessGroup] = None,
                 compute: Optional[Callable] = None):
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        # compute(a_slab, b, c_slab, alpha, beta) -> None (in place on c_slab)
        self.compute = compute or (lambda a, b, c, alpha, beta: _gpu_gemm(a, b, c, alpha, beta))

    def partition(self, m: int) -> tuple[int, int]:
        """(row0, rows) of this rank's C slab."""
        return slab_rows(m, self.world, self.rank)

    def broadcast_b(self, b: torch.Tensor, src: int = 0) -> torch.Tensor:
        """Replicate B from `src` into `b` on every rank (in place), once."""
        dist.broadcast(b, src=src, group=self.group)
        return b

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
