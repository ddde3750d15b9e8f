"""Host logic of the multi-GPU row-slab launcher on CPU ranks (gloo, world size 2).

The compute step is the CPU oracle (tests may use it as the checker), so these
cover partition, broadcast of B, per-rank slab work and reassembly without a
GPU. The failure tests inject on the host, with no GPU involved: one rank dies
before the broadcast, and the surviving rank must get an error from its
collective within the process-group timeout instead of hanging; or one rank
stays alive but never joins, and the other's host deadline (shorter than the
process-group timeout) must end its broadcast with CommDeadlineExceeded.
"""
import multiprocessing as mp
import os
import socket
import sys
import time
import traceback
from datetime import timedelta
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, scenario, q):
    try:
        sys.path[:0] = [str(REPO), str(REPO / "gemm-project_b200")]
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        import torch
        import torch.distributed as dist
        from oracle import oracle
        from gemm_b200.slab import SlabGemm

        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=timedelta(seconds=5))
        m, n, k, alpha, beta = 37, 24, 40, 0.75, -0.25
        if scenario == "overlapped":
            n = 37  # column blocks of 16, 16 and 5 (widths rounded up to multiples of 8)
        a, b_full, c = oracle.make_inputs(m, n, k, "uniform", seed=11)

        def cpu_compute(a_s, b_s, c_s, al, be):
            c_s.copy_(oracle.c_gemm(a_s, b_s, c_s, al, be))

        def cpu_compute_sub(a_s, b_s, c_v, al, be, max_sms):  # c_v: a column block of C
            c_v.copy_(oracle.c_gemm(a_s, b_s.contiguous(), c_v.contiguous(), al, be))

        sg = SlabGemm(compute=cpu_compute, compute_sub=cpu_compute_sub)
        row0, rows = sg.partition(m)
        if scenario == "overlapped":
            b = b_full.clone() if rank == 0 else torch.full_like(b_full, float("nan"))
            a_slab = a[row0:row0 + rows].contiguous()
            c_slab = c[row0:row0 + rows].clone()
            blocks = sg.broadcast_and_run(a_slab, b, c_slab, alpha, beta, chunks=3)
            assert [t.shape[1] for t in blocks] == [16, 16, 5]
            assert torch.equal(torch.cat(blocks, dim=1), b_full)
            plain = c[row0:row0 + rows].clone()
            cpu_compute(a_slab, b_full, plain, alpha, beta)
            assert torch.equal(c_slab, plain), "column blocks change the arithmetic"
            full = sg.gather_c(c_slab, m)
            if rank == 0:
                chk = oracle.check(full, oracle.reference_fp32(a, b_full, c, alpha, beta))
                q.put((rank, "ok" if chk.passed else f"mismatch {chk}", rows, row0))
            else:
                q.put((rank, "ok", rows, row0))
            dist.barrier()
            dist.destroy_process_group()
            return
        if scenario == "die_before_broadcast" and rank == 1:
            os._exit(3)  # this rank disappears without joining the collective
        if scenario == "stall_before_broadcast" and rank == 1:
            time.sleep(12)  # alive, but never joins the collective
            q.put((rank, "stalled", None, None))
            os._exit(0)
        b = b_full.clone() if rank == 0 else torch.zeros_like(b_full)
        t0 = time.time()
        try:
            if scenario == "stall_before_broadcast":
                # host deadline well below the 5 s process-group timeout
                sg.broadcast_b(b, deadline_s=1.0)
            else:
                sg.broadcast_b(b)
        except Exception as e:  # the surviving rank must see an error, not hang
            q.put((rank, "collective_error", round(time.time() - t0, 2), type(e).__name__))
            return
        assert torch.equal(b, b_full)
        a_slab = a[row0:row0 + rows].contiguous()
        c_slab = c[row0:row0 + rows].clone()
        sg.run(a_slab, b, c_slab, alpha, beta)
        full = sg.gather_c(c_slab, m)
        if rank == 0:
            ref = oracle.reference_fp32(a, b_full, c, alpha, beta)
            chk = oracle.check(full, ref)
            q.put((rank, "ok" if chk.passed else f"mismatch {chk}", rows, row0))
        else:
            q.put((rank, "ok", rows, row0))
        dist.barrier()
        dist.destroy_process_group()
    except Exception:
        q.put((rank, "exception", traceback.format_exc(), None))


def _spawn(world, scenario, wait_s=60):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, scenario, q)) for r in range(world)]
    for p in procs:
        p.start()
    deadline = time.time() + wait_s
    for p in procs:
        p.join(max(0.1, deadline - time.time()))
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
        p.join()
    out = []
    while not q.empty():
        out.append(q.get())
    return sorted(out, key=lambda x: x[0]), alive


def test_slab_gemm_two_ranks_matches_oracle():
    results, alive = _spawn(2, "normal")
    assert not alive, "a rank hung"
    assert [r[1] for r in results] == ["ok", "ok"], results
    # M = 37 over 2 ranks: 19 + 18 rows, remainder on rank 0
    assert (results[0][2], results[0][3]) == (19, 0)
    assert (results[1][2], results[1][3]) == (18, 19)


def test_overlapped_broadcast_two_ranks_matches_plain_path():
    """B broadcast as column blocks, each consumed as it lands (broadcast_and_run)."""
    results, alive = _spawn(2, "overlapped")
    assert not alive, "a rank hung"
    assert [r[1] for r in results] == ["ok", "ok"], results


def test_dead_rank_surfaces_as_error_not_hang():
    results, alive = _spawn(2, "die_before_broadcast", wait_s=60)
    assert not alive, "surviving rank hung instead of failing"
    assert len(results) == 1 and results[0][0] == 0, results
    assert results[0][1] == "collective_error", results
    assert results[0][2] < 30


def test_stalled_rank_hits_host_deadline():
    """A peer that is alive but never joins: the broadcast's host deadline (1 s)
    ends the wait well before the 5 s process-group timeout."""
    results, alive = _spawn(2, "stall_before_broadcast", wait_s=60)
    assert not alive, "a rank hung"
    by_rank = {r[0]: r for r in results}
    assert by_rank[0][1] == "collective_error", results
    assert by_rank[0][3] == "CommDeadlineExceeded", results
    assert by_rank[0][2] < 4.0, results


def test_reserve_schedule():
    """broadcast_and_run leaves SMs free only for blocks whose GEMM starts
    before the broadcast's modelled end (with its margin), never for the last."""
    sys.path.insert(0, str(REPO / "gemm-project_b200"))
    from gemm_b200.slab import SlabGemm

    k, widths = 16384, [4096] * 8
    # 4096-row slab: one block's GEMM (0.42 ms) is about twice one block's
    # broadcast (0.22 ms); the broadcast's end (1.8 ms, x1.5) falls in block 5
    assert SlabGemm.reserve_schedule(4096, k, widths) == [True] * 6 + [False] * 2
    # 8192-row slab: blocks 0-2 start before it
    assert SlabGemm.reserve_schedule(8192, k, widths) == [True] * 3 + [False] * 5
    # a slab so small that every GEMM finishes before the next block lands
    assert SlabGemm.reserve_schedule(16, k, widths) == [True] * 7 + [False]
    assert SlabGemm.reserve_schedule(4096, k, [8]) == [False]
    assert SlabGemm.reserve_schedule(4096, k, []) == []
