"""One rank of tests/test_multigpu_nccl.py (launched by torchrun, one process per GPU).

Runs the multi-GPU row-slab launcher on real GPUs over NCCL and checks it against
the CPU oracle: SlabGemm.broadcast_b + run, the overlapped
broadcast_and_run (B in column blocks), and PeerRing (B along a ring of
copy-engine copies, three calls in a row with B rewritten on the source before
the last), each on a ragged shape (M not a
multiple of the rank count or of the tile heights, N and K not multiples of
the tile widths), with beta != 0 and with beta == 0 over a NaN-filled C. The
slabs are gathered with gather_c and rank 0 compares the whole C with the
oracle; every rank also checks its own replica of B. Each rank prints one line
`RESULT <rank> <ok|failure text>`.
"""
import os
import sys
import traceback
from datetime import timedelta
from pathlib import Path

REPO = Path(__file__).resolve().parent.parent
sys.path[:0] = [str(REPO), str(REPO / "gemm-project_b200")]


def main():
    import torch
    import torch.distributed as dist
    import gemm_b200
    from gemm_b200.slab import PeerRing, SlabGemm
    from oracle import oracle

    rank = int(os.environ["RANK"])
    world = int(os.environ["WORLD_SIZE"])
    dev = torch.device("cuda", int(os.environ["LOCAL_RANK"]))
    torch.cuda.set_device(dev)
    gemm_b200.load()
    dist.init_process_group("nccl", timeout=timedelta(seconds=60), device_id=dev)
    failures = []
    try:
        m, n, k = 1037, 2056, 1000
        a, b_full, c0 = oracle.make_inputs(m, n, k, "uniform", seed=41)
        for alpha, beta in ((0.75, -0.25), (1.0, 0.0)):
            sg = SlabGemm()
            row0, rows = sg.partition(m)
            b = b_full.to(dev) if rank == 0 else torch.full((k, n), float("nan"), device=dev,
                                                            dtype=torch.float16)
            sg.broadcast_b(b, deadline_s=30.0)
            if not torch.equal(b.cpu(), b_full):
                failures.append(f"B replica differs (beta={beta})")
            a_slab = a[row0:row0 + rows].to(dev)
            c_init = c0[row0:row0 + rows] if beta != 0 else torch.full((rows, n), float("nan"),
                                                                       dtype=torch.float16)
            ref = oracle.reference_fp32(a, b_full, c0, alpha, beta) if rank == 0 else None
            # plain: broadcast, then each rank's slab GEMM
            c_slab = c_init.to(dev)
            sg.run(a_slab, b, c_slab, alpha, beta)
            torch.cuda.synchronize()
            full = sg.gather_c(c_slab, m)
            if rank == 0:
                chk = oracle.check(full, ref)
                if not chk.passed:
                    failures.append(f"run beta={beta}: {chk}")
            # overlapped: B in 3 column blocks, each consumed as it lands
            bgroup = SlabGemm.broadcast_group(list(range(world)), 16)
            sg2 = SlabGemm(bcast_group=bgroup)
            b2 = b_full.to(dev) if rank == 0 else torch.full((k, n), float("nan"), device=dev,
                                                             dtype=torch.float16)
            c2 = c_init.to(dev)
            blocks = sg2.broadcast_and_run(a_slab, b2, c2, alpha, beta, chunks=3, reserve_sms=16,
                                           deadline_s=30.0)
            torch.cuda.synchronize()
            if [t.shape[1] for t in blocks] != [688, 688, 680]:
                failures.append(f"block widths {[t.shape[1] for t in blocks]}")
            if not torch.equal(torch.cat([t.cpu() for t in blocks], dim=1), b_full):
                failures.append(f"column blocks of B differ (beta={beta})")
            full2 = sg.gather_c(c2, m)
            if rank == 0:
                chk = oracle.check(full2, ref)
                if not chk.passed:
                    failures.append(f"broadcast_and_run beta={beta}: {chk}")
            del blocks
            dist.destroy_process_group(bgroup)
            st = gemm_b200.status()
            if st != 0:
                failures.append(f"library status {st}")
        # copy-engine ring: three calls in a row on one PeerRing, B rewritten on
        # the source before the third; 9 chunks (8 of 256 columns and one of 8)
        # in GEMM blocks of 3 chunks
        b_alt = oracle.make_inputs(m, n, k, "normal", seed=43)[1]
        row0, rows = SlabGemm().partition(m)
        a_slab = a[row0:row0 + rows].to(dev)
        b_ring = b_full.to(dev) if rank == 0 else torch.full((k, n), float("nan"), device=dev,
                                                             dtype=torch.float16)
        ring = PeerRing(b_ring, chunk_cols=256, block_cols=768, first_chunk_cols=256,
                        first_block_cols=768, timeout_s=20.0)
        if ring.blocks != [(0, 768), (768, 1536), (1536, 2056)]:
            failures.append(f"ring blocks {ring.blocks}")
        for call, (alpha, beta, b_src) in enumerate(((0.75, -0.25, b_full), (1.0, 0.0, b_full),
                                                     (0.5, 0.25, b_alt))):
            if rank == 0 and call == 2:
                b_ring.copy_(b_alt.to(dev))
            c_init = c0[row0:row0 + rows] if beta != 0 else torch.full((rows, n), float("nan"),
                                                                       dtype=torch.float16)
            c3 = c_init.to(dev)
            ring.broadcast_and_run(a_slab, c3, alpha, beta, deadline_s=30.0)
            if not torch.equal(b_ring.cpu(), b_src):
                failures.append(f"ring call {call}: replica of B differs")
            full3 = SlabGemm().gather_c(c3, m)
            if rank == 0:
                chk = oracle.check(full3, oracle.reference_fp32(a, b_src, c0, alpha, beta))
                if not chk.passed:
                    failures.append(f"ring call {call} beta={beta}: {chk}")
        ring.close()
        st = gemm_b200.status()
        if st != 0:
            failures.append(f"library status {st} after the ring")
        dist.barrier()
    except Exception:
        failures.append(traceback.format_exc().replace("\n", " | "))
    # one write() per line: the ranks share the pipe, and a single write of up to
    # PIPE_BUF bytes is never interleaved with another process's
    line = f"RESULT {rank} {'ok' if not failures else '; '.join(failures)}"[:3000] + "\n"
    sys.stdout.flush()
    os.write(1, line.encode())
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
