"""The copy-engine ring's protocol (gemm_b200.slab.ring_program), run on CPU.

A discrete-event simulator executes every rank's copy and compute streams, as
the ops lists say, under random interleavings of the streams, for several calls
in a row enqueued up front (as the host does). It checks that:
- every copy reads the chunk of the same call from its predecessor;
- every GEMM block reads chunks of the same call;
- no chunk is overwritten while a successor copies it or a GEMM reads it;
- the caller's rewrite of B on the source waits for the same;
- every flag word only grows;
- nothing deadlocks.
Planted protocol bugs (a wait taken out) must be caught. No GPU is involved."""
import random
import sys
from pathlib import Path

import pytest

sys.path.insert(0, str(Path(__file__).resolve().parent.parent / "gemm-project_b200"))
from gemm_b200.slab import ring_layout, ring_program  # noqa: E402


def _ends(n_chunks, cpb):
    return [min(n_chunks, g + cpb) for g in range(0, n_chunks, cpb)]


class RingViolation(AssertionError):
    pass


def simulate(world, n_chunks, cpb, calls, seed, program=ring_program):
    rng = random.Random(seed)
    block_ends = _ends(n_chunks, cpb)
    blocks = [list(range(j0, j1)) for j0, j1 in zip([0] + block_ends[:-1], block_ends)]
    flags = [{"ready": 0, "consumed": 0} for _ in range(world)]
    ver = [[0] * n_chunks for _ in range(world)]       # call whose data the chunk holds
    reading = [[0] * n_chunks for _ in range(world)]   # in-flight readers of each chunk
    events = set()                                     # (rank, call, block) recorded
    # host: enqueue every call's ops on both streams of every rank, in order
    streams = {}
    for r in range(world):
        cq, mq = [], []
        for seq in range(1, calls + 1):
            copy_ops, compute_ops = program(r, world, n_chunks, block_ends, seq)
            if r == 0:
                mq.append((seq, ("write_b",)))
            for op in copy_ops:
                cq.append((seq, op, len(mq)) if op[0] == "join_compute" else (seq, op))
            mq += [(seq, op) for op in compute_ops]
        streams[(r, "copy")] = {"q": cq, "i": 0, "busy": None}
        streams[(r, "compute")] = {"q": mq, "i": 0, "busy": None}

    def target(r, who):
        return r + 1 if who == "succ" else r - 1

    def ready(r, item):
        seq, op = item[0], item[1]
        if op[0] == "join_compute":
            return streams[(r, "compute")]["i"] >= item[2]
        if op[0] == "flags":
            return all(flags[r][which] - value >= 0 for which, value in op[2])
        if op[0] == "gemm" and r > 0:
            return (r, seq, op[1]) in events
        return True

    def start(r, item):
        seq, op = item[0], item[1]
        if op[0] == "copy":
            j = op[1]
            if ver[r - 1][j] != seq:
                raise RingViolation(f"rank {r} call {seq} copied chunk {j} of call {ver[r - 1][j]}")
            reading[r - 1][j] += 1
        elif op[0] == "gemm":
            for j in blocks[op[1]]:
                if ver[r][j] != seq:
                    raise RingViolation(f"rank {r} call {seq} GEMM read chunk {j} of call {ver[r][j]}")
                reading[r][j] += 1
        return True

    def finish(r, item):
        seq, op = item[0], item[1]
        if op[0] == "copy":
            j = op[1]
            reading[r - 1][j] -= 1
            if reading[r][j]:
                raise RingViolation(f"rank {r} overwrote chunk {j} while it was being read")
            ver[r][j] = seq
        elif op[0] == "gemm":
            for j in blocks[op[1]]:
                reading[r][j] -= 1
        elif op[0] == "write_b":
            if any(reading[0]):
                raise RingViolation(f"call {seq}: B rewritten on the source while being read")
            ver[0] = [seq] * n_chunks
        elif op[0] == "flags":
            for who, which, value in op[1]:
                t = target(r, who)
                if value < flags[t][which]:
                    raise RingViolation(f"flag {which} of rank {t} went back")
                flags[t][which] = value
        elif op[0] == "block_ready":
            events.add((r, seq, op[1]))

    while True:
        live = [k for k, s in streams.items() if s["i"] < len(s["q"])]
        if not live:
            break
        runnable = [k for k in live if streams[k]["busy"] is not None
                    or ready(k[0], streams[k]["q"][streams[k]["i"]])]
        if not runnable:
            raise RingViolation(f"deadlock at {[(k, streams[k]['q'][streams[k]['i']]) for k in live]}")
        k = rng.choice(runnable)
        s = streams[k]
        item = s["q"][s["i"]]
        if s["busy"] is None and item[1][0] in ("copy", "gemm"):
            s["busy"] = start(k[0], item)        # two-phase: readers stay in flight
            continue
        finish(k[0], item)
        s["busy"] = None
        s["i"] += 1
    for r in range(world):
        if ver[r] != [calls] * n_chunks:
            raise RingViolation(f"rank {r} ends with chunk versions {ver[r]}")
    return True


@pytest.mark.parametrize("world", [1, 2, 3, 5, 8])
@pytest.mark.parametrize("n_chunks,cpb", [(1, 1), (3, 1), (7, 2), (8, 4), (5, 8)])
def test_ring_protocol_random_interleavings(world, n_chunks, cpb):
    for seed in range(40):
        assert simulate(world, n_chunks, cpb, calls=3, seed=seed)


def test_ring_program_shape():
    """Counters of call 2 with 5 chunks start at 5; the last block's event comes
    after the final signal; the source only signals once and waits once."""
    copy_ops, compute_ops = ring_program(1, 3, 5, [2, 4, 5], 2)
    assert copy_ops[0] == ("join_compute",)
    assert copy_ops[1] == ("flags", [], [("ready", 6)])
    assert copy_ops[-2] == ("flags", [("succ", "ready", 10), ("pred", "consumed", 10)], [])
    assert copy_ops[-1] == ("block_ready", 2)
    assert [op for op in compute_ops if op[0] == "gemm"] == [("gemm", 0, True), ("gemm", 1, True),
                                                             ("gemm", 2, False)]
    assert compute_ops[-1] == ("flags", [], [("consumed", 10)])
    src_copy, src_compute = ring_program(0, 3, 5, [2, 4, 5], 2)
    assert src_copy == []
    assert src_compute[0] == ("flags", [("succ", "ready", 10)], [])
    last_copy, last_compute = ring_program(2, 3, 5, [2, 4, 5], 2)
    assert all(op[1] == [] or op[1] == [("pred", "consumed", 10)]
               for op in last_copy if op[0] == "flags")
    assert last_compute[-1][0] == "gemm"
    with pytest.raises(ValueError):
        ring_program(3, 3, 5, [2, 4, 5], 1)
    with pytest.raises(ValueError):
        ring_program(1, 3, 5, [2, 4], 1)    # blocks must cover every chunk


def test_ring_layout():
    """Chunks grow 512, 1024, 2048 and stay there (the last takes the rest);
    blocks end at the first chunk boundary at or past 2048 columns, then every
    4096 or more, and the 512-column remainder joins the last block."""
    bounds, ends = ring_layout(32768)
    widths = [c1 - c0 for c0, c1 in bounds]
    assert widths[:4] == [512, 1024, 2048, 2048] and set(widths[3:-1]) == {2048}
    assert widths[-1] == 512
    assert sum(widths) == 32768 and bounds[0][0] == 0
    assert all(a[1] == b[0] for a, b in zip(bounds, bounds[1:]))
    block_cols = [bounds[e - 1][1] for e in ends]
    assert block_cols[:3] == [3584, 7680, 11776] and block_cols[-2:] == [28160, 32768]
    assert ends[-1] == len(bounds)
    # ragged N: the last chunk and block take the rest; uniform when first == chunk
    bounds, ends = ring_layout(2056, 256, 768, 256, 768)
    assert [c1 - c0 for c0, c1 in bounds] == [256] * 8 + [8] and ends == [3, 6, 9]
    bounds, ends = ring_layout(100, 2048, 4096, 512, 2048)
    assert bounds == [(0, 100)] and ends == [1]
    with pytest.raises(ValueError):
        ring_layout(1024, 1004)


def _without_end_wait(position, world, n_chunks, block_ends, seq):
    """A planted bug: the compute stream's end-of-call wait for the successor."""
    copy_ops, compute_ops = ring_program(position, world, n_chunks, block_ends, seq)
    return copy_ops, [op for op in compute_ops if not (op[0] == "flags" and op[2])]


def _without_ready_wait(position, world, n_chunks, block_ends, seq):
    """A planted bug: copies that do not wait for the predecessor."""
    copy_ops, compute_ops = ring_program(position, world, n_chunks, block_ends, seq)
    return [("flags", op[1], []) if op[0] == "flags" else op for op in copy_ops], compute_ops


@pytest.mark.parametrize("bug", [_without_end_wait, _without_ready_wait])
def test_simulator_catches_planted_bugs(bug):
    caught = 0
    for seed in range(200):
        try:
            simulate(3, 4, 2, calls=3, seed=seed, program=bug)
        except RingViolation:
            caught += 1
    assert caught > 0


def test_peer_ring_rejects_host_and_strided_replicas():
    """The replica must be a contiguous FP16 CUDA tensor; checked before any
    collective, so a bad argument fails on the calling rank alone."""
    import torch
    from gemm_b200.slab import PeerRing

    with pytest.raises(ValueError):
        PeerRing(torch.zeros((16, 32), dtype=torch.float16))          # host memory
    with pytest.raises(ValueError):
        PeerRing(torch.zeros((16, 32), dtype=torch.float32))
