"""The multi-GPU row-slab launcher on real GPUs, over NCCL and over the
copy-engine ring (needs >= 2 B200s; uses up to 4).

Marked `multigpu`, not `gpu`: the single-GPU suite (`-m gpu`) runs on one B200,
so this test runs on its own on a two-GPU box
(`python -m pytest tests/test_multigpu_nccl.py -m multigpu`) and is skipped
wherever fewer than two GPUs are visible. It launches tests/nccl_slab_worker.py
under torchrun (one process per GPU, rendezvous on 127.0.0.1, a 60 s process
group timeout and an outer `timeout` as the last bound) and requires every rank
to report that its results and its replica of B match the CPU oracle.
"""
import os
import re
import socket
import subprocess
import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent

pytestmark = pytest.mark.multigpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_slab_launcher_multi_gpu_matches_oracle():
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    # up to four ranks, so that the ring has a rank with both neighbours
    world = min(torch.cuda.device_count(), 4)
    env = dict(os.environ, GEMM_LAUNCH_LOG="0")
    cmd = ["timeout", "-k", "60", "400", sys.executable, "-m", "torch.distributed.run",
           "--nnodes=1", f"--nproc-per-node={world}", "--master-addr", "127.0.0.1",
           "--master-port", str(_free_port()), str(REPO / "tests" / "nccl_slab_worker.py")]
    proc = subprocess.run(cmd, capture_output=True, text=True, env=env, timeout=500)
    lines = re.findall(r"RESULT \d+ .*", proc.stdout)
    assert proc.returncode == 0, proc.stdout[-4000:] + proc.stderr[-4000:]
    assert sorted(lines) == [f"RESULT {r} ok" for r in range(world)], \
        "\n".join(lines) + proc.stderr[-3000:]
