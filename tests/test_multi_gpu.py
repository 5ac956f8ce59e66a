"""GPU: sharded execution over 2+ GPUs equals the unsharded run (NCCL gather for
verification only), and a rank that leaves between steps is detected on the
host before the next collective.  Needs at least 2 visible GPUs; NVLS is
switched off."""

import os
import socket
import subprocess
import sys

import pytest
import torch

from conftest import ROOT

pytestmark = pytest.mark.gpu


def test_two_gpu_shards_match_single_gpu():
    n = torch.cuda.device_count()
    if n < 2:
        pytest.skip(f"needs >= 2 GPUs, {n} visible")
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "240", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={min(n, 2)}", "--master-addr=127.0.0.1", f"--master-port={port}",
           os.path.join(ROOT, "tests", "multi_gpu_worker.py")]
    res = subprocess.run(cmd, capture_output=True, text=True, env=env, timeout=300)
    print(res.stdout[-2000:], res.stderr[-2000:])
    assert res.returncode == 0
    assert "DIFFERS" not in res.stdout and res.stdout.count("identical") == 5


def test_two_gpu_dead_rank_detected_on_the_host():
    """Rank 1 leaves between steps; rank 0's heartbeat wait reports it before
    step 1's NCCL collective (no GPU fault, nothing in flight; NVLS off)."""
    n = torch.cuda.device_count()
    if n < 2:
        pytest.skip(f"needs >= 2 GPUs, {n} visible")
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    worker = os.path.join(ROOT, "tests", "multi_gpu_worker.py")
    procs = []
    for r in range(2):
        env = dict(os.environ, NCCL_NVLS_ENABLE="0", MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(r),
                   LOCAL_RANK=str(r), WORLD_SIZE="2")
        procs.append(subprocess.Popen(["timeout", "-k", "30", "120", sys.executable, worker, "--dead-rank"],
                                      stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True, env=env))
    outs = [p.communicate(timeout=200)[0] for p in procs]
    print(outs[0][-2000:], outs[1][-2000:])
    assert procs[1].returncode == 3, outs[1][-2000:]
    assert procs[0].returncode == 0 and "detected: rank(s) [1]" in outs[0], outs[0][-2000:]
