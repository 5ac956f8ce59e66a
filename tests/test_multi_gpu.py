"""GPU: sharded execution over 2+ GPUs equals the unsharded run (NCCL gather for
verification only).  Needs at least 2 visible GPUs; NVLS is switched off."""

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
