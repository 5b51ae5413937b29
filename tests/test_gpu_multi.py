"""Multi-GPU partitions over NCCL (needs >= 2 GPUs; skipped otherwise)."""

import os
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu

WORKER = os.path.join(os.path.dirname(os.path.abspath(__file__)), "multigpu", "partition_worker.py")


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs at least 2 GPUs")
def test_batch_and_head_partitions_nccl():
    n = min(torch.cuda.device_count(), 8)
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run",
           "--nnodes=1", f"--nproc-per-node={n}", "--master-addr", "127.0.0.1",
           "--master-port", "29611", WORKER]
    res = subprocess.run(cmd, capture_output=True, text=True, env=env)
    print(res.stdout[-4000:])
    assert res.returncode == 0, res.stderr[-4000:]
