"""The peer-memory column split on two GPUs (skipped with fewer).

The worker (tests/nsplit_peer_worker.py) runs as two torchrun processes, one per
GPU, and compares the split layer with the unsplit one bit for bit on every
rank; see its docstring for the cases.
"""
import os
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))


def test_peer_column_split_two_gpus():
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node", "2", "--master-addr", "127.0.0.1", "--master-port", "29561",
           os.path.join(HERE, "nsplit_peer_worker.py")]
    cp = subprocess.run(cmd, capture_output=True, text=True, env=env, timeout=400)
    assert cp.returncode == 0, cp.stdout[-3000:] + cp.stderr[-3000:]
    assert "ok 0" in cp.stdout and "ok 1" in cp.stdout
