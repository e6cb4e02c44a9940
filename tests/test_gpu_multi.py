"""Batch-sharded execution on two GPUs (NCCL) against the single-GPU result;
skipped on boxes with fewer than two GPUs (the CPU suite covers the
sharding logic with two gloo ranks)."""
import os
import socket
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_sharded_network_matches_single_gpu():
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node", "2", "--master-addr", "127.0.0.1", "--master-port", str(_free_port()),
           os.path.join(HERE, "multi_rank_check.py")]
    res = subprocess.run(cmd, capture_output=True, text=True, env=env, timeout=400)
    assert res.returncode == 0, res.stdout[-2000:] + res.stderr[-4000:]
    assert "indices_equal=True features_equal=True" in res.stdout
