"""GPU, 2 or more devices: the row-split LM head and the expert-parallel MoE
block over NCCL, bit for bit against one GPU (tests/mgpu_worker.py, one rank
per GPU under torchrun). Skipped on a box with fewer than two GPUs."""
from __future__ import annotations

import os
import socket
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def test_two_ranks_match_one_gpu():
    import torch

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    cmd = ["timeout", "-k", "30", "400", sys.executable, "-m", "torch.distributed.run", "--nnodes", "1",
           "--nproc-per-node", "2", "--master-addr", "127.0.0.1", "--master-port", str(_free_port()),
           os.path.join(HERE, "mgpu_worker.py")]
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=460)
    out = r.stdout + r.stderr
    assert r.returncode == 0, out[-3000:]
    assert "rank 0 MGPU OK" in out and "rank 1 MGPU OK" in out, out[-3000:]
