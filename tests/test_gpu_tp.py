"""GPU: the row-split (tensor-parallel) decode stack and the library's NCCL
control path.

- One GPU: a communicator of two ranks of which only rank 0 ever joins:
  bh_tp_comm_init returns BH_ETIMEDOUT within its limit (the non-blocking
  init is polled and then aborted) instead of hanging.
- Two or more GPUs (tests/tp_worker.py under torchrun, one rank per GPU):
  the row-split stack at a small shape and at the full config-2 shape
  (36 layers, 4096 / 12288, 151936-row LM head) gives the one-GPU stack's
  tokens and hidden states bit for bit, step after step; the library's
  all-gather and all-reduce over the same communicator. Skipped with fewer
  than two GPUs."""
from __future__ import annotations

import os
import socket
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def test_nccl_rank_that_never_joins_times_out():
    code = (
        "import sys, time; sys.path.insert(0, %r)\n"
        "import burnhard as bh\n"
        "uid = bh.tp_unique_id()\n"
        "t0 = time.monotonic()\n"
        "rc, comm = bh.tp_comm_init_rc(0, uid, 2, 0, 3000)\n"
        "dt = time.monotonic() - t0\n"
        "print('RC', rc, 'DT', round(dt, 2), flush=True)\n"
        "sys.exit(0 if (rc == bh.BH_ETIMEDOUT and 2.5 < dt < 30) else 1)\n"
    ) % os.path.join(ROOT, "shannon-prime-burnhard_b200")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    r = subprocess.run(["timeout", "-k", "10", "120", sys.executable, "-c", code], capture_output=True, text=True,
                       timeout=150, env=env)
    assert r.returncode == 0, (r.stdout + r.stderr)[-3000:]


def test_row_split_stack_matches_one_gpu():
    import torch

    n = torch.cuda.device_count()
    if n < 2:
        pytest.skip("needs two GPUs")
    world = 2
    cmd = ["timeout", "-k", "30", "600", sys.executable, "-m", "torch.distributed.run", "--nnodes", "1",
           "--nproc-per-node", str(world), "--master-addr", "127.0.0.1", "--master-port", str(_free_port()),
           os.path.join(HERE, "tp_worker.py")]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=660, env=env)
    out = r.stdout + r.stderr
    assert r.returncode == 0, out[-4000:]
    for q in range(world):
        assert f"rank {q} TP OK" in out, out[-4000:]
