"""GPU: the row-split (tensor-parallel) decode stack and the library's NCCL
control path.

- One GPU: a communicator of two ranks of which only rank 0 ever joins:
  bh_tp_comm_init returns BH_ETIMEDOUT within its limit (the non-blocking
  init is polled and then aborted) instead of hanging.
- Two, four and eight GPUs, as many as there are (tests/tp_worker.py under
  torchrun, one rank per GPU):
  the row-split stack at a small shape and at the full config-2 shape
  (36 layers, 4096 / 12288, 151936-row LM head) gives the one-GPU stack's
  tokens and hidden states bit for bit, step after step; the library's
  all-gather and all-reduce over the same communicator. A world size is
  skipped when there are fewer GPUs than ranks."""
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


@pytest.mark.parametrize("world", [2, 4, 8])
def test_row_split_stack_matches_one_gpu(world):
    import torch

    n = torch.cuda.device_count()
    if n < world:
        pytest.skip(f"needs {world} GPUs")
    cmd = ["timeout", "-k", "30", "600", sys.executable, "-m", "torch.distributed.run", "--nnodes", "1",
           "--nproc-per-node", str(world), "--master-addr", "127.0.0.1", "--master-port", str(_free_port()),
           os.path.join(HERE, "tp_worker.py")]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=660, env=env)
    out = r.stdout + r.stderr
    assert r.returncode == 0, out[-4000:]
    for q in range(world):
        assert f"rank {q} TP OK" in out, out[-4000:]


_HOLDER = r"""
import sys
sys.path.insert(0, %r)
import burnhard as bh
ctx = bh.Context(0)
cfg = bh.default_stack_config(n_layer=2, n_embd=1024, n_head=16, n_head_kv=8, n_ff=2048, n_vocab=5000)
st = bh.Stack(ctx, cfg, 11, rank=1, world=2)
print(st.tp_handle().hex(), flush=True)
sys.stdin.readline()      # holds its exchange region until told; launches no kernel that waits
st.close()
"""


def test_row_split_wait_runs_out_when_a_peer_never_decodes(bh, ctx):
    """Rank 0 of a two-rank split decodes while rank 1 (another process on
    the same GPU) only holds its exchange region and never decodes: the pairs
    rank 0 waits for never arrive, its bounded waits run out (the first after
    about a second, the rest at once since the status already holds the
    error), the step ends, the token is -1 and bh_device_status reports
    BH_ETIMEDOUT; the context stays usable."""
    import time

    import numpy as np
    import torch

    holder = subprocess.Popen([sys.executable, "-c", _HOLDER % os.path.join(ROOT, "shannon-prime-burnhard_b200")],
                              stdin=subprocess.PIPE, stdout=subprocess.PIPE, text=True)
    try:
        peer = bytes.fromhex(holder.stdout.readline().strip())
        cfg = bh.default_stack_config(n_layer=2, n_embd=1024, n_head=16, n_head_kv=8, n_ff=2048, n_vocab=5000)
        st = bh.Stack(ctx, cfg, 11, rank=0, world=2)
        st.tp_connect([st.tp_handle(), peer])
        st.fill_kv(5, 13)
        st.set_pos(5)
        x = torch.from_numpy(np.random.default_rng(3).standard_normal(1024).astype(np.float32)).cuda()
        tok = torch.zeros(1, dtype=torch.int32, device="cuda")
        ctx.status()
        t0 = time.monotonic()
        st.decode(x, tok)
        torch.cuda.synchronize()
        dt = time.monotonic() - t0
        assert ctx.status() == bh.BH_ETIMEDOUT
        assert int(tok.item()) == -1
        assert dt < 30, dt
        st.close()
        # the context still works
        y = ctx.matvec_f32(ctx.q4k_quantize(torch.randn((256, 256), device="cuda") * 0.02), 256, 256,
                           torch.randn((1, 256), device="cuda"))
        torch.cuda.synchronize()
        assert torch.isfinite(y).all() and ctx.status() == 0
    finally:
        holder.stdin.write("done\n")
        holder.stdin.flush()
        holder.wait(timeout=60)
