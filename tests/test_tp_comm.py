"""Host-only: the bounded waits of the NCCL control path (bh_tp_comm_init).

Two gloo ranks on CPU share a unique id; the library resolves its NCCL
entry points from tests/fake_nccl.c (BH_NCCL_LIB), whose communicators stay
in progress until every rank has joined. When both ranks join, both
bh_tp_comm_init calls return 0; when rank 1 never joins, rank 0's call
returns BH_ETIMEDOUT within its limit and the communicator is aborted
(the fake leaves a marker), instead of hanging."""
from __future__ import annotations

import os
import subprocess
import sys
import time

import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)


@pytest.fixture(scope="module")
def fake_lib(tmp_path_factory):
    out = tmp_path_factory.mktemp("fake_nccl") / "libfake_nccl.so"
    subprocess.run(["gcc", "-shared", "-fPIC", "-O1", "-o", str(out), os.path.join(HERE, "fake_nccl.c")], check=True)
    return str(out)


def _worker(rank: int, world: int, port: int, fake: str, q) -> None:
    os.environ["BH_NCCL_LIB"] = fake
    sys.path.insert(0, os.path.join(ROOT, "shannon-prime-burnhard_b200"))
    import torch.distributed as dist

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    import burnhard as bh

    res = {}
    # 1. every rank joins
    obj = [bh.tp_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(obj, src=0)
    rc, comm = bh.tp_comm_init_rc(-1, obj[0], world, rank, 5000)
    res["join_rc"] = rc
    if rc == 0:
        res["free_rc"] = bh.lib.bh_tp_comm_free(comm, 5000)
    dist.barrier()
    # 2. rank 1 never joins: rank 0 gives up after 800 ms and aborts
    obj = [bh.tp_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(obj, src=0)
    if rank == 0:
        t0 = time.monotonic()
        rc, _ = bh.tp_comm_init_rc(-1, obj[0], world, rank, 800)
        res["alone_rc"] = rc
        res["alone_s"] = time.monotonic() - t0
        res["aborted"] = os.path.exists(os.path.join(obj[0].split(b"\0")[0].decode(), "aborted_0"))
    dist.barrier()
    dist.destroy_process_group()
    q.put((rank, res))


def test_rank_that_never_joins_times_out(fake_lib):
    import socket

    import torch.multiprocessing as mp

    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, fake_lib, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    import burnhard as bh

    for r in (0, 1):
        assert out[r]["join_rc"] == 0, out
        assert out[r]["free_rc"] == 0, out
    assert out[0]["alone_rc"] == bh.BH_ETIMEDOUT, out
    assert 0.7 < out[0]["alone_s"] < 10.0, out
    assert out[0]["aborted"], out


def test_tp_entry_points_reject_bad_arguments(bh):
    assert bh.lib.bh_tp_comm_init(-1, None, 2, 0, 100, None) == bh.BH_EINVAL
    assert bh.lib.bh_tp_comm_init(-1, b"\0" * 128, 2, 2, 100, None) == bh.BH_EINVAL
    assert bh.lib.bh_tp_allgather(None, None, None, 0, None, 100) == bh.BH_EINVAL
    assert bh.lib.bh_tp_comm_free(None, 100) == bh.BH_EINVAL
    assert bh.lib.bh_stack_tp_connect(None, None) == bh.BH_EINVAL
