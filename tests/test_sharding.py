"""CPU: the multi-GPU host logic (sharding.py) as world_size-2 gloo ranks.

The per-rank compute is the oracle (CPU restatement) on that rank's share;
the collective steps are the product's own functions. Checked: the row-split
LM head (all-gather of logit slices, and the candidate merge) picks exactly
the single-device greedy token, including ties across the shard boundary;
the expert-parallel sum of -0.0-filled expert outputs reproduces every
value bit for bit, so the slot-order combine equals the single-device block.
"""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle as om
import sharding


def test_even_shards():
    assert sharding.even_shards(151936, 8) == [(18992 * r, 18992 * (r + 1)) for r in range(8)]
    assert sharding.even_shards(128, 8)[3] == (48, 64)
    s = sharding.even_shards(10, 3)
    assert s[0][0] == 0 and s[-1][1] == 10 and all(a[1] == b[0] for a, b in zip(s, s[1:]))
    with pytest.raises(ValueError):
        sharding.even_shards(3, 4)


def test_merge_argmax_first_index_on_ties():
    vals = torch.tensor([[1.0, 5.0, 2.0], [3.0, 5.0, 2.0]])
    idxs = torch.tensor([[10, 11, 12], [40, 41, 42]])
    best_i, best_v = sharding.merge_argmax(vals, idxs)
    assert best_i.tolist() == [40, 11, 12]
    assert best_v.tolist() == [3.0, 5.0, 2.0]


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank: int, world: int, port: int, case: str, q):
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=__import__("datetime").timedelta(seconds=60))
        o = om.Oracle()
        if case == "lmhead":
            n, k, b = 4000, 512, 3
            w = o.quantize_q4k(o.normal((n, k), 11, 0.0, 0.02))
            x = o.normal((b, k), 12, 0.0, 1.0)
            xq = o.quantize_q8k(x)
            full = o.matvec(w, n, k, xq, b)
            # plant a tie across the shard boundary in column 1, and one inside rank 1's rows in column 2
            lo, hi = sharding.even_shards(n, world)[rank]
            row = w.shape[1]
            local = o.matvec(w[lo:hi], hi - lo, k, xq, b)
            tie = full[1].max() + 1.0
            for (c, r_) in ((1, n // 2 - 1), (1, n // 2), (2, n // 2 + 5), (2, n - 1)):
                full[c, r_] = tie if c == 1 else tie + 1.0
                if lo <= r_ < hi:
                    local[c, r_ - lo] = full[c, r_]
            loc_t = torch.from_numpy(local)
            gathered = sharding.gather_rows(loc_t, world)
            ok_g = bool((gathered.numpy().view(np.uint32) == full.view(np.uint32)).all())
            li = torch.from_numpy(np.array([np.argmax(local[c]) for c in range(b)], dtype=np.int64)) + lo
            lv = torch.from_numpy(local.max(axis=1))
            vals, idxs = sharding.gather_candidates(lv, li, world)
            tok, _ = sharding.merge_argmax(vals, idxs)
            want = [o.argmax(full[c]) for c in range(b)]
            q.put((rank, ok_g and tok.tolist() == want and want[1] == n // 2 - 1 and want[2] == n // 2 + 5))
        elif case == "ep":
            E, D, F, k, T = 8, 512, 256, 3, 3
            gate = o.quantize_q4k(o.normal((E * F, D), 21, 0.0, 0.02))
            up = o.quantize_q4k(o.normal((E * F, D), 22, 0.0, 0.02))
            down = o.quantize_q4k(o.normal((E * D, F), 23, 0.0, 0.02))
            cur = o.normal((T, D), 24, 0.0, 1.0)
            ids, w = o.moe_route(o.normal((T, E), 25), k)
            ref, _, dout_full = o.moe_ffn(cur, ids, w, gate, up, down, D, F)
            lo, hi = sharding.even_shards(E, world)[rank]
            mine = (ids.reshape(-1) >= lo) & (ids.reshape(-1) < hi)
            dout = np.where(mine[:, None], dout_full, np.float32(-0.0)).astype(np.float32)
            summed = sharding.sum_expert_outputs(torch.from_numpy(dout), world).numpy()
            exact = bool((summed.view(np.uint32) == dout_full.view(np.uint32)).all())
            out = np.zeros((T, D), np.float32)
            for t in range(T):
                acc = np.zeros(D, np.float64)
                for s in range(k):
                    acc += (summed[t * k + s] * w[t, s]).astype(np.float64)
                out[t] = acc.astype(np.float32)
            q.put((rank, exact and bool((out.view(np.uint32) == ref.view(np.uint32)).all())))
        dist.barrier()
        dist.destroy_process_group()
    except Exception as e:  # report instead of hanging the parent
        q.put((rank, f"error: {e!r}"))


@pytest.mark.parametrize("case", ["lmhead", "ep"])
def test_two_gloo_ranks(case):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, case, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=180) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert results == {0: True, 1: True}, results


def _peer_map_worker(rank, world, port, q, fail_rank):
    import os

    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    import sharding

    class FakeBuf:
        # stands in for bh.PeerMailbox: a "handle" and an "open" that maps it
        def __init__(self, r):
            self.ptr = 1000 + r

        def handle(self):
            return bytes([rank]) * 64

        def open(self, h):
            if rank == fail_rank:
                raise RuntimeError("cannot map")
            return 1000 + h[0]

    try:
        out = sharding._map_peers([FakeBuf(rank)], rank, world)
        q.put((rank, "ok", out))
    except RuntimeError as e:
        q.put((rank, "raised", str(e)))
    dist.destroy_process_group()


@pytest.mark.parametrize("fail_rank", [-1, 1])
def test_peer_mapping_all_or_nothing(fail_rank):
    """The IPC handle exchange of the peer-memory paths (host logic, gloo):
    every rank gets every rank's buffer at its rank's position; when one
    rank cannot map, every rank raises instead of waiting."""
    import multiprocessing as mp
    import socket

    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_peer_map_worker, args=(r, 2, port, q, fail_rank)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(60)
    if fail_rank < 0:
        assert [r[1] for r in res] == ["ok", "ok"]
        assert res[0][2] == [[1000, 1001]] and res[1][2] == [[1000, 1001]]
    else:
        assert [r[1] for r in res] == ["raised", "raised"]
