"""One rank of the row-split decode check (launched by tests/test_gpu_tp.py
under torchrun, one rank per GPU): the NCCL communicator comes from the
library's own non-blocking bh_tp_comm_init (the unique id is broadcast over a
gloo group), the ranks' exchange regions are connected through it, and the
row-split stack decodes several tokens. Every rank also builds the one-GPU
stack from the same seed on its own GPU; tokens and the whole hidden state
after every step must be equal bit for bit."""
import datetime
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "shannon-prime-burnhard_b200"))

import numpy as np
import torch
import torch.distributed as dist


def run(bh, ctx, rank, world, comm, cfg_kw, steps, seed, fails):
    cfg = bh.default_stack_config(**cfg_kw)
    one = bh.Stack(ctx, cfg, seed)
    tp = bh.Stack(ctx, cfg, seed, rank=rank, world=world)
    tp.tp_connect_comm(comm, 30000)
    info = tp.tp_info()
    n_embd = cfg.n_embd
    rng = np.random.default_rng(seed + 1)
    pos0 = 5
    for st in (one, tp):
        st.fill_kv(pos0, seed + 2)
    h_one = one.view(0, bh.T_HIDDEN)
    h_tp = tp.view(0, bh.T_HIDDEN)
    tok1 = torch.zeros(1, dtype=torch.int32, device="cuda")
    tok2 = torch.zeros(1, dtype=torch.int32, device="cuda")
    for s in range(steps):
        x = torch.from_numpy(rng.standard_normal(n_embd).astype(np.float32)).cuda()
        for st in (one, tp):
            st.set_pos(pos0 + s)
        one.decode(x, tok1)
        tp.decode(x, tok2)
        torch.cuda.synchronize()
        if ctx.status() != 0:
            fails.append(f"{cfg_kw} step {s}: device status {ctx.status()}")
            break
        if int(tok1.item()) != int(tok2.item()):
            fails.append(f"{cfg_kw} step {s}: token {tok2.item()} vs one GPU {tok1.item()}")
        h_vals = h_tp.reshape(-1)[0::2]  # (value, generation) pairs on a split
        if not torch.equal(h_one.reshape(-1).view(torch.int32), h_vals.contiguous().view(torch.int32)):
            d = (h_one.reshape(-1) - h_vals).abs().max().item()
            fails.append(f"{cfg_kw} step {s}: hidden differs (max {d})")
    # this rank's K cache rows equal the one-GPU cache's columns of its KV heads
    kv0, kvn = info["kv_heads"]
    hd = cfg.head_dim
    kc1 = one.view(cfg.n_layer - 1, bh.T_K_CACHE)[: pos0 + steps, kv0 * hd:(kv0 + kvn) * hd]
    kc2 = tp.view(cfg.n_layer - 1, bh.T_K_CACHE)[: pos0 + steps]
    if not torch.equal(kc1.contiguous().view(torch.int32), kc2.contiguous().view(torch.int32)):
        fails.append(f"{cfg_kw}: K cache rows differ")
    torch.cuda.synchronize()
    dist.barrier()  # every rank done with the peers' regions before any is freed
    tp.close()
    one.close()


def main() -> int:
    rank, world, local = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"]), int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=120))
    import burnhard as bh

    ctx = bh.Context(local)
    obj = [bh.tp_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(obj, src=0)
    comm = bh.tp_comm_init(local, obj[0], world, rank, 60000)
    fails = []
    run(bh, ctx, rank, world, comm, dict(n_layer=3, n_embd=1024, n_head=16, n_head_kv=8, n_ff=2048, n_vocab=5000),
        6, 11, fails)
    run(bh, ctx, rank, world, comm, {}, 4, 20261201, fails)
    # the NCCL all-gather through the library, against the ranks' values
    n = 1000
    mine = torch.full((n,), float(rank + 1), device="cuda")
    allv = torch.empty(world * n, device="cuda")
    bh.tp_allgather(comm, mine, allv)
    want = torch.cat([torch.full((n,), float(r + 1), device="cuda") for r in range(world)])
    if not torch.equal(allv, want):
        fails.append("bh_tp_allgather result")
    buf = torch.full((n,), float(rank + 1), device="cuda")
    bh.tp_allreduce_sum(comm, buf)
    if not torch.equal(buf, torch.full((n,), float(world * (world + 1) // 2), device="cuda")):
        fails.append("bh_tp_allreduce_sum_f32 result")
    bh.tp_comm_free(comm)
    for f in fails:
        print(f"rank {rank} FAIL {f}", flush=True)
    if not fails:
        print(f"rank {rank} TP OK", flush=True)
    dist.barrier()
    dist.destroy_process_group()
    return 0 if not fails else 1


if __name__ == "__main__":
    sys.exit(main())
