"""One rank of the 2+ GPU check (launched by tests/test_gpu_multi.py under
torchrun): the row-split LM head and the expert-parallel MoE block against
the single-GPU entry points on the same seeded inputs, bit for bit.

Shapes are the C5 LM head (151936 x 4096, batch 1 and 4) and the C4 expert
block (128 experts, 2048 -> 768 -> 2048, top-8, 1 and 4 tokens)."""
import datetime
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "shannon-prime-burnhard_b200"))

import torch
import torch.distributed as dist


def main() -> int:
    rank, world, local = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"]), int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    import burnhard as bh
    import sharding

    ctx = bh.Context(local)
    fails = []
    # ---- row-split LM head
    N, K = 151936, 4096
    g = torch.Generator(device="cuda").manual_seed(7)
    w = ctx.q4k_quantize(torch.randn((N, K), generator=g, device="cuda") * 0.02)
    lo, hi = sharding.even_shards(N, world)[rank]
    head = sharding.TPLMHead(ctx, N, K, rank, world, sharding.TPLMHead.slice_rows(w, N, K, lo, hi))
    head.enable_peer_exchange()
    for B in (1, 4, 1, 8):
        x = torch.randn((B, K), generator=g, device="cuda")
        full = torch.empty((B, N), device="cuda")
        tok1, _ = bh.lmhead_argmax(ctx, w, N, K, x, logits=full)
        tok_g, logits_g = head.forward(x, gather_logits=True)
        tok_c, _ = head.forward(x, gather_logits=False)
        tok_p = head.forward_peer(x)
        torch.cuda.synchronize()
        if not torch.equal(logits_g.view(torch.int32), full.view(torch.int32)):
            fails.append(f"lmhead B={B}: gathered logits differ")
        if not (torch.equal(tok_g, tok1.to(torch.int64)) and torch.equal(tok_c, tok1.to(torch.int64))):
            fails.append(f"lmhead B={B}: tokens {tok_g.tolist()} {tok_c.tolist()} vs {tok1.tolist()}")
        if not torch.equal(tok_p, tok1):
            fails.append(f"lmhead B={B}: peer-exchange tokens {tok_p.tolist()} vs {tok1.tolist()}")
    head.close_peer_exchange()
    del w, head
    # ---- expert-parallel MoE block
    E, D, F, k = 128, 2048, 768, 8
    banks = {}
    for name, rows, cols in (("gate", E * F, D), ("up", E * F, D), ("down", E * D, F)):
        banks[name] = ctx.q4k_quantize(torch.randn((rows, cols), generator=g, device="cuda") * 0.02)
    elo, ehi = sharding.even_shards(E, world)[rank]
    own = {n: sharding.EPMoE.slice_experts(b, E, elo, ehi) for n, b in banks.items()}
    ep = sharding.EPMoE(ctx, E, D, F, k, rank, world, own["gate"], own["up"], own["down"])
    ep.enable_peer_exchange()
    for T in (1, 4, 8, 1):
        cur = torch.randn((T, D), generator=g, device="cuda")
        lg = torch.randn((T, E), generator=g, device="cuda")
        ref, _, _ = bh.moe(ctx, cur, banks["gate"], banks["up"], banks["down"], E, F, k, logits=lg)
        out = ep.forward(cur, logits=lg)
        outp = ep.forward_peer(cur, logits=lg)
        torch.cuda.synchronize()
        if not torch.equal(out.view(torch.int32), ref.view(torch.int32)):
            fails.append(f"moe T={T}: expert-parallel output differs")
        if not torch.equal(outp.view(torch.int32), ref.view(torch.int32)):
            fails.append(f"moe T={T}: peer-exchange expert-parallel output differs")
    ep.close_peer_exchange()
    torch.cuda.synchronize()
    st = ctx.status()
    if st != 0:
        fails.append(f"device status {st}")
    dist.barrier()
    dist.destroy_process_group()
    if fails:
        print(f"rank {rank} FAIL: " + "; ".join(fails), flush=True)
        return 1
    print(f"rank {rank} MGPU OK", flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
