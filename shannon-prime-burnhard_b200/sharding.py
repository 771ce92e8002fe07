"""Multi-GPU partitioning of the Q4_K path: one process per GPU, plumbing by
torch.distributed (NCCL over NVLink on B200s, gloo for the CPU tests).

Only the two partitions the path admits:

- row split (tensor parallel) of a matrix, e.g. the LM head
  (desktop/engine/src/forward.cpp:3413): rank r owns rows [lo_r, hi_r) of the
  Q4_K weight, computes that slice of the logits with the same kernel as one
  GPU (rows are independent, so each slice is bit-identical to the
  single-GPU rows), then an all-gather assembles the full fp32 logits on
  every rank and the greedy pick (engine.cpp:36-43, first index of the
  maximum) is taken identically everywhere. The per-rank (max, first index)
  candidates give the same token without the logits; both are exposed.
- expert parallelism for the routed-expert FFN (forward.cpp:1001-1118):
  rank r owns experts [lo_r, hi_r); every rank routes the batch identically,
  computes the expert outputs of the (token, slot) pairs routed to its
  experts (-0.0 in the other rows), an all-reduce sum assembles every pair's
  output exactly (one nonzero term per element), and each rank combines in
  slot order, so the result is bit-identical to one GPU.

The collective steps are plain functions over torch tensors so that the CPU
tests can run them as gloo ranks.
"""
from __future__ import annotations

import torch
import torch.distributed as dist


def even_shards(n: int, world: int) -> list[tuple[int, int]]:
    """Contiguous near-even split of n items over world ranks: rank r gets
    [n*r//world, n*(r+1)//world). Row shards of a Q4_K matrix (151936 rows =
    8 x 18992) and expert ranges (128 experts = 8 x 16) divide evenly."""
    if world < 1 or n < world:
        raise ValueError(f"cannot split {n} items over {world} ranks")
    return [(n * r // world, n * (r + 1) // world) for r in range(world)]


def merge_argmax(vals, idxs):
    """Global greedy pick from per-rank candidates [world, B] (value, global
    index), ranks in row order: the maximum value, first index among equals."""
    world, b = vals.shape
    best_v = vals[0].clone()
    best_i = idxs[0].clone()
    for r in range(1, world):
        take = (vals[r] > best_v) | ((vals[r] == best_v) & (idxs[r] < best_i))
        best_v = torch.where(take, vals[r], best_v)
        best_i = torch.where(take, idxs[r], best_i)
    return best_i, best_v


def gather_rows(local, world: int, group=None):
    """All-gather of row slices: local [B, n_r] from every rank (equal n_r)
    -> full [B, world * n_r] in rank order."""
    b, n_r = local.shape
    if world == 1:
        return local.clone()
    parts = [torch.empty_like(local) for _ in range(world)]
    dist.all_gather(parts, local.contiguous(), group=group)
    return torch.cat(parts, dim=1)


def gather_candidates(val, idx, world: int, group=None):
    """All-gather of the per-rank (max, global index) pairs [B] -> [world, B]."""
    if world == 1:
        return val[None].clone(), idx[None].clone()
    vals = [torch.empty_like(val) for _ in range(world)]
    idxs = [torch.empty_like(idx) for _ in range(world)]
    dist.all_gather(vals, val.contiguous(), group=group)
    dist.all_gather(idxs, idx.contiguous(), group=group)
    return torch.stack(vals), torch.stack(idxs)


def sum_expert_outputs(dout, world: int, group=None):
    """In-place all-reduce sum of the per-rank expert outputs [T*k, n_embd]
    (each element nonzero on at most one rank, -0.0 on the others)."""
    if world > 1:
        dist.all_reduce(dout, op=dist.ReduceOp.SUM, group=group)
    return dout


def _all_ok(ok: bool, world: int, group=None) -> bool:
    """True on every rank iff ok on every rank (all ranks call it)."""
    if world == 1:
        return ok
    flags = [None] * world
    dist.all_gather_object(flags, bool(ok), group=group)
    return all(flags)


def _map_peers(bufs, rank: int, world: int, group=None) -> list[list[int]]:
    """Exchange the CUDA IPC handles of this rank's buffers (bh.PeerMailbox)
    and map the other ranks' ones: per buffer, every rank's pointer as seen
    from this process (own at [rank]). All-or-nothing across the ranks: a
    failure on any rank closes the mappings and raises on every rank, so no
    rank is left waiting in a later collective."""
    if world == 1:
        return [[b.ptr] for b in bufs]
    handles = None
    try:
        handles = [b.handle() for b in bufs]
        ok = True
    except Exception:
        ok = False
    if not _all_ok(ok, world, group):
        raise RuntimeError("peer exchange: a rank could not export its buffers")
    hs = [None] * world
    dist.all_gather_object(hs, handles, group=group)
    try:
        out = [[b.ptr if r == rank else b.open(hs[r][i]) for r in range(world)] for i, b in enumerate(bufs)]
        ok = True
    except Exception:
        out, ok = None, False
    if not _all_ok(ok, world, group):
        raise RuntimeError("peer exchange: a rank could not map the others' buffers")
    dist.barrier(group=group)  # every rank's buffers are mapped before the first exchange
    return out


class TPLMHead:
    """Row-split Q4_K LM head with the greedy pick.

    w_full_q4k: the full [N rows] Q4_K weight on this rank's device, or
    w_local: this rank's rows already sliced (bytes of rows [lo, hi))."""

    def __init__(self, ctx, n: int, k: int, rank: int, world: int, w_local, group=None):
        import burnhard as bh

        self.bh = bh
        self.ctx, self.n, self.k, self.rank, self.world, self.group = ctx, n, k, rank, world, group
        self.lo, self.hi = even_shards(n, world)[rank]
        if len(set(hi - lo for lo, hi in even_shards(n, world))) != 1:
            raise ValueError("the all-gather needs equal row shards: N % world == 0")
        self.w = w_local

    @staticmethod
    def slice_rows(w_full_q4k, n: int, k: int, lo: int, hi: int):
        """Rows [lo, hi) of a Q4_K matrix (k/256 blocks of 144 bytes per row)."""
        row = (k // 256) * 144
        return w_full_q4k.view(-1)[lo * row:hi * row].clone()

    def forward(self, x, gather_logits: bool = True):
        """x [B, K] fp32 on this rank's device -> (tokens [B] int64, logits
        [B, N] or None). Every rank returns the same tokens."""
        b = x.shape[0]
        n_r = self.hi - self.lo
        local = torch.empty((b, n_r), dtype=torch.float32, device=x.device)
        tok, mx = self.bh.lmhead_argmax(self.ctx, self.w, n_r, self.k, x, logits=local)
        if gather_logits:
            full = gather_rows(local, self.world, self.group)
            # engine.cpp:36-43 over the assembled logits: first index of the maximum
            mxv = full.max(dim=1, keepdim=True).values
            first = (full == mxv).to(torch.int8).argmax(dim=1)
            return first.to(torch.int64), full
        vals, idxs = gather_candidates(mx, tok.to(torch.int64) + self.lo, self.world, self.group)
        best_i, _ = merge_argmax(vals, idxs)
        return best_i, None

    def enable_peer_exchange(self) -> None:
        """Map every rank's exchange mailbox into this process (CUDA IPC; the
        64-byte handles travel through the process group once). Afterwards
        forward_peer() exchanges the greedy pick through peer memory."""
        self.mbox = self.bh.PeerMailbox(self.ctx)
        self.epoch = 0
        (self.boxes,) = _map_peers([self.mbox], self.rank, self.world, self.group)

    def forward_peer(self, x):
        """x [B, K] -> global tokens [B] (int32, on the device), the same on
        every rank: this rank's rows, then the (max, first index) pairs
        exchanged through the mailboxes by the reducing kernel itself (no
        collective call). Every rank calls it the same number of times."""
        self.epoch += 1
        n_r = self.hi - self.lo
        tok, _ = self.bh.lmhead_argmax_tp(self.ctx, self.w, n_r, self.k, x, self.lo, self.rank, self.boxes,
                                          self.epoch)
        return tok

    def close_peer_exchange(self) -> None:
        if getattr(self, "mbox", None) is not None:
            if self.world > 1:
                dist.barrier(group=self.group)  # no rank still writes into a mailbox being unmapped
            self.mbox.close()
            self.mbox = None


class EPMoE:
    """Expert-parallel routed-expert FFN: this rank holds the banks of experts
    [lo, hi) (gate_own / up_own / down_own)."""

    def __init__(self, ctx, n_expert: int, n_embd: int, n_ff: int, k: int, rank: int, world: int, gate_own, up_own,
                 down_own, group=None):
        import burnhard as bh

        self.bh = bh
        self.ctx, self.n_expert, self.n_embd, self.n_ff, self.k = ctx, n_expert, n_embd, n_ff, k
        self.rank, self.world, self.group = rank, world, group
        self.lo, self.hi = even_shards(n_expert, world)[rank]
        self.gate, self.up, self.down = gate_own, up_own, down_own

    @staticmethod
    def slice_experts(bank, n_expert: int, lo: int, hi: int):
        """Experts [lo, hi) of a bundled expert bank (equal bytes per expert)."""
        per = bank.numel() // n_expert
        return bank.view(-1)[lo * per:hi * per].clone()

    def forward(self, cur, logits=None, selected=None, weights=None, out=None, residual: bool = False):
        """cur [T, n_embd] -> out [T, n_embd], identical on every rank."""
        dout, sel, w = self.bh.moe_ep(self.ctx, cur, self.gate, self.up, self.down, self.n_expert, self.lo, self.hi,
                                      self.n_ff, self.k, selected=selected, weights=weights, logits=logits)
        sum_expert_outputs(dout, self.world, self.group)
        return self.bh.moe_combine(self.ctx, dout, w, out=out, residual=residual)

    def enable_peer_exchange(self) -> None:
        """Map every rank's receive buffer and flag mailbox into this process
        (CUDA IPC handles exchanged once over the process group)."""
        bh = self.bh
        self.recv = bh.PeerMailbox(self.ctx, bh.lib.bh_moe_xchg_recv_bytes(self.n_embd))
        self.mbox = bh.PeerMailbox(self.ctx)
        self.epoch = 0
        self.recvs, self.boxes = _map_peers([self.recv, self.mbox], self.rank, self.world, self.group)

    def forward_peer(self, cur, logits=None, selected=None, weights=None, out=None, residual: bool = False):
        """As forward(), with the owned pairs exchanged through peer memory by
        the combining kernel instead of an all-reduce."""
        dout, sel, w = self.bh.moe_ep(self.ctx, cur, self.gate, self.up, self.down, self.n_expert, self.lo, self.hi,
                                      self.n_ff, self.k, selected=selected, weights=weights, logits=logits)
        self.epoch += 1
        return self.bh.moe_ep_exchange_combine(self.ctx, dout, sel, w, self.lo, self.hi, self.rank, self.recvs,
                                               self.boxes, self.epoch, out=out, residual=residual)

    def close_peer_exchange(self) -> None:
        if getattr(self, "mbox", None) is not None:
            if self.world > 1:
                dist.barrier(group=self.group)
            self.recv.close()
            self.mbox.close()
            self.recv = self.mbox = None
