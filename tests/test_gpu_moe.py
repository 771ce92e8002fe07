"""GPU: the routed-expert FFN (bh_moe_route, bh_q4k_moe, bh_moe_stack_*)
against the oracle's restatement of the reference's stock MoE block
(desktop/engine/src/forward.cpp:1001-1118) and BURN_MOE's given-routing
contract (burn_moe_op.cpp:202-372).

The device evaluates the same binary32/binary64 operation sequence as the
oracle (its own Cody-Waite exp on both sides, the reference's reduction
orders), so routing, gate|up, expert outputs and the weighted sum are
compared bit for bit."""
from __future__ import annotations

import numpy as np
import pytest

import oracle as om

pytestmark = pytest.mark.gpu


def to_dev(a):
    import torch

    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def banks(oracle, n_expert, n_embd, n_ff, seed):
    gate = oracle.quantize_q4k(oracle.normal((n_expert * n_ff, n_embd), seed, 0.0, 0.02))
    up = oracle.quantize_q4k(oracle.normal((n_expert * n_ff, n_embd), seed + 1, 0.0, 0.02))
    down = oracle.quantize_q4k(oracle.normal((n_expert * n_embd, n_ff), seed + 2, 0.0, 0.02))
    return gate, up, down


@pytest.mark.parametrize("T,E,k", [(1, 128, 8), (8, 128, 8), (5, 64, 4), (3, 256, 8), (2, 16, 1), (4, 9, 2)])
def test_route_bit_exact(ctx, bh, oracle, T, E, k):
    logits = oracle.normal((T, E), 500 + T * E + k, 0.0, 1.0)
    ids, w = bh.moe_route(ctx, to_dev(logits), k)
    rids, rw = oracle.moe_route(logits, k)
    assert (ids.cpu().numpy() == rids).all()
    assert (w.cpu().numpy().view(np.uint32) == rw.view(np.uint32)).all()
    assert ctx.status() == 0


def test_route_ties(ctx, bh, oracle):
    logits = np.zeros((2, 32), np.float32)
    logits[0, [5, 17, 30]] = 1.5
    logits[1, :] = 0.25  # all equal
    ids, w = bh.moe_route(ctx, to_dev(logits), 4)
    rids, rw = oracle.moe_route(logits, 4)
    assert (ids.cpu().numpy() == rids).all()
    assert (w.cpu().numpy() == rw).all()


@pytest.mark.parametrize("fold", [om.FOLD_X86, om.FOLD_GENERIC])
@pytest.mark.parametrize("T", [1, 3, 8])
def test_moe_logits_bit_exact(ctx, bh, oracle, T, fold):
    E, D, F, k = 16, 512, 256, 4
    gate, up, down = banks(oracle, E, D, F, 900)
    cur = oracle.normal((T, D), 910 + T, 0.0, 1.0)
    logits = oracle.normal((T, E), 920 + T, 0.0, 1.0)
    out, ids, w = bh.moe(ctx, to_dev(cur), to_dev(gate), to_dev(up), to_dev(down), E, F, k,
                         logits=to_dev(logits), fold=fold)
    rids, rw = oracle.moe_route(logits, k)
    assert (ids.cpu().numpy() == rids).all() and (w.cpu().numpy() == rw).all()
    ref, _, _ = oracle.moe_ffn(cur, rids, rw, gate, up, down, D, F, fold=fold)
    assert (out.cpu().numpy().view(np.uint32) == ref.view(np.uint32)).all()
    assert ctx.status() == 0


@pytest.mark.parametrize("T", [1, 2, 8])
def test_moe_given_routing_shared_experts(ctx, bh, oracle, T):
    """BURN_MOE's contract: selected / weights given. Tokens share experts, so
    each shared expert is streamed once for several columns."""
    E, D, F, k = 12, 768, 512, 3
    gate, up, down = banks(oracle, E, D, F, 930)
    cur = oracle.normal((T, D), 940 + T, 0.0, 1.0)
    rng = np.random.default_rng(T)
    ids = np.stack([rng.choice([1, 4, 7, 11, 2], size=k, replace=False) for _ in range(T)]).astype(np.int32)
    w = rng.random((T, k)).astype(np.float32)
    out, _, _ = bh.moe(ctx, to_dev(cur), to_dev(gate), to_dev(up), to_dev(down), E, F, k,
                       selected=to_dev(ids), weights=to_dev(w))
    ref, _, _ = oracle.moe_ffn(cur, ids, w, gate, up, down, D, F)
    assert (out.cpu().numpy().view(np.uint32) == ref.view(np.uint32)).all()
    assert ctx.status() == 0


@pytest.mark.parametrize("T", [1, 4])
def test_moe_config_shape(ctx, bh, oracle, T):
    """The 30B-A3B expert shape: 128 experts of 2048 -> 768 -> 2048, top-8.
    Banks are quantized on the device (bit-exact with the oracle's quantizer,
    tested elsewhere) and copied back for the oracle."""
    import torch

    E, D, F, k = 128, 2048, 768, 8
    g = torch.Generator(device="cuda").manual_seed(T)
    dev = {}
    for name, rows, cols in (("gate", E * F, D), ("up", E * F, D), ("down", E * D, F)):
        wf = torch.randn((rows, cols), generator=g, device="cuda") * 0.02
        dev[name] = ctx.q4k_quantize(wf)
        del wf
    cur = oracle.normal((T, D), 950 + T, 0.0, 1.0)
    logits = oracle.normal((T, E), 960 + T, 0.0, 1.0)
    out, ids, w = bh.moe(ctx, to_dev(cur), dev["gate"], dev["up"], dev["down"], E, F, k, logits=to_dev(logits))
    rids, rw = oracle.moe_route(logits, k)
    assert (ids.cpu().numpy() == rids).all()
    host = {n: t.cpu().numpy() for n, t in dev.items()}
    ref, _, _ = oracle.moe_ffn(cur, rids, rw, host["gate"], host["up"], host["down"], D, F)
    assert (out.cpu().numpy().view(np.uint32) == ref.view(np.uint32)).all()


def test_moe_bad_expert_id_reports(ctx, bh, oracle):
    import torch

    E, D, F, k = 8, 256, 256, 2
    gate, up, down = banks(oracle, E, D, F, 970)
    cur = oracle.normal((1, D), 971, 0.0, 1.0)
    for bad in ([[1, 8]], [[3, 3]]):  # out of range; repeated within the token
        ids = np.array(bad, np.int32)
        w = np.array([[0.5, 0.5]], np.float32)
        bh.moe(ctx, to_dev(cur), to_dev(gate), to_dev(up), to_dev(down), E, F, k, selected=to_dev(ids),
               weights=to_dev(w))
        torch.cuda.synchronize()
        assert ctx.status() == bh.BH_EINVAL
        assert ctx.status() == 0  # cleared by the read


def test_moe_invalid_args(ctx, bh, oracle):
    import torch

    cur = torch.zeros((1, 256), device="cuda")
    wb = torch.zeros(256 * 144, dtype=torch.uint8, device="cuda")
    lg = torch.zeros((1, 8), device="cuda")
    for kw in (dict(T=9), dict(k=9), dict(n_ff=100)):
        T = kw.get("T", 1)
        with pytest.raises(bh.BHError):
            bh.moe(ctx, torch.zeros((T, 256), device="cuda"), wb, wb, wb, 8, kw.get("n_ff", 256), kw.get("k", 2),
                   logits=torch.zeros((T, 8), device="cuda"))
    with pytest.raises(bh.BHError):  # both routing sources
        bh.moe(ctx, cur, wb, wb, wb, 8, 256, 2, selected=torch.zeros((1, 2), dtype=torch.int32, device="cuda"),
               weights=torch.zeros((1, 2), device="cuda"), logits=lg)


# ---------------------------------------------------------------------------
# the MoE layer stack
# ---------------------------------------------------------------------------
SMALL = dict(n_layer=3, n_embd=512, n_ff=256, n_expert=16, k=4)


def stack_oracle_step(oracle, st, bh, h):
    cfg = st.cfg
    D, F, E, k = cfg.n_embd, cfg.n_ff, cfg.n_expert, cfg.k
    h = h.copy()
    for l in range(cfg.n_layer):
        gate = st.to_host(l, bh.MOE_GATE)
        up = st.to_host(l, bh.MOE_UP)
        down = st.to_host(l, bh.MOE_DOWN)
        logits = st.to_host(l, bh.MOE_LOGITS).reshape(cfg.n_tok, E)
        norm = st.to_host(l, bh.MOE_NORM)
        x = oracle.rmsnorm(h, norm, cfg.rms_eps)
        ids, w = oracle.moe_route(logits, k)
        out, _, _ = oracle.moe_ffn(x, ids, w, gate, up, down, D, F)
        h = h + out
    return h


@pytest.mark.parametrize("n_tok", [1, 2, 8])
def test_moe_stack_bit_exact(ctx, bh, oracle, n_tok):
    import torch

    cfg = bh.default_moe_config(**SMALL, n_tok=n_tok)
    st = bh.MoeStack(ctx, cfg, seed=31 + n_tok)
    h0 = oracle.normal((n_tok, cfg.n_embd), 32 + n_tok, 0.0, 1.0)
    out = torch.empty((n_tok, cfg.n_embd), device="cuda")
    st.step(to_dev(h0), out)
    torch.cuda.synchronize()
    ref = stack_oracle_step(oracle, st, bh, h0)
    assert (out.cpu().numpy().view(np.uint32) == ref.view(np.uint32)).all()
    # the host path gives the same bits, and steps are repeatable
    host_out = np.empty_like(h0)
    st.step_host(h0, host_out)
    assert (host_out.view(np.uint32) == ref.view(np.uint32)).all()
    assert st.info()["launches"] == cfg.n_layer
    assert ctx.status() == 0
    st.close()


def test_moe_stack_info_counts_distinct_experts(ctx, bh, oracle):
    cfg = bh.default_moe_config(**SMALL, n_tok=4)
    st = bh.MoeStack(ctx, cfg, seed=5)
    h0 = oracle.normal((4, cfg.n_embd), 6, 0.0, 1.0)
    out = np.empty_like(h0)
    st.step_host(h0, out)
    per_expert = (2 * cfg.n_ff * (cfg.n_embd // 256) + cfg.n_embd * (cfg.n_ff // 256)) * 144
    pairs = 4 * cfg.k
    act = 4 * cfg.n_embd * 8 + pairs * 2 * cfg.n_ff * 8 + pairs * cfg.n_embd * 8
    want = 0
    for l in range(cfg.n_layer):
        ids = st.to_host(l, bh.MOE_SELECTED)
        want += len(set(ids.tolist())) * per_expert + act
    assert st.info()["step_bytes"] == want
    st.close()


def test_moe_peer_exchange_one_rank_matches_moe(ctx, bh):
    """The expert-parallel exchange fused with the combine, one rank owning
    every expert (its own receive buffer and mailbox): bit-identical to
    bh_q4k_moe over consecutive epochs."""
    import torch

    E, D, F, k = 16, 512, 256, 4
    g = torch.Generator(device="cuda").manual_seed(21)
    gate = ctx.q4k_quantize(torch.randn((E * F, D), generator=g, device="cuda") * 0.02)
    up = ctx.q4k_quantize(torch.randn((E * F, D), generator=g, device="cuda") * 0.02)
    down = ctx.q4k_quantize(torch.randn((E * D, F), generator=g, device="cuda") * 0.02)
    recv = bh.PeerMailbox(ctx, bh.lib.bh_moe_xchg_recv_bytes(D))
    box = bh.PeerMailbox(ctx)
    try:
        for epoch, T in enumerate((1, 3, 8, 2), start=1):
            cur = torch.randn((T, D), generator=g, device="cuda")
            lg = torch.randn((T, E), generator=g, device="cuda")
            ref, _, _ = bh.moe(ctx, cur, gate, up, down, E, F, k, logits=lg)
            dout, sel, w = bh.moe_ep(ctx, cur, gate, up, down, E, 0, E, F, k, logits=lg)
            out = bh.moe_ep_exchange_combine(ctx, dout, sel, w, 0, E, 0, [recv.ptr], [box.ptr], epoch)
            torch.cuda.synchronize()
            assert torch.equal(out.view(torch.int32), ref.view(torch.int32))
        assert ctx.status() == 0
    finally:
        recv.close()
        box.close()


def test_moe_barrier_timeout_then_bit_exact(bh, oracle):
    """A grid-barrier wait that runs out leaves its arrivals counted; clearing
    the timeout through bh_device_status resets the barrier, and the next
    step is bit-exact again. The timeout is made without a fault: the barrier
    word is preset so that no arrival is ever the last one (a flag nothing
    sets), with a short wait bound, so every CTA gives up and returns."""
    import torch

    ctx = bh.Context(0)
    try:
        ctx.tune(bh.TUNE_BARRIER_WAIT, 20)  # ~0.5 ms per barrier wait
        cfg = bh.default_moe_config(**SMALL, n_tok=2)
        st = bh.MoeStack(ctx, cfg, seed=41)
        h0 = oracle.normal((2, cfg.n_embd), 42, 0.0, 1.0)
        ref = stack_oracle_step(oracle, st, bh, h0)
        out = torch.empty((2, cfg.n_embd), device="cuda")
        st.step(to_dev(h0), out)
        torch.cuda.synchronize()
        assert (out.cpu().numpy().view(np.uint32) == ref.view(np.uint32)).all()
        ptr, nbytes = st.tensor(-1, bh.MOE_BARRIER)
        words = bh.device_view(ptr, nbytes // 4, "<u4")
        words[0] = 0x8000  # arrivals start at 32768: the count never reaches the grid size
        torch.cuda.synchronize()
        st.step(to_dev(h0), out)
        assert ctx.status(clear=True) == bh.BH_ETIMEDOUT
        assert int(words.cpu()[0]) == 0  # reset with the clear
        out.fill_(0)
        st.step(to_dev(h0), out)
        torch.cuda.synchronize()
        assert (out.cpu().numpy().view(np.uint32) == ref.view(np.uint32)).all()
        assert ctx.status() == 0
        st.close()
    finally:
        ctx.close()
