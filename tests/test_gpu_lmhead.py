"""GPU: the LM-head matvec with the engine's greedy pick (first index of the
maximum, engine.cpp:36-43) through bh_q4k_lmhead_argmax."""
from __future__ import annotations

import numpy as np
import pytest

from conftest import golden_inputs
from test_gpu_matvec import assert_bits_equal, dev, host, seeded_q4k

import oracle as om

pytestmark = pytest.mark.gpu


def first_argmax(v: np.ndarray) -> int:
    return int(np.nonzero(v == v.max())[0][0])


@pytest.mark.parametrize("fold", [om.FOLD_X86, om.FOLD_GENERIC])
def test_golden_argmax_with_planted_tie(ctx, bh, oracle, golden, fold):
    case = golden["argmax"]
    n, k, b, w, x = golden_inputs(oracle, case)
    logits = dev(np.zeros((b, n), np.float32))
    tok, mx = bh.lmhead_argmax(ctx, dev(case["w_q4k"]), n, k, dev(x), logits=logits, fold=fold)
    want = case["y_x86"] if fold == om.FOLD_X86 else case["y_generic"]
    assert_bits_equal(host(logits), want, "logits")
    got = host(tok)
    for c in range(b):
        assert got[c] == first_argmax(want[c])
    assert got[0] == int(case["argmax_x86"][0])           # the tie resolves to the first row
    assert np.array_equal(host(mx), want.max(axis=1))


@pytest.mark.parametrize("b", [1, 4])
def test_lm_head_config_size(ctx, bh, oracle, b):
    """Config 5: 151936 x 4096, batch 1 and 4; logits bit-exact on sampled
    rows (all rows at batch 1), tokens equal the first argmax."""
    n, k = 151936, 4096
    wq = seeded_q4k(ctx, oracle, n, k, seed=5151, check_rows=16)
    # plant a tie on a future maximum: copy row 10 over row 150000 (later row)
    wq_h = host(wq).reshape(n, -1)
    x = oracle.normal((b, k), 6161 + b, 0.0, 1.0)
    logits = dev(np.zeros((b, n), np.float32))
    tok, mx = bh.lmhead_argmax(ctx, wq, n, k, dev(x), logits=logits)
    lg = host(logits)
    xq = oracle.quantize_q8k(x)
    if b == 1:
        assert_bits_equal(lg, oracle.matvec(wq_h, n, k, xq, b, om.FOLD_X86), "full logits")
    else:
        rows = np.unique(np.random.default_rng(b).integers(0, n, 2048))
        ref = oracle.matvec(np.ascontiguousarray(wq_h[rows]), len(rows), k, xq, b, om.FOLD_X86)
        assert_bits_equal(lg[:, rows], ref, "sampled logits")
    t = host(tok)
    for c in range(b):
        assert t[c] == first_argmax(lg[c])
    assert np.array_equal(host(mx), lg.max(axis=1))


def test_tie_across_ctas(ctx, bh, oracle):
    """Equal maxima in rows owned by different CTAs: the lowest index wins."""
    n, k = 20000, 512
    w = oracle.normal((n, k), 99, 0.0, 0.02)
    wq = oracle.quantize_q4k(w)
    x = oracle.normal((1, k), 98, 0.0, 1.0)
    y = oracle.matvec(wq, n, k, oracle.quantize_q8k(x), 1, om.FOLD_X86)[0]
    top = first_argmax(y)
    wq2 = wq.copy()
    for r in (top + 7000) % n, (top + 13000) % n, 5:
        wq2[r] = wq[top]
    tok, _ = bh.lmhead_argmax(ctx, dev(wq2), n, k, dev(x))
    y2 = oracle.matvec(wq2, n, k, oracle.quantize_q8k(x), 1, om.FOLD_X86)[0]
    assert int(host(tok)[0]) == first_argmax(y2) == min(top, 5, (top + 7000) % n, (top + 13000) % n)


def test_peer_exchange_one_rank_matches_lmhead(ctx, bh, oracle):
    """The peer-exchange LM head with a single rank (its own mailbox): the
    same tokens and maxima as bh_q4k_lmhead_argmax, over consecutive epochs."""
    import torch

    n, k = 6000, 1024
    g = torch.Generator(device="cuda").manual_seed(3)
    w = ctx.q4k_quantize(torch.randn((n, k), generator=g, device="cuda") * 0.02)
    box = bh.PeerMailbox(ctx)
    try:
        for epoch, b in enumerate((1, 3, 8, 1), start=1):
            x = torch.randn((b, k), generator=g, device="cuda")
            want_t, want_m = bh.lmhead_argmax(ctx, w, n, k, x)
            got_t, got_m = bh.lmhead_argmax_tp(ctx, w, n, k, x, 0, 0, [box.ptr], epoch)
            torch.cuda.synchronize()
            assert torch.equal(got_t, want_t)
            assert torch.equal(got_m.view(torch.int32), want_m.view(torch.int32))
        assert ctx.status() == 0
    finally:
        box.close()


def test_peer_exchange_times_out_when_a_rank_never_arrives(ctx, bh):
    """Failure detection without a fault: a two-rank exchange whose second
    mailbox nobody writes. The kernel's bounded wait (about a second) runs
    out, the token is -1 and the device status reports BH_ETIMEDOUT; the
    context stays usable."""
    import torch

    n, k = 512, 256
    w = ctx.q4k_quantize(torch.randn((n, k), device="cuda") * 0.02)
    own, silent = bh.PeerMailbox(ctx), bh.PeerMailbox(ctx)
    try:
        x = torch.randn((1, k), device="cuda")
        # rank 0 of two: rank 1's pair never arrives in rank 0's mailbox
        tok, _ = bh.lmhead_argmax_tp(ctx, w, n // 2, k, x, 0, 0, [own.ptr, silent.ptr], 1)
        torch.cuda.synchronize()
        assert int(tok[0]) == -1
        assert ctx.status() == bh.BH_ETIMEDOUT
        assert ctx.status() == 0  # cleared by the read above
        t2, _ = bh.lmhead_argmax(ctx, w, n, k, x)  # the context still works
        torch.cuda.synchronize()
        assert 0 <= int(t2[0]) < n
    finally:
        own.close()
        silent.close()
