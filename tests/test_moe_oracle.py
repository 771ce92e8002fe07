"""CPU: the routed-expert FFN restatement (oracle) against the reference's own
code compiled in oracle/_ref (ggml's soft_max, SiLU and Q4_K x Q8_K vec_dot)
and against the reference's top-k / renormalisation rules
(desktop/engine/src/forward.cpp:1018-1107, ggml-cpu/ops.cpp:8157-8194)."""
from __future__ import annotations

import numpy as np
import pytest

import oracle as om


def test_expf_bit_exact_with_reference(oracle, reference):
    """The oracle's exp is one lane of ggml's AVX2 ggml_v_expf: equal bit for
    bit to the reference's compiled kernel over the whole range it is used
    on, including the two-factor scaling (|n| > 126) and saturation
    (|n| > 192) branches, and within ggml's stated bound (1.45 + 0.5 ulp) of
    the true exponential."""
    x = np.concatenate([np.linspace(-110.0, 95.0, 800_000, dtype=np.float32),
                        oracle.normal((200_000,), 5, 0.0, 8.0),
                        np.array([0.0, -0.0, 88.3, 88.8, -87.0, -100.0, -104.0, 1e-30, -1e-30,
                                  np.inf, -np.inf, np.nan, 200.0, -200.0, 135.0, -135.0], np.float32)])
    x = np.concatenate([x, np.zeros((-x.size) % 8, np.float32)]).astype(np.float32)
    a, b = oracle.expf(x), reference.expf(x)
    nan = np.isnan(x)
    assert np.isnan(a[nan]).all() and np.isnan(b[nan]).all()  # (NaN payloads may differ)
    assert np.array_equal(a[~nan].view(np.uint32), b[~nan].view(np.uint32))
    y = a.astype(np.float64)
    ref = np.exp(x.astype(np.float64))
    normal = np.isfinite(x) & (ref > 1.2e-38) & (ref < 3.4e38)
    ulp = np.spacing(ref[normal].astype(np.float32)).astype(np.float64)
    assert (np.abs(y[normal] - ref[normal]) / ulp).max() <= 1.96


def test_silu_bit_exact_with_reference(oracle, reference):
    x = np.concatenate([oracle.normal((200_000,), 3, 0.0, 4.0),
                        np.linspace(-120.0, 120.0, 4000, dtype=np.float32)]).astype(np.float32)
    a, b = oracle.silu(x), reference.silu(x)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


def ref_route(reference, logits, k, norm=True):
    """Top-k as the reference's ops.cpp writes it, over the reference's own soft_max."""
    p = reference.soft_max(logits)
    ids = np.empty((logits.shape[0], k), np.int32)
    w = np.empty((logits.shape[0], k), np.float32)
    for t in range(logits.shape[0]):
        order = np.argsort(-p[t], kind="stable")[:k]
        if k > 1:
            order[[0, 1]] = order[[1, 0]]
        ids[t] = order
        ww = p[t][order]
        if norm:
            ww = ww / np.float32(np.sum(ww.astype(np.float64)))
        w[t] = ww
    return ids, w


@pytest.mark.parametrize("n_expert,k", [(128, 8), (64, 4), (256, 8), (16, 1), (9, 2)])
def test_route_matches_reference(oracle, reference, n_expert, k):
    """Routing equals the reference's soft_max + top-k + renormalisation bit
    for bit when n_expert is a multiple of 8 (all through ggml_v_expf); the
    reference's n % 8 tail goes through libm expf, which the restatement does
    not reproduce, so 9 experts are held to 1e-5 / 1e-6."""
    logits = oracle.normal((32, n_expert), 100 + n_expert + k, 0.0, 1.0)
    ids, w = oracle.moe_route(logits, k)
    rids, rw = ref_route(reference, logits, k)
    assert (ids == rids).all()
    if n_expert % 8 == 0:
        assert np.array_equal(w.view(np.uint32), rw.view(np.uint32))
    else:
        np.testing.assert_allclose(w, rw, rtol=1e-5, atol=1e-6)
    assert np.allclose(w.sum(1), 1.0, atol=1e-6)


def test_route_ties_take_lower_index(oracle):
    logits = np.zeros((1, 16), np.float32)
    logits[0, [3, 9, 12]] = 2.0
    ids, w = oracle.moe_route(logits, 4)
    # ranks: 3, 9, 12 (equal, index order), then 0; slots 0 and 1 swapped
    assert ids[0].tolist() == [9, 3, 12, 0]
    assert w[0][0] == w[0][1] == w[0][2]


def test_route_unnormalised_is_softmax(oracle, reference):
    logits = oracle.normal((8, 128), 77, 0.0, 1.0)
    ids, w = oracle.moe_route(logits, 8, norm=False)
    p = reference.soft_max(logits)
    for t in range(8):
        assert np.array_equal(w[t].view(np.uint32), p[t][ids[t]].view(np.uint32))


def test_rmsnorm_restatement(oracle):
    x = oracle.normal((4, 2048), 9, 0.0, 1.0)
    g = oracle.normal((2048,), 10, 1.0, 0.02)
    y = oracle.rmsnorm(x, g, 1e-6)
    for r in range(4):
        ss = float(np.sum((x[r] * x[r]).astype(np.float64)))
        mean = np.float32(ss / 2048)
        scale = np.float32(1.0) / np.sqrt(np.float32(mean + np.float32(1e-6)))
        assert (y[r] == (x[r] * scale) * g).all()


def small_banks(oracle, n_expert, n_embd, n_ff, seed):
    gate = oracle.quantize_q4k(oracle.normal((n_expert * n_ff, n_embd), seed, 0.0, 0.02))
    up = oracle.quantize_q4k(oracle.normal((n_expert * n_ff, n_embd), seed + 1, 0.0, 0.02))
    down = oracle.quantize_q4k(oracle.normal((n_expert * n_embd, n_ff), seed + 2, 0.0, 0.02))
    return gate, up, down


def test_moe_ffn_internal_consistency(oracle):
    E, D, F, k, T = 8, 512, 256, 3, 3
    gate, up, down = small_banks(oracle, E, D, F, 50)
    cur = oracle.normal((T, D), 60, 0.0, 1.0)
    ids, w = oracle.moe_route(oracle.normal((T, E), 61), k)
    out, gu, dout = oracle.moe_ffn(cur, ids, w, gate, up, down, D, F)
    gb, ub, db = gate.reshape(E, -1), up.reshape(E, -1), down.reshape(E, -1)
    for t in range(T):
        xq = oracle.quantize_q8k(cur[t:t + 1])
        acc = np.zeros(D, np.float64)
        for s in range(k):
            e = ids[t, s]
            g = oracle.matvec(gb[e], F, D, xq, 1)[0]
            u = oracle.matvec(ub[e], F, D, xq, 1)[0]
            assert (gu[t * k + s, :F] == g).all() and (gu[t * k + s, F:] == u).all()
            par = oracle.silu(g) * u
            d = oracle.matvec(db[e], D, F, oracle.quantize_q8k(par[None]), 1)[0]
            assert (dout[t * k + s] == d).all()
            acc += (d * w[t, s]).astype(np.float64)
        assert (out[t] == acc.astype(np.float32)).all()


def test_moe_ffn_vs_reference_kernels(oracle, reference):
    """The same block composed from the reference's own Q8_K quantizer, x86
    vec_dot and SiLU (ggml_vec_silu_f32) with the slot-order double sum: the
    restatement equals it bit for bit."""
    E, D, F, k, T = 8, 512, 256, 4, 2
    gate, up, down = small_banks(oracle, E, D, F, 70)
    cur = oracle.normal((T, D), 80, 0.0, 1.0)
    ids, w = ref_route(reference, oracle.normal((T, E), 81), k)
    out, _, _ = oracle.moe_ffn(cur, ids, w, gate, up, down, D, F)
    gb, ub, db = gate.reshape(E, -1), up.reshape(E, -1), down.reshape(E, -1)
    for t in range(T):
        xq = reference.quantize_q8k(cur[t:t + 1])
        acc = np.zeros(D, np.float64)
        for s in range(k):
            e = ids[t, s]
            g = reference.matvec_rows(gb[e], F, D, xq, 1, om.FOLD_X86)[0]
            u = reference.matvec_rows(ub[e], F, D, xq, 1, om.FOLD_X86)[0]
            par = reference.silu(g) * u
            d = reference.matvec_rows(db[e], D, F, reference.quantize_q8k(par[None]), 1, om.FOLD_X86)[0]
            acc += (d * w[t, s]).astype(np.float64)
        ref_out = acc.astype(np.float32)
        assert np.array_equal(out[t].view(np.uint32), ref_out.view(np.uint32))
