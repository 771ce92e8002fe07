"""CPU: the reference's own ggml CPU backend, driven through its graph API
(oracle/_ref/libggml_graph.so, built from the reference tree), against the
oracle.

- one ggml_mul_mat node (Q4_K weight, f32 activations: ggml quantizes them to
  Q8_K and runs ggml_vec_dot_q4_K_q8_K in its chunks, ggml-cpu.c:1241-1439)
  equals the oracle's x86-fold matvec bit for bit, at 1 and several threads;
- ggml_quantize_chunk equals the oracle's Q4_K quantizer byte for byte;
- the decode step built as the reference engine builds it (forward.cpp
  build_block_decode, LM head, argmax) agrees with the oracle's CPU stack
  (cpu_stack.CpuStack) within the attention's float tolerance, and its
  greedy token equals the stack's wherever the top-2 margin is not a tie.
"""
from __future__ import annotations

import os

import numpy as np
import pytest

import oracle as om

pytestmark = pytest.mark.skipif(not os.path.exists(om.GRAPH_SO), reason="oracle/_ref not built (reference tree absent)")


@pytest.mark.parametrize("n,k,b", [(4096, 4096, 1), (1000, 2048, 3), (768, 12288, 2), (33, 256, 8)])
@pytest.mark.parametrize("threads", [1, 4])
def test_graph_mul_mat_equals_oracle(oracle, n, k, b, threads):
    w = oracle.quantize_q4k(oracle.normal((n, k), 11 + n, 0.0, 0.02))
    x = oracle.normal((b, k), 12 + k, 0.0, 1.0)
    got = om.graph_mul_mat(w, n, k, x, threads)
    want = oracle.matvec(w, n, k, oracle.quantize_q8k(x), b, om.FOLD_X86)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_graph_quantize_equals_oracle(oracle):
    x = oracle.normal((64, 4096), 5, 0.0, 0.02)
    assert np.array_equal(om.graph_quantize_q4k(x, 4), oracle.quantize_q4k(x).reshape(-1))


def test_graph_fill_normal_equals_oracle(oracle):
    L = om.graph_lib()
    out = np.empty(10001, np.float32)
    L.rg_fill_normal(om._ptr(out), out.size, 77, 1234, 0.5, 0.02, 3)
    assert np.array_equal(out, oracle.normal((10001,), 1234, 0.5, 0.02, first=77))


SMALL = dict(n_layer=2, n_embd=512, n_head=4, n_head_kv=2, head_dim=128, n_ff=1024, n_vocab=2000, n_ctx=16,
             rms_eps=1e-6, rope_theta=1e6)


def small_weights(oracle, c, seed=3):
    qd, kvd = c["n_head"] * c["head_dim"], c["n_head_kv"] * c["head_dim"]
    dims = [(qd, c["n_embd"]), (kvd, c["n_embd"]), (kvd, c["n_embd"]), (c["n_embd"], qd), (c["n_ff"], c["n_embd"]),
            (c["n_ff"], c["n_embd"]), (c["n_embd"], c["n_ff"])]
    w, s = {}, seed
    for l in range(c["n_layer"]):
        for which, (r, k) in enumerate(dims):
            w[(l, which)] = oracle.quantize_q4k(oracle.normal((r, k), s, 0.0, 0.02))
            s += 1
    w[(-1, 7)] = oracle.quantize_q4k(oracle.normal((c["n_vocab"], c["n_embd"]), s, 0.0, 0.02))
    L = c["n_layer"]
    norms = {"attn_norm": [oracle.normal((c["n_embd"],), 100 + l, 1.0, 0.02) for l in range(L)],
             "ffn_norm": [oracle.normal((c["n_embd"],), 200 + l, 1.0, 0.02) for l in range(L)],
             "q_norm": [oracle.normal((c["head_dim"],), 300 + l, 1.0, 0.02) for l in range(L)],
             "k_norm": [oracle.normal((c["head_dim"],), 400 + l, 1.0, 0.02) for l in range(L)],
             "out_norm": oracle.normal((c["n_embd"],), 500, 1.0, 0.02)}
    kc = [oracle.normal((c["n_ctx"], kvd), 600 + l, 0.0, 1.0) for l in range(L)]
    vc = [oracle.normal((c["n_ctx"], kvd), 700 + l, 0.0, 1.0) for l in range(L)]
    return w, norms, kc, vc


def test_graph_stack_matches_cpu_stack(oracle):
    from cpu_stack import CpuStack

    c = SMALL
    w, norms, kc, vc = small_weights(oracle, c)
    g = om.graph_stack_from_cpu(c, w, norms, kc, vc)

    def mv(wb, n, k, x):
        return oracle.matvec(wb, n, k, oracle.quantize_q8k(x), x.shape[0], om.FOLD_X86)

    cpu = CpuStack(c, w, norms, kc, vc, mv)
    agree = 0
    for pos in range(c["n_ctx"]):
        x = oracle.normal((c["n_embd"],), 900 + pos, 0.0, 1.0)
        t_g, lg_g, h_g = g.decode(x, pos, 2)
        t_c, lg_c, h_c = cpu.step(x, pos)
        assert np.abs(h_g - h_c).max() <= 2e-3 * np.abs(h_c).max()
        assert np.abs(lg_g - lg_c).max() <= 2e-2 * np.abs(lg_c).max()
        srt = np.sort(lg_c)
        if srt[-1] - srt[-2] > 1e-2 * np.abs(lg_c).max():
            assert t_g == t_c
        agree += t_g == t_c
    assert agree >= c["n_ctx"] - 1
    # the graph wrote each step's K/V into its cache at pos
    assert np.abs(g.tensor(0, 14).reshape(c["n_ctx"], -1) - cpu.vc[0].reshape(c["n_ctx"], -1)).max() <= \
        2e-3 * np.abs(cpu.vc[0]).max()
    g.close()


def test_graph_direct_row_loop_equals_oracle(oracle):
    n, k = 300, 4096
    w = oracle.quantize_q4k(oracle.normal((n, k), 21, 0.0, 0.02))
    x = oracle.normal((1, k), 22, 0.0, 1.0)
    y = np.empty(n, np.float32)
    assert om.graph_lib().rg_vec_dot_rows(om._ptr(np.ascontiguousarray(w)), n, k, om._ptr(x), om._ptr(y)) == 0
    want = oracle.matvec(w, n, k, oracle.quantize_q8k(x), 1, om.FOLD_X86)[0]
    assert np.array_equal(y.view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("n,k", [(64, 256), (100, 768), (200, 4096), (16, 12288)])
def test_q6k_oracle_equals_reference_vec_dot(oracle, n, k):
    """The oracle's Q6_K restatement (the AVX2 lane structure) equals the
    reference's own ggml_vec_dot_q6_K_q8_K bit for bit, on weights from the
    reference's Q6_K quantizer."""
    w = om.graph_quantize_q6k(oracle.normal((n, k), 40 + k, 0.0, 0.02))
    x = oracle.normal((1, k), 41 + n, 0.0, 1.0)
    want = om.graph_vec_dot_rows(om.GGML_TYPE_Q6_K, w, n, k, x)
    got = oracle.matvec_q6k(w, n, k, oracle.quantize_q8k(x), 1)[0]
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
