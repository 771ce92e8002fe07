"""GPU: the decode step's own fused launches at the Qwen3-8B width, bit for bit.

One layer of BASELINE config 2 (n_embd 4096, 32 query / 8 KV heads of 128,
n_ff 12288) and the full 151936-row LM head, decoded through the same launch
plan the 36-layer step uses (the stack's SM-budget plan: 16-warp CTAs, 1440-
byte stages, 8 threads per row for the 4096-row matrices). Each fused launch
is checked against the oracle on the inputs the device itself produced:

  QKV        RMSNorm(x) * attn_norm -> Q8_K -> [Wq; Wk; Wv] (3 segments)
  O          h1 = x + Wo . Q8_K(attn)           (residual-add epilogue)
  gate|up    Wg, Wu . Q8_K(RMSNorm(h1) * ffn_norm)  (3-D-TMA pair launch)
  SwiGLU     silu(gate) * up with ggml_v_silu's exp (pair epilogue)
  down       h2 = h1 + Wd . Q8_K(silu(gate) * up)
  LM head    logits = Wout . Q8_K(RMSNorm(h2) * out_norm), first-index argmax

All of these are bit-exact. The attention between QKV and O evaluates RoPE
with the device's sin/cos and its own summation order, so it is held to a
relative tolerance of 1e-4 against a float64 restatement instead.
"""
from __future__ import annotations

import numpy as np
import pytest

import oracle as om
from cpu_stack import rope_neox, stack_to_cpu

pytestmark = pytest.mark.gpu

CFG = dict(n_layer=1, n_embd=4096, n_head=32, n_head_kv=8, head_dim=128, n_ff=12288, n_vocab=151936, n_ctx=128)


def same_bits(a, b):
    a = np.ascontiguousarray(a, dtype=np.float32)
    b = np.ascontiguousarray(b, dtype=np.float32)
    return a.shape == b.shape and np.array_equal(a.view(np.uint32), b.view(np.uint32))


@pytest.mark.parametrize("pos", [0, 127])
def test_config2_layer_launches_bit_exact(ctx, bh, oracle, pos):
    import torch

    st = bh.Stack(ctx, bh.default_stack_config(**CFG), seed=2026 + pos)
    st.fill_kv(pos, 77)
    st.set_pos(pos)
    kc0 = st.to_host(0, bh.T_K_CACHE).copy()
    vc0 = st.to_host(0, bh.T_V_CACHE).copy()
    x = oracle.normal((CFG["n_embd"],), 31 + pos, 0.0, 1.0)
    tok = torch.zeros(1, dtype=torch.int32, device="cuda")
    st.decode(torch.from_numpy(x).cuda(), tok)
    torch.cuda.synchronize()
    assert ctx.status() == 0
    cfg, w, norms, _, _ = stack_to_cpu(st, with_caches=False)
    E, F, V = cfg["n_embd"], cfg["n_ff"], cfg["n_vocab"]
    hd, nh, nkv, eps = cfg["head_dim"], cfg["n_head"], cfg["n_head_kv"], cfg["rms_eps"]
    qd, kvd = nh * hd, nkv * hd

    def mv(which, n, k, a, layer=0):
        return oracle.matvec(w[(layer, which)], n, k, oracle.quantize_q8k(a[None]), 1, om.FOLD_X86)[0]

    # QKV after the RMSNorm prologue
    xn = oracle.rmsnorm(x, norms["attn_norm"][0], eps)
    qkv_want = np.concatenate([mv(bh.W_Q, qd, E, xn), mv(bh.W_K, kvd, E, xn), mv(bh.W_V, kvd, E, xn)])
    qkv = st.to_host(-1, bh.T_QKV)[0]
    assert same_bits(qkv, qkv_want)

    # attention (tolerance): q/k per-head RMSNorm, NeoX RoPE, softmax over 0..pos
    q = qkv[:qd].reshape(nh, hd)
    k = qkv[qd:qd + kvd].reshape(nkv, hd)
    v = qkv[qd + kvd:].reshape(nkv, hd)
    qr = rope_neox(oracle.rmsnorm(q, norms["q_norm"][0], eps), pos, cfg["rope_theta"])
    kr = rope_neox(oracle.rmsnorm(k, norms["k_norm"][0], eps), pos, cfg["rope_theta"])
    kc = kc0.reshape(CFG["n_ctx"], nkv, hd)
    vc = vc0.reshape(CFG["n_ctx"], nkv, hd)
    kc[pos], vc[pos] = kr, v
    attn = st.to_host(-1, bh.T_ATTN)[0]
    want = np.empty((nh, hd))
    for h in range(nh):
        g = h // (nh // nkv)
        s = (kc[: pos + 1, g].astype(np.float64) @ qr[h].astype(np.float64)) / np.sqrt(hd)
        e = np.exp(s - s.max())
        want[h] = (e @ vc[: pos + 1, g].astype(np.float64)) / e.sum()
    assert np.abs(attn.reshape(nh, hd) - want).max() <= 1e-4 * np.abs(want).max()

    # O projection and residual add, from the device's attention output
    h1 = (x + mv(bh.W_O, E, qd, attn)).astype(np.float32)
    assert same_bits(st.to_host(-1, bh.T_H_ATTN)[0], h1)

    # gate | up rows of the 3-D-TMA pair launch, before the SwiGLU
    xn2 = oracle.rmsnorm(h1, norms["ffn_norm"][0], eps)
    gate, up = mv(bh.W_GATE, F, E, xn2), mv(bh.W_UP, F, E, xn2)
    cap = st.to_host(-1, bh.T_GATE_UP)[0]
    assert same_bits(cap[:F], gate)
    assert same_bits(cap[F:], up)

    # SwiGLU epilogue: ggml_silu (ggml_v_silu) then ggml_mul
    act = (oracle.silu(gate) * up).astype(np.float32)
    assert same_bits(st.to_host(-1, bh.T_FFN_ACT)[0], act)

    # down projection and residual add
    h2 = (h1 + mv(bh.W_DOWN, E, F, act)).astype(np.float32)
    assert same_bits(st.to_host(-1, bh.T_HIDDEN)[0], h2)

    # LM head over all 151936 rows and the greedy pick
    xo = oracle.rmsnorm(h2, norms["out_norm"], eps)
    logits = oracle.matvec(w[(-1, 7)], V, E, oracle.quantize_q8k(xo[None]), 1, om.FOLD_X86)[0]
    assert same_bits(st.to_host(-1, bh.T_LOGITS)[0], logits)
    assert int(tok.cpu()[0]) == oracle.argmax(logits)
    st.close()
