"""GPU: the decode block stack (bh_stack_*) against its CPU restatement.

Every matvec is bit-exact given identical inputs (tested elsewhere); here the
whole step is compared within a float tolerance, because the glue between
matvecs (RMSNorm, RoPE, softmax, SiLU) sums in a different order on the CPU.
The greedy token must equal the first argmax of the device's own logits."""
from __future__ import annotations

import numpy as np
import pytest

import oracle as om
from cpu_stack import CpuStack, stack_to_cpu

pytestmark = pytest.mark.gpu

SMALL = dict(n_layer=2, n_embd=512, n_head=4, n_head_kv=2, head_dim=128, n_ff=1024, n_vocab=2000, n_ctx=16)


def make_stack(bh, ctx, seed=7, **cfg):
    c = bh.default_stack_config(**{**SMALL, **cfg})
    return bh.Stack(ctx, c, seed)


def oracle_matvec(o):
    def mv(w, n, k, x):
        return o.matvec(w, n, k, o.quantize_q8k(x), x.shape[0], om.FOLD_X86)
    return mv


@pytest.mark.parametrize("pos", [0, 5, 15])
def test_stack_step_matches_cpu(ctx, bh, oracle, pos):
    check_step(ctx, bh, oracle, pos)


# query heads per KV group 1, 2, 4, 8 and positions past one round of the
# attention's position chunks (several rounds per warp)
@pytest.mark.parametrize(
    "n_head,n_head_kv,n_ctx,pos", [(8, 2, 300, 200), (4, 4, 64, 40), (8, 1, 200, 150), (4, 2, 600, 599)]
)
def test_stack_attention_shapes(ctx, bh, oracle, n_head, n_head_kv, n_ctx, pos):
    # logits within 1e-2 of their maximum: the last RMSNorm output is Q8_K-
    # quantized, and a code that rounds the other way on the device (its glue
    # sums in another order) moves every logit; the attention launch itself
    # is held to 1e-4 in test_stack_attention_kernel
    check_step(ctx, bh, oracle, pos, lg_tol=1e-2, n_head=n_head, n_head_kv=n_head_kv, n_ctx=n_ctx)


def check_step(ctx, bh, oracle, pos, lg_tol=2e-3, **cfg_over):
    import torch

    st = make_stack(bh, ctx, **cfg_over)
    st.fill_kv(pos, 1234)
    st.set_pos(pos)
    cfg, w, norms, kc, vc = stack_to_cpu(st)
    x = oracle.normal((cfg["n_embd"],), 4321 + pos, 0.0, 1.0)
    tok = torch.zeros(1, dtype=torch.int32, device="cuda")
    st.decode(torch.from_numpy(x).cuda(), tok)
    torch.cuda.synchronize()
    logits = st.to_host(-1, bh.T_LOGITS)[0]
    hidden = st.to_host(-1, bh.T_HIDDEN)[0]
    t_gpu = int(tok.cpu()[0])
    assert t_gpu == int(np.nonzero(logits == logits.max())[0][0])
    cpu = CpuStack(cfg, w, norms, kc, vc, oracle_matvec(oracle))
    t_cpu, lg_cpu, h_cpu = cpu.step(x, pos)
    scale = np.abs(h_cpu).max()
    assert np.abs(hidden - h_cpu).max() <= 2e-3 * scale, np.abs(hidden - h_cpu).max() / scale
    assert np.abs(logits - lg_cpu).max() <= lg_tol * np.abs(lg_cpu).max()
    srt = np.sort(lg_cpu)
    if srt[-1] - srt[-2] > 1e-2 * np.abs(lg_cpu).max():
        assert t_gpu == t_cpu
    # the KV append wrote this token's K/V at pos in every layer
    for l in range(cfg["n_layer"]):
        assert np.abs(st.to_host(l, bh.T_V_CACHE)[pos] - cpu.vc[l][pos]).max() <= 2e-3 * np.abs(cpu.vc[l][pos]).max()
    assert ctx.status() == 0


def test_stack_host_path_and_repeatability(ctx, bh, oracle):
    import torch

    st = make_stack(bh, ctx, seed=11)
    st.fill_kv(8, 99)
    st.set_pos(8)
    x = oracle.normal((SMALL["n_embd"],), 77, 0.0, 1.0)
    t_host = st.decode_host(x)
    tok = torch.zeros(1, dtype=torch.int32, device="cuda")
    lg1 = st.to_host(-1, bh.T_LOGITS)[0].copy()
    st.decode(torch.from_numpy(x).cuda(), tok)
    torch.cuda.synchronize()
    lg2 = st.to_host(-1, bh.T_LOGITS)[0]
    assert int(tok.cpu()[0]) == t_host
    assert np.array_equal(lg1.view(np.uint32), lg2.view(np.uint32))  # deterministic
    info = st.info()
    assert info["launches"] == 5 * SMALL["n_layer"] + 2
    assert info["weight_bytes"] >= sum(
        r * (c // 256) * 144 for r, c in [(512, 512), (256, 512), (256, 512), (512, 512), (1024, 512), (1024, 512), (512, 1024)]
    ) * SMALL["n_layer"]


def test_stack_rejects_bad_config(ctx, bh):
    with pytest.raises(bh.BHError):
        make_stack(bh, ctx, n_embd=500)
    with pytest.raises(bh.BHError):
        make_stack(bh, ctx, n_head=3, n_head_kv=2)
    make_stack(bh, ctx, n_head=6, n_head_kv=2).close()  # 3 query heads per group: supported
    st = make_stack(bh, ctx)
    with pytest.raises(bh.BHError):
        st.set_pos(SMALL["n_ctx"])


@pytest.mark.parametrize(
    "n_head,n_head_kv,n_ctx,pos",
    [(4, 2, 16, 0), (4, 2, 16, 15), (8, 2, 300, 200), (4, 4, 64, 40), (8, 1, 200, 150), (4, 2, 600, 599)],
)
def test_stack_attention_kernel(ctx, bh, oracle, n_head, n_head_kv, n_ctx, pos):
    """The attention launch alone: the last layer's q|k|v as the device
    projected them, through per-head RMSNorm, NeoX RoPE, the KV append and
    softmax attention over positions 0..pos, against a float64 restatement
    (the device follows the reference's binary32 order; the reference graph
    comparison of tests/test_gpu_stack_reference.py checks that bit for bit)."""
    import torch

    from cpu_stack import rmsnorm, rope_neox

    st = make_stack(bh, ctx, n_head=n_head, n_head_kv=n_head_kv, n_ctx=n_ctx)
    st.fill_kv(pos, 99)
    st.set_pos(pos)
    kc0 = st.to_host(SMALL["n_layer"] - 1, bh.T_K_CACHE).copy()
    vc0 = st.to_host(SMALL["n_layer"] - 1, bh.T_V_CACHE).copy()
    x = oracle.normal((SMALL["n_embd"],), 5 + pos, 0.0, 1.0)
    tok = torch.zeros(1, dtype=torch.int32, device="cuda")
    st.decode(torch.from_numpy(x).cuda(), tok)
    torch.cuda.synchronize()
    L = SMALL["n_layer"] - 1
    cfg = st.cfg.as_dict()
    hd, eps = cfg["head_dim"], cfg["rms_eps"]
    qkv = st.to_host(-1, bh.T_QKV)[0]
    got = st.to_host(-1, bh.T_ATTN)[0].reshape(n_head, hd)
    qn_w, kn_w = st.to_host(L, bh.T_Q_NORM)[0], st.to_host(L, bh.T_K_NORM)[0]
    q = qkv[: n_head * hd].reshape(n_head, hd)
    k = qkv[n_head * hd : (n_head + n_head_kv) * hd].reshape(n_head_kv, hd)
    v = qkv[(n_head + n_head_kv) * hd :].reshape(n_head_kv, hd)
    qr = rope_neox(np.stack([rmsnorm(q[h], qn_w, eps) for h in range(n_head)]), pos, cfg["rope_theta"])
    kr = rope_neox(np.stack([rmsnorm(k[g], kn_w, eps) for g in range(n_head_kv)]), pos, cfg["rope_theta"])
    kc = kc0.reshape(n_ctx, n_head_kv, hd)
    vc = vc0.reshape(n_ctx, n_head_kv, hd)
    kc[pos], vc[pos] = kr, v
    # the append
    kc_dev = st.to_host(L, bh.T_K_CACHE).reshape(n_ctx, n_head_kv, hd)
    vc_dev = st.to_host(L, bh.T_V_CACHE).reshape(n_ctx, n_head_kv, hd)
    assert np.array_equal(vc_dev[pos], v)
    # RMSNorm and the ggml rotation table: equal up to the double sum's order
    assert np.abs(kc_dev[pos] - kr).max() <= 1e-6 * np.abs(kr).max()
    group = n_head // n_head_kv
    scale = np.float32(1.0) / np.sqrt(np.float32(hd))
    want = np.empty((n_head, hd), dtype=np.float64)
    for h in range(n_head):
        g = h // group
        s = (kc[: pos + 1, g, :].astype(np.float64) @ qr[h].astype(np.float64)) * float(scale)
        e = np.exp(s - s.max())
        want[h] = (e @ vc[: pos + 1, g, :].astype(np.float64)) / e.sum()
    err = np.abs(got - want).max() / np.abs(want).max()
    assert err <= 1e-4, err
    assert ctx.status() == 0
