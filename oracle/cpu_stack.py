"""CPU restatement of the decode block stack (one token, batch 1).

TEST INFRASTRUCTURE ONLY: the checker for bh_stack_decode and the timed CPU
path of bench.py's reference arm. The Q4_K matvecs go through a caller-chosen
function: the reference's own ggml mul_mat compiled into oracle/_ref
(quantize_row_q8_K + ggml_vec_dot_q4_K_q8_K, ggml-cpu.c:1241-1439), or the
oracle's restatement of it. RMSNorm and SiLU(gate)*up are the oracle's
C restatements of the reference's rms_norm_f32 and ggml_v_silu (bit-exact
with the device); the per-head q/k RMSNorm, NeoX RoPE and GQA softmax
attention are float32 numpy following the same formulas as the device
kernels but not their summation order or sin/cos, so the stack as a whole is
compared within a tolerance, while each matvec, RMSNorm and SwiGLU is
bit-exact given identical inputs; residual adds and the first-index argmax of
engine.cpp:36-43 are exact.
"""
from __future__ import annotations

import numpy as np

W_Q, W_K, W_V, W_O, W_GATE, W_UP, W_DOWN = range(7)


_ORACLE = None


def _oracle():
    global _ORACLE
    if _ORACLE is None:
        import oracle as om

        _ORACLE = om.Oracle()
    return _ORACLE


def rmsnorm(x: np.ndarray, g: np.ndarray, eps: float) -> np.ndarray:
    """rms_norm_f32 then ggml_mul (the oracle's C restatement: binary32
    squares summed sequentially in double, mean = (float)(sum / n),
    1 / sqrtf(mean + eps), x * scale * g)."""
    return _oracle().rmsnorm(np.asarray(x, dtype=np.float32), g, eps)


def swiglu(g: np.ndarray, u: np.ndarray) -> np.ndarray:
    """ggml_silu (ggml_v_silu lane by lane) then ggml_mul."""
    return (_oracle().silu(np.asarray(g, dtype=np.float32)) * u).astype(np.float32)


_LIBM = None


def _libm():
    global _LIBM
    if _LIBM is None:
        import ctypes as C
        import ctypes.util

        L = C.CDLL(ctypes.util.find_library("m") or "libm.so.6")
        for f in ("powf", "cosf", "sinf"):
            getattr(L, f).restype = C.c_float
        L.powf.argtypes = [C.c_float, C.c_float]
        L.cosf.argtypes = [C.c_float]
        L.sinf.argtypes = [C.c_float]
        _LIBM = L
    return _LIBM


def rope_table(pos: int, head_dim: int, theta: float):
    """(cos, sin) of the NeoX rotation angles of one position, as the
    reference's CPU backend fills its rope cache (ggml-cpu/ops.cpp
    ggml_rope_cache_init): theta_scale = powf(base, -2.0f / n_dims); theta
    starts at (float)pos and is multiplied by theta_scale after every pair in
    binary32; cosf / sinf of the host C library."""
    L = _libm()
    half = head_dim // 2
    scale = np.float32(L.powf(np.float32(theta), np.float32(-2.0) / np.float32(head_dim)))
    c = np.empty(half, np.float32)
    s = np.empty(half, np.float32)
    th = np.float32(pos)
    for i in range(half):
        c[i] = L.cosf(th)
        s[i] = L.sinf(th)
        th = np.float32(th * scale)
    return c, s


def rope_neox(x: np.ndarray, pos: int, theta: float) -> np.ndarray:
    """NeoX rotation of the pairs (i, i + head_dim/2): x0 c - x1 s, x0 s + x1 c
    in binary32 (ggml-cpu/ops.cpp rotate_pairs)."""
    x = np.asarray(x, dtype=np.float32)
    hd = x.shape[-1]
    half = hd // 2
    c, s = rope_table(pos, hd, theta)
    x1, x2 = x[..., :half], x[..., half:]
    return np.concatenate([(x1 * c) - (x2 * s), (x1 * s) + (x2 * c)], axis=-1).astype(np.float32)


class CpuStack:
    """weights[(layer, which)] -> Q4_K bytes; out weights under (-1, 7)."""

    def __init__(self, cfg: dict, weights: dict, norms: dict, k_cache: list, v_cache: list, matvec):
        self.cfg = cfg
        self.w = weights
        self.norms = norms
        self.kc = [np.array(a, dtype=np.float32, copy=True) for a in k_cache]
        self.vc = [np.array(a, dtype=np.float32, copy=True) for a in v_cache]
        self.matvec = matvec  # (w_bytes, n, k, x[1][k]) -> y[1][n]

    def mv(self, layer: int, which: int, n: int, k: int, x: np.ndarray) -> np.ndarray:
        return self.matvec(self.w[(layer, which)], n, k, x.reshape(1, k))[0]

    def attention(self, l: int, q: np.ndarray, k: np.ndarray, v: np.ndarray, pos: int) -> np.ndarray:
        c = self.cfg
        hd, nh, nkv = c["head_dim"], c["n_head"], c["n_head_kv"]
        eps = c["rms_eps"]
        q = q.reshape(nh, hd)
        k = k.reshape(nkv, hd)
        v = v.reshape(nkv, hd)
        qn = np.stack([rmsnorm(q[h], self.norms["q_norm"][l], eps) for h in range(nh)])
        kn = np.stack([rmsnorm(k[g], self.norms["k_norm"][l], eps) for g in range(nkv)])
        qr = rope_neox(qn, pos, c["rope_theta"])
        kr = rope_neox(kn, pos, c["rope_theta"])
        kc = self.kc[l].reshape(c["n_ctx"], nkv, hd)
        vc = self.vc[l].reshape(c["n_ctx"], nkv, hd)
        kc[pos] = kr
        vc[pos] = v
        out = np.empty((nh, hd), dtype=np.float32)
        group = nh // nkv
        scale = np.float32(1.0) / np.sqrt(np.float32(hd))
        for h in range(nh):
            g = h // group
            s = (kc[: pos + 1, g, :] @ qr[h]).astype(np.float32) * scale
            e = np.exp(s - s.max()).astype(np.float32)
            out[h] = (e @ vc[: pos + 1, g, :]) / np.float32(e.sum())
        return out.reshape(-1)

    def step(self, x: np.ndarray, pos: int):
        c = self.cfg
        E, F = c["n_embd"], c["n_ff"]
        qd, kvd = c["n_head"] * c["head_dim"], c["n_head_kv"] * c["head_dim"]
        eps = c["rms_eps"]
        h = np.array(x, dtype=np.float32, copy=True)
        for l in range(c["n_layer"]):
            xn = rmsnorm(h, self.norms["attn_norm"][l], eps)
            q = self.mv(l, W_Q, qd, E, xn)
            k = self.mv(l, W_K, kvd, E, xn)
            v = self.mv(l, W_V, kvd, E, xn)
            a = self.attention(l, q, k, v, pos)
            h = (h + self.mv(l, W_O, E, qd, a)).astype(np.float32)
            xn = rmsnorm(h, self.norms["ffn_norm"][l], eps)
            g = self.mv(l, W_GATE, F, E, xn)
            u = self.mv(l, W_UP, F, E, xn)
            act = swiglu(g, u)
            h = (h + self.mv(l, W_DOWN, E, F, act)).astype(np.float32)
        xn = rmsnorm(h, self.norms["out_norm"], eps)
        logits = self.matvec(self.w[(-1, 7)], c["n_vocab"], E, xn.reshape(1, E))[0]
        m = logits.max()
        tok = int(np.nonzero(logits == m)[0][0])
        return tok, logits, h


def stack_to_cpu(st, with_caches: bool = True):
    """Copy a device stack's weights, norms and KV caches to host arrays."""
    import burnhard as bh

    c = st.cfg.as_dict()
    w = {}
    for l in range(c["n_layer"]):
        for which in range(bh.W_PER_LAYER):
            w[(l, which)] = st.to_host(l, which)
    w[(-1, 7)] = st.to_host(-1, bh.W_OUTPUT)
    norms = {
        "attn_norm": [st.to_host(l, bh.T_ATTN_NORM)[0] for l in range(c["n_layer"])],
        "ffn_norm": [st.to_host(l, bh.T_FFN_NORM)[0] for l in range(c["n_layer"])],
        "q_norm": [st.to_host(l, bh.T_Q_NORM)[0] for l in range(c["n_layer"])],
        "k_norm": [st.to_host(l, bh.T_K_NORM)[0] for l in range(c["n_layer"])],
        "out_norm": st.to_host(-1, bh.T_OUT_NORM)[0],
    }
    kc = [st.to_host(l, bh.T_K_CACHE) for l in range(c["n_layer"])] if with_caches else None
    vc = [st.to_host(l, bh.T_V_CACHE) for l in range(c["n_layer"])] if with_caches else None
    return c, w, norms, kc, vc
