"""The reference arm's CPU decode step, built entirely on the host.

TEST INFRASTRUCTURE / CPU BASELINE ONLY. The Qwen3-8B-shaped stack of
BASELINE config 2 as the reference engine's ggml graph (oracle.GraphStack on
oracle/_ref/libggml_graph.so, the reference's own ggml CPU backend), with
weights generated and quantized on the host: seeded N(0, 0.02) values from
the splitmix64 + Box-Muller generator, quantized by ggml_quantize_chunk
(quantize_row_q4_K_ref) over all host threads. Nothing here loads the
product library.

Quantizing all 36 layers on the host takes minutes, so `n_distinct` layers
get their own weights and layer l uses those of l % n_distinct: every step
still runs all 36 layers' matvecs over 4.26 GB of weight bytes, and with 4
distinct layers plus the LM head the working set (784 MB) is several times
any host's last-level cache, so the weights stream from DRAM every step.
"""
from __future__ import annotations

import numpy as np

import oracle as om

# tensor ids of include/bh_q4k.h
W_Q, W_K, W_V, W_O, W_GATE, W_UP, W_DOWN, W_OUTPUT = range(8)
T_ATTN_NORM, T_FFN_NORM, T_Q_NORM, T_K_NORM, T_OUT_NORM, T_K_CACHE, T_V_CACHE = range(8, 15)

CHUNK_ROWS = 16384


def _seed(seed: int, layer: int, which: int) -> int:
    z = (seed ^ (0x51ED2701A3B4C5D6 + (layer * 0x9E3779B97F4A7C15) + which * 0xD6E8FEB86659FD93)) & (2**64 - 1)
    z = ((z ^ (z >> 31)) * 0x7FB5D329728EA185) & (2**64 - 1)
    return z ^ (z >> 27)


def _fill(L, out: np.ndarray, seed: int, mean: float, std: float, nthreads: int, first: int = 0) -> None:
    L.rg_fill_normal(om._ptr(out), out.size, first, seed, mean, std, nthreads)


def _quantized(L, rows: int, k: int, seed: int, nthreads: int, dst: np.ndarray) -> None:
    """dst (rows * k/256 * 144 bytes) <- Q4_K of seeded N(0, 0.02) [rows][k]."""
    rb = om.q4k_row_bytes(k)
    tmp = np.empty((min(rows, CHUNK_ROWS), k), np.float32)
    for r0 in range(0, rows, CHUNK_ROWS):
        nr = min(CHUNK_ROWS, rows - r0)
        t = tmp[:nr]
        _fill(L, t, seed, 0.0, 0.02, nthreads, first=r0 * k)
        L.rg_quantize_q4k(om._ptr(t), om._ptr(dst[r0 * rb:(r0 + nr) * rb]), nr, k, nthreads)


def make_host_stack(cfg: dict, seed: int, nthreads: int, n_distinct: int = 4, kv_pos: int = 0) -> om.GraphStack:
    """A GraphStack of config cfg with host-generated weights and norms
    (norms ~ 1 + N(0, 0.02)) and seeded N(0, 1) K/V history for [0, kv_pos)."""
    L = om.graph_lib()
    g = om.GraphStack(cfg, n_distinct=n_distinct)
    c = cfg
    qd, kvd = c["n_head"] * c["head_dim"], c["n_head_kv"] * c["head_dim"]
    dims = {W_Q: (qd, c["n_embd"]), W_K: (kvd, c["n_embd"]), W_V: (kvd, c["n_embd"]), W_O: (c["n_embd"], qd),
            W_GATE: (c["n_ff"], c["n_embd"]), W_UP: (c["n_ff"], c["n_embd"]), W_DOWN: (c["n_embd"], c["n_ff"])}
    nd = min(n_distinct, c["n_layer"]) if n_distinct > 0 else c["n_layer"]
    for l in range(nd):
        for which, (r, k) in dims.items():
            _quantized(L, r, k, _seed(seed, l, which), nthreads, g.tensor(l, which))
        for which, n in ((T_ATTN_NORM, c["n_embd"]), (T_FFN_NORM, c["n_embd"]), (T_Q_NORM, c["head_dim"]),
                         (T_K_NORM, c["head_dim"])):
            _fill(L, g.tensor(l, which), _seed(seed, l, which), 1.0, 0.02, nthreads)
    _quantized(L, c["n_vocab"], c["n_embd"], _seed(seed, -1, W_OUTPUT), nthreads, g.tensor(-1, W_OUTPUT))
    _fill(L, g.tensor(-1, T_OUT_NORM), _seed(seed, -1, T_OUT_NORM), 1.0, 0.02, nthreads)
    if kv_pos > 0:
        for l in range(c["n_layer"]):
            for which in (T_K_CACHE, T_V_CACHE):
                t = g.tensor(l, which)
                _fill(L, t[: kv_pos * kvd], _seed(seed, l, 100 + which), 0.0, 1.0, nthreads)
    return g
