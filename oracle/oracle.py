"""ctypes bindings for the test-infrastructure libraries in this folder.

TEST INFRASTRUCTURE ONLY: the parity checker (``Oracle`` -> liboracle.so, the
CPU restatement of the reference's Q4_K x Q8_K arithmetic), the compiled
reference (``Reference`` -> _ref/libq4k_ref.so, the reference's own
ggml-quants.c / ggml-cpu quants sources) and the reference's whole ggml CPU
backend driven through its graph API (``GraphStack`` / ``graph_mul_mat`` ->
_ref/libggml_graph.so). Nothing on the product path imports this module;
tests/, __graft_entry__.smoke() and bench.py's CPU legs do.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "liboracle.so")
REF_SO = os.path.join(HERE, "_ref", "libq4k_ref.so")
GRAPH_SO = os.path.join(HERE, "_ref", "libggml_graph.so")
MMVQ_SO = os.path.join(HERE, "_ref", "libmmvq_ref.so")

QK = 256
Q4K_BYTES = 144
Q6K_BYTES = 210
GGML_TYPE_Q4_K = 12
GGML_TYPE_Q6_K = 14
Q8K_BYTES = 292
FOLD_X86 = 0
FOLD_GENERIC = 1

_f32p = C.POINTER(C.c_float)
_vp = C.c_void_p


def build(ref_root: str | None = None) -> None:
    """Compile liboracle.so (and _ref when the reference tree is present)."""
    cmd = ["make", "-s", "-C", HERE, "all"]
    if ref_root:
        cmd.append(f"REF_ROOT={ref_root}")
    subprocess.run(cmd, check=True)


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(_vp)


def q4k_row_bytes(k: int) -> int:
    return k // QK * Q4K_BYTES


def q8k_row_bytes(k: int) -> int:
    return k // QK * Q8K_BYTES


class Oracle:
    """The CPU restatement (q4k_oracle.c)."""

    def __init__(self, path: str = ORACLE_SO):
        if not os.path.exists(path):
            build()
        L = C.CDLL(path)
        self.lib = L
        L.bho_fp16_to_fp32.argtypes = [C.c_uint16]
        L.bho_fp16_to_fp32.restype = C.c_float
        L.bho_fp32_to_fp16.argtypes = [C.c_float]
        L.bho_fp32_to_fp16.restype = C.c_uint16
        L.bho_fill_normal_range.argtypes = [_vp, C.c_int64, C.c_int64, C.c_uint64, C.c_double, C.c_double]
        L.bho_quantize_q4k.argtypes = [_vp, _vp, C.c_int64, C.c_int64, C.c_int]
        L.bho_dequantize_row_q4k.argtypes = [_vp, _vp, C.c_int64]
        L.bho_quantize_row_q8k.argtypes = [_vp, _vp, C.c_int64]
        L.bho_vec_dot_generic.argtypes = [C.c_int, _vp, _vp]
        L.bho_vec_dot_generic.restype = C.c_float
        L.bho_vec_dot_x86.argtypes = [C.c_int, _vp, _vp]
        L.bho_vec_dot_x86.restype = C.c_float
        L.bho_matvec.argtypes = [_vp, C.c_int64, C.c_int64, _vp, C.c_int, _vp, C.c_int, C.c_int]
        L.bho_partials.argtypes = [_vp, C.c_int64, C.c_int64, _vp, C.c_int, _vp]
        L.bho_argmax.argtypes = [_vp, C.c_int64]
        L.bho_argmax.restype = C.c_int64
        L.bho_expf_n.argtypes = [_vp, C.c_int64, _vp]
        L.bho_matvec_q6k.argtypes = [_vp, C.c_int64, C.c_int64, _vp, C.c_int, _vp, C.c_int]
        L.bho_silu_n.argtypes = [_vp, C.c_int64, _vp]
        L.bho_rmsnorm.argtypes = [_vp, _vp, C.c_int, C.c_float, _vp]
        L.bho_moe_route.argtypes = [_vp, C.c_int, C.c_int, C.c_int, _vp, _vp]
        L.bho_moe_ffn.argtypes = [_vp, C.c_int, _vp, _vp, C.c_int, _vp, _vp, _vp, C.c_int, C.c_int,
                                  _vp, _vp, _vp, C.c_int, C.c_int]

    def normal(self, shape, seed: int, mean: float = 0.0, std: float = 1.0, first: int = 0) -> np.ndarray:
        out = np.empty(shape, dtype=np.float32)
        self.lib.bho_fill_normal_range(_ptr(out), first, out.size, seed & (2**64 - 1), mean, std)
        return out

    def quantize_q4k(self, x: np.ndarray, nthreads: int = 0) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=np.float32)
        n, k = x.shape
        out = np.zeros((n, q4k_row_bytes(k)), dtype=np.uint8)
        self.lib.bho_quantize_q4k(_ptr(x), _ptr(out), n, k, nthreads or (os.cpu_count() or 1))
        return out

    def dequantize_q4k(self, w: np.ndarray, k: int) -> np.ndarray:
        w = np.ascontiguousarray(w, dtype=np.uint8)
        n = w.size // q4k_row_bytes(k)
        out = np.empty((n, k), dtype=np.float32)
        self.lib.bho_dequantize_row_q4k(_ptr(w), _ptr(out), n * k)
        return out

    def quantize_q8k(self, x: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=np.float32)
        rows = x.reshape(-1, x.shape[-1])
        k = rows.shape[1]
        out = np.zeros((rows.shape[0], q8k_row_bytes(k)), dtype=np.uint8)
        self.lib.bho_quantize_row_q8k(_ptr(rows), _ptr(out), rows.size)
        return out

    def matvec(self, w: np.ndarray, n: int, k: int, xq: np.ndarray, b: int,
               fold: int = FOLD_X86, nthreads: int = 0) -> np.ndarray:
        y = np.empty((b, n), dtype=np.float32)
        self.lib.bho_matvec(_ptr(np.ascontiguousarray(w)), n, k, _ptr(np.ascontiguousarray(xq)), b,
                            _ptr(y), fold, nthreads or (os.cpu_count() or 1))
        return y

    def matvec_q6k(self, w: np.ndarray, n: int, k: int, xq: np.ndarray, b: int, nthreads: int = 0) -> np.ndarray:
        """Q6_K rows x Q8_K columns, the x86 fold: y [b][n]."""
        y = np.empty((b, n), dtype=np.float32)
        self.lib.bho_matvec_q6k(_ptr(np.ascontiguousarray(w)), n, k, _ptr(np.ascontiguousarray(xq)), b, _ptr(y),
                                nthreads or (os.cpu_count() or 1))
        return y

    def partials(self, w: np.ndarray, n: int, k: int, xq: np.ndarray, b: int) -> np.ndarray:
        out = np.empty((b, n, k // QK, 9), dtype=np.int32)
        self.lib.bho_partials(_ptr(np.ascontiguousarray(w)), n, k, _ptr(np.ascontiguousarray(xq)), b, _ptr(out))
        return out

    def vec_dot(self, k: int, w_row: np.ndarray, x_row: np.ndarray, fold: int = FOLD_X86) -> float:
        f = self.lib.bho_vec_dot_generic if fold == FOLD_GENERIC else self.lib.bho_vec_dot_x86
        return float(f(k, _ptr(np.ascontiguousarray(w_row)), _ptr(np.ascontiguousarray(x_row))))

    def argmax(self, v: np.ndarray) -> int:
        v = np.ascontiguousarray(v, dtype=np.float32)
        return int(self.lib.bho_argmax(_ptr(v), v.size))

    def fp32_to_fp16(self, f: float) -> int:
        return int(self.lib.bho_fp32_to_fp16(f))

    # ---- routed-expert FFN glue -------------------------------------------
    def expf(self, x: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=np.float32)
        y = np.empty_like(x)
        self.lib.bho_expf_n(_ptr(x), x.size, _ptr(y))
        return y

    def silu(self, x: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=np.float32)
        y = np.empty_like(x)
        self.lib.bho_silu_n(_ptr(x), x.size, _ptr(y))
        return y

    def rmsnorm(self, x: np.ndarray, gamma: np.ndarray | None, eps: float) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=np.float32)
        rows = x.reshape(-1, x.shape[-1])
        y = np.empty_like(rows)
        g = None if gamma is None else np.ascontiguousarray(gamma, dtype=np.float32)
        for i in range(rows.shape[0]):
            self.lib.bho_rmsnorm(_ptr(rows[i]), None if g is None else _ptr(g), rows.shape[1], eps, _ptr(y[i]))
        return y.reshape(x.shape)

    def moe_route(self, logits: np.ndarray, k: int, norm: bool = True):
        """logits [T, n_expert] -> (ids [T, k] int32, w [T, k] float32)."""
        logits = np.ascontiguousarray(logits, dtype=np.float32)
        t, e = logits.shape
        ids = np.empty((t, k), dtype=np.int32)
        w = np.empty((t, k), dtype=np.float32)
        for i in range(t):
            self.lib.bho_moe_route(_ptr(logits[i]), e, k, int(norm), _ptr(ids[i]), _ptr(w[i]))
        return ids, w

    def moe_ffn(self, cur: np.ndarray, ids: np.ndarray, w: np.ndarray, gate: np.ndarray, up: np.ndarray,
                down: np.ndarray, n_embd: int, n_ff: int, fold: int = FOLD_X86, nthreads: int = 0):
        """cur [T, n_embd] -> (out [T, n_embd], gu [T*k, 2*n_ff], dout [T*k, n_embd])."""
        cur = np.ascontiguousarray(cur, dtype=np.float32)
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        w = np.ascontiguousarray(w, dtype=np.float32)
        t, k = ids.shape
        out = np.empty((t, n_embd), dtype=np.float32)
        gu = np.empty((t * k, 2 * n_ff), dtype=np.float32)
        dout = np.empty((t * k, n_embd), dtype=np.float32)
        self.lib.bho_moe_ffn(_ptr(cur), t, _ptr(ids), _ptr(w), k, _ptr(np.ascontiguousarray(gate)),
                             _ptr(np.ascontiguousarray(up)), _ptr(np.ascontiguousarray(down)), n_embd, n_ff,
                             _ptr(out), _ptr(gu), _ptr(dout), fold, nthreads or (os.cpu_count() or 1))
        return out, gu, dout

    def fp16_to_fp32(self, h: int) -> float:
        return float(self.lib.bho_fp16_to_fp32(h))


class Reference:
    """The reference's own code, compiled from its tree (oracle/_ref)."""

    def __init__(self, path: str = REF_SO):
        if not os.path.exists(path):
            raise FileNotFoundError(f"{path} not built (make -C oracle ref)")
        L = C.CDLL(path)
        self.lib = L
        L.ref_has_avx2.restype = C.c_int
        for name in ("ref_quantize_row_q4k", "ref_quantize_row_q8k", "ref_quantize_row_q8k_ref"):
            getattr(L, name).argtypes = [_vp, _vp, C.c_int64]
        L.ref_dequantize_row_q4k.argtypes = [_vp, _vp, C.c_int64]
        for name in ("ref_vec_dot_generic", "ref_vec_dot_x86"):
            getattr(L, name).argtypes = [C.c_int, _vp, _vp]
            getattr(L, name).restype = C.c_float
        L.ref_pool_create.argtypes = [C.c_int]
        L.ref_pool_create.restype = _vp
        L.ref_pool_free.argtypes = [_vp]
        L.ref_pool_threads.argtypes = [_vp]
        L.ref_pool_threads.restype = C.c_int
        L.ref_mul_mat.argtypes = [_vp, _vp, C.c_int64, C.c_int64, _vp, C.c_int, _vp, _vp]
        L.ref_soft_max.argtypes = [_vp, C.c_int, _vp]
        L.ref_silu.argtypes = [_vp, C.c_int, _vp]
        L.ref_vexpf.argtypes = [_vp, C.c_int, _vp]
        self.has_avx2 = bool(L.ref_has_avx2())
        self._pool = None

    def quantize_q4k(self, x: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=np.float32)
        n, k = x.shape
        out = np.zeros((n, q4k_row_bytes(k)), dtype=np.uint8)
        self.lib.ref_quantize_row_q4k(_ptr(x), _ptr(out), n * k)
        return out

    def quantize_q8k(self, x: np.ndarray, x86: bool = True) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=np.float32)
        rows = x.reshape(-1, x.shape[-1])
        out = np.zeros((rows.shape[0], q8k_row_bytes(rows.shape[1])), dtype=np.uint8)
        f = self.lib.ref_quantize_row_q8k if x86 else self.lib.ref_quantize_row_q8k_ref
        f(_ptr(rows), _ptr(out), rows.size)
        return out

    def dequantize_q4k(self, w: np.ndarray, k: int) -> np.ndarray:
        w = np.ascontiguousarray(w, dtype=np.uint8)
        n = w.size // q4k_row_bytes(k)
        out = np.empty((n, k), dtype=np.float32)
        self.lib.ref_dequantize_row_q4k(_ptr(w), _ptr(out), n * k)
        return out

    def matvec_rows(self, w: np.ndarray, n: int, k: int, xq: np.ndarray, b: int, fold: int) -> np.ndarray:
        """Row-by-row vec_dot, single thread (fold selects generic or AVX2)."""
        f = self.lib.ref_vec_dot_generic if fold == FOLD_GENERIC else self.lib.ref_vec_dot_x86
        w = np.ascontiguousarray(w, dtype=np.uint8).reshape(n, -1)
        xq = np.ascontiguousarray(xq, dtype=np.uint8).reshape(b, -1)
        y = np.empty((b, n), dtype=np.float32)
        for c in range(b):
            xp = _ptr(xq[c])
            for r in range(n):
                y[c, r] = f(k, w[r].ctypes.data_as(_vp), xp)
        return y

    def soft_max(self, x: np.ndarray) -> np.ndarray:
        """Row-wise ggml soft_max of x [T, n] through the reference's vec.cpp."""
        x = np.ascontiguousarray(x, dtype=np.float32)
        y = np.empty_like(x)
        for i in range(x.shape[0]):
            self.lib.ref_soft_max(_ptr(x[i]), x.shape[1], _ptr(y[i]))
        return y

    def expf(self, x: np.ndarray) -> np.ndarray:
        """ggml_v_expf (AVX2) of every element; x.size must be a multiple of 8."""
        x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1)
        assert x.size % 8 == 0
        y = np.empty_like(x)
        self.lib.ref_vexpf(_ptr(x), x.size, _ptr(y))
        return y

    def silu(self, x: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=np.float32)
        y = np.empty_like(x)
        self.lib.ref_silu(_ptr(x), x.size, _ptr(y))
        return y

    def pool(self, nthreads: int):
        if self._pool is None or self.lib.ref_pool_threads(self._pool) != nthreads:
            if self._pool is not None:
                self.lib.ref_pool_free(self._pool)
            self._pool = self.lib.ref_pool_create(nthreads)
        return self._pool

    def mul_mat(self, w: np.ndarray, n: int, k: int, x: np.ndarray, nthreads: int,
                xq_scratch: np.ndarray | None = None, out: np.ndarray | None = None) -> np.ndarray:
        """ggml-style threaded mul_mat: fp32 activations [B][K] -> Y [B][N]."""
        x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, k)
        b = x.shape[0]
        if xq_scratch is None:
            xq_scratch = np.empty(b * q8k_row_bytes(k), dtype=np.uint8)
        y = out if out is not None else np.empty((b, n), dtype=np.float32)
        self.lib.ref_mul_mat(self.pool(nthreads), _ptr(w), n, k, _ptr(x), b, _ptr(xq_scratch), _ptr(y))
        return y

    def __del__(self):
        try:
            if self._pool is not None:
                self.lib.ref_pool_free(self._pool)
        except Exception:
            pass


# ---------------------------------------------------------------------------
# the reference's ggml CPU backend through its graph API (oracle/_ref)
# ---------------------------------------------------------------------------
class RgConfig(C.Structure):
    _fields_ = [("n_layer", C.c_int), ("n_embd", C.c_int), ("n_head", C.c_int), ("n_head_kv", C.c_int),
                ("head_dim", C.c_int), ("n_ff", C.c_int), ("n_vocab", C.c_int), ("n_ctx", C.c_int),
                ("rms_eps", C.c_float), ("rope_theta", C.c_float), ("n_distinct", C.c_int)]


_GRAPH = None


def graph_lib():
    global _GRAPH
    if _GRAPH is None:
        if not os.path.exists(GRAPH_SO):
            raise FileNotFoundError(f"{GRAPH_SO} not built (make -C oracle graph)")
        L = C.CDLL(GRAPH_SO)
        L.rg_stack_create.argtypes = [C.POINTER(RgConfig)]
        L.rg_stack_create.restype = _vp
        L.rg_stack_free.argtypes = [_vp]
        L.rg_stack_tensor.argtypes = [_vp, C.c_int, C.c_int, C.POINTER(C.c_size_t)]
        L.rg_stack_tensor.restype = _vp
        L.rg_stack_decode.argtypes = [_vp, _vp, C.c_int, C.c_int, _vp, _vp]
        L.rg_mul_mat.argtypes = [_vp, C.c_int64, C.c_int64, _vp, C.c_int, _vp, C.c_int]
        L.rg_quantize_q4k.argtypes = [_vp, _vp, C.c_int64, C.c_int64, C.c_int]
        L.rg_fill_normal.argtypes = [_vp, C.c_int64, C.c_int64, C.c_uint64, C.c_double, C.c_double, C.c_int]
        L.rg_has_avx2.restype = C.c_int
        L.rg_vec_dot_rows.argtypes = [_vp, C.c_int64, C.c_int64, _vp, _vp]
        L.rg_vec_dot_rows_type.argtypes = [C.c_int, _vp, C.c_int64, C.c_int64, _vp, _vp]
        L.rg_quantize_q6k.argtypes = [_vp, _vp, C.c_int64, C.c_int64]
        L.rg_gguf_write.argtypes = [C.c_char_p, C.c_int, C.POINTER(C.c_char_p), C.POINTER(C.c_int),
                                    C.POINTER(C.c_int64), C.POINTER(C.c_int64), C.POINTER(_vp), C.c_int,
                                    C.POINTER(C.c_char_p), C.POINTER(C.c_uint32), C.c_char_p, C.c_char_p,
                                    C.c_char_p, C.c_float]
        _GRAPH = L
    return _GRAPH


def graph_mul_mat(w: np.ndarray, n: int, k: int, x: np.ndarray, nthreads: int, out: np.ndarray | None = None):
    """One ggml_mul_mat node (Q4_K weight, f32 activations [B][K]) computed by
    the reference's CPU backend on nthreads threads: y [B][N]."""
    L = graph_lib()
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, k)
    y = out if out is not None else np.empty((x.shape[0], n), dtype=np.float32)
    if L.rg_mul_mat(_ptr(np.ascontiguousarray(w)), n, k, _ptr(x), x.shape[0], _ptr(y), nthreads) != 0:
        raise RuntimeError("rg_mul_mat failed")
    return y


def graph_quantize_q4k(w: np.ndarray, nthreads: int) -> np.ndarray:
    """fp32 [rows][k] -> Q4_K bytes through ggml_quantize_chunk, rows over threads."""
    L = graph_lib()
    w = np.ascontiguousarray(w, dtype=np.float32)
    rows, k = w.shape
    out = np.empty(rows * q4k_row_bytes(k), dtype=np.uint8)
    L.rg_quantize_q4k(_ptr(w), _ptr(out), rows, k, nthreads)
    return out


class GraphStack:
    """The decode step as the reference engine's ggml graph (forward.cpp
    build_block_decode + LM head) on the reference's CPU backend. Tensor ids
    follow include/bh_q4k.h; ``fill(layer, which, array)`` copies host data in."""

    def __init__(self, cfg: dict, n_distinct: int = 0):
        L = graph_lib()
        c = RgConfig(**{f: cfg[f] for f, _ in RgConfig._fields_ if f != "n_distinct"}, n_distinct=n_distinct)
        self.cfg = dict(cfg)
        self.h = L.rg_stack_create(C.byref(c))
        if not self.h:
            raise MemoryError("rg_stack_create failed")
        self.L = L

    def tensor(self, layer: int, which: int) -> np.ndarray:
        """A numpy view of one tensor's host memory (uint8 for Q4_K weights, else float32)."""
        nb = C.c_size_t(0)
        p = self.L.rg_stack_tensor(self.h, layer, which, C.byref(nb))
        if not p:
            raise IndexError((layer, which))
        dt = np.uint8 if which <= 7 else np.float32
        n = nb.value // np.dtype(dt).itemsize
        return np.ctypeslib.as_array(C.cast(p, C.POINTER(C.c_uint8 if dt == np.uint8 else C.c_float)), shape=(n,))

    def fill(self, layer: int, which: int, a: np.ndarray) -> None:
        t = self.tensor(layer, which)
        src = np.ascontiguousarray(a).reshape(-1).view(t.dtype)
        assert src.size == t.size, (layer, which, src.size, t.size)
        t[:] = src

    def decode(self, x: np.ndarray, pos: int, nthreads: int, logits: bool = True):
        """(token, logits [n_vocab] or None, hidden [n_embd]) of one step at pos."""
        x = np.ascontiguousarray(x, dtype=np.float32)
        lg = np.empty(self.cfg["n_vocab"], np.float32) if logits else None
        hid = np.empty(self.cfg["n_embd"], np.float32)
        tok = self.L.rg_stack_decode(self.h, _ptr(x), pos, nthreads, _ptr(lg) if logits else None, _ptr(hid))
        if tok < 0:
            raise RuntimeError("rg_stack_decode failed")
        return tok, lg, hid

    def close(self) -> None:
        if self.h:
            self.L.rg_stack_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def graph_stack_from_cpu(cfg: dict, w: dict, norms: dict, kc: list | None, vc: list | None) -> GraphStack:
    """A GraphStack holding the given host copies (cpu_stack.stack_to_cpu's layout)."""
    g = GraphStack(cfg)
    for l in range(cfg["n_layer"]):
        for which in range(7):
            g.fill(l, which, w[(l, which)])
        g.fill(l, 8, norms["attn_norm"][l])
        g.fill(l, 9, norms["ffn_norm"][l])
        g.fill(l, 10, norms["q_norm"][l])
        g.fill(l, 11, norms["k_norm"][l])
        if kc is not None:
            g.fill(l, 13, kc[l])
            g.fill(l, 14, vc[l])
    g.fill(-1, 7, w[(-1, 7)])
    g.fill(-1, 12, norms["out_norm"])
    return g


# ---------------------------------------------------------------------------
# the reference's own GPU Q4_K matvec (ggml-cuda mul_mat_vec_q, oracle/_ref)
# ---------------------------------------------------------------------------
class RefMMVQ:
    """ggml-cuda's mul_mat_vec_q<Q4_K> with its Q8_1 activation quantizer,
    built for sm_100a from the reference tree: the GPU comparison point. Its
    activations are Q8_1 (32-value blocks), so its results are close to, not
    equal to, the Q4_K x Q8_K path."""

    def __init__(self, path: str = MMVQ_SO):
        if not os.path.exists(path):
            raise FileNotFoundError(f"{path} not built (make -C oracle mmvq)")
        L = C.CDLL(path)
        L.refmmvq_xq_bytes.argtypes = [C.c_int]
        L.refmmvq_xq_bytes.restype = C.c_size_t
        L.refmmvq_q4k.argtypes = [_vp, C.c_int, C.c_int, _vp, C.c_int, _vp, _vp, _vp]
        self.lib = L

    def xq_bytes(self, k: int, b: int) -> int:
        return int(self.lib.refmmvq_xq_bytes(k)) * b

    def matvec(self, w_ptr: int, n: int, k: int, x_ptr: int, b: int, xq_ptr: int, y_ptr: int, stream: int = 0) -> None:
        """Device pointers: y [b][n] = W . x [b][k]; xq scratch of xq_bytes(k, b)."""
        if self.lib.refmmvq_q4k(w_ptr, n, k, x_ptr, b, xq_ptr, y_ptr, stream) != 0:
            raise RuntimeError("refmmvq_q4k failed")


def graph_quantize_q6k(w: np.ndarray) -> np.ndarray:
    """fp32 [rows][k] -> Q6_K bytes through the reference's ggml_quantize_chunk."""
    L = graph_lib()
    w = np.ascontiguousarray(w, dtype=np.float32)
    rows, k = w.shape
    out = np.empty(rows * (k // QK) * Q6K_BYTES, dtype=np.uint8)
    L.rg_quantize_q6k(_ptr(w), _ptr(out), rows, k)
    return out


def graph_vec_dot_rows(ggml_type: int, w: np.ndarray, n: int, k: int, x: np.ndarray) -> np.ndarray:
    """The reference CPU backend's vec_dot for each row against from_float(x) (one column)."""
    y = np.empty(n, np.float32)
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1)
    if graph_lib().rg_vec_dot_rows_type(ggml_type, _ptr(np.ascontiguousarray(w)), n, k, _ptr(x), _ptr(y)) != 0:
        raise RuntimeError("rg_vec_dot_rows_type failed")
    return y


def graph_gguf_write(path: str, tensors: list, u32: dict, strs: tuple | None = None, f32: tuple | None = None):
    """Write a GGUF file with the reference's own writer: tensors = [(name,
    ggml_type, ne0, ne1, bytes ndarray)], u32 = {key: value}."""
    L = graph_lib()
    n = len(tensors)
    names = (C.c_char_p * n)(*[t[0].encode() for t in tensors])
    types = (C.c_int * n)(*[t[1] for t in tensors])
    ne0 = (C.c_int64 * n)(*[t[2] for t in tensors])
    ne1 = (C.c_int64 * n)(*[t[3] for t in tensors])
    bufs = [np.ascontiguousarray(t[4]) for t in tensors]
    data = (_vp * n)(*[b.ctypes.data for b in bufs])
    keys = list(u32)
    ks = (C.c_char_p * max(1, len(keys)))(*[k.encode() for k in keys])
    vs = (C.c_uint32 * max(1, len(keys)))(*[u32[k] for k in keys])
    rc = L.rg_gguf_write(path.encode(), n, names, types, ne0, ne1, data, len(keys), ks, vs,
                         strs[0].encode() if strs else None, strs[1].encode() if strs else None,
                         f32[0].encode() if f32 else None, f32[1] if f32 else 0.0)
    if rc != 0:
        raise RuntimeError("rg_gguf_write failed")
