"""Python mirror of the C ABI in include/bh_q4k.h (ctypes over libbh_q4k.so).

This is host plumbing for tests and the bench: torch supplies device memory
and streams; all arithmetic happens in the sm_100a kernels of libbh_q4k.so.
There is no CPU fallback: if the library is missing, importing this module
raises, and every compute call fails loudly on a non-zero status.
"""
from __future__ import annotations

import ctypes as C
import os
import re

HERE = os.path.dirname(os.path.abspath(__file__))
# the in-tree build, unless BH_Q4K_LIB names another build of the same library
LIB_PATH = os.environ.get("BH_Q4K_LIB") or os.path.join(HERE, "libbh_q4k.so")
HEADER = os.path.join(os.path.dirname(HERE), "include", "bh_q4k.h")

QK = 256
Q4K_BYTES = 144
Q8K_BYTES = 292
FOLD_X86 = 0
FOLD_GENERIC = 1
MAX_BATCH = 8

BH_OK = 0
TUNE_CTAS_PER_SM = 1
TUNE_STAGE_BYTES = 2
TUNE_SMEM_CAP = 3
TUNE_TPR = 4
TUNE_SM_BUDGET = 5
TUNE_SMALL_ACT = 7
TUNE_PREFILL = 8
TUNE_BARRIER_WAIT = 9
TUNE_PREFETCH_MB = 10
TUNE_PDL = 11
BH_EIO = -5
BH_ENOMEM = -12
BH_ENODEV = -19
BH_EINVAL = -22
BH_ETIMEDOUT = -110

_vp = C.c_void_p
_i64 = C.c_int64


class BHError(RuntimeError):
    def __init__(self, code: int, what: str):
        super().__init__(f"{what} failed: {code} ({strerror(code)})")
        self.code = code


def header_functions(path: str = HEADER) -> list[str]:
    """Names of the functions declared in the public header."""
    src = open(path).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return re.findall(r"^\s*(?:const\s+)?[A-Za-z_][A-Za-z0-9_]*\s*\**\s*(bh_[A-Za-z0-9_]+)\s*\(", src, flags=re.M)


class StackConfig(C.Structure):
    _fields_ = [("n_layer", C.c_int), ("n_embd", C.c_int), ("n_head", C.c_int), ("n_head_kv", C.c_int),
                ("head_dim", C.c_int), ("n_ff", C.c_int), ("n_vocab", C.c_int), ("n_ctx", C.c_int),
                ("rms_eps", C.c_float), ("rope_theta", C.c_float)]

    def as_dict(self) -> dict:
        return {name: getattr(self, name) for name, _ in self._fields_}


class MoeConfig(C.Structure):
    _fields_ = [("n_layer", C.c_int), ("n_embd", C.c_int), ("n_ff", C.c_int), ("n_expert", C.c_int),
                ("k", C.c_int), ("n_tok", C.c_int), ("rms_eps", C.c_float)]

    def as_dict(self) -> dict:
        return {name: getattr(self, name) for name, _ in self._fields_}


MOE_GATE, MOE_UP, MOE_DOWN, MOE_LOGITS, MOE_NORM, MOE_SELECTED, MOE_WEIGHTS, MOE_HIDDEN, MOE_BARRIER = range(9)

W_Q, W_K, W_V, W_O, W_GATE, W_UP, W_DOWN = range(7)
W_PER_LAYER = 7
W_OUTPUT = 7
OP_QKV, OP_O, OP_GATE_UP, OP_DOWN, OP_LMHEAD, OP_ATTN = range(6)
(T_ATTN_NORM, T_FFN_NORM, T_Q_NORM, T_K_NORM, T_OUT_NORM, T_K_CACHE, T_V_CACHE, T_LOGITS, T_HIDDEN, T_QKV, T_ATTN,
 T_H_ATTN, T_GATE_UP, T_FFN_ACT) = range(8, 22)


def load(path: str = LIB_PATH) -> C.CDLL:
    if not os.path.exists(path):
        raise ImportError(f"{path} is not built: run `make -C {HERE}` (nvcc, sm_100a)")
    L = C.CDLL(path)
    L.bh_version.restype = C.c_int
    L.bh_strerror.argtypes = [C.c_int]
    L.bh_strerror.restype = C.c_char_p
    L.bh_init.argtypes = [C.c_int, C.POINTER(_vp)]
    L.bh_free.argtypes = [_vp]
    L.bh_device_status.argtypes = [_vp, C.c_int]
    L.bh_tune.argtypes = [_vp, C.c_int, C.c_int]
    L.bh_q8k_quantize.argtypes = [_vp, _vp, _i64, C.c_int, _vp, _vp]
    L.bh_q4k_matvec.argtypes = [_vp, _vp, _i64, _i64, _vp, C.c_int, _vp, _vp, C.c_int, _vp]
    L.bh_q4k_matvec_f32.argtypes = [_vp, _vp, _i64, _i64, _vp, C.c_int, _vp, C.c_int, _vp]
    L.bh_q6k_matvec.argtypes = [_vp, _vp, _i64, _i64, _vp, C.c_int, _vp, C.c_int, _vp]
    L.bh_q4k_quantize.argtypes = [_vp, _vp, _i64, _i64, _vp, _vp]
    L.bh_q4k_dequantize.argtypes = [_vp, _vp, _i64, _i64, _vp, _vp]
    L.bh_q4k_mul_mat_host.argtypes = [_vp, _vp, _i64, _i64, _vp, C.c_int, _vp, C.c_int]
    L.bh_q4k_lmhead_argmax.argtypes = [_vp, _vp, _i64, _i64, _vp, C.c_int, _vp, _vp, _vp, C.c_int, _vp]
    L.bh_q4k_lmhead_argmax_noalloc.argtypes = [_vp, _i64, _i64, _vp, C.c_int, _vp, _vp, _vp, C.c_int, _vp]
    L.bh_noalloc_status.argtypes = [C.c_int]
    L.bh_xchg_mailbox_bytes.restype = C.c_size_t
    L.bh_xchg_mailbox_alloc.argtypes = [_vp, C.POINTER(_vp)]
    L.bh_xchg_mailbox_free.argtypes = [_vp, _vp]
    L.bh_xchg_ipc_handle.argtypes = [_vp, _vp, _vp]
    L.bh_xchg_ipc_open.argtypes = [_vp, _vp, C.POINTER(_vp)]
    L.bh_xchg_ipc_close.argtypes = [_vp, _vp]
    L.bh_q4k_lmhead_argmax_tp.argtypes = [_vp, _vp, _i64, _i64, _vp, C.c_int, _i64, C.c_int, C.c_int, _vp,
                                          C.c_uint32, _vp, _vp, C.c_int, _vp]
    L.bh_xchg_alloc.argtypes = [_vp, C.c_size_t, C.POINTER(_vp)]
    L.bh_moe_xchg_recv_bytes.argtypes = [C.c_int]
    L.bh_moe_xchg_recv_bytes.restype = C.c_size_t
    L.bh_moe_ep_exchange_combine.argtypes = [_vp, _vp, _vp, _vp, _vp, _vp, C.c_int, C.c_int, C.c_int, C.c_int,
                                             C.c_int, C.c_int, C.c_int, C.c_uint32, _vp, C.c_int, _vp]
    L.bh_gguf_open.argtypes = [C.c_char_p, C.POINTER(_vp)]
    L.bh_gguf_close.argtypes = [_vp]
    L.bh_gguf_n_tensors.argtypes = [_vp]
    L.bh_gguf_n_tensors.restype = _i64
    L.bh_gguf_n_keys.argtypes = [_vp]
    L.bh_gguf_n_keys.restype = _i64
    L.bh_gguf_find_tensor.argtypes = [_vp, C.c_char_p]
    L.bh_gguf_find_tensor.restype = _i64
    L.bh_gguf_find_key.argtypes = [_vp, C.c_char_p]
    L.bh_gguf_find_key.restype = _i64
    L.bh_gguf_tensor_info.argtypes = [_vp, _i64, C.POINTER(C.c_char_p), C.POINTER(C.c_int), C.POINTER(C.c_int),
                                      C.POINTER(_i64), C.POINTER(C.c_uint64), C.POINTER(C.c_uint64)]
    L.bh_gguf_tensor_host.argtypes = [_vp, _i64]
    L.bh_gguf_tensor_host.restype = _vp
    L.bh_gguf_upload.argtypes = [_vp, _vp, _i64, _vp, C.c_size_t, _vp]
    L.bh_gguf_key.argtypes = [_vp, _i64, C.POINTER(C.c_char_p), C.POINTER(C.c_int)]
    L.bh_gguf_get_int.argtypes = [_vp, _i64, C.POINTER(_i64)]
    L.bh_gguf_get_float.argtypes = [_vp, _i64, C.POINTER(C.c_double)]
    L.bh_gguf_get_str.argtypes = [_vp, _i64, C.POINTER(C.c_void_p), C.POINTER(C.c_uint64)]
    L.bh_stack_default_config.argtypes = [C.POINTER(StackConfig)]
    L.bh_stack_default_config.restype = None
    L.bh_stack_create.argtypes = [_vp, C.POINTER(StackConfig), C.c_uint64, C.POINTER(_vp)]
    L.bh_stack_free.argtypes = [_vp]
    L.bh_stack_set_pos.argtypes = [_vp, C.c_int]
    L.bh_stack_fill_kv.argtypes = [_vp, C.c_int, C.c_uint64]
    L.bh_stack_decode.argtypes = [_vp, _vp, _vp, _vp]
    L.bh_stack_decode_host.argtypes = [_vp, _vp, _vp]
    L.bh_stack_info.argtypes = [_vp, C.POINTER(_i64), C.POINTER(_i64), C.POINTER(_i64)]
    L.bh_stack_time_op.argtypes = [_vp, C.c_int, C.c_int, C.POINTER(C.c_float), C.POINTER(_i64)]
    L.bh_stack_tensor.argtypes = [_vp, C.c_int, C.c_int, C.POINTER(_vp), C.POINTER(_i64), C.POINTER(_i64)]
    L.bh_stack_create_tp.argtypes = [_vp, C.POINTER(StackConfig), C.c_uint64, C.c_int, C.c_int, C.POINTER(_vp)]
    L.bh_stack_tp_handle.argtypes = [_vp, _vp]
    L.bh_stack_tp_connect.argtypes = [_vp, _vp]
    L.bh_stack_tp_info.argtypes = [_vp, C.POINTER(C.c_int), C.POINTER(C.c_int), C.POINTER(_i64)]
    L.bh_stack_tp_connect_comm.argtypes = [_vp, _vp, C.c_int]
    L.bh_mm_registry_create.argtypes = [_vp, C.POINTER(_vp)]
    L.bh_mm_registry_add.argtypes = [_vp, _vp, _vp, C.c_int, C.c_int]
    L.bh_mm_registry_free.argtypes = [_vp]
    L.bh_mm_dispatch.argtypes = [_vp, _vp, _vp, C.c_int, C.c_int, C.c_int, _vp]
    L.bh_ctx_device.argtypes = [_vp]
    L.bh_moe_combine_split.argtypes = [_vp, _vp, _vp, _vp, C.c_int, C.c_int, C.c_int, _vp, C.c_int, _vp]
    L.bh_tp_unique_id.argtypes = [_vp]
    L.bh_tp_comm_init.argtypes = [C.c_int, _vp, C.c_int, C.c_int, C.c_int, C.POINTER(_vp)]
    L.bh_tp_comm_abort.argtypes = [_vp]
    L.bh_tp_comm_free.argtypes = [_vp, C.c_int]
    L.bh_tp_comm_info.argtypes = [_vp, C.POINTER(C.c_int), C.POINTER(C.c_int)]
    L.bh_tp_allgather.argtypes = [_vp, _vp, _vp, C.c_size_t, _vp, C.c_int]
    L.bh_tp_allreduce_sum_f32.argtypes = [_vp, _vp, C.c_size_t, _vp, C.c_int]
    L.bh_moe_route.argtypes = [_vp, _vp, C.c_int, C.c_int, C.c_int, C.c_int, _vp, _vp, _vp]
    L.bh_q4k_moe.argtypes = [_vp, _vp, C.c_int, _vp, _vp, _vp, C.c_int, _vp, _vp, _vp, C.c_int, C.c_int, C.c_int,
                             C.c_int, _vp, _vp, _vp, C.c_int, _vp]
    L.bh_q4k_moe_ep.argtypes = [_vp, _vp, C.c_int, _vp, _vp, _vp, C.c_int, _vp, _vp, _vp, C.c_int, C.c_int,
                                C.c_int, C.c_int, C.c_int, C.c_int, _vp, _vp, _vp, C.c_int, _vp]
    L.bh_moe_combine.argtypes = [_vp, _vp, _vp, C.c_int, C.c_int, C.c_int, _vp, C.c_int, _vp]
    L.bh_moe_default_config.argtypes = [C.POINTER(MoeConfig)]
    L.bh_moe_default_config.restype = None
    L.bh_moe_stack_create.argtypes = [_vp, C.POINTER(MoeConfig), C.c_uint64, C.POINTER(_vp)]
    L.bh_moe_stack_free.argtypes = [_vp]
    L.bh_moe_stack_step.argtypes = [_vp, _vp, _vp, _vp]
    L.bh_moe_stack_step_host.argtypes = [_vp, _vp, _vp]
    L.bh_moe_stack_info.argtypes = [_vp, C.POINTER(_i64), C.POINTER(_i64), C.POINTER(_i64)]
    L.bh_moe_stack_tensor.argtypes = [_vp, C.c_int, C.c_int, C.POINTER(_vp), C.POINTER(_i64)]
    L.bh_ggml_vec_dot_q4_K_q8_K.argtypes = [C.c_int, _vp, C.c_size_t, _vp, C.c_size_t, _vp, C.c_size_t, C.c_int]
    L.bh_ggml_vec_dot_q4_K_q8_K.restype = None
    return L


lib = load()


def strerror(code: int) -> str:
    return lib.bh_strerror(code).decode()


def _check(rc: int, what: str) -> None:
    if rc != BH_OK:
        raise BHError(rc, what)


def _dp(t) -> int | None:
    """Device pointer of a torch tensor (or pass through ints / None)."""
    if t is None:
        return None
    if isinstance(t, int):
        return t
    return t.data_ptr()


def _stream(stream) -> int | None:
    if stream is None:
        import torch

        return torch.cuda.current_stream().cuda_stream
    return stream if isinstance(stream, int) else stream.cuda_stream


def q4k_row_bytes(k: int) -> int:
    return k // QK * Q4K_BYTES


def q8k_row_bytes(k: int) -> int:
    return k // QK * Q8K_BYTES


class Context:
    """One bh_ctx bound to a CUDA device (bh_init / bh_free)."""

    def __init__(self, device: int = 0):
        h = _vp()
        _check(lib.bh_init(device, C.byref(h)), "bh_init")
        self.h = h
        self.device = device

    def close(self) -> None:
        if self.h:
            lib.bh_free(self.h)
            self.h = _vp()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def tune(self, key: int, value: int) -> None:
        _check(lib.bh_tune(self.h, key, value), "bh_tune")

    def status(self, clear: bool = True) -> int:
        return lib.bh_device_status(self.h, 1 if clear else 0)

    # -- compute entry points (torch tensors on this device) --
    def q8k_quantize(self, x, out=None, stream=None):
        import torch

        B, K = x.shape
        if out is None:
            out = torch.empty(B * q8k_row_bytes(K), dtype=torch.uint8, device=x.device)
        _check(lib.bh_q8k_quantize(self.h, _dp(x), K, B, _dp(out), _stream(stream)), "bh_q8k_quantize")
        return out

    def matvec(self, w, n: int, k: int, xq, b: int, y=None, partials=None, fold: int = FOLD_X86, stream=None):
        import torch

        if y is None:
            y = torch.empty((b, n), dtype=torch.float32, device=w.device)
        _check(lib.bh_q4k_matvec(self.h, _dp(w), n, k, _dp(xq), b, _dp(y), _dp(partials), fold, _stream(stream)),
               "bh_q4k_matvec")
        return y

    def matvec_f32(self, w, n: int, k: int, x, y=None, fold: int = FOLD_X86, stream=None):
        import torch

        b = x.shape[0]
        if y is None:
            y = torch.empty((b, n), dtype=torch.float32, device=w.device)
        _check(lib.bh_q4k_matvec_f32(self.h, _dp(w), n, k, _dp(x), b, _dp(y), fold, _stream(stream)),
               "bh_q4k_matvec_f32")
        return y

    def q6k_matvec(self, w, n: int, k: int, xq, b: int, y=None, stream=None):
        """Q6_K weights [n rows of k] x Q8_K columns xq [b]: y [b][n] (x86 fold)."""
        import torch

        if y is None:
            y = torch.empty((b, n), dtype=torch.float32, device=w.device)
        _check(lib.bh_q6k_matvec(self.h, _dp(w), n, k, _dp(xq), b, _dp(y), FOLD_X86, _stream(stream)),
               "bh_q6k_matvec")
        return y

    def q4k_quantize(self, w_f32, out=None, stream=None):
        import torch

        n, k = w_f32.shape
        if out is None:
            out = torch.empty(n * q4k_row_bytes(k), dtype=torch.uint8, device=w_f32.device)
        _check(lib.bh_q4k_quantize(self.h, _dp(w_f32), n, k, _dp(out), _stream(stream)), "bh_q4k_quantize")
        return out

    def q4k_dequantize(self, w, n: int, k: int, out=None, stream=None):
        import torch

        if out is None:
            out = torch.empty((n, k), dtype=torch.float32, device=w.device)
        _check(lib.bh_q4k_dequantize(self.h, _dp(w), n, k, _dp(out), _stream(stream)), "bh_q4k_dequantize")
        return out

    def mul_mat_host(self, w, n: int, k: int, host_x, host_y, fold: int = FOLD_X86):
        """host_x / host_y: numpy float32 arrays [B][K] / [B][N] (or pinned tensors)."""
        b = host_x.shape[0]
        xp = host_x.ctypes.data if hasattr(host_x, "ctypes") else host_x.data_ptr()
        yp = host_y.ctypes.data if hasattr(host_y, "ctypes") else host_y.data_ptr()
        _check(lib.bh_q4k_mul_mat_host(self.h, _dp(w), n, k, xp, b, yp, fold), "bh_q4k_mul_mat_host")
        return host_y


def tp_unique_id() -> bytes:
    """ncclGetUniqueId through the library (bh_tp_unique_id): 128 bytes."""
    buf = C.create_string_buffer(128)
    _check(lib.bh_tp_unique_id(buf), "bh_tp_unique_id")
    return buf.raw


def tp_comm_init(device: int, unique_id: bytes, world: int, rank: int, timeout_ms: int = 30000):
    """A non-blocking NCCL communicator (bh_tp_comm_init): returns the
    ncclComm_t as an int, or raises BHError (BH_ETIMEDOUT when a rank never
    joined within timeout_ms; the communicator was then aborted)."""
    comm = _vp()
    _check(lib.bh_tp_comm_init(device, unique_id, world, rank, timeout_ms, C.byref(comm)), "bh_tp_comm_init")
    return comm.value


def tp_comm_init_rc(device: int, unique_id: bytes, world: int, rank: int, timeout_ms: int):
    """bh_tp_comm_init's status code and communicator, without raising."""
    comm = _vp()
    rc = lib.bh_tp_comm_init(device, unique_id, world, rank, timeout_ms, C.byref(comm))
    return rc, comm.value


def tp_comm_free(comm, timeout_ms: int = 30000) -> None:
    _check(lib.bh_tp_comm_free(comm, timeout_ms), "bh_tp_comm_free")


def tp_allgather(comm, send, recv, timeout_ms: int = 30000, stream=None) -> None:
    """recv [world * n] <- every rank's send [n] (device tensors)."""
    nbytes = send.numel() * send.element_size()
    _check(lib.bh_tp_allgather(comm, _dp(send), _dp(recv), nbytes, _stream(stream), timeout_ms), "bh_tp_allgather")


def tp_allreduce_sum(comm, buf, timeout_ms: int = 30000, stream=None) -> None:
    """buf (fp32, device) <- elementwise sum over ranks."""
    _check(lib.bh_tp_allreduce_sum_f32(comm, _dp(buf), buf.numel(), _stream(stream), timeout_ms),
           "bh_tp_allreduce_sum_f32")


def default_stack_config(**overrides) -> StackConfig:
    cfg = StackConfig()
    lib.bh_stack_default_config(C.byref(cfg))
    for k, v in overrides.items():
        setattr(cfg, k, v)
    return cfg


class Stack:
    """A decode block stack (bh_stack_*) on a Context's device; with world >
    1, rank `rank`'s share of a row-split stack (bh_stack_create_tp), to be
    connected to its peers (tp_connect / tp_connect_comm) before decoding."""

    def __init__(self, ctx: Context, cfg: StackConfig, seed: int, rank: int = 0, world: int = 1):
        h = _vp()
        if world == 1:
            _check(lib.bh_stack_create(ctx.h, C.byref(cfg), seed & (2**64 - 1), C.byref(h)), "bh_stack_create")
        else:
            _check(lib.bh_stack_create_tp(ctx.h, C.byref(cfg), seed & (2**64 - 1), rank, world, C.byref(h)),
                   "bh_stack_create_tp")
        self.h = h
        self.ctx = ctx
        self.cfg = cfg
        self.rank, self.world = rank, world

    def tp_handle(self) -> bytes:
        buf = C.create_string_buffer(64)
        _check(lib.bh_stack_tp_handle(self.h, buf), "bh_stack_tp_handle")
        return buf.raw

    def tp_connect(self, handles) -> None:
        """handles: every rank's tp_handle() in rank order."""
        blob = b"".join(handles)
        _check(lib.bh_stack_tp_connect(self.h, blob), "bh_stack_tp_connect")

    def tp_connect_comm(self, comm, timeout_ms: int = 30000) -> None:
        _check(lib.bh_stack_tp_connect_comm(self.h, comm, timeout_ms), "bh_stack_tp_connect_comm")

    def tp_info(self) -> dict:
        r, w = C.c_int(0), C.c_int(0)
        rr = (_i64 * 10)()
        _check(lib.bh_stack_tp_info(self.h, C.byref(r), C.byref(w), rr), "bh_stack_tp_info")
        v = list(rr)
        return {"rank": r.value, "world": w.value, "q_heads": (v[0], v[1]), "kv_heads": (v[2], v[3]),
                "embd_rows": (v[4], v[5]), "ff_rows": (v[6], v[7]), "vocab_rows": (v[8], v[9])}

    def close(self) -> None:
        if self.h:
            lib.bh_stack_free(self.h)
            self.h = _vp()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def set_pos(self, pos: int) -> None:
        _check(lib.bh_stack_set_pos(self.h, pos), "bh_stack_set_pos")

    def fill_kv(self, n_pos: int, seed: int) -> None:
        _check(lib.bh_stack_fill_kv(self.h, n_pos, seed & (2**64 - 1)), "bh_stack_fill_kv")

    def decode(self, x, tok, stream=None) -> None:
        _check(lib.bh_stack_decode(self.h, _dp(x), _dp(tok), _stream(stream)), "bh_stack_decode")

    def decode_host(self, host_x) -> int:
        tok = C.c_int32(0)
        xp = host_x.ctypes.data if hasattr(host_x, "ctypes") else host_x.data_ptr()
        _check(lib.bh_stack_decode_host(self.h, xp, C.byref(tok)), "bh_stack_decode_host")
        return tok.value

    def info(self) -> dict:
        wb, sb, nl = _i64(), _i64(), _i64()
        _check(lib.bh_stack_info(self.h, C.byref(wb), C.byref(sb), C.byref(nl)), "bh_stack_info")
        return {"weight_bytes": wb.value, "step_bytes": sb.value, "launches": nl.value}

    def time_op(self, op: int, reps: int = 5):
        """(average ms per launch, algorithmic bytes per launch) of one op."""
        ms, nb = C.c_float(0), _i64()
        _check(lib.bh_stack_time_op(self.h, op, reps, C.byref(ms), C.byref(nb)), "bh_stack_time_op")
        return ms.value, nb.value

    def tensor(self, layer: int, which: int):
        """(device pointer, rows, cols) of one stack tensor."""
        p, r, c = _vp(), _i64(), _i64()
        _check(lib.bh_stack_tensor(self.h, layer, which, C.byref(p), C.byref(r), C.byref(c)), "bh_stack_tensor")
        return p.value, r.value, c.value

    def view(self, layer: int, which: int):
        """A torch tensor aliasing one stack tensor on the device (uint8 Q4_K
        bytes, or float32 rows x cols)."""
        ptr, r, c = self.tensor(layer, which)
        if which <= W_OUTPUT:
            return device_view(ptr, r * (c // QK) * Q4K_BYTES, "|u1")
        return device_view(ptr, r * c, "<f4").view(r, c)

    def to_host(self, layer: int, which: int):
        import torch

        t = self.view(layer, which)
        torch.cuda.synchronize()
        return t.cpu().numpy()


def device_view(ptr: int, n: int, typestr: str):
    """Wrap n elements of device memory at ptr as a torch tensor (no copy)."""
    import torch

    class _Dev:
        __cuda_array_interface__ = {"shape": (n,), "typestr": typestr, "data": (ptr, False), "version": 3}

    return torch.as_tensor(_Dev(), device="cuda")


def lmhead_argmax(ctx: Context, w, n: int, k: int, x, logits=None, fold: int = FOLD_X86, stream=None):
    """Token ids (and maxima) of the greedy pick over W . x; x [B][K] fp32 on the device."""
    import torch

    b = x.shape[0]
    tok = torch.empty(b, dtype=torch.int32, device=x.device)
    mx = torch.empty(b, dtype=torch.float32, device=x.device)
    _check(lib.bh_q4k_lmhead_argmax(ctx.h, _dp(w), n, k, _dp(x), b, _dp(logits), _dp(tok), _dp(mx), fold,
                                    _stream(stream)), "bh_q4k_lmhead_argmax")
    return tok, mx


class PeerMailbox:
    """A zeroed device buffer of this rank for the peer-memory exchanges
    (bh_xchg_*): the flag mailbox by default, or `nbytes` for a receive
    buffer. handle() gives the 64-byte CUDA IPC handle to share with the other
    ranks, open(handle) maps a peer's buffer into this process."""

    def __init__(self, ctx: Context, nbytes: int | None = None):
        self.ctx = ctx
        p = _vp()
        if nbytes is None:
            _check(lib.bh_xchg_mailbox_alloc(ctx.h, C.byref(p)), "bh_xchg_mailbox_alloc")
        else:
            _check(lib.bh_xchg_alloc(ctx.h, nbytes, C.byref(p)), "bh_xchg_alloc")
        self.ptr = p.value
        self.opened: list[int] = []

    def handle(self) -> bytes:
        buf = C.create_string_buffer(64)
        _check(lib.bh_xchg_ipc_handle(self.ctx.h, self.ptr, buf), "bh_xchg_ipc_handle")
        return buf.raw

    def open(self, handle: bytes) -> int:
        buf = C.create_string_buffer(bytes(handle), 64)
        p = _vp()
        _check(lib.bh_xchg_ipc_open(self.ctx.h, buf, C.byref(p)), "bh_xchg_ipc_open")
        self.opened.append(p.value)
        return p.value

    def close(self) -> None:
        for q in self.opened:
            lib.bh_xchg_ipc_close(self.ctx.h, q)
        self.opened = []
        if self.ptr:
            lib.bh_xchg_mailbox_free(self.ctx.h, self.ptr)
            self.ptr = None


def lmhead_argmax_tp(ctx: Context, w_local, n_local: int, k: int, x, row_offset: int, rank: int, mailboxes,
                     epoch: int, fold: int = FOLD_X86, stream=None):
    """Global greedy pick of a row-split LM head (bh_q4k_lmhead_argmax_tp):
    mailboxes = every rank's mailbox pointer as seen from this process (own
    at [rank]); epoch = the call's number (1, 2, ...), the same on every
    rank. Returns (tok [B] int32, max [B] fp32) on the device; a timed-out
    exchange raises BHError(BH_ETIMEDOUT) once the stream is synchronized."""
    import torch

    b = x.shape[0]
    tok = torch.empty(b, dtype=torch.int32, device=x.device)
    mx = torch.empty(b, dtype=torch.float32, device=x.device)
    arr = (_vp * len(mailboxes))(*mailboxes)
    _check(lib.bh_q4k_lmhead_argmax_tp(ctx.h, _dp(w_local), n_local, k, _dp(x), b, row_offset, rank,
                                       len(mailboxes), arr, epoch, _dp(tok), _dp(mx), fold, _stream(stream)),
           "bh_q4k_lmhead_argmax_tp")
    return tok, mx


def moe_ep_exchange_combine(ctx: Context, dout, selected, weights, expert_lo: int, expert_hi: int, rank: int,
                            recv, mailboxes, epoch: int, out=None, residual: bool = False, stream=None):
    """out [T, n_embd] of the expert-parallel block with the owned pairs
    exchanged through peer memory (bh_moe_ep_exchange_combine)."""
    import torch

    t, k = selected.shape
    n_embd = dout.shape[1]
    if out is None:
        out = torch.empty((t, n_embd), dtype=torch.float32, device=dout.device)
    world = len(mailboxes)
    ra = (_vp * world)(*recv)
    ma = (_vp * world)(*mailboxes)
    _check(lib.bh_moe_ep_exchange_combine(ctx.h, _dp(dout), ra, ma, _dp(selected), _dp(weights), t, k, n_embd,
                                          expert_lo, expert_hi, rank, world, epoch, _dp(out), int(residual),
                                          _stream(stream)), "bh_moe_ep_exchange_combine")
    return out


# ---------------------------------------------------------------------------
# routed-expert FFN
# ---------------------------------------------------------------------------
def moe_route(ctx: Context, logits, k: int, norm_topk: bool = True, stream=None):
    """(selected [T, k] int32, weights [T, k] fp32) of router logits [T, n_expert] on the device."""
    import torch

    t, e = logits.shape
    ids = torch.empty((t, k), dtype=torch.int32, device=logits.device)
    w = torch.empty((t, k), dtype=torch.float32, device=logits.device)
    _check(lib.bh_moe_route(ctx.h, _dp(logits), t, e, k, int(norm_topk), _dp(ids), _dp(w), _stream(stream)),
           "bh_moe_route")
    return ids, w


def moe(ctx: Context, cur, gate, up, down, n_expert: int, n_ff: int, k: int, selected=None, weights=None,
        logits=None, norm_topk: bool = True, out=None, fold: int = FOLD_X86, stream=None):
    """Routed-expert FFN of cur [T, n_embd] (device fp32). Routing is given
    (selected, weights) or computed from logits; returns (out, selected, weights)."""
    import torch

    t, n_embd = cur.shape
    if out is None:
        out = torch.empty((t, n_embd), dtype=torch.float32, device=cur.device)
    sel_out = w_out = None
    if logits is not None:
        sel_out = torch.empty((t, k), dtype=torch.int32, device=cur.device)
        w_out = torch.empty((t, k), dtype=torch.float32, device=cur.device)
    _check(lib.bh_q4k_moe(ctx.h, _dp(cur), t, _dp(selected), _dp(weights), _dp(logits), int(norm_topk), _dp(gate),
                          _dp(up), _dp(down), n_expert, n_embd, n_ff, k, _dp(out), _dp(sel_out), _dp(w_out), fold,
                          _stream(stream)), "bh_q4k_moe")
    if logits is not None:
        return out, sel_out, w_out
    return out, selected, weights


def moe_ep(ctx: Context, cur, gate_own, up_own, down_own, n_expert: int, expert_lo: int, expert_hi: int, n_ff: int,
           k: int, selected=None, weights=None, logits=None, norm_topk: bool = True, dout=None,
           fold: int = FOLD_X86, stream=None):
    """This rank's expert outputs (bh_q4k_moe_ep): dout [T*k, n_embd] holds the
    owned pairs' outputs and -0.0 elsewhere; returns (dout, selected, weights)."""
    import torch

    t, n_embd = cur.shape
    if dout is None:
        dout = torch.empty((t * k, n_embd), dtype=torch.float32, device=cur.device)
    sel_out = w_out = None
    if logits is not None:
        sel_out = torch.empty((t, k), dtype=torch.int32, device=cur.device)
        w_out = torch.empty((t, k), dtype=torch.float32, device=cur.device)
    _check(lib.bh_q4k_moe_ep(ctx.h, _dp(cur), t, _dp(selected), _dp(weights), _dp(logits), int(norm_topk),
                             _dp(gate_own), _dp(up_own), _dp(down_own), n_expert, expert_lo, expert_hi, n_embd, n_ff,
                             k, _dp(dout), _dp(sel_out), _dp(w_out), fold, _stream(stream)), "bh_q4k_moe_ep")
    if logits is not None:
        return dout, sel_out, w_out
    return dout, selected, weights


def moe_combine(ctx: Context, dout, weights, out=None, residual: bool = False, stream=None):
    """out [T, n_embd] = sum over slots of weights * dout (bh_moe_combine)."""
    import torch

    t, k = weights.shape
    n_embd = dout.shape[1]
    if out is None:
        out = torch.empty((t, n_embd), dtype=torch.float32, device=dout.device)
    _check(lib.bh_moe_combine(ctx.h, _dp(dout), _dp(weights), t, k, n_embd, _dp(out), int(residual),
                              _stream(stream)), "bh_moe_combine")
    return out


def default_moe_config(**overrides) -> MoeConfig:
    cfg = MoeConfig()
    lib.bh_moe_default_config(C.byref(cfg))
    for key, v in overrides.items():
        setattr(cfg, key, v)
    return cfg


class MoeStack:
    """The MoE layer stack (bh_moe_stack_*) on a Context's device."""

    def __init__(self, ctx: Context, cfg: MoeConfig, seed: int):
        h = _vp()
        _check(lib.bh_moe_stack_create(ctx.h, C.byref(cfg), seed & (2**64 - 1), C.byref(h)), "bh_moe_stack_create")
        self.h = h
        self.ctx = ctx
        self.cfg = cfg

    def close(self) -> None:
        if self.h:
            lib.bh_moe_stack_free(self.h)
            self.h = _vp()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def step(self, h_in, h_out, stream=None) -> None:
        _check(lib.bh_moe_stack_step(self.h, _dp(h_in), _dp(h_out), _stream(stream)), "bh_moe_stack_step")

    def step_host(self, host_h, host_out) -> None:
        hp = host_h.ctypes.data if hasattr(host_h, "ctypes") else host_h.data_ptr()
        op = host_out.ctypes.data if hasattr(host_out, "ctypes") else host_out.data_ptr()
        _check(lib.bh_moe_stack_step_host(self.h, hp, op), "bh_moe_stack_step_host")

    def info(self) -> dict:
        wb, sb, nl = _i64(), _i64(), _i64()
        _check(lib.bh_moe_stack_info(self.h, C.byref(wb), C.byref(sb), C.byref(nl)), "bh_moe_stack_info")
        return {"weight_bytes": wb.value, "step_bytes": sb.value, "launches": nl.value}

    def tensor(self, layer: int, which: int):
        p, nb = _vp(), _i64()
        _check(lib.bh_moe_stack_tensor(self.h, layer, which, C.byref(p), C.byref(nb)), "bh_moe_stack_tensor")
        return p.value, nb.value

    def to_host(self, layer: int, which: int):
        """A host copy of one tensor (uint8 for the banks, int32 routing ids, else fp32)."""
        import torch

        ptr, nb = self.tensor(layer, which)
        if which in (MOE_GATE, MOE_UP, MOE_DOWN):
            t = device_view(ptr, nb, "|u1")
        elif which in (MOE_SELECTED, MOE_BARRIER):
            t = device_view(ptr, nb // 4, "<i4")
        else:
            t = device_view(ptr, nb // 4, "<f4")
        torch.cuda.synchronize()
        return t.cpu().numpy()


class GGUF:
    """A GGUF model file opened by bh_gguf_open (host parsing; upload to a
    Context's device)."""

    def __init__(self, path: str):
        h = _vp()
        _check(lib.bh_gguf_open(path.encode(), C.byref(h)), "bh_gguf_open")
        self.h = h

    def close(self) -> None:
        if self.h:
            lib.bh_gguf_close(self.h)
            self.h = _vp()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def n_tensors(self) -> int:
        return int(lib.bh_gguf_n_tensors(self.h))

    def find(self, name: str) -> int:
        return int(lib.bh_gguf_find_tensor(self.h, name.encode()))

    def info(self, i: int) -> dict:
        nm, ty, nd = C.c_char_p(), C.c_int(), C.c_int()
        ne = (_i64 * 4)()
        off, nb = C.c_uint64(), C.c_uint64()
        _check(lib.bh_gguf_tensor_info(self.h, i, C.byref(nm), C.byref(ty), C.byref(nd), ne, C.byref(off),
                                       C.byref(nb)), "bh_gguf_tensor_info")
        return {"name": nm.value.decode(), "type": ty.value, "n_dims": nd.value, "ne": list(ne)[: nd.value],
                "offset": off.value, "bytes": nb.value}

    def host_bytes(self, i: int):
        import numpy as np

        p = lib.bh_gguf_tensor_host(self.h, i)
        nb = self.info(i)["bytes"]
        return np.ctypeslib.as_array(C.cast(p, C.POINTER(C.c_uint8)), shape=(nb,)).copy()

    def upload(self, ctx: "Context", i: int, dst=None, stream=None):
        import torch

        nb = self.info(i)["bytes"]
        if dst is None:
            dst = torch.empty(nb, dtype=torch.uint8, device="cuda")
        _check(lib.bh_gguf_upload(ctx.h, self.h, i, _dp(dst), nb, _stream(stream)), "bh_gguf_upload")
        return dst

    def key(self, name: str):
        k = int(lib.bh_gguf_find_key(self.h, name.encode()))
        if k < 0:
            raise KeyError(name)
        ty = C.c_int()
        _check(lib.bh_gguf_key(self.h, k, None, C.byref(ty)), "bh_gguf_key")
        if ty.value == 8:
            p, n = C.c_void_p(), C.c_uint64()
            _check(lib.bh_gguf_get_str(self.h, k, C.byref(p), C.byref(n)), "bh_gguf_get_str")
            return C.string_at(p, n.value).decode()
        if ty.value in (6, 12):
            v = C.c_double()
            _check(lib.bh_gguf_get_float(self.h, k, C.byref(v)), "bh_gguf_get_float")
            return v.value
        v = _i64()
        _check(lib.bh_gguf_get_int(self.h, k, C.byref(v)), "bh_gguf_get_int")
        return v.value
