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
LIB_PATH = os.path.join(HERE, "libbh_q4k.so")
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
    L.bh_q4k_quantize.argtypes = [_vp, _vp, _i64, _i64, _vp, _vp]
    L.bh_q4k_dequantize.argtypes = [_vp, _vp, _i64, _i64, _vp, _vp]
    L.bh_q4k_mul_mat_host.argtypes = [_vp, _vp, _i64, _i64, _vp, C.c_int, _vp, C.c_int]
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
