"""GPU: the native engine's dense-matmul hook (bh_mm_dispatch, the
mm_dispatch_fn_t of forward_native.h:115-119) on registered Q4_K weights:
out [M][N] for host lhs [M][K] equals the oracle's Q4_K x Q8_K matmul bit
for bit (M above 8 in chunks); an unregistered key or a mismatched shape
returns non-zero so that the engine falls through to its CPU matmul."""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

from test_gpu_matvec import assert_bits_equal, dev

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("m,n,k", [(1, 4096, 4096), (5, 1000, 768), (13, 2048, 2048)])
def test_mm_dispatch_matches_oracle(ctx, bh, oracle, m, n, k):
    w = oracle.normal((n, k), 300 + n + m, 0.0, 0.02)
    wq = oracle.quantize_q4k(w)
    wd = dev(wq)
    lhs = np.ascontiguousarray(oracle.normal((m, k), 301 + k, 0.0, 1.0), dtype=np.float32)
    out = np.zeros((m, n), np.float32)
    key = np.zeros(16, np.uint16)  # stands for the engine's fp16 copy of the weight
    reg = C.c_void_p()
    assert bh.lib.bh_mm_registry_create(ctx.h, C.byref(reg)) == 0
    try:
        assert bh.lib.bh_mm_registry_add(reg, key.ctypes.data, wd.data_ptr(), n, k) == 0
        rc = bh.lib.bh_mm_dispatch(reg, lhs.ctypes.data, key.ctypes.data, m, k, n, out.ctypes.data)
        assert rc == 0
        want = oracle.matvec(wq, n, k, oracle.quantize_q8k(lhs), m, 0).reshape(m, n)
        assert_bits_equal(out, want, f"mm_dispatch {m}x{k} . {n}x{k}")
        other = np.zeros(16, np.uint16)
        assert bh.lib.bh_mm_dispatch(reg, lhs.ctypes.data, other.ctypes.data, m, k, n, out.ctypes.data) != 0
        assert bh.lib.bh_mm_dispatch(reg, lhs.ctypes.data, key.ctypes.data, m, k, n + 1, out.ctypes.data) != 0
    finally:
        bh.lib.bh_mm_registry_free(reg)
