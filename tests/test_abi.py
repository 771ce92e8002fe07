"""CPU: the C-ABI library loads, exports every symbol the header declares,
and rejects invalid arguments on the host before any launch."""
from __future__ import annotations

import ctypes as C
import os

import pytest


def test_library_exports_every_header_symbol(bh):
    names = bh.header_functions()
    assert len(names) >= 10
    for name in names:
        assert hasattr(bh.lib, name), name
    assert bh.lib.bh_version() >> 16 == 1


def test_strerror_codes(bh):
    for code in (bh.BH_OK, bh.BH_EIO, bh.BH_ENOMEM, bh.BH_ENODEV, bh.BH_EINVAL, bh.BH_ETIMEDOUT):
        assert bh.strerror(code) != "unknown status"


def test_null_context_is_einval(bh):
    L = bh.lib
    assert L.bh_q4k_matvec(None, None, 16, 256, None, 1, None, None, 0, None) == bh.BH_EINVAL
    assert L.bh_q4k_matvec_f32(None, None, 16, 256, None, 1, None, 0, None) == bh.BH_EINVAL
    assert L.bh_q8k_quantize(None, None, 256, 1, None, None) == bh.BH_EINVAL
    assert L.bh_q4k_quantize(None, None, 1, 256, None, None) == bh.BH_EINVAL
    assert L.bh_q4k_dequantize(None, None, 1, 256, None, None) == bh.BH_EINVAL
    assert L.bh_free(None) == bh.BH_EINVAL
    assert L.bh_device_status(None, 0) == bh.BH_EINVAL
    assert L.bh_init(0, None) == bh.BH_EINVAL


def test_vec_dot_shim_rejects_bad_nrc(bh):
    s = C.c_float(123.0)
    bh.lib.bh_ggml_vec_dot_q4_K_q8_K(256, C.byref(s), 0, None, 0, None, 0, 2)
    assert s.value == 0.0


@pytest.mark.skipif(os.environ.get("CUDA_VISIBLE_DEVICES", None) is not None, reason="device list pinned")
def test_init_without_device_is_enodev(bh):
    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    h = C.c_void_p()
    assert bh.lib.bh_init(0, C.byref(h)) == bh.BH_ENODEV
