"""Host-only: the ggml graph-node library (shannon-prime-burnhard_b200/
adapters/libbh_ggml_ops.so) loads into a process that provides ggml (here
the reference's ggml built under oracle/_ref) and exports the entry points
its header declares."""
from __future__ import annotations

import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB = os.path.join(ROOT, "shannon-prime-burnhard_b200", "adapters", "libbh_ggml_ops.so")
GGML = os.path.join(ROOT, "oracle", "_ref", "libggml_graph.so")
HDR = os.path.join(ROOT, "shannon-prime-burnhard_b200", "adapters", "bh_ggml_ops.h")


def test_adapter_library_exports_its_header():
    if not (os.path.exists(LIB) and os.path.exists(GGML)):
        pytest.skip("built only where the reference's ggml headers are")
    ctypes.CDLL(GGML, mode=ctypes.RTLD_GLOBAL)
    lib = ctypes.CDLL(LIB)
    names = re.findall(r"\b(bh_\w+)\s*\(", open(HDR).read())
    assert {"bh_build_burn_moe_op", "bh_ggml_mul_mat"} <= set(names)
    for n in names:
        assert hasattr(lib, n), n
    assert lib.bh_ggml_ops_last_error() == 0
    assert lib.bh_ggml_ops_cached_weights() == 0
