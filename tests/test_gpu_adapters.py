"""GPU: the ggml graph nodes of shannon-prime-burnhard_b200/adapters against
the stock ggml path of the reference engine, bit for bit (the C check
tests/c/test_ggml_ops.c, compiled against the reference's ggml headers where
the reference tree is present and run here): BURN_MOE with one expert bank
and with the banks split at a pivot (bh_build_burn_moe_op, the argument list
of sp_build_burn_moe_op) against ggml_mul_mat_id + ggml_silu + ggml_mul +
the weighted ggml_sum_rows of forward.cpp:1096-1107, and the Q4_K branch of
sp_crt_mul_mat (bh_ggml_mul_mat) against ggml_mul_mat, both on the
reference's own x86 CPU backend."""
from __future__ import annotations

import os
import subprocess

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
BIN = os.path.join(ROOT, "tests", "c", "_bin", "test_ggml_ops")


def test_ggml_nodes_match_stock_ggml_path():
    if not os.path.exists(BIN):
        pytest.skip("the C check is built only where the reference's ggml headers are")
    r = subprocess.run(["timeout", "-k", "10", "600", BIN], capture_output=True, text=True, timeout=650)
    out = r.stdout + r.stderr
    assert r.returncode == 0, out[-4000:]
    assert "GGML OPS OK" in out, out[-4000:]
