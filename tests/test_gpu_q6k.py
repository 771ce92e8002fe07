"""GPU: the Q6_K x Q8_K matvec (bh_q6k_matvec) against the oracle's
restatement of the reference's x86 ggml_vec_dot_q6_K_q8_K, which
tests/test_graph_reference.py pins to the reference's own compiled function;
weights from the reference's own Q6_K quantizer (oracle/_ref), bit for bit."""
from __future__ import annotations

import os

import numpy as np
import pytest

import oracle as om

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not os.path.exists(om.GRAPH_SO), reason="oracle/_ref not built (no reference tree)")]


@pytest.mark.parametrize("n,k,b", [(1, 256, 1), (33, 768, 3), (768, 2048, 8), (4096, 4096, 1), (1000, 12288, 4),
                                   (2048, 768, 2), (151, 4096, 8)])
def test_q6k_matvec_bit_exact(ctx, bh, oracle, n, k, b):
    import torch

    w = om.graph_quantize_q6k(oracle.normal((n, k), 900 + n + k, 0.0, 0.02))
    x = oracle.normal((b, k), 901 + b, 0.0, 1.0)
    xq = oracle.quantize_q8k(x)
    y = ctx.q6k_matvec(torch.from_numpy(w).cuda(), n, k, torch.from_numpy(xq.reshape(-1)).cuda(), b)
    torch.cuda.synchronize()
    want = oracle.matvec_q6k(w, n, k, xq, b)
    assert np.array_equal(y.cpu().numpy().view(np.uint32), want.view(np.uint32))
    assert ctx.status() == 0


def test_q6k_rejects_generic_fold_and_bad_sizes(ctx, bh):
    import torch

    w = torch.zeros(210 * 4, dtype=torch.uint8, device="cuda")
    xq = torch.zeros(292, dtype=torch.uint8, device="cuda")
    y = torch.zeros(4, device="cuda")
    assert bh.lib.bh_q6k_matvec(ctx.h, w.data_ptr(), 4, 256, xq.data_ptr(), 1, y.data_ptr(), bh.FOLD_GENERIC, None) \
        == bh.BH_EINVAL
    assert bh.lib.bh_q6k_matvec(ctx.h, w.data_ptr(), 4, 300, xq.data_ptr(), 1, y.data_ptr(), bh.FOLD_X86, None) \
        == bh.BH_EINVAL
    assert bh.lib.bh_q6k_matvec(ctx.h, w.data_ptr(), 4, 256, xq.data_ptr(), 9, y.data_ptr(), bh.FOLD_X86, None) \
        == bh.BH_EINVAL
