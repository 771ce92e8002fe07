"""GPU: the reference's own GPU Q4_K matvec (ggml-cuda mul_mat_vec_q<Q4_K>,
built for sm_100a from the reference tree into oracle/_ref) computes the
same product as this library on the same weights. It quantizes the
activations to Q8_1 (32-value blocks) instead of Q8_K, so the two agree
within the activation quantization error, not bit for bit; the benchmark
times it beside bh_q4k_matvec_f32 as the GPU comparison point."""
from __future__ import annotations

import os

import numpy as np
import pytest

import oracle as om

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not os.path.exists(om.MMVQ_SO), reason="oracle/_ref not built (no reference tree)")]


@pytest.mark.parametrize("n,k,b", [(4096, 4096, 1), (12288, 4096, 4), (4096, 12288, 8)])
def test_reference_gpu_matvec_agrees(ctx, bh, oracle, n, k, b):
    import torch

    ref = om.RefMMVQ()
    wq = oracle.quantize_q4k(oracle.normal((n, k), 300 + n, 0.0, 0.02))
    x = oracle.normal((b, k), 301 + k, 0.0, 1.0)
    w_d = torch.from_numpy(wq.reshape(-1)).cuda()
    x_d = torch.from_numpy(x).cuda()
    y_ref = torch.empty((b, n), device="cuda")
    xq = torch.empty(ref.xq_bytes(k, b), dtype=torch.uint8, device="cuda")
    ref.matvec(w_d.data_ptr(), n, k, x_d.data_ptr(), b, xq.data_ptr(), y_ref.data_ptr())
    y = ctx.matvec_f32(w_d, n, k, x_d)
    torch.cuda.synchronize()
    a, r = y.cpu().numpy(), y_ref.cpu().numpy()
    want = oracle.matvec(wq, n, k, oracle.quantize_q8k(x), b, om.FOLD_X86)
    assert np.array_equal(a.view(np.uint32), want.view(np.uint32))
    # Q8_1 vs Q8_K activations: within the activation quantization error
    assert np.abs(r - want).max() <= 2e-2 * np.abs(want).max()
