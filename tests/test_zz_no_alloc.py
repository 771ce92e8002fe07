"""GPU: the no-allocation LM-head entry point (collected last on purpose).

bh_q4k_lmhead_argmax_noalloc exists for callers that may not allocate device
memory and therefore cannot create a context; its argmax candidates live in a
static device array of the library. It is called here through the C ABI,
several times in a row (batch 4, 1 and 8, the last one the largest candidate
footprint), and must give the same logits, maxima and tokens, bit for bit, as
the context-based bh_q4k_lmhead_argmax on the same inputs. A rejected call
(bad K) launches nothing, and the valid call after it is still bit-exact: the
array's stale contents from earlier calls do not leak into a result.
"""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _call_and_compare(bh, oracle, ctx, wq, n, k, b, seed, stream):
    import torch

    x = torch.from_numpy(oracle.normal((b, k), seed, 0.0, 1.0)).cuda()
    lg_ref = torch.zeros((b, n), device="cuda")
    tok_ref, mx_ref = bh.lmhead_argmax(ctx, wq, n, k, x, logits=lg_ref)
    lg = torch.full((b, n), -1.0, device="cuda")
    tok = torch.full((b,), -7, dtype=torch.int32, device="cuda")
    mx = torch.zeros(b, device="cuda")
    rc = bh.lib.bh_q4k_lmhead_argmax_noalloc(wq.data_ptr(), n, k, x.data_ptr(), b, lg.data_ptr(), tok.data_ptr(),
                                            mx.data_ptr(), bh.FOLD_X86, stream)
    assert rc == bh.BH_OK, bh.strerror(rc)
    torch.cuda.synchronize()
    assert np.array_equal(lg.cpu().numpy().view(np.uint32), lg_ref.cpu().numpy().view(np.uint32))
    assert np.array_equal(tok.cpu().numpy(), tok_ref.cpu().numpy())
    assert np.array_equal(mx.cpu().numpy().view(np.uint32), mx_ref.cpu().numpy().view(np.uint32))
    return x, tok


def test_noalloc_lmhead_matches_context_entry(bh, oracle):
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    ctx = bh.Context(0)
    n, k = 20000, 4096
    wq = torch.from_numpy(oracle.quantize_q4k(oracle.normal((n, k), 2024, 0.0, 0.02)).reshape(-1)).cuda()
    stream = torch.cuda.current_stream().cuda_stream
    for call, b in enumerate((4, 1, 8)):  # calls in a row, different batches
        x, tok = _call_and_compare(bh, oracle, ctx, wq, n, k, b, 7 + call, stream)
    # invalid sizes are rejected before any launch
    bad = bh.lib.bh_q4k_lmhead_argmax_noalloc(wq.data_ptr(), n, 300, x.data_ptr(), 1, None, tok.data_ptr(), None,
                                             bh.FOLD_X86, stream)
    assert bad == bh.BH_EINVAL
    # the next valid call after the rejected one
    _call_and_compare(bh, oracle, ctx, wq, n, k, 2, 99, stream)
    assert bh.lib.bh_noalloc_status(1) == bh.BH_OK
    assert ctx.status() == 0
    ctx.close()
