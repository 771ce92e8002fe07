"""The GGUF tensor reader (bh_gguf_*) on files written by the reference's own
GGUF writer (vendor/ggml/src/gguf.cpp, compiled into oracle/_ref): tensor
names, ggml types, shapes, data offsets and bytes, key/values, and rejection
of truncated files. CPU tests parse and read host bytes; the GPU tests upload
Q4_K and Q6_K tensors and multiply with them, bit for bit against the oracle."""
from __future__ import annotations

import os

import numpy as np
import pytest

import oracle as om

needs_ref = pytest.mark.skipif(not os.path.exists(om.GRAPH_SO), reason="oracle/_ref not built (no reference tree)")


def write_model(oracle, path):
    q4 = oracle.quantize_q4k(oracle.normal((96, 512), 1, 0.0, 0.02)).reshape(-1)
    q6 = om.graph_quantize_q6k(oracle.normal((40, 768), 2, 0.0, 0.02))
    f32 = oracle.normal((7, 33), 3, 0.0, 1.0)
    tensors = [("blk.0.attn_q.weight", om.GGML_TYPE_Q4_K, 512, 96, q4),
               ("output.weight", om.GGML_TYPE_Q6_K, 768, 40, q6),
               ("output_norm.weight", 0, 33, 7, f32)]
    om.graph_gguf_write(path, tensors, {"qwen3.block_count": 1, "qwen3.embedding_length": 512},
                        strs=("general.architecture", "qwen3"), f32=("qwen3.rope.freq_base", 1000000.0))
    return tensors


@needs_ref
def test_gguf_reader_parses_reference_written_file(bh, oracle, tmp_path):
    path = str(tmp_path / "m.gguf")
    tensors = write_model(oracle, path)
    g = bh.GGUF(path)
    assert g.n_tensors() == 3
    for name, ty, ne0, ne1, data in tensors:
        i = g.find(name)
        assert i >= 0
        info = g.info(i)
        assert info["type"] == ty and info["ne"] == [ne0, ne1] and info["n_dims"] == 2
        assert info["offset"] % 32 == 0
        raw = np.ascontiguousarray(data).view(np.uint8).reshape(-1)
        assert info["bytes"] == raw.size
        assert np.array_equal(g.host_bytes(i), raw)
        # the bytes also sit at that offset of the file itself
        with open(path, "rb") as f:
            f.seek(info["offset"])
            assert f.read(16) == raw[:16].tobytes()
    assert g.find("missing.weight") == -1
    assert g.key("general.architecture") == "qwen3"
    assert g.key("qwen3.block_count") == 1 and g.key("qwen3.embedding_length") == 512
    assert g.key("qwen3.rope.freq_base") == 1000000.0
    with pytest.raises(KeyError):
        g.key("no.such.key")
    g.close()


@needs_ref
def test_gguf_reader_rejects_truncated_and_foreign_files(bh, oracle, tmp_path):
    path = str(tmp_path / "m.gguf")
    write_model(oracle, path)
    blob = open(path, "rb").read()
    for cut in (10, 100, len(blob) // 2, len(blob) - 7):
        p = str(tmp_path / f"cut{cut}.gguf")
        open(p, "wb").write(blob[:cut])
        with pytest.raises(bh.BHError):
            bh.GGUF(p)
    p = str(tmp_path / "bad.gguf")
    open(p, "wb").write(b"GGML" + blob[4:])
    with pytest.raises(bh.BHError):
        bh.GGUF(p)


@needs_ref
@pytest.mark.gpu
def test_gguf_upload_then_matvec_bit_exact(ctx, bh, oracle, tmp_path):
    import torch

    path = str(tmp_path / "m.gguf")
    tensors = write_model(oracle, path)
    g = bh.GGUF(path)
    # Q4_K tensor: uploaded bytes, then the matvec from them
    i = g.find("blk.0.attn_q.weight")
    w = g.upload(ctx, i)
    torch.cuda.synchronize()
    assert np.array_equal(w.cpu().numpy(), tensors[0][4])
    x = oracle.normal((2, 512), 9, 0.0, 1.0)
    y = ctx.matvec_f32(w, 96, 512, torch.from_numpy(x).cuda())
    want = oracle.matvec(tensors[0][4], 96, 512, oracle.quantize_q8k(x), 2, om.FOLD_X86)
    assert np.array_equal(y.cpu().numpy().view(np.uint32), want.view(np.uint32))
    # Q6_K tensor
    j = g.find("output.weight")
    w6 = g.upload(ctx, j)
    x6 = oracle.normal((1, 768), 10, 0.0, 1.0)
    xq = oracle.quantize_q8k(x6)
    y6 = ctx.q6k_matvec(w6, 40, 768, torch.from_numpy(xq.reshape(-1)).cuda(), 1)
    want6 = oracle.matvec_q6k(tensors[1][4], 40, 768, xq, 1)
    assert np.array_equal(y6.cpu().numpy().view(np.uint32), want6.view(np.uint32))
    g.close()
