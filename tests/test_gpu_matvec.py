"""GPU parity: the sm_100a kernels through the C ABI against the oracle and
the reference's golden vectors. Integer work, quantizer bytes and fp32
outputs must all be bit-exact."""
from __future__ import annotations

import numpy as np
import pytest

from conftest import golden_inputs

import oracle as om

pytestmark = pytest.mark.gpu

CASES = ["basic", "ragged", "k768_b8", "c1rows", "k12288", "edge", "argmax"]
FOLDS = [om.FOLD_X86, om.FOLD_GENERIC]


def dev(a):
    import torch

    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def host(t):
    import torch

    torch.cuda.synchronize()
    return t.cpu().numpy()


def bits(a):
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


def assert_bits_equal(got, want, what=""):
    g, w = bits(got), bits(want)
    if not np.array_equal(g, w):
        bad = np.nonzero(g.reshape(-1) != w.reshape(-1))[0]
        raise AssertionError(f"{what}: {bad.size} of {g.size} differ, first at {bad[:5]}: "
                             f"{np.asarray(got).reshape(-1)[bad[:5]]} vs {np.asarray(want).reshape(-1)[bad[:5]]}")


# ---------------------------------------------------------------- golden
@pytest.mark.parametrize("name", CASES)
def test_q8k_quantize_golden(ctx, oracle, golden, name):
    case = golden[name]
    n, k, b, w, x = golden_inputs(oracle, case)
    xq = host(ctx.q8k_quantize(dev(x)))
    assert np.array_equal(xq, case["x_q8k"])


@pytest.mark.parametrize("name", CASES)
@pytest.mark.parametrize("fold", FOLDS)
def test_matvec_golden_bit_exact(ctx, golden, name, fold):
    case = golden[name]
    n, k, b = (int(v) for v in case["shape"][:3])
    y = host(ctx.matvec(dev(case["w_q4k"]), n, k, dev(case["x_q8k"]), b, fold=fold))
    assert_bits_equal(y, case["y_x86"] if fold == om.FOLD_X86 else case["y_generic"], f"{name}/fold{fold}")


@pytest.mark.parametrize("name", CASES)
@pytest.mark.parametrize("fold", FOLDS)
def test_matvec_f32_prologue_golden(ctx, oracle, golden, name, fold):
    """Quantizing inside the matvec prologue gives the same bits."""
    case = golden[name]
    n, k, b, w, x = golden_inputs(oracle, case)
    y = host(ctx.matvec_f32(dev(case["w_q4k"]), n, k, dev(x), fold=fold))
    assert_bits_equal(y, case["y_x86"] if fold == om.FOLD_X86 else case["y_generic"], name)


@pytest.mark.parametrize("name", CASES)
@pytest.mark.parametrize("fold", FOLDS)
def test_partials_exact(ctx, oracle, golden, name, fold):
    import torch

    case = golden[name]
    n, k, b = (int(v) for v in case["shape"][:3])
    P = torch.zeros((b, n, k // 256, 9), dtype=torch.int32, device="cuda")
    y = ctx.matvec(dev(case["w_q4k"]), n, k, dev(case["x_q8k"]), b, partials=P, fold=fold)
    want = oracle.partials(case["w_q4k"].reshape(n, -1), n, k, case["x_q8k"].reshape(b, -1), b)
    assert np.array_equal(host(P), want)
    assert_bits_equal(host(y), case["y_x86"] if fold == om.FOLD_X86 else case["y_generic"], name)


@pytest.mark.parametrize("name", CASES)
def test_q4k_quantize_golden(ctx, oracle, golden, name):
    case = golden[name]
    n, k, b, w, x = golden_inputs(oracle, case)
    got = host(ctx.q4k_quantize(dev(w)))
    want = oracle.quantize_q4k(w).reshape(-1)  # == fixture bytes (pinned on CPU)
    assert np.array_equal(got, want)


@pytest.mark.parametrize("name", CASES)
def test_dequantize_golden(ctx, oracle, golden, name):
    case = golden[name]
    n, k = int(case["shape"][0]), int(case["shape"][1])
    got = host(ctx.q4k_dequantize(dev(case["w_q4k"]), n, k))
    assert_bits_equal(got, oracle.dequantize_q4k(case["w_q4k"], k), name)


# ---------------------------------------------------------------- config sizes
def seeded_q4k(ctx, oracle, n, k, seed, check_rows=48):
    """Seeded N(0, 0.02) weights quantized on the GPU; a sample of rows is
    checked byte-for-byte against the oracle quantizer."""
    w = oracle.normal((n, k), seed, 0.0, 0.02)
    wq = ctx.q4k_quantize(dev(w))
    rng = np.random.default_rng(seed)
    rows = np.unique(np.concatenate([[0, n - 1], rng.integers(0, n, check_rows)]))
    got = host(wq).reshape(n, -1)[rows]
    assert np.array_equal(got, oracle.quantize_q4k(w[rows]))
    return wq


@pytest.mark.parametrize("n,k", [(4096, 4096), (12288, 4096), (4096, 12288), (6144, 4096), (768, 2048), (2048, 768)])
@pytest.mark.parametrize("b", [1, 2, 3, 4, 8])
def test_config_shapes_bit_exact(ctx, oracle, n, k, b):
    wq = seeded_q4k(ctx, oracle, n, k, seed=1000 + n + k)
    x = oracle.normal((b, k), 2000 + b, 0.0, 1.0)
    xq = ctx.q8k_quantize(dev(x))
    xq_h = host(xq)
    assert np.array_equal(xq_h, oracle.quantize_q8k(x).reshape(-1))
    wq_h = host(wq)
    for fold in FOLDS:
        y = host(ctx.matvec(wq, n, k, xq, b, fold=fold))
        assert_bits_equal(y, oracle.matvec(wq_h, n, k, xq_h, b, fold), f"{n}x{k} b{b} fold{fold}")


@pytest.mark.parametrize("n,k,b", [(1, 256, 1), (33, 256, 3), (148 * 32 + 5, 512, 2), (7, 768, 8), (300, 1024, 5),
                                   (31, 16384, 1), (2, 65536, 1)])
def test_ragged_shapes(ctx, oracle, n, k, b):
    w = oracle.normal((n, k), 77 + n, 0.0, 0.02)
    wq = oracle.quantize_q4k(w)
    x = oracle.normal((b, k), 88 + k, 0.0, 1.0)
    xq = oracle.quantize_q8k(x)
    for fold in FOLDS:
        y = host(ctx.matvec(dev(wq), n, k, dev(xq), b, fold=fold))
        assert_bits_equal(y, oracle.matvec(wq, n, k, xq, b, fold), f"{n}x{k} b{b}")


# ---------------------------------------------------------------- boundary forms
def test_mul_mat_host(ctx, oracle):
    n, k, b = 1000, 2048, 3
    wq = oracle.quantize_q4k(oracle.normal((n, k), 5, 0.0, 0.02))
    x = oracle.normal((b, k), 6, 0.0, 1.0)
    y = np.empty((b, n), np.float32)
    ctx.mul_mat_host(dev(wq), n, k, x, y)
    assert_bits_equal(y, oracle.matvec(wq, n, k, oracle.quantize_q8k(x), b, om.FOLD_X86), "host path")


def test_ggml_vec_dot_shim(ctx, bh, oracle, golden):
    import ctypes as C

    case = golden["c1rows"]
    n, k = int(case["shape"][0]), int(case["shape"][1])
    wq = case["w_q4k"].reshape(n, -1)
    xq = case["x_q8k"]
    for r in range(n):
        s = C.c_float(0)
        bh.lib.bh_ggml_vec_dot_q4_K_q8_K(k, C.byref(s), 0, wq[r].ctypes.data, 0, xq.ctypes.data, 0, 1)
        assert np.float32(s.value).view(np.uint32) == case["y_x86"][0, r].view(np.uint32)


def test_invalid_arguments_launch_nothing(ctx, bh):
    import torch

    w = torch.zeros(144 * 4, dtype=torch.uint8, device="cuda")
    xq = torch.zeros(292, dtype=torch.uint8, device="cuda")
    y = torch.full((4,), 7.0, device="cuda")
    L = bh.lib
    assert L.bh_q4k_matvec(ctx.h, w.data_ptr(), 4, 300, xq.data_ptr(), 1, y.data_ptr(), None, 0, None) == bh.BH_EINVAL
    assert L.bh_q4k_matvec(ctx.h, w.data_ptr(), 4, 256, xq.data_ptr(), 9, y.data_ptr(), None, 0, None) == bh.BH_EINVAL
    assert L.bh_q4k_matvec(ctx.h, w.data_ptr() + 8, 4, 256, xq.data_ptr(), 1, y.data_ptr(), None, 0, None) == bh.BH_EINVAL
    assert L.bh_q4k_matvec(ctx.h, w.data_ptr(), 4, 256, xq.data_ptr(), 1, y.data_ptr(), None, 7, None) == bh.BH_EINVAL
    torch.cuda.synchronize()
    assert (y == 7.0).all()
    # empty inputs are no-ops; K == 0 gives zeros (a dot product of nothing)
    assert L.bh_q4k_matvec(ctx.h, w.data_ptr(), 0, 256, xq.data_ptr(), 1, y.data_ptr(), None, 0, None) == 0
    assert L.bh_q4k_matvec(ctx.h, w.data_ptr(), 4, 0, xq.data_ptr(), 1, y.data_ptr(), None, 0, None) == 0
    torch.cuda.synchronize()
    assert (y == 0.0).all()
    assert ctx.status() == 0


def test_fp16_scale_conversion_matches_oracle(ctx, oracle):
    """The GPU quantizer's fp32->fp16 scale rounding equals the reference's
    on values spanning normal, subnormal and near-overflow ranges."""
    rng = np.random.default_rng(3)
    # rows whose super-block maxima land in many binades, incl. fp16-subnormal scales
    scales = np.float32(10.0) ** rng.uniform(-9, 3, 256).astype(np.float32)
    w = (oracle.normal((256, 256), 9, 0.0, 1.0) * scales[:, None]).astype(np.float32)
    assert np.array_equal(host(ctx.q4k_quantize(dev(w))), oracle.quantize_q4k(w).reshape(-1))


@pytest.mark.parametrize("tpr", [4, 8, 16])
@pytest.mark.parametrize("n,k,b", [(4096, 4096, 1), (4096, 12288, 2), (1000, 768, 1), (33, 2048, 2), (151936 // 16, 4096, 1)])
def test_forced_threads_per_row_bit_exact(ctx, bh, oracle, tpr, n, k, b):
    """4, 8 or 16 threads per row (the planner picks by shape; 16 falls back
    to 8 for the generic fold and the partials) give the same bits."""
    w = oracle.normal((n, k), 31 + n + k, 0.0, 0.02)
    wq = oracle.quantize_q4k(w)
    x = oracle.normal((b, k), 41 + k, 0.0, 1.0)
    xq = oracle.quantize_q8k(x)
    ctx.tune(bh.TUNE_TPR, tpr)
    try:
        for fold in FOLDS:
            y = host(ctx.matvec(dev(wq), n, k, dev(xq), b, fold=fold))
            assert_bits_equal(y, oracle.matvec(wq, n, k, xq, b, fold), f"tpr{tpr} {n}x{k} b{b} fold{fold}")
            y2 = host(ctx.matvec_f32(dev(wq), n, k, dev(x), fold=fold))
            assert_bits_equal(y2, oracle.matvec(wq, n, k, xq, b, fold), f"f32 tpr{tpr}")
            P = torch_zeros_int((b, n, k // 256, 9))
            ctx.matvec(dev(wq), n, k, dev(xq), b, partials=P, fold=fold)
            assert np.array_equal(host(P), oracle.partials(wq, n, k, xq, b))
    finally:
        ctx.tune(bh.TUNE_TPR, 0)


@pytest.mark.parametrize("tpr", [8, 16])
@pytest.mark.parametrize("n,k,b", [(4096, 4096, 1), (2000, 12288, 2), (4736, 4096, 1)])
def test_threads_per_row_argmax(ctx, bh, oracle, tpr, n, k, b):
    """The LM-head argmax epilogue (fp32 input quantized in the prologue) at 8
    and 16 threads per row gives the oracle's logits, maxima and tokens."""
    w = oracle.normal((n, k), 77 + n + k, 0.0, 0.02)
    wq = oracle.quantize_q4k(w)
    x = oracle.normal((b, k), 78 + k, 0.0, 1.0)
    xq = oracle.quantize_q8k(x)
    want = oracle.matvec(wq, n, k, xq, b, 0).reshape(b, n)
    ctx.tune(bh.TUNE_TPR, tpr)
    try:
        logits = dev(np.zeros((b, n), np.float32))
        tok, mx = bh.lmhead_argmax(ctx, dev(wq), n, k, dev(x), logits=logits)
        assert_bits_equal(host(logits).reshape(b, n), want, f"argmax logits tpr{tpr}")
        assert list(host(tok)) == [int(np.argmax(want[i])) for i in range(b)]
        assert np.array_equal(host(mx), want.max(axis=1))
    finally:
        ctx.tune(bh.TUNE_TPR, 0)


@pytest.mark.parametrize("prefill", [0, 1, 2, -1])
@pytest.mark.parametrize("n,k,b", [(4096, 4096, 1), (4096, 12288, 2), (33, 2048, 1), (12288, 4096, 4)])
def test_split_prefill_bit_exact(ctx, bh, oracle, prefill, n, k, b):
    """Issuing all, part or none of each warp's ring before the programmatic
    wait (the rest after the activation loads) gives the same bits."""
    w = oracle.normal((n, k), 7 + n + k, 0.0, 0.02)
    wq = oracle.quantize_q4k(w)
    x = oracle.normal((b, k), 5 + k, 0.0, 1.0)
    xq = oracle.quantize_q8k(x)
    ctx.tune(bh.TUNE_PREFILL, prefill)
    try:
        for fold in FOLDS:
            want = oracle.matvec(wq, n, k, xq, b, fold)
            assert_bits_equal(host(ctx.matvec(dev(wq), n, k, dev(xq), b, fold=fold)), want, f"q8k prefill{prefill}")
            assert_bits_equal(host(ctx.matvec_f32(dev(wq), n, k, dev(x), fold=fold)), want, f"f32 prefill{prefill}")
    finally:
        ctx.tune(bh.TUNE_PREFILL, 1)  # the default


def torch_zeros_int(shape):
    import torch

    return torch.zeros(shape, dtype=torch.int32, device="cuda")


def test_pdl_sequence_bit_exact(ctx, bh, oracle):
    """Back-to-back matvecs launched with programmatic dependent launch
    (BH_TUNE_PDL): each result equals the plain launch's bits, including
    launches whose input is computed from the output of the one before."""
    import torch

    n, k = 4096, 4096
    w = oracle.normal((n, k), 4242, 0.0, 0.02)
    wq = dev(oracle.quantize_q4k(w))
    x = dev(oracle.normal((1, k), 4343, 0.0, 1.0))
    want = [host(ctx.matvec_f32(wq, n, k, x))]
    for i in range(3):
        want.append(host(ctx.matvec_f32(wq, n, k, dev(want[-1] * np.float32(0.05)))))
    ys = [torch.empty((1, n), device="cuda") for _ in range(4)]
    xs = [torch.empty((1, n), device="cuda") for _ in range(3)]
    ctx.tune(bh.TUNE_PDL, 1)
    try:
        s = torch.cuda.Stream()
        with torch.cuda.stream(s):
            ctx.matvec_f32(wq, n, k, x, y=ys[0], stream=s)
            for i in range(3):
                torch.mul(ys[i], 0.05, out=xs[i])
                ctx.matvec_f32(wq, n, k, xs[i], y=ys[i + 1], stream=s)
        s.synchronize()
    finally:
        ctx.tune(bh.TUNE_PDL, 0)
    for i in range(4):
        assert_bits_equal(host(ys[i]), want[i], f"pdl step {i}")
