"""CPU: the oracle restatement against the reference's golden vectors and,
where it is built, against the reference's own compiled code."""
from __future__ import annotations

import numpy as np
import pytest

from conftest import golden_inputs

import oracle as om

CASES = ["basic", "ragged", "k768_b8", "c1rows", "k12288", "edge", "argmax"]


def bits(a):
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


@pytest.mark.parametrize("name", CASES)
def test_q4k_quantizer_matches_golden(oracle, golden, name):
    case = golden[name]
    n, k, b, w, x = golden_inputs(oracle, case)
    wq = oracle.quantize_q4k(w).reshape(-1)
    ref = case["w_q4k"].copy()
    if name == "argmax":  # the fixture carries one planted duplicate row
        rb = om.q4k_row_bytes(k)
        diff_rows = np.nonzero((wq.reshape(n, rb) != ref.reshape(n, rb)).any(axis=1))[0]
        assert len(diff_rows) == 1
        return
    assert np.array_equal(wq, ref)


@pytest.mark.parametrize("name", CASES)
def test_q8k_quantizer_matches_golden(oracle, golden, name):
    case = golden[name]
    n, k, b, w, x = golden_inputs(oracle, case)
    assert np.array_equal(oracle.quantize_q8k(x).reshape(-1), case["x_q8k"])


@pytest.mark.parametrize("name", CASES)
@pytest.mark.parametrize("fold", [om.FOLD_X86, om.FOLD_GENERIC])
def test_vec_dot_matches_golden_bit_exact(oracle, golden, name, fold):
    case = golden[name]
    n, k, b = (int(v) for v in case["shape"][:3])
    y = oracle.matvec(case["w_q4k"], n, k, case["x_q8k"], b, fold)
    want = case["y_x86"] if fold == om.FOLD_X86 else case["y_generic"]
    assert np.array_equal(bits(y), bits(want))


@pytest.mark.parametrize("name", CASES)
def test_partials_reproduce_outputs(oracle, golden, name):
    """The exact integer partials, folded in fp64, agree with both fp32 folds
    to the reference's own tolerance (|a-b| <= 1e-6 + 1e-5 |a|)."""
    case = golden[name]
    n, k, b = (int(v) for v in case["shape"][:3])
    wq = case["w_q4k"].reshape(n, -1)
    xq = case["x_q8k"].reshape(b, -1)
    P = oracle.partials(wq, n, k, xq, b).astype(np.int64)
    nb = k // 256
    hdr = wq.reshape(n, nb, 144)
    d = hdr[:, :, 0:2].copy().view(np.float16)[..., 0].astype(np.float64)
    dmin = hdr[:, :, 2:4].copy().view(np.float16)[..., 0].astype(np.float64)
    sc = np.zeros((n, nb, 8), np.int64)
    for r in range(n):
        for i in range(nb):
            s12 = hdr[r, i, 4:16]
            for j in range(8):
                if j < 4:
                    sc[r, i, j] = s12[j] & 63
                else:
                    sc[r, i, j] = (s12[j + 4] & 0xF) | ((s12[j - 4] >> 6) << 4)
    yd = xq.reshape(b, nb, 292)[:, :, 0:4].copy().view(np.float32)[..., 0].astype(np.float64)
    ints = (P[..., :8] * sc[None]).sum(-1)
    y64 = (yd[:, None, :] * (d[None] * ints - dmin[None] * P[..., 8])).sum(-1)
    for key in ("y_x86", "y_generic"):
        got = case[key].astype(np.float64)
        bad = np.abs(got - y64) > 1e-6 + 1e-5 * np.abs(y64)
        # the reference's own folds exceed this bar on a few rows of large K
        assert bad.sum() <= max(1, n * b // 1000), (key, bad.sum())


def test_argmax_tie_first_index(golden, oracle):
    case = golden["argmax"]
    y = case["y_x86"]
    for c in range(y.shape[0]):
        assert oracle.argmax(y[c]) == int(case["argmax_x86"][c])
    assert (y[0] == y[0].max()).sum() == 2  # the planted tie is present


def test_dequantize_matches_golden(oracle, golden):
    import hashlib

    for name in CASES:
        case = golden[name]
        n, k = int(case["shape"][0]), int(case["shape"][1])
        deq = oracle.dequantize_q4k(case["w_q4k"], k)
        assert hashlib.sha256(deq.tobytes()).hexdigest() == str(case["deq_sha"]), name


def test_fp16_conversions_exhaustive(oracle):
    """fp16 -> fp32 for all 2^16 codes and fp32 -> fp16 on a sweep, against numpy."""
    import ctypes as C

    lib = oracle.lib
    codes = np.arange(1 << 16, dtype=np.uint16)
    want = codes.view(np.float16).astype(np.float32)
    got = np.array([lib.bho_fp16_to_fp32(int(h)) for h in codes], dtype=np.float32)
    nan = np.isnan(want)
    assert np.array_equal(bits(got[~nan]), bits(want[~nan]))
    assert np.isnan(got[nan]).all()
    rng = np.random.default_rng(7)
    vals = np.concatenate([
        rng.standard_normal(20000).astype(np.float32) * np.float32(10.0) ** rng.integers(-9, 6, 20000).astype(np.float32),
        np.array([0.0, -0.0, 65504.0, 65519.99, 65520.0, 1e-8, 2.0**-25, 2.0**-24, 5.96e-8, 6.1e-5], dtype=np.float32),
    ]).astype(np.float32)
    got16 = np.array([lib.bho_fp32_to_fp16(C.c_float(float(v))) for v in vals], dtype=np.uint16)
    with np.errstate(over="ignore"):
        want16 = vals.astype(np.float16).view(np.uint16)
    assert np.array_equal(got16, want16)


@pytest.mark.parametrize("n,k,b,seed", [(96, 2048, 3, 11), (7, 768, 8, 12), (40, 12288, 1, 13)])
def test_oracle_against_compiled_reference(oracle, reference, n, k, b, seed):
    w = oracle.normal((n, k), seed, 0.0, 0.02)
    x = oracle.normal((b, k), seed + 1, 0.0, 1.0)
    wq = reference.quantize_q4k(w)
    assert np.array_equal(oracle.quantize_q4k(w), wq)
    xq = reference.quantize_q8k(x)
    assert np.array_equal(oracle.quantize_q8k(x), xq)
    for fold in (om.FOLD_X86, om.FOLD_GENERIC):
        assert np.array_equal(bits(oracle.matvec(wq, n, k, xq, b, fold)), bits(reference.matvec_rows(wq, n, k, xq, b, fold)))
    # ggml-style threaded mul_mat (fp32 activations) equals the AVX2 row loop
    ym = reference.mul_mat(wq, n, k, x, 4)
    assert np.array_equal(bits(ym), bits(reference.matvec_rows(wq, n, k, xq, b, om.FOLD_X86)))
