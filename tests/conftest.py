"""Shared fixtures. GPU tests are marked `gpu`; everything else runs on CPU."""
from __future__ import annotations

import os
import subprocess
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "shannon-prime-burnhard_b200")
ORACLE_DIR = os.path.join(ROOT, "oracle")
GOLDEN = os.path.join(ROOT, "tests", "golden", "q4k_golden.npz")

for p in (PKG, ORACLE_DIR):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (B200, sm_100a) device")


def _ensure_built():
    if not os.path.exists(os.path.join(ORACLE_DIR, "liboracle.so")):
        subprocess.run(["make", "-s", "-C", ORACLE_DIR, "oracle"], check=True)
    if not os.path.exists(os.path.join(PKG, "libbh_q4k.so")):
        subprocess.run(["make", "-s", "-C", PKG], check=True)


_ensure_built()


@pytest.fixture(scope="session")
def oracle():
    import oracle as om

    return om.Oracle()


@pytest.fixture(scope="session")
def reference():
    """The reference's own code (oracle/_ref); skipped where it is not built."""
    import oracle as om

    if not os.path.exists(om.REF_SO):
        pytest.skip("oracle/_ref not built (the reference tree is absent)")
    r = om.Reference()
    if not r.has_avx2:
        pytest.skip("host CPU lacks AVX2/FMA/F16C for the reference's x86 path")
    return r


@pytest.fixture(scope="session")
def golden():
    d = np.load(GOLDEN)
    cases = {}
    for key in d.files:
        name, field = key.split("__", 1)
        cases.setdefault(name, {})[field] = d[key]
    return cases


def golden_inputs(oracle, case: dict):
    """Regenerate a case's seeded fp32 inputs and check them against the fixture."""
    import hashlib

    n, k, b, ws, xs = (int(v) for v in case["shape"])
    if "w_f32" in case:
        w, x = case["w_f32"], case["x_f32"]
    else:
        w = oracle.normal((n, k), ws, 0.0, 0.02)
        x = oracle.normal((b, k), xs, 0.0, 1.0)
    assert hashlib.sha256(np.ascontiguousarray(w).tobytes()).hexdigest() == str(case["w_sha"])
    assert hashlib.sha256(np.ascontiguousarray(x).tobytes()).hexdigest() == str(case["x_sha"])
    return n, k, b, w, x


@pytest.fixture(scope="session")
def bh():
    import burnhard

    return burnhard


@pytest.fixture(scope="session")
def ctx(bh):
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    c = bh.Context(0)
    yield c
    assert c.status() == 0, "a kernel reported a device-side timeout"
    c.close()
