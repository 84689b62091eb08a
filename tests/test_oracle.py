"""The oracle itself: pinned against the reference's own CPU path.

The golden fixtures were written by the reference's cpu_gemm_ref /
pax_verify_gemm (src/host_bridge.c:397-445) compiled from its sources
(tests/golden/make_golden.py).  The oracle must reproduce them bit for bit.
"""
from __future__ import annotations

import glob
import math
import os

import numpy as np
import pytest

import oracle

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
GEMM_CASES = sorted(glob.glob(os.path.join(GOLDEN, "gemm_*.npz")))


def test_golden_fixtures_present():
    assert len(GEMM_CASES) >= 7


@pytest.mark.parametrize("path", GEMM_CASES, ids=lambda p: os.path.basename(p)[5:-4])
def test_oracle_matches_reference_golden(path):
    d = np.load(path)
    A, B, C = d["A"], d["B"], d["C"]
    lit = oracle.cpu_gemm_ref(A.astype(np.float32), B.astype(np.float32))
    assert np.array_equal(lit.view(np.uint32), C.view(np.uint32)), "literal restatement differs from reference"
    fast = oracle.gemm_f16(A, B, nthreads=2)
    assert np.array_equal(fast.view(np.uint32), C.view(np.uint32)), "row-parallel oracle differs from reference"


def test_integer_kat_is_exact():
    d = np.load(os.path.join(GOLDEN, "gemm_int_kat.npz"))
    exact = d["A"].astype(np.int64) @ d["B"].astype(np.int64)
    assert np.array_equal(d["C"], exact.astype(np.float32))


def test_identity_and_permutation_kat():
    d = np.load(os.path.join(GOLDEN, "gemm_identity.npz"))
    assert np.array_equal(d["C"], d["B"].astype(np.float32))
    d = np.load(os.path.join(GOLDEN, "gemm_permutation.npz"))
    perm = np.argmax(d["A"].astype(np.float32), axis=1)
    assert np.array_equal(d["C"], d["B"].astype(np.float32)[perm])


def test_verify_matches_reference_decisions():
    d = np.load(os.path.join(GOLDEN, "verify_decisions.npz"))
    for i in range(d["C_gpu"].shape[0]):
        for j, tol in enumerate(d["tols"]):
            ok, _, _ = oracle.verify(d["C_gpu"][i], d["C_ref"], float(tol))
            assert int(ok) == int(d["decisions"][i, j])


def test_reference_build_matches_restatement_when_present(rng):
    if oracle.ref_lib() is None:
        pytest.skip("oracle/_ref not built here")
    for (m, n, k) in [(1, 1, 1), (7, 9, 300), (64, 33, 129)]:
        A = rng.uniform(-1, 1, (m, k)).astype(np.float16).astype(np.float32)
        B = rng.uniform(-1, 1, (k, n)).astype(np.float16).astype(np.float32)
        a = oracle.reference_cpu_gemm_ref(A, B)
        b = oracle.cpu_gemm_ref(A, B)
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


def test_fp16_widening_exhaustive():
    h = np.arange(65536, dtype=np.uint16)
    w = oracle.f16_to_f32(h)
    ref = h.view(np.float16).astype(np.float32)
    nan = np.isnan(ref)
    assert np.array_equal(w[~nan].view(np.uint32), ref[~nan].view(np.uint32))
    assert np.isnan(w[nan]).all()


def test_fp16_rounding_matches_ieee(rng):
    x = np.concatenate([
        rng.standard_normal(200000).astype(np.float32) * np.float32(3e4),
        rng.standard_normal(200000).astype(np.float32) * np.float32(1e-5),
        np.array([65504, 65519.996, 65520, 1e9, 2.0 ** -25, 2.0 ** -24, 3 * 2.0 ** -26, 0.0, -0.0, np.inf, -np.inf],
                 np.float32),
    ])
    with np.errstate(over="ignore"):
        ref = x.astype(np.float16)
    assert np.array_equal(oracle.f32_to_f16(x).view(np.uint16), ref.view(np.uint16))


def test_gelu_known_values():
    for x in (0.0, 1.0, -1.0, 3.0, -3.0, 0.5):
        t = 0.5 * x * (1 + math.tanh(math.sqrt(2 / math.pi) * (x + 0.044715 * x ** 3)))
        e = 0.5 * x * (1 + math.erf(x / math.sqrt(2)))
        assert abs(oracle.gelu_tanh(x) - t) <= 2e-7 * max(1.0, abs(t))
        assert abs(oracle.gelu_erf(x) - e) <= 2e-7 * max(1.0, abs(e))


def test_gelu_bound_stated_by_reference():
    """|GeLU_tanh - GeLU_exact| <= 1e-3 |x| (README.md:43, PAX/GEMM.lean:150-152)."""
    xs = np.linspace(-12, 12, 48001, dtype=np.float32)
    worst = 0.0
    for x in xs[::7]:
        d = abs(oracle.gelu_tanh(float(x)) - oracle.gelu_erf(float(x)))
        if x != 0:
            worst = max(worst, d / abs(float(x)))
    assert worst <= 1e-3
    assert worst > 1e-5  # the two forms do differ


def test_epilogue_order_scale_bias_gelu(rng):
    C = rng.standard_normal((4, 8)).astype(np.float32)
    bias = rng.standard_normal(8).astype(np.float16)
    out = oracle.epilogue(C.copy(), "bias_gelu_tanh", alpha=0.5, bias=bias)
    for i in range(4):
        for j in range(8):
            v = np.float32(C[i, j] * np.float32(0.5)) + np.float32(bias[j])
            assert out[i, j] == np.float32(oracle.gelu_tanh(float(v)))


def test_residual_indexing(rng):
    C = np.zeros((3, 5), np.float32)
    R = rng.standard_normal((3, 5)).astype(np.float32)
    out = oracle.epilogue(C.copy(), "residual", residual=R)
    assert np.array_equal(out, R)
    rows = np.array([2, 0], np.int64)
    out = oracle.epilogue(np.zeros((2, 5), np.float32), "residual", residual=R, rows=rows)
    assert np.array_equal(out, R[rows])


def test_row_subset(rng):
    A = rng.uniform(-1, 1, (50, 70)).astype(np.float16)
    B = rng.uniform(-1, 1, (70, 30)).astype(np.float16)
    full = oracle.gemm_f16(A, B)
    rows = np.array([49, 0, 17], np.int64)
    part = oracle.gemm_f16(A, B, rows=rows)
    assert np.array_equal(part, full[rows])
