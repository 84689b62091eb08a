"""pax_gemm_skinny_noalloc: the skinny GEMM without any allocation.

Callers whose GPU memory belongs to their own allocator (a framework's caching
allocator, a server that reserves memory at start-up) or that cannot afford
the device synchronisation of cudaMalloc/cudaFree need an entry point that
allocates nothing.  This one keeps the split-K scratch in a fixed 8 MiB array
inside the library.  Its output must match the ordinary skinny entry point
(pax_gemm_ex with PAX_ALGO_SKINNY, per-stream workspace) within the tolerances
of the other parity tests, on consecutive calls that reuse the shared array.

This file is collected last so that a failure here cannot hide others.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

import oracle
import pax_b200
from _helpers import TIGHT, check, inputs, to_dev

pytestmark = pytest.mark.gpu


def _noalloc(A, B, C, epilogue="none", bias=None, residual=None):
    d = pax_b200.make_desc(A, B, C, epilogue=epilogue, bias=bias, residual=residual)
    s = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    return pax_b200.lib.pax_gemm_skinny_noalloc(ctypes.byref(d), s)


@pytest.mark.parametrize("M,N,K,epi", [(16, 16384, 4096, "bias"), (33, 4096, 1024, "bias_gelu_erf"),
                                         (1, 1000, 320, "none"), (16, 20480, 2048, "bias")])
def test_noalloc_matches_workspace_entry_point_twice(cuda, rng, M, N, K, epi):
    A, B = inputs(rng, M, N, K, dist="normal")
    bias = rng.standard_normal(N).astype(np.float16)
    tA, tB, tb = to_dev(A, cuda), to_dev(B, cuda), to_dev(bias, cuda)
    tbias = tb if "bias" in epi else None
    ref = pax_b200.gemm(tA, tB, epilogue=epi, bias=tbias, algo="skinny")
    for _ in range(2):  # two calls in a row on the same shared scratch array
        C = torch.full_like(ref, float("nan"))
        st = _noalloc(tA, tB, C, epilogue=epi, bias=tbias)
        assert st == 0, pax_b200.lib.pax_status_string(st)
        torch.cuda.synchronize()
        got = C.cpu().numpy()
        check(got, ref.cpu().numpy(), np.float16)
        # and against the oracle, as every parity test
        check(got, oracle.gemm(A, B, epi=epi, bias=bias, out_dtype=np.float16), np.float16)
    assert oracle.normwise_error(got, ref.cpu().numpy()) <= TIGHT[np.float16]


def test_noalloc_rejects_problems_above_its_scratch_limit(cuda, rng):
    # m = 64, n = 20480 at 148 SMs: 160 column tiles, more than SMs, so the
    # stream-K layout (256-column units); its 148 CTAs need
    # 148 x 2 x 64 x 256 x 4 B = 19 MB of partial sums, above the 8 MiB array.
    A, B = inputs(rng, 64, 20480, 4096, dist="normal")
    tA, tB = to_dev(A, cuda), to_dev(B, cuda)
    C = torch.zeros((64, 20480), dtype=torch.float16, device=cuda)
    if torch.cuda.get_device_properties(0).multi_processor_count < 140:
        pytest.skip("scratch need depends on the SM count")
    st = _noalloc(tA, tB, C)
    assert st == pax_b200.Status.UNSUPPORTED
    torch.cuda.synchronize()
    assert (C == 0).all()  # nothing was launched
    big = torch.zeros((80, 20480), dtype=torch.float16, device=cuda)
    A80 = torch.zeros((80, 4096), dtype=torch.float16, device=cuda)
    assert _noalloc(A80, tB, big) == pax_b200.Status.UNSUPPORTED  # m > 64


def test_noalloc_leaves_no_device_error(cuda):
    assert pax_b200.device_error() == pax_b200.Status.OK
