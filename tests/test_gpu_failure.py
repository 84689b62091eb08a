"""Failure detection on the GPU without a fault: bounded waits that run out.

pax_selftest_bounded_wait launches one thread that waits, with the kernels'
own bounded mbarrier wait, on a barrier nothing arrives on.  The wait must
give up after its 2 s limit, record a timeout that pax_device_error() reports,
and leave the CUDA context usable for the next GEMM.
"""
from __future__ import annotations

import time

import numpy as np
import pytest
import torch

import oracle
import pax_b200
from _helpers import check, inputs, run_gemm

pytestmark = pytest.mark.gpu


def test_bounded_wait_times_out_and_context_survives(cuda, rng):
    pax_b200.device_error()  # start from a clear error word
    s = torch.cuda.current_stream(cuda).cuda_stream
    t0 = time.time()
    assert pax_b200.lib.pax_selftest_bounded_wait(s) == 0
    torch.cuda.synchronize()
    waited = time.time() - t0
    assert pax_b200.device_error() == pax_b200.Status.TIMEOUT
    assert 1.5 < waited < 60, waited
    assert pax_b200.device_error() == pax_b200.Status.OK  # read and cleared
    # The context still runs GEMMs correctly.
    A, B = inputs(rng, 512, 768, 384)
    bias = rng.standard_normal(768).astype(np.float16)
    got = run_gemm(A, B, cuda, epi="bias_gelu_tanh", bias=bias, out_dtype=np.float16)
    check(got, oracle.gemm(A, B, epi="bias_gelu_tanh", bias=bias, out_dtype=np.float16), np.float16)
    assert pax_b200.device_error() == pax_b200.Status.OK


# ----------------------------------------------------------------- abort paths
# The GEMM kernels' own waits run out when a test shortens the limit of the
# waits a CTA may abandon (pax_selftest_set_wait_limit).  The kernel then
# takes its abort path: its issued TMA loads land, its issued MMAs drain,
# TMEM is freed, a timeout is recorded, and it ends.  Nothing faults or hangs:
# the abort path's own waits keep the 2 s limit.  The next GEMM in the same
# context must be correct.  In the CTA-pair kernels both CTAs' loads complete
# on the leader's barriers; the non-leader reports how many k-blocks it
# issued and the leader settles every stage before the pair tears down.
SHORT_NS = 2000


def _abort_run(fn):
    lib = pax_b200.lib
    pax_b200.device_error()  # start from a clear error word
    assert lib.pax_selftest_set_wait_limit(SHORT_NS) == 0
    try:
        fn()
        torch.cuda.synchronize()
    finally:
        assert lib.pax_selftest_set_wait_limit(0) == 0
    return pax_b200.device_error()


@pytest.mark.parametrize("shape", ["128", "256"])
def test_tc_one_cta_kernel_abort_path(cuda, rng, monkeypatch, shape):
    monkeypatch.setenv("PAX_TC_BN", shape)
    g = torch.Generator(device=cuda)
    g.manual_seed(7)
    A = torch.randn((1024, 65536), generator=g, device=cuda).half()
    B = torch.randn((65536, 1024), generator=g, device=cuda).half()
    bias = torch.randn((1024,), generator=g, device=cuda).half()
    C = torch.empty((1024, 1024), dtype=torch.float16, device=cuda)
    st = _abort_run(lambda: pax_b200.gemm(A, B, out=C, epilogue="bias_gelu_tanh", bias=bias, algo="tc"))
    assert st == pax_b200.Status.TIMEOUT
    assert pax_b200.device_error() == pax_b200.Status.OK
    del A, B
    # The same kernel, with the default limit, is correct afterwards.
    A2, B2 = inputs(rng, 640, 1024, 512)
    b2 = rng.standard_normal(1024).astype(np.float16)
    got = run_gemm(A2, B2, cuda, epi="bias_gelu_tanh", bias=b2, out_dtype=np.float16, algo="tc")
    check(got, oracle.gemm(A2, B2, epi="bias_gelu_tanh", bias=b2, out_dtype=np.float16), np.float16)
    assert pax_b200.device_error() == pax_b200.Status.OK


@pytest.mark.parametrize("shape", ["2", "4"])
def test_tc_pair_kernel_abort_path(cuda, rng, monkeypatch, shape):
    # 2: CTA pairs on 256 x 256 tiles; 4: CTA pairs on 256 x 512 tiles.
    monkeypatch.setenv("PAX_TC_SHAPE", shape)
    g = torch.Generator(device=cuda)
    g.manual_seed(9)
    A = torch.randn((1024, 65536), generator=g, device=cuda).half()
    B = torch.randn((65536, 1024), generator=g, device=cuda).half()
    bias = torch.randn((1024,), generator=g, device=cuda).half()
    C = torch.empty((1024, 1024), dtype=torch.float16, device=cuda)
    assert pax_b200.select_algo(A, B, C, epilogue="bias_gelu_tanh", bias=bias) == pax_b200.Algo.TC2
    for _ in range(3):  # the two CTAs give up at different points each time
        st = _abort_run(lambda: pax_b200.gemm(A, B, out=C, epilogue="bias_gelu_tanh", bias=bias))
        assert st == pax_b200.Status.TIMEOUT
        assert pax_b200.device_error() == pax_b200.Status.OK
    del A, B
    A2, B2 = inputs(rng, 640, 1536, 512)
    b2 = rng.standard_normal(1536).astype(np.float16)
    got = run_gemm(A2, B2, cuda, epi="bias_gelu_tanh", bias=b2, out_dtype=np.float16)
    check(got, oracle.gemm(A2, B2, epi="bias_gelu_tanh", bias=b2, out_dtype=np.float16), np.float16)
    assert pax_b200.device_error() == pax_b200.Status.OK


@pytest.mark.parametrize("N", [16384, 4096])
def test_skinny_kernel_abort_path(cuda, rng, N):
    # N = 16384: 128 tiles, one CTA each.  N = 4096: 32 tiles with K split
    # over 4 CTAs each, so the abort can leave split-tile arrival counters
    # behind in this stream's workspace.
    g = torch.Generator(device=cuda)
    g.manual_seed(8)
    K = 65536
    A = torch.randn((16, K), generator=g, device=cuda).half()
    B = (torch.randn((K, N), generator=g, device=cuda) * 0.02).half()
    C = torch.empty((16, N), dtype=torch.float16, device=cuda)
    st = _abort_run(lambda: pax_b200.gemm(A, B, out=C, algo="skinny"))
    assert st == pax_b200.Status.TIMEOUT
    assert pax_b200.device_error() == pax_b200.Status.OK
    del A, B
    # A split-tile problem on the same stream (same workspace) afterwards.
    A2, B2 = inputs(rng, 16, 4096, 4096, dist="normal")
    got = run_gemm(A2, B2, cuda, out_dtype=np.float16, algo="skinny")
    check(got, oracle.gemm(A2, B2, out_dtype=np.float16), np.float16)
    assert pax_b200.device_error() == pax_b200.Status.OK


def test_wait_limit_hook_rejects_sub_microsecond_limits(cuda):
    assert pax_b200.lib.pax_selftest_set_wait_limit(10) == pax_b200.Status.INVALID
    assert pax_b200.lib.pax_selftest_set_wait_limit(0) == 0
