"""Failure detection on the GPU without a fault: a bounded wait that runs out.

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
