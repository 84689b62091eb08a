"""Host-bridge entry points on the GPU, through the C ABI: the reference's
bench harness (src/host_bridge.c:543-566), the shared-memory queries of the
reference-named launchers, and the skinny kernel's workspace handling
(publication flags left by an aborted launch, cudaStreamPerThread)."""
from __future__ import annotations

import ctypes
import math
import re
import threading

import numpy as np
import pytest
import torch

import oracle
import pax_b200
from _helpers import check, inputs, run_gemm, to_dev

pytestmark = pytest.mark.gpu


def test_bench_all_times_every_variant(cuda, capfd):
    """pax_bench_setup + pax_bench_all on a small shape, as the reference's
    harness runs its variants: one row per variant, each with a finite,
    positive time."""
    s = torch.cuda.current_stream(cuda).cuda_stream
    lib = pax_b200.lib
    assert lib.pax_bench_setup(256, 512, 384, s) == 1
    try:
        lib.pax_bench_all(3)
        torch.cuda.synchronize()
    finally:
        lib.pax_bench_teardown()
    out = capfd.readouterr().out
    assert "[PAX] Benchmark  m=256  n=512  k=384  iters=3" in out
    rows = {}
    for line in out.splitlines():
        m = re.match(r"^(\w+)\s+([0-9.eE+-]+|nan|inf)\s+([0-9.eE+-]+|nan|inf)\s*$", line.strip())
        if m:
            rows[m.group(1)] = (float(m.group(2)), float(m.group(3)))
    for name in ["wmma", "ptx", "pipeline", "bias_gelu", "residual_gelu", "bias_gelu_f16", "residual_gelu_erf_f16"]:
        assert name in rows, (name, out)
        ms, tflops = rows[name]
        assert math.isfinite(ms) and ms > 0, (name, ms)
        assert math.isfinite(tflops) and tflops > 0, (name, tflops)
    assert pax_b200.device_error() == pax_b200.Status.OK


def test_bench_all_without_setup_is_rejected(cuda, capfd):
    pax_b200.lib.pax_bench_teardown()
    pax_b200.lib.pax_bench_all(1)
    assert pax_b200.lib.pax_last_error() == pax_b200.Status.INVALID
    assert "pax_bench_setup" in capfd.readouterr().err


def test_smem_queries_on_the_device(cuda):
    """On the B200 the launchers' queries name the kernels chosen for 4096^3
    fp32 C, and fit the per-CTA limit of the device."""
    limit = torch.cuda.get_device_properties(0).shared_memory_per_block_optin
    lib = pax_b200.lib
    for f in (lib.pax_gemm_ptx_smem_bytes, lib.pax_gemm_pipeline_smem_bytes, lib.pax_gemm_tma_smem_bytes):
        assert 0 < f() <= limit
    A = torch.empty((4096, 4096), dtype=torch.float16, device=cuda)
    C = torch.empty((4096, 4096), dtype=torch.float32, device=cuda)
    d = pax_b200.make_desc(A, A, C)
    assert lib.pax_gemm_smem_bytes(ctypes.byref(d)) == lib.pax_gemm_ptx_smem_bytes()


def test_skinny_ignores_flags_left_by_an_aborted_launch(cuda, rng):
    """A launch that gave up on a timed-out wait can leave split-tile
    publication flags behind.  The next launch on that stream must ignore
    them (they carry an older launch epoch): its reducing CTAs must wait for
    this launch's partial sums, not read stale ones."""
    s = torch.cuda.current_stream(cuda).cuda_stream
    # 32 column tiles: the lockstep layout splits each tile's K over 4 CTAs,
    # so every tile is reduced through flags; then stream-K.
    for M, N, K, nt in [(16, 4096, 4096, "0"), (16, 16384, 4096, "128")]:
        A, B = inputs(rng, M, N, K, dist="normal")
        ref = oracle.gemm(A, B, out_dtype=np.float16)
        with pytest.MonkeyPatch.context() as mp:
            mp.setenv("PAX_SKINNY_NT", nt)
            check(run_gemm(A, B, cuda, out_dtype=np.float16, algo="skinny"), ref, np.float16)
            for _ in range(2):
                assert pax_b200.lib.pax_selftest_stale_counters(s) == 0
                check(run_gemm(A, B, cuda, out_dtype=np.float16, algo="skinny"), ref, np.float16)
    assert pax_b200.device_error() == pax_b200.Status.OK


def test_per_thread_default_stream_from_two_threads(cuda, rng):
    """cudaStreamPerThread is one handle value that names a different stream
    in each host thread.  Skinny GEMMs on it from two threads at once must
    not share a workspace (they would race on its flags and partials)."""
    A, B = inputs(rng, 16, 4096, 4096, dist="normal")
    ref = oracle.gemm(A, B, out_dtype=np.float16)
    tA, tB = to_dev(A, cuda), to_dev(B, cuda)
    per_thread = ctypes.c_void_p(2)  # cudaStreamPerThread
    errors = []

    def worker():
        try:
            torch.cuda.set_device(0)
            outs = [torch.empty((16, 4096), dtype=torch.float16, device=cuda) for _ in range(20)]
            torch.cuda.synchronize()
            for C in outs:
                d = pax_b200.make_desc(tA, tB, C, algo="skinny")
                st = pax_b200.lib.pax_gemm_ex(ctypes.byref(d), per_thread)
                if st != 0:
                    errors.append(st)
            torch.cuda.synchronize()
            for C in outs:
                check(C.cpu().numpy(), ref, np.float16)
        except Exception as e:  # reported below, on the main thread
            errors.append(e)

    ts = [threading.Thread(target=worker) for _ in range(2)]
    for t in ts:
        t.start()
    for t in ts:
        t.join()
    assert not errors, errors
    assert pax_b200.device_error() == pax_b200.Status.OK


def test_peer_barrier_on_one_gpu(cuda):
    """pax_peer_barrier with both ranks' flag arrays on this GPU: rank 0's
    barrier signals its epoch into the peer's array and passes once rank 1's
    slot of its own array holds that epoch or a later one."""
    own = torch.zeros(2, dtype=torch.int64, device=cuda)
    peer = torch.zeros(2, dtype=torch.int64, device=cuda)
    own[1] = 5  # rank 1 has already reached epoch 5
    torch.cuda.synchronize()
    for epoch in (3, 5):
        pax_b200.peer_barrier(own.data_ptr(), [peer.data_ptr()], 0, epoch, timeout_ns=1_000_000_000)
        torch.cuda.synchronize()
        assert peer.cpu().tolist() == [epoch, 0]
    assert own.cpu().tolist() == [0, 5]
    assert pax_b200.device_error() == pax_b200.Status.OK


def test_peer_barrier_times_out_without_the_peer(cuda):
    """A peer that never signals: the barrier's wait gives up after its
    limit, the timeout is reported once, and the device keeps working."""
    own = torch.zeros(2, dtype=torch.int64, device=cuda)
    peer = torch.zeros(2, dtype=torch.int64, device=cuda)
    torch.cuda.synchronize()
    pax_b200.peer_barrier(own.data_ptr(), [peer.data_ptr()], 0, 1, timeout_ns=2_000_000)
    torch.cuda.synchronize()
    assert peer.cpu().tolist() == [1, 0]
    assert pax_b200.device_error() == pax_b200.Status.TIMEOUT
    assert pax_b200.device_error() == pax_b200.Status.OK
    A = torch.randn((256, 128), device=cuda).half()
    B = torch.randn((128, 256), device=cuda).half()
    C = pax_b200.gemm(A, B)
    torch.cuda.synchronize()
    ref = (A.float() @ B.float()).half()
    assert torch.allclose(C.float(), ref.float(), rtol=2e-2, atol=2e-2)
