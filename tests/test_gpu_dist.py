"""Column-slab GEMM on 2 GPUs (NCCL, one process per GPU): each rank runs the
library kernel on its slab of B and C, the slabs are all-gathered, and the
replicated C must match the oracle on every rank."""
from __future__ import annotations

import os
import queue
import socket
import time

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, M, N, K, q):
    import torch.distributed as dist
    from datetime import timedelta

    import pax_b200
    from pax_b200.dist import ReplicatedC, gather_columns, local_slab_gemm

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60), device_id=dev)
    try:
        g = torch.Generator().manual_seed(11)  # identical full inputs on every rank
        A = (torch.rand((M, K), generator=g) * 2 - 1).half()
        B = (torch.rand((K, N), generator=g) * 2 - 1).half()
        bias = torch.randn((N,), generator=g).half()
        C_slab = local_slab_gemm(A.to(dev), B.to(dev), rank, world, epilogue="bias_gelu_tanh", bias=bias.to(dev))
        C = gather_columns(C_slab)
        # Fused: each rank's kernel also copies its slab into the peer's C,
        # ordered by peer flag barriers, then by NCCL all-reduces.
        fused = []
        for ordering in ("flags", "collective"):
            rc = ReplicatedC(M, N, device=dev, ordering=ordering, barrier_timeout_ns=20_000_000_000)
            for _ in range(3):  # later calls overwrite the same buffers
                rc.full.zero_()
                fused.append(rc.gemm(A.to(dev), B.to(dev), "bias_gelu_tanh", bias=bias.to(dev)).cpu().numpy())
            torch.cuda.synchronize()
            dist.barrier()
            rc.close()
        q.put((rank, C.cpu().numpy(), int(pax_b200.device_error()), fused))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_two_gpu_slabs_and_gather(cuda):
    import oracle

    world, M, N, K = 2, 512, 2048, 768
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, world, port, M, N, K, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = {}
    deadline = time.time() + 240
    while len(got) < world and time.time() < deadline:
        try:
            r, C, err, fused = q.get(timeout=1)
            got[r] = (C, err, fused)
        except queue.Empty:
            if any(p.exitcode not in (None, 0) for p in procs):
                break
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert len(got) == world, f"ranks failed: {[p.exitcode for p in procs]}"
    g = torch.Generator().manual_seed(11)
    A = (torch.rand((M, K), generator=g) * 2 - 1).half().numpy()
    B = (torch.rand((K, N), generator=g) * 2 - 1).half().numpy()
    bias = torch.randn((N,), generator=g).half().numpy()
    ref = oracle.gemm(A, B, epi="bias_gelu_tanh", bias=bias, out_dtype=np.float16)
    for r, (C, err, fused) in got.items():
        assert err == 0
        assert oracle.normwise_error(C, ref) <= 2e-3
        for F in fused:  # the fused all-gather delivers the same bits as NCCL
            assert np.array_equal(F.view(np.uint16), C.view(np.uint16))
    assert np.array_equal(got[0][0].view(np.uint16), got[1][0].view(np.uint16))
