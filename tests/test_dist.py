"""Column-slab partitioning and the C all-gather, on CPU ranks (gloo,
world_size 2 and 4).  The per-slab GEMM is the oracle here; on GPUs it is the
library kernel (bench.py --gpus N)."""
from __future__ import annotations

import os
import queue
import socket
import time

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
from pax_b200.dist import equal_slabs, gather_columns, local_slab_gemm, slab_bounds


def test_slab_bounds_cover_all_columns():
    for n, w in [(32768, 8), (4096, 2), (1000, 4), (16, 4), (8200, 3)]:
        spans = [slab_bounds(n, w, r) for r in range(w)]
        assert spans[0][0] == 0 and spans[-1][1] == n
        for (a, b), (c, d) in zip(spans, spans[1:]):
            assert b == c and a <= b
        for a, b in spans[:-1]:
            assert a % 8 == 0 and b % 8 == 0
    assert equal_slabs(32768, 8) and not equal_slabs(1000, 3)


def _oracle_gemm(A, B, epilogue="none", bias=None, residual=None, out_dtype=torch.float16):
    a = A.numpy()
    b = np.ascontiguousarray(B.numpy())
    bi = None if bias is None else bias.numpy()
    r = None if residual is None else np.ascontiguousarray(residual.numpy())
    out = oracle.gemm(a, b, epi=epilogue, bias=bi, residual=r,
                      out_dtype=np.float16 if out_dtype == torch.float16 else np.float32, nthreads=1)
    return torch.from_numpy(out)


def _worker(rank, world, port, M, N, K, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        g = torch.Generator().manual_seed(7)  # identical full inputs on every rank
        A = (torch.rand((M, K), generator=g) * 2 - 1).half()
        B = (torch.rand((K, N), generator=g) * 2 - 1).half()
        bias = torch.randn((N,), generator=g).half()
        C_slab = local_slab_gemm(A, B, rank, world, epilogue="bias_gelu_tanh", bias=bias, gemm=_oracle_gemm)
        C = gather_columns(C_slab)
        if rank == 0:
            q.put(C.numpy())
    finally:
        dist.destroy_process_group()


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world", [2, 4])
def test_split_and_gather_equal_single_rank(world):
    M, N, K = 24, 64 * world, 40
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, M, N, K, q)) for r in range(world)]
    for p in procs:
        p.start()
    C = None
    deadline = time.time() + 180
    while C is None and time.time() < deadline:
        try:
            C = q.get(timeout=1)
        except queue.Empty:
            if any(p.exitcode not in (None, 0) for p in procs):
                break
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert C is not None, f"ranks failed: {[p.exitcode for p in procs]}"
    assert all(p.exitcode == 0 for p in procs)
    g = torch.Generator().manual_seed(7)
    A = (torch.rand((M, K), generator=g) * 2 - 1).half()
    B = (torch.rand((K, N), generator=g) * 2 - 1).half()
    bias = torch.randn((N,), generator=g).half()
    full = oracle.gemm(A.numpy(), B.numpy(), epi="bias_gelu_tanh", bias=bias.numpy(), out_dtype=np.float16)
    assert np.array_equal(C.view(np.uint16), full.view(np.uint16))


def _replicated_worker(rank, world, port, M, N, K, q):
    """ReplicatedC host logic with stand-ins for the IPC calls and the kernel:
    each rank's kernel call must get its own column slab as `out` and, as
    replicas, every peer's base address plus that slab's byte offset."""
    from pax_b200.dist import ReplicatedC

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        fake_base = lambda r: (r + 1) << 40  # noqa: E731
        calls = []

        def fake_gemm(A, B, *, epilogue, bias, residual, out, replicas):
            calls.append((B.shape, out.data_ptr() - rc.full.data_ptr(), out.shape, out.stride(), list(replicas)))
            out.copy_(_oracle_gemm(A, B, epilogue=epilogue, bias=bias, residual=residual))

        rc = ReplicatedC(M, N, device="cpu", _export=lambda t: str(dist.get_rank()).encode(),
                         _import=lambda h: fake_base(int(h.decode())), _close=lambda p: None)
        g = torch.Generator().manual_seed(7)
        A = (torch.rand((M, K), generator=g) * 2 - 1).half()
        B = (torch.rand((K, N), generator=g) * 2 - 1).half()
        bias = torch.randn((N,), generator=g).half()
        rc.gemm(A, B, "bias_gelu_tanh", bias=bias, gemm_fn=fake_gemm)
        rc.close()
        q.put((rank, calls, sorted(rc.peers.items()), rc.slab))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_replicated_c_host_logic(world):
    M, N, K = 16, 32 * world, 24
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_replicated_worker, args=(r, world, port, M, N, K, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = {}
    deadline = time.time() + 180
    while len(got) < world and time.time() < deadline:
        try:
            r, calls, peers, slab = q.get(timeout=1)
            got[r] = (calls, peers, slab)
        except queue.Empty:
            if any(p.exitcode not in (None, 0) for p in procs):
                break
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert len(got) == world, f"ranks failed: {[p.exitcode for p in procs]}"
    Ns = N // world
    for r, (calls, peers, slab) in got.items():
        assert slab == (r * Ns, (r + 1) * Ns)
        assert peers == []  # closed
        (bshape, out_off, out_shape, out_stride, replicas), = calls
        assert tuple(bshape) == (K, Ns)
        assert out_off == r * Ns * 2 and tuple(out_shape) == (M, Ns) and out_stride == (N, 1)  # bytes
        expect = [((p + 1) << 40) + r * Ns * 2 for p in range(world) if p != r]
        assert replicas == expect


def _flags_worker(rank, world, port, M, N, K, q):
    """ReplicatedC with flag ordering, with stand-ins for IPC and the
    barrier kernel: every call is bracketed by two barriers with growing
    epochs, each given this rank's flag array, the peers' mapped arrays in
    rank order and this rank as the slot; close unmaps C and flags."""
    from pax_b200.dist import ReplicatedC

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        events, closed = [], []

        def fake_gemm(A, B, *, epilogue, bias, residual, out, replicas):
            events.append(("gemm",))

        def fake_barrier(own, peers, slot, epoch, timeout_ns):
            events.append(("barrier", own == rc.sync.data_ptr(), list(peers), slot, epoch, timeout_ns))

        # The fake mapping puts rank r's C at (r + 1) << 40; its flags follow
        # C in the same allocation.
        rc = ReplicatedC(M, N, device="cpu", ordering="flags", barrier_timeout_ns=5_000_000,
                         _export=lambda t: str(dist.get_rank()).encode(),
                         _import=lambda h: (int(h.decode()) + 1) << 40, _close=closed.append, _barrier=fake_barrier)
        assert rc.sync_offset % 256 == 0 and rc.sync_offset >= M * N * 2
        assert rc.sync.data_ptr() - rc.full.data_ptr() == rc.sync_offset and rc.sync.tolist() == [0] * world
        A = torch.zeros((M, K), dtype=torch.float16)
        B = torch.zeros((K, N), dtype=torch.float16)
        for _ in range(2):
            rc.gemm(A, B, gemm_fn=fake_gemm)
        off = rc.sync_offset
        rc.close()
        q.put((rank, events, sorted(closed), off))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_replicated_c_flag_ordering_host_logic(world):
    M, N, K = 8, 16 * world, 16
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_flags_worker, args=(r, world, port, M, N, K, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = {}
    deadline = time.time() + 180
    while len(got) < world and time.time() < deadline:
        try:
            r, events, closed, off = q.get(timeout=1)
            got[r] = (events, closed, off)
        except queue.Empty:
            if any(p.exitcode not in (None, 0) for p in procs):
                break
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert len(got) == world, f"ranks failed: {[p.exitcode for p in procs]}"
    for r, (events, closed, off) in got.items():
        peer_flags = [((p + 1) << 40) + off for p in range(world) if p != r]
        kinds = [e[0] for e in events]
        assert kinds == ["barrier", "gemm", "barrier"] * 2
        barriers = [e for e in events if e[0] == "barrier"]
        assert [b[4] for b in barriers] == [1, 2, 3, 4]  # epochs grow, the same on every rank
        for _, own_ok, peers, slot, _, timeout_ns in barriers:
            assert own_ok and peers == peer_flags and slot == r and timeout_ns == 5_000_000
        assert closed == [(p + 1) << 40 for p in range(world) if p != r]  # one mapping per peer


def test_replicated_c_rejects_unknown_ordering():
    from pax_b200.dist import ReplicatedC

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(_free_port())
    dist.init_process_group("gloo", rank=0, world_size=1)
    try:
        with pytest.raises(ValueError, match="ordering"):
            ReplicatedC(8, 16, device="cpu", ordering="nccl", _export=lambda t: b"h", _import=lambda h: 1 << 40,
                        _close=lambda p: None)
    finally:
        dist.destroy_process_group()
