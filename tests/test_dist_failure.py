"""Failure detection for the multi-rank path, on CPU ranks (gloo).

Every failure is made on the host: a rank that leaves between steps, a rank
that exits without a word, a rank that never starts.  The surviving ranks
must end with an error within a bound instead of waiting forever:

  * PeerMonitor.step() raises RankFailure before the next launch when a peer
    has left (at once) or has stopped publishing steps (after its timeout);
  * ReplicatedC with a monitor raises before its first collective;
  * without a monitor, the collective itself ends with an error (the peer's
    connection closes), and a rank that never joins ends the process group's
    set-up after its timeout.

Ranks wait for the parent's release before they exit, so the rank that hosts
the store outlives every other rank's last store access.
"""
from __future__ import annotations

import os
import queue
import socket
import time
from datetime import timedelta

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from pax_b200.dist import PeerMonitor, RankFailure


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port, timeout_s=30):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=timeout_s))


def _run(target, world, n_started=None, extra=(), budget=90.0):
    """Start `n_started` of `world` ranks, collect one result per started
    rank (or per rank that reports), release them, and return the results."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    release = ctx.Event()
    port = _free_port()
    n = world if n_started is None else n_started
    procs = [ctx.Process(target=target, args=(r, world, port, q, release, *extra)) for r in range(n)]
    for p in procs:
        p.start()
    got = {}
    deadline = time.time() + budget
    while time.time() < deadline:
        try:
            r, res = q.get(timeout=0.5)
            got[r] = res
        except queue.Empty:
            pass
        # done when every rank has reported or exited
        if all(r in got or p.exitcode is not None for r, p in enumerate(procs)) and q.empty():
            break
    release.set()
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
            p.join(timeout=10)
    return got, [p.exitcode for p in procs]


# ---------------------------------------------------------------- leave
def _leave_worker(rank, world, port, q, release, leaver, steps):
    _init(rank, world, port)
    mon = PeerMonitor(timeout=20.0)
    t = torch.ones(4)
    for _ in range(steps):
        mon.step()
        dist.all_reduce(t)
    if rank == leaver:
        mon.leave("test")
        q.put((rank, ("left", None, None, 0.0)))
    else:
        t0 = time.monotonic()
        try:
            mon.step()
            q.put((rank, ("no error", None, None, time.monotonic() - t0)))
        except RankFailure as e:
            q.put((rank, ("failure", e.rank, e.reason, time.monotonic() - t0)))
    release.wait(60)


@pytest.mark.parametrize("world,leaver", [(2, 1), (3, 2), (3, 0)])
def test_rank_leaving_between_steps_is_seen_before_the_next_launch(world, leaver):
    got, codes = _run(_leave_worker, world, extra=(leaver, 3))
    assert len(got) == world, (got, codes)
    for r, (kind, who, reason, dt) in got.items():
        if r == leaver:
            assert kind == "left"
            continue
        assert kind == "failure", got
        assert who == leaver and "left" in reason and "step 3" in reason
        assert dt < 5.0  # at once, not after the 20 s timeout
    assert all(c == 0 for c in codes), codes


# ---------------------------------------------------------------- crash
def _crash_worker(rank, world, port, q, release, victim, timeout):
    _init(rank, world, port)
    mon = PeerMonitor(timeout=timeout)
    t = torch.ones(4)
    for _ in range(2):
        mon.step()
        dist.all_reduce(t)
    if rank == victim:
        os._exit(0)  # no leave(): the peers see only that its steps stop
    t0 = time.monotonic()
    try:
        mon.step()
        q.put((rank, ("no error", None, None, time.monotonic() - t0)))
    except RankFailure as e:
        q.put((rank, ("failure", e.rank, e.reason, time.monotonic() - t0)))
    release.wait(60)


def test_rank_that_stops_is_reported_after_the_monitor_timeout():
    world, victim, timeout = 3, 2, 1.5
    got, codes = _run(_crash_worker, world, extra=(victim, timeout))
    assert set(got) == {0, 1}, (got, codes)
    for r, (kind, who, reason, dt) in got.items():
        assert kind == "failure", got
        assert who == victim and "stopped responding" in reason and "last step 1" in reason
        assert timeout <= dt < timeout + 5.0


# ------------------------------------------- ReplicatedC with a monitor
def _replicated_leave_worker(rank, world, port, q, release):
    from pax_b200.dist import ReplicatedC

    _init(rank, world, port)
    mon = PeerMonitor(timeout=20.0)
    calls = []

    def fake_gemm(A, B, *, epilogue, bias, residual, out, replicas):
        calls.append(out.shape)

    rc = ReplicatedC(8, 16 * world, device="cpu", monitor=mon, _export=lambda t: b"h",
                     _import=lambda h: 1 << 40, _close=lambda p: None)
    A = torch.zeros((8, 8), dtype=torch.float16)
    B = torch.zeros((8, 16 * world), dtype=torch.float16)
    rc.gemm(A, B, gemm_fn=fake_gemm)
    if rank == world - 1:
        mon.leave("done early")
        q.put((rank, ("left", len(calls))))
    else:
        try:
            rc.gemm(A, B, gemm_fn=fake_gemm)
            q.put((rank, ("no error", len(calls))))
        except RankFailure as e:
            q.put((rank, ("failure", len(calls), e.rank)))
    rc.close()
    release.wait(60)


def test_replicated_c_raises_before_its_collective_when_a_peer_left():
    world = 3
    got, codes = _run(_replicated_leave_worker, world)
    assert len(got) == world, (got, codes)
    for r, res in got.items():
        if r == world - 1:
            assert res == ("left", 1)
        else:
            # one finished call; the second raised before launching anything
            assert res == ("failure", 1, world - 1), got
    assert all(c == 0 for c in codes), codes


# ------------------------------------------------ without a monitor
def _collective_worker(rank, world, port, q, release):
    _init(rank, world, port, timeout_s=5)
    t = torch.ones(4)
    dist.all_reduce(t)
    if rank == 1:
        os._exit(0)
    time.sleep(0.3)
    t0 = time.monotonic()
    try:
        dist.all_reduce(t)
        q.put((rank, ("no error", time.monotonic() - t0)))
    except RuntimeError as e:
        q.put((rank, ("error", time.monotonic() - t0, str(e)[:120])))
    release.wait(60)


def test_collective_with_a_departed_peer_ends_with_an_error():
    got, codes = _run(_collective_worker, 2)
    assert set(got) == {0}, (got, codes)
    kind, dt = got[0][0], got[0][1]
    assert kind == "error", got
    assert dt < 10.0  # bounded by the 5 s process-group timeout at most


def _never_joined_worker(rank, world, port, q, release):
    t0 = time.monotonic()
    try:
        _init(rank, world, port, timeout_s=2)
        q.put((rank, ("joined", time.monotonic() - t0)))
    except Exception as e:  # the store's set-up timeout (DistStoreError)
        q.put((rank, ("timeout", time.monotonic() - t0, type(e).__name__)))
    release.wait(60)


def test_rank_that_never_joins_ends_set_up_with_an_error():
    got, codes = _run(_never_joined_worker, 2, n_started=1)
    assert set(got) == {0}, (got, codes)
    kind, dt = got[0][0], got[0][1]
    assert kind == "timeout", got
    assert 1.5 <= dt < 15.0
