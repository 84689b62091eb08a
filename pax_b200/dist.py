"""Multi-GPU GEMM by column slabs (one process per GPU).

The product C = epi(A . B) has independent output columns, so P ranks split
B, bias and C along N: rank p owns columns [p*Ns, (p+1)*Ns), holds all of A
and computes its slab with the single-GPU kernels, with no communication.
When the caller wants C replicated on every rank, `ReplicatedC` fuses the
all-gather into the GEMM: each rank's kernel also stores its tiles straight
into the peers' C over NVLink.  `gather_columns` is the unfused baseline:
one NCCL all-gather of the contiguous slabs into a [P][M][Ns] staging buffer,
packed into row-major M x N.  The reference has no multi-GPU code; this is
the partitioning its large benchmark configuration (32768^3 over 1 to 8
GPUs, B and C split along N) calls for.
"""
from __future__ import annotations

import time
from typing import Callable

import torch
import torch.distributed as dist


def slab_bounds(n_total: int, world: int, rank: int, align: int = 8) -> tuple[int, int]:
    """Column range [start, stop) of `rank`: equal slabs of a multiple of
    `align` columns (16-byte fp16 rows for the TMA kernels); the last slab
    takes the remainder."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("bad rank/world")
    per = (n_total // world) // align * align
    if per == 0:
        per = align
    start = min(rank * per, n_total)
    stop = n_total if rank == world - 1 else min(start + per, n_total)
    return start, stop


def equal_slabs(n_total: int, world: int, align: int = 8) -> bool:
    """True when every slab has the same width (what all_gather needs)."""
    return n_total % world == 0 and (n_total // world) % align == 0


def local_slab_gemm(A: torch.Tensor, B: torch.Tensor, rank: int, world: int, epilogue: str = "none",
                    bias: torch.Tensor | None = None, residual: torch.Tensor | None = None,
                    out_dtype: torch.dtype = torch.float16,
                    gemm: Callable | None = None) -> torch.Tensor:
    """This rank's slab C[:, s:e] = epi(A . B[:, s:e]) from the full-width B
    (and bias/residual).  `gemm` defaults to pax_b200.gemm; tests pass a
    CPU stand-in."""
    if gemm is None:
        from .api import gemm as _g

        gemm = _g
    s, e = slab_bounds(B.shape[1], world, rank)
    Bs = B[:, s:e]
    bs = bias[s:e] if bias is not None else None
    rs = residual[:, s:e] if residual is not None else None
    return gemm(A, Bs, epilogue=epilogue, bias=bs, residual=rs, out_dtype=out_dtype)


def gather_columns(C_slab: torch.Tensor, group=None) -> torch.Tensor:
    """All-gather equal-width column slabs of every rank into the full
    row-major C (M x P*Ns) on every rank."""
    world = dist.get_world_size(group)
    M, Ns = C_slab.shape
    staging = C_slab.new_empty((world * M, Ns))  # rank-major stack of slabs
    dist.all_gather_into_tensor(staging, C_slab.contiguous(), group=group)
    return staging.view(world, M, Ns).permute(1, 0, 2).reshape(M, world * Ns)


class ReplicatedC:
    """C [M, N_total] replicated on every rank, filled by one fused kernel per
    rank instead of a GEMM followed by an all-gather.

    Every rank allocates the full C and maps the other ranks' C buffers
    (CUDA IPC, pax_ipc_export / pax_ipc_import).  `gemm` computes this rank's
    column slab with pax_gemm_replicated_ex: the epilogue stores each finished
    tile into the local C and, over NVLink, into the same place of every
    peer's C while the kernel goes on with later tiles.  Stores only: no
    kernel reads another GPU's memory.

    Ordering: a rank barrier before the kernel (every rank has finished
    reading the previous contents) and one after it (every rank's slab has
    landed everywhere) bracket each call, on the current stream.  With
    ``ordering="flags"`` (the default for CUDA buffers) each barrier is
    pax_peer_barrier: one small kernel that release-stores an epoch into the
    peers' flag arrays over NVLink and waits, bounded, for theirs.  With
    ``ordering="collective"`` (the default elsewhere) it is a one-element
    all-reduce of the process group.

    With a `monitor` (a PeerMonitor), each call first checks on the host
    that every peer is alive and at the same step, and raises RankFailure
    before the first barrier if one has left or stopped responding.

    `_export`, `_import`, `_close`, `_barrier` and `gemm_fn` exist so that
    the host logic can be tested without GPUs.
    """

    def __init__(self, M: int, N_total: int, dtype: torch.dtype = torch.float16, device=None, group=None, *,
                 monitor: PeerMonitor | None = None, ordering: str | None = None, barrier_timeout_ns: int = 0,
                 _export: Callable | None = None, _import: Callable | None = None, _close: Callable | None = None,
                 _barrier: Callable | None = None):
        from . import api

        self.group = group
        self.monitor = monitor
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if not equal_slabs(N_total, self.world):
            raise ValueError("replicated C needs N_total divisible by 8 * ranks")
        if ordering is None:
            ordering = "flags" if torch.device(device if device is not None else "cpu").type == "cuda" else \
                "collective"
        if ordering not in ("flags", "collective"):
            raise ValueError(f"ordering must be 'flags' or 'collective', not {ordering!r}")
        self.ordering = ordering
        self.barrier_timeout_ns = int(barrier_timeout_ns)
        # One allocation holds C and, after it, this rank's barrier flags (one
        # 64-bit slot per rank), so a peer maps both with one IPC handle.  The
        # flags are zero before any peer can see them: the fill completes
        # before the handles are exchanged.
        c_bytes = M * N_total * torch.empty((), dtype=dtype).element_size()
        self.sync_offset = (c_bytes + 255) // 256 * 256
        buf = torch.empty(self.sync_offset + 8 * self.world, dtype=torch.uint8, device=device)
        self.full = buf[:c_bytes].view(dtype).view(M, N_total)
        self.sync = buf[self.sync_offset:].view(torch.int64)
        self.sync.zero_()
        if self.sync.is_cuda:
            torch.cuda.current_stream(self.sync.device).synchronize()
        self._epoch = 0
        self._close = _close or api.ipc_close
        self._barrier_fn = _barrier or api.peer_barrier
        mine = (_export or api.ipc_export)(self.full)
        handles: list = [None] * self.world
        dist.all_gather_object(handles, mine, group=group)
        imp = _import or api.ipc_import
        self.peers = {r: imp(h) for r, h in enumerate(handles) if r != self.rank}
        self.slab = slab_bounds(N_total, self.world, self.rank)
        self._flag = torch.zeros(1, dtype=torch.float32, device=device)

    def replica_addresses(self) -> list[int]:
        """Where this rank's slab goes in every peer's C (same offset as here)."""
        off = self.slab[0] * self.full.element_size()
        return [base + off for _, base in sorted(self.peers.items())]

    def gemm(self, A: torch.Tensor, B: torch.Tensor, epilogue: str = "none", bias: torch.Tensor | None = None,
             residual: torch.Tensor | None = None, gemm_fn: Callable | None = None) -> torch.Tensor:
        """full = epi(A . B) on every rank, from the full-width B (and bias /
        residual); this rank computes its column slab."""
        s, e = self.slab
        return self.gemm_slab(A, B[:, s:e], epilogue, bias[s:e] if bias is not None else None,
                              residual[:, s:e] if residual is not None else None, gemm_fn)

    def gemm_slab(self, A: torch.Tensor, B_slab: torch.Tensor, epilogue: str = "none",
                  bias_slab: torch.Tensor | None = None, residual_slab: torch.Tensor | None = None,
                  gemm_fn: Callable | None = None) -> torch.Tensor:
        """As `gemm`, from this rank's slabs of B, bias and residual only."""
        if gemm_fn is None:
            from .api import gemm as gemm_fn
        s, e = self.slab
        if self.monitor is not None:
            self.monitor.step()
        self.barrier()
        gemm_fn(A, B_slab, epilogue=epilogue, bias=bias_slab, residual=residual_slab, out=self.full[:, s:e],
                replicas=self.replica_addresses())
        self.barrier()
        return self.full

    def barrier(self) -> None:
        """Every rank's work queued on its current stream before this point
        is complete before anything queued after it runs (on every rank)."""
        if self.ordering == "collective":
            dist.all_reduce(self._flag, group=self.group)
            return
        self._epoch += 1
        peers = [base + self.sync_offset for _, base in sorted(self.peers.items())]
        self._barrier_fn(self.sync.data_ptr(), peers, self.rank, self._epoch, self.barrier_timeout_ns)

    def close(self) -> None:
        for ptr in self.peers.values():
            self._close(ptr)
        self.peers = {}


class RankFailure(RuntimeError):
    """A peer rank left the job or stopped making progress.

    Raised on the host by `PeerMonitor.step` before this rank's next launch,
    so none of this rank's kernels or collectives is left waiting on the
    missing peer."""

    def __init__(self, rank: int, reason: str):
        super().__init__(f"rank {rank} {reason}")
        self.rank = rank
        self.reason = reason


class PeerMonitor:
    """Host-side failure detection between steps, through the c10d store.

    Ranks of a slab-partitioned job run the same steps in the same order,
    and a step with a collective (the all-gather of C, or the barriers of
    `ReplicatedC`) cannot finish while a peer is missing.
    Before each step's launches every rank calls `step()`:

    * it publishes its own step number under ``<name>/step/<rank>``;
    * it waits until every peer has published the same step number, i.e.
      every peer is alive and about to launch the same step;
    * a peer that called `leave()` (a rank leaving between steps) raises
      `RankFailure(peer, "left ...")` at once;
    * a peer that has not arrived after `timeout` seconds (a rank that
      crashed, hangs on the host or never started) raises
      `RankFailure(peer, "stopped responding ...")`.

    The check costs one store round trip per peer per step (tens of
    microseconds each on one node), so it suits steps of a millisecond or
    more.  It does not replace the process group's own timeout, which still
    bounds a collective whose peer dies inside the step.
    """

    def __init__(self, timeout: float = 30.0, name: str = "pax_monitor", store=None, group=None,
                 poll: float = 0.001):
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.timeout = float(timeout)
        self.poll = float(poll)
        self.name = name
        self._store = store if store is not None else dist.distributed_c10d._get_default_store()
        self._step = 0

    def _key(self, kind: str, rank: int) -> str:
        return f"{self.name}/{kind}/{rank}"

    def step(self) -> int:
        """Announce this rank's next step and wait for every peer to reach it.
        Returns the step number (0 for the first call)."""
        s = self._step
        self._store.set(self._key("step", self.rank), str(s))
        pending = [p for p in range(self.world) if p != self.rank]
        last = {p: -1 for p in pending}
        deadline = time.monotonic() + self.timeout
        wait = self.poll
        while pending:
            still = []
            for p in pending:
                if self._store.check([self._key("left", p)]):
                    why = self._store.get(self._key("left", p)).decode()
                    raise RankFailure(p, f"left the job ({why}) before step {s}")
                if self._store.check([self._key("step", p)]):
                    last[p] = int(self._store.get(self._key("step", p)))
                if last[p] < s:
                    still.append(p)
            pending = still
            if not pending:
                break
            if time.monotonic() > deadline:
                p = pending[0]
                raise RankFailure(p, f"stopped responding: last step {last[p]}, waited {self.timeout:.1f} s "
                                     f"at step {s}")
            time.sleep(wait)
            wait = min(wait * 2, 0.05)
        self._step = s + 1
        return s

    def leave(self, reason: str = "shutdown") -> None:
        """Tell the peers, between steps, that this rank will launch nothing
        more.  Their next `step()` raises RankFailure instead of waiting."""
        self._store.set(self._key("left", self.rank), reason)
