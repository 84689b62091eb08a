"""Multi-GPU GEMM by column slabs (one process per GPU).

The product C = epi(A . B) has independent output columns, so P ranks split
B, bias and C along N: rank p owns columns [p*Ns, (p+1)*Ns), holds all of A
and computes its slab with the single-GPU kernels, with no communication.
When the caller wants C replicated on every rank, `gather_columns` runs one
NCCL all-gather of the contiguous slabs into a [P][M][Ns] staging buffer and
packs it into row-major M x N.  The reference has no multi-GPU code; this is
the partitioning BASELINE's configuration 5 asks for.
"""
from __future__ import annotations

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
