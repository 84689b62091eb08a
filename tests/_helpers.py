"""Helpers shared by the GPU tests: run the library on numpy inputs and
compare with the oracle under the north-star tolerance."""
from __future__ import annotations

import numpy as np
import torch

import oracle
import pax_b200

# North-star parity bound: max|C - C_ref| <= 1e-2 * max|C_ref| for K <= 32768.
NORTH_STAR = 1e-2
# Tighter bounds that catch dropped k-blocks or mis-mapped tiles well below
# fp16 output carries <= 2^-11 relative rounding.
TIGHT = {np.float16: 2e-3, np.float32: 1e-4}


def to_dev(a: np.ndarray | None, dev) -> torch.Tensor | None:
    if a is None:
        return None
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def run_gemm(A, B, dev, epi="none", out_dtype=np.float16, bias=None, residual=None, alpha=1.0, algo="auto"):
    tA, tB = to_dev(A, dev), to_dev(B, dev)
    td = torch.float16 if out_dtype == np.float16 else torch.float32
    C = pax_b200.gemm(tA, tB, epilogue=epi, bias=to_dev(bias, dev), residual=to_dev(residual, dev), alpha=alpha,
                      out_dtype=td, algo=algo)
    torch.cuda.synchronize()
    return C.cpu().numpy()


def check(got: np.ndarray, ref: np.ndarray, out_dtype) -> float:
    nw = oracle.normwise_error(got, ref)
    assert np.isfinite(got).all(), "non-finite output"
    assert nw <= NORTH_STAR, f"normwise error {nw:.3e} above the north-star bound"
    assert nw <= TIGHT[out_dtype], f"normwise error {nw:.3e} above {TIGHT[out_dtype]:.0e}"
    return nw


def inputs(rng, M, N, K, dist="uniform"):
    if dist == "uniform":
        A = rng.uniform(-1, 1, (M, K)).astype(np.float16)
        B = rng.uniform(-1, 1, (K, N)).astype(np.float16)
    else:
        A = rng.standard_normal((M, K)).astype(np.float16)
        B = (rng.standard_normal((K, N)) * 0.02).astype(np.float16)
    return A, B
