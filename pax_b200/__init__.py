"""pax_b200 -- FP16 GEMM with fused Bias / GeLU / residual epilogues for
NVIDIA B200 (sm_100a), behind the C ABI of PAX's host bridge (include/pax.h).

Kernels: a persistent warp-specialised tcgen05 GEMM (TMA, mbarrier ring,
TMEM accumulators), a swap-AB stream-K variant for small M, and a CUDA-core
kernel for problems that are not 16-byte aligned.  Importing the package
loads libpax_b200.so and fails if it has not been built; there is no CPU
fallback.
"""
from ._lib import LIB_PATH, GemmDesc, LibraryNotBuilt, PaxBuffer, lib
from .api import Algo, DType, Epilogue, PaxError, Status, device_error, gemm, last_error, make_desc, select_algo

__all__ = [
    "LIB_PATH", "GemmDesc", "LibraryNotBuilt", "PaxBuffer", "lib", "Algo", "DType", "Epilogue", "PaxError",
    "Status", "device_error", "gemm", "last_error", "make_desc", "select_algo",
]
