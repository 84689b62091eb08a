"""pax_b200 -- FP16 GEMM with fused Bias / GeLU / residual epilogues for
NVIDIA B200 (sm_100a), behind the C ABI of PAX's host bridge (include/pax.h).

Kernels: a persistent warp-specialised tcgen05 GEMM (TMA, mbarrier ring,
TMEM accumulators), a swap-AB stream-K variant for small M, and a CUDA-core
kernel for problems that are not 16-byte aligned.  libpax_b200.so is loaded
on first use (``pax_b200.lib`` or any call) and its absence raises
LibraryNotBuilt; there is no CPU fallback.
"""
from . import _lib
from ._lib import LIB_PATH, GemmDesc, LibraryNotBuilt, PaxBuffer
from .api import (Algo, DType, Epilogue, PaxError, Status, device_error, gemm, gemm_batched, ipc_close, ipc_export,
                  ipc_import, last_error, make_desc, peer_barrier, pipeline_stages, select_algo)

__all__ = [
    "LIB_PATH", "GemmDesc", "LibraryNotBuilt", "PaxBuffer", "lib", "Algo", "DType", "Epilogue", "PaxError",
    "Status", "device_error", "gemm", "gemm_batched", "ipc_close", "ipc_export", "ipc_import", "last_error",
    "make_desc", "peer_barrier", "pipeline_stages", "select_algo",
]


def __getattr__(name):
    if name == "lib":
        return _lib.get()
    raise AttributeError(name)
