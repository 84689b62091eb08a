"""Tensor-level front end of the C ABI: ``gemm(A, B, ...)`` on torch CUDA
tensors.  torch supplies device memory and the stream; every FLOP runs in
libpax_b200.so (pax_gemm_ex)."""
from __future__ import annotations

import ctypes
from enum import IntEnum

import torch

from . import _lib
from ._lib import GemmDesc


class Status(IntEnum):
    OK = 0
    INVALID = 1
    UNSUPPORTED = 2
    CUDA = 3
    TIMEOUT = 4
    NO_DEVICE = 5
    ALLOC = 6


class Epilogue(IntEnum):
    NONE = 0
    BIAS = 1
    BIAS_GELU_TANH = 2
    BIAS_GELU_ERF = 3
    RESIDUAL_GELU_TANH = 4
    RESIDUAL_GELU_ERF = 5
    GELU_TANH = 6
    GELU_ERF = 7
    RESIDUAL = 8


class DType(IntEnum):
    F32 = 0
    F16 = 1


class Algo(IntEnum):
    AUTO = 0
    TC = 1
    TC2 = 2
    SKINNY = 3
    SIMT = 4


PAX_GEMM_B_CONST = 0x100  # hint bit of pax_gemm_desc_t.algo (include/pax.h)


class PaxError(RuntimeError):
    def __init__(self, status: int, what: str = ""):
        self.status = Status(status)
        msg = _lib.get().pax_status_string(int(status)).decode()
        super().__init__(f"{what}: {msg} ({self.status.name})" if what else msg)


_EPI_NAMES = {e.name.lower(): e for e in Epilogue}
_DT = {torch.float32: DType.F32, torch.float16: DType.F16}


def _row_major_ld(t: torch.Tensor, name: str) -> int:
    if t.dim() != 2 or t.stride(1) != 1:
        raise ValueError(f"{name} must be a 2-D tensor with unit column stride")
    return t.stride(0)


def make_desc(A: torch.Tensor, B: torch.Tensor, C: torch.Tensor, epilogue="none", bias=None, residual=None,
              alpha: float = 1.0, algo="auto") -> GemmDesc:
    epi = _EPI_NAMES[epilogue] if isinstance(epilogue, str) else Epilogue(epilogue)
    al = Algo[algo.upper()] if isinstance(algo, str) else Algo(algo)
    if A.dtype != torch.float16 or B.dtype != torch.float16:
        raise TypeError("A and B must be float16")
    if C.dtype not in _DT:
        raise TypeError("C must be float32 or float16")
    M, K = A.shape
    K2, N = B.shape
    if K2 != K or tuple(C.shape) != (M, N):
        raise ValueError(f"shape mismatch: A {tuple(A.shape)} B {tuple(B.shape)} C {tuple(C.shape)}")
    d = GemmDesc()
    d.A, d.B, d.C = A.data_ptr(), B.data_ptr(), C.data_ptr()
    d.M, d.N, d.K = M, N, K
    d.lda = _row_major_ld(A, "A") if A.numel() else 0
    d.ldb = _row_major_ld(B, "B") if B.numel() else 0
    d.ldc = _row_major_ld(C, "C") if C.numel() else 0
    d.c_dtype = int(_DT[C.dtype])
    d.epilogue = int(epi)
    d.alpha = float(alpha)
    if bias is not None:
        if bias.dtype != torch.float16 or bias.numel() != N:
            raise ValueError("bias must be float16 with N elements")
        d.bias = bias.data_ptr()
    if residual is not None:
        if residual.dtype not in _DT or tuple(residual.shape) != (M, N):
            raise ValueError("residual must be float32/float16 of shape (M, N)")
        d.residual = residual.data_ptr()
        d.residual_dtype = int(_DT[residual.dtype])
        d.ld_res = _row_major_ld(residual, "residual")
    d.algo = int(al)
    return d


def gemm(A: torch.Tensor, B: torch.Tensor, *, epilogue="none", bias=None, residual=None, alpha: float = 1.0,
         out: torch.Tensor | None = None, out_dtype: torch.dtype = torch.float16, algo="auto",
         stream: torch.cuda.Stream | None = None, replicas: list[int] | None = None,
         b_const: bool = False) -> torch.Tensor:
    """C = epilogue(alpha * A @ B) on the current (or given) CUDA stream.

    A [M, K] and B [K, N] are float16 row-major CUDA tensors; C is float16 or
    float32.  epilogue is one of none, bias, bias_gelu_tanh, bias_gelu_erf,
    residual_gelu_tanh, residual_gelu_erf, gelu_tanh, gelu_erf, residual.
    replicas: device addresses of further buffers with out's shape and pitch
    (usually other GPUs' memory, see pax_b200.dist.ReplicatedC) that the same
    kernel also writes C to.
    b_const: B is not written by the kernel launched just before on this
    stream (weights); the skinny kernel may then start reading B before that
    kernel ends (PAX_GEMM_B_CONST).
    """
    if out is None:
        out = torch.empty((A.shape[0], B.shape[1]), dtype=out_dtype, device=A.device)
    d = make_desc(A, B, out, epilogue, bias, residual, alpha, algo)
    if b_const:
        d.algo |= PAX_GEMM_B_CONST
    s = stream if stream is not None else torch.cuda.current_stream(A.device)
    if replicas:
        arr = (ctypes.c_void_p * len(replicas))(*replicas)
        st = _lib.get().pax_gemm_replicated_ex(ctypes.byref(d), arr, len(replicas), ctypes.c_void_p(s.cuda_stream))
        if st != 0:
            raise PaxError(st, "pax_gemm_replicated_ex")
        return out
    st = _lib.get().pax_gemm_ex(ctypes.byref(d), ctypes.c_void_p(s.cuda_stream))
    if st != 0:
        raise PaxError(st, "pax_gemm_ex")
    return out


def _batch_view(t: torch.Tensor | None, ndim_item: int, name: str):
    """(item-0 view, element stride between items) of a batched operand;
    an operand without the batch dimension is shared (stride 0)."""
    if t is None:
        return None, 0
    if t.dim() == ndim_item:
        return t, 0
    if t.dim() != ndim_item + 1:
        raise ValueError(f"{name} must have {ndim_item} or {ndim_item + 1} dimensions")
    return t[0], t.stride(0)


def gemm_batched(A: torch.Tensor, B: torch.Tensor, *, epilogue="none", bias=None, residual=None,
                 alpha: float = 1.0, out: torch.Tensor | None = None, out_dtype: torch.dtype = torch.float16,
                 algo="auto", stream: torch.cuda.Stream | None = None) -> torch.Tensor:
    """C[b] = epilogue(alpha * A[b] @ B[b]) for every batch item b, through
    pax_gemm_batched_ex.  A is [batch, M, K] or a shared [M, K]; B is
    [batch, K, N] or a shared [K, N]; bias [batch, N] or [N]; residual
    [batch, M, N] or [M, N].  C is [batch, M, N]."""
    nb = max(A.shape[0] if A.dim() == 3 else 1, B.shape[0] if B.dim() == 3 else 1)
    for t, d, name in ((A, 3, "A"), (B, 3, "B"), (bias, 2, "bias"), (residual, 3, "residual")):
        if t is not None and t.dim() == d and t.shape[0] != nb:
            raise ValueError(f"{name} has batch {t.shape[0]}, expected {nb}")
    A0, sa = _batch_view(A, 2, "A")
    B0, sb = _batch_view(B, 2, "B")
    b0, sbias = _batch_view(bias, 1, "bias")
    r0, sres = _batch_view(residual, 2, "residual")
    M, N = A0.shape[0], B0.shape[1]
    if out is None:
        out = torch.empty((nb, M, N), dtype=out_dtype, device=A.device)
    if out.dim() != 3 or out.shape[0] != nb:
        raise ValueError("out must be [batch, M, N]")
    d = _lib.GemmBatchedDesc()
    d.gemm = make_desc(A0, B0, out[0], epilogue, b0, r0, alpha, algo)
    d.batch = nb
    d.stride_a, d.stride_b, d.stride_c = sa, sb, out.stride(0)
    d.stride_bias, d.stride_residual = sbias, sres
    s = stream if stream is not None else torch.cuda.current_stream(A.device)
    st = _lib.get().pax_gemm_batched_ex(ctypes.byref(d), ctypes.c_void_p(s.cuda_stream))
    if st != 0:
        raise PaxError(st, "pax_gemm_batched_ex")
    return out


def select_algo(A: torch.Tensor, B: torch.Tensor, C: torch.Tensor, **kw) -> Algo:
    """The algorithm pax_gemm_ex would run (host-only)."""
    d = make_desc(A, B, C, **kw)
    return Algo(_lib.get().pax_gemm_select_algo(ctypes.byref(d)))


def pipeline_stages(A: torch.Tensor, B: torch.Tensor, C: torch.Tensor, **kw) -> int:
    """TMA ring depth of the kernel pax_gemm_ex would run (host-only; 0 for
    the CUDA-core kernel)."""
    d = make_desc(A, B, C, **kw)
    return int(_lib.get().pax_gemm_pipeline_stages(ctypes.byref(d)))


def ipc_export(t: torch.Tensor) -> bytes:
    """CUDA IPC handle (72 bytes) of the memory at t.data_ptr()."""
    h = _lib.IpcHandle()
    st = _lib.get().pax_ipc_export(ctypes.c_void_p(t.data_ptr()), ctypes.byref(h))
    if st != 0:
        raise PaxError(st, "pax_ipc_export")
    return bytes(h)


def ipc_import(handle: bytes) -> int:
    """Map another process's exported device memory; returns its address here."""
    h = _lib.IpcHandle.from_buffer_copy(handle)
    ptr = ctypes.c_void_p()
    st = _lib.get().pax_ipc_import(ctypes.byref(h), ctypes.byref(ptr))
    if st != 0:
        raise PaxError(st, "pax_ipc_import")
    return int(ptr.value)


def ipc_close(ptr: int) -> None:
    st = _lib.get().pax_ipc_close(ctypes.c_void_p(ptr))
    if st != 0:
        raise PaxError(st, "pax_ipc_close")


def peer_barrier(own: int, peers: list[int], slot: int, epoch: int, timeout_ns: int = 0,
                 stream: torch.cuda.Stream | None = None) -> None:
    """pax_peer_barrier on `stream` (default: the current stream): signal
    `epoch` into slot `slot` of every peer's flag array, then wait until
    every other slot of `own` holds at least `epoch`.  Addresses are device
    pointers (the peers' mapped with ipc_import)."""
    s = stream if stream is not None else torch.cuda.current_stream()
    arr = (ctypes.c_void_p * max(1, len(peers)))(*peers)
    st = _lib.get().pax_peer_barrier(ctypes.c_void_p(own), arr, len(peers), slot, epoch, timeout_ns,
                                     ctypes.c_void_p(s.cuda_stream))
    if st != 0:
        raise PaxError(st, "pax_peer_barrier")


def device_error() -> Status:
    """Read and clear the device error word (synchronises the device)."""
    return Status(_lib.get().pax_device_error())


def last_error() -> Status:
    return Status(_lib.get().pax_last_error())
