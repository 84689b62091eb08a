"""Loads ``libpax_b200.so`` (the C ABI of include/pax.h) on first use and
declares its signatures.  There is no fallback: if the library is missing,
the first call raises LibraryNotBuilt with instructions to build it."""
from __future__ import annotations

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libpax_b200.so")


class LibraryNotBuilt(ImportError):
    pass


class PaxBuffer(ctypes.Structure):
    """pax_buffer_t (include/pax.h; reference src/host_bridge.c:38-60)."""
    _fields_ = [
        ("base", ctypes.c_void_p),
        ("elem_size", ctypes.c_size_t),
        ("shape", ctypes.c_int64 * 3),
        ("stride", ctypes.c_int64 * 3),
        ("ndim", ctypes.c_int),
        ("alignment", ctypes.c_size_t),
        ("ownership", ctypes.c_int),
        ("stream", ctypes.c_void_p),
    ]


class GemmDesc(ctypes.Structure):
    """pax_gemm_desc_t (include/pax.h)."""
    _fields_ = [
        ("A", ctypes.c_void_p),
        ("B", ctypes.c_void_p),
        ("C", ctypes.c_void_p),
        ("M", ctypes.c_int64),
        ("N", ctypes.c_int64),
        ("K", ctypes.c_int64),
        ("lda", ctypes.c_int64),
        ("ldb", ctypes.c_int64),
        ("ldc", ctypes.c_int64),
        ("c_dtype", ctypes.c_int),
        ("epilogue", ctypes.c_int),
        ("alpha", ctypes.c_float),
        ("bias", ctypes.c_void_p),
        ("residual", ctypes.c_void_p),
        ("residual_dtype", ctypes.c_int),
        ("ld_res", ctypes.c_int64),
        ("algo", ctypes.c_int),
    ]


class IpcHandle(ctypes.Structure):
    """pax_ipc_handle_t (include/pax.h)."""
    _fields_ = [("handle", ctypes.c_ubyte * 64), ("offset", ctypes.c_uint64)]


class GemmBatchedDesc(ctypes.Structure):
    """pax_gemm_batched_desc_t (include/pax.h)."""
    _fields_ = [
        ("gemm", GemmDesc),
        ("batch", ctypes.c_int64),
        ("stride_a", ctypes.c_int64),
        ("stride_b", ctypes.c_int64),
        ("stride_c", ctypes.c_int64),
        ("stride_bias", ctypes.c_int64),
        ("stride_residual", ctypes.c_int64),
    ]


def _declare(L: ctypes.CDLL) -> None:
    P = ctypes.c_void_p
    i = ctypes.c_int
    f = ctypes.c_float
    sz = ctypes.c_size_t
    buf_p = ctypes.POINTER(PaxBuffer)
    launch7 = [P, P, P, i, i, i, P]
    u64, u16 = ctypes.c_uint64, ctypes.c_uint16
    sigs = {
        # launchers (reference names, fp32 C)
        "pax_gemm_wmma_launch": (launch7, None),
        "pax_gemm_ptx_launch": (launch7, None),
        "pax_gemm_pipeline_launch": (launch7, None),
        "pax_gemm_ptx_smem_bytes": ([], sz),
        "pax_gemm_pipeline_smem_bytes": ([], sz),
        "pax_gemm_tma_smem_bytes": ([], sz),
        "pax_gemm_bias_gelu_launch": ([P, P, P, i, i, i, P, P], None),
        "pax_gemm_residual_gelu_launch": ([P, P, P, i, i, i, P, P], None),
        "pax_gemm_scale_bias_gelu_launch": ([P, P, P, i, i, i, f, P, P], None),
        "pax_gemm_tma_cluster_launch": ([P, P, P, i, i, i, P, P, P, P], None),
        # fp16 twins
        "pax_gemm_f16_launch": (launch7, None),
        "pax_gemm_bias_f16_launch": ([P, P, P, i, i, i, P, P], None),
        "pax_gemm_bias_gelu_f16_launch": ([P, P, P, i, i, i, P, P], None),
        "pax_gemm_bias_gelu_erf_f16_launch": ([P, P, P, i, i, i, P, P], None),
        "pax_gemm_residual_gelu_f16_launch": ([P, P, P, i, i, i, P, P], None),
        "pax_gemm_residual_gelu_erf_f16_launch": ([P, P, P, i, i, i, P, P], None),
        "pax_gemm_ex": ([ctypes.POINTER(GemmDesc), P], i),
        "pax_gemm_batched_ex": ([ctypes.POINTER(GemmBatchedDesc), P], i),
        "pax_gemm_replicated_ex": ([ctypes.POINTER(GemmDesc), ctypes.POINTER(P), i, P], i),
        "pax_ipc_export": ([P, ctypes.POINTER(IpcHandle)], i),
        "pax_ipc_import": ([ctypes.POINTER(IpcHandle), ctypes.POINTER(P)], i),
        "pax_ipc_close": ([P], i),
        "pax_peer_barrier": ([P, ctypes.POINTER(P), i, i, u64, u64, P], i),
        "pax_gemm_select_algo": ([ctypes.POINTER(GemmDesc)], i),
        "pax_gemm_pipeline_stages": ([ctypes.POINTER(GemmDesc)], i),
        "pax_gemm_smem_bytes": ([ctypes.POINTER(GemmDesc)], sz),
        "pax_gemm_skinny_noalloc": ([ctypes.POINTER(GemmDesc), P], i),
        # Lean-extraction names (64-bit sizes, pointers as integers)
        "pax_gemm_wmma_verified": ([u64] * 6, None),
        "pax_gemm_ptx_verified": ([u64] * 6, None),
        "pax_gemm_pipeline3_verified": ([u64] * 6, None),
        "pax_gemm_bias_gelu_verified": ([u64] * 7, None),
        "pax_gemm_residual_gelu_verified": ([u64] * 7, None),
        "pax_fp16_add_verified": ([u16] * 2, u16),
        "pax_fp16_mul_verified": ([u16] * 2, u16),
        "pax_fp16_fma_verified": ([u16] * 3, u16),
        # bridge
        "pax_validate_buffer": ([buf_p], i),
        "pax_alloc_device_1d": ([sz, sz, P], PaxBuffer),
        "pax_alloc_device_2d": ([sz, sz, sz, P], PaxBuffer),
        "pax_alloc_host_1d": ([sz, sz, P], PaxBuffer),
        "pax_alloc_host_2d": ([sz, sz, sz, P], PaxBuffer),
        "pax_free_device": ([buf_p], None),
        "pax_free_host": ([buf_p], None),
        "pax_dispatch_wmma_gemm": ([buf_p, buf_p, buf_p, P], None),
        "pax_dispatch_ptx_gemm": ([buf_p, buf_p, buf_p, P], None),
        "pax_dispatch_pipeline_gemm": ([buf_p, buf_p, buf_p, P], None),
        "pax_dispatch_bias_gelu": ([buf_p, buf_p, buf_p, P, P], None),
        "pax_dispatch_residual_gelu": ([buf_p, buf_p, buf_p, P, P], None),
        "pax_dispatch_scale_bias_gelu": ([buf_p, buf_p, buf_p, f, P, P], None),
        "cpu_gemm_ref": ([P, P, P, i, i, i], None),
        "pax_verify_gemm": ([P, P, i, i, f], i),
        "pax_bench_all": ([i], None),
        "pax_bench_setup": ([i, i, i, P], i),
        "pax_bench_teardown": ([], None),
        # status
        "pax_last_error": ([], i),
        "pax_status_string": ([i], ctypes.c_char_p),
        "pax_device_error": ([], i),
        "pax_selftest_bounded_wait": ([P], i),
        "pax_selftest_stale_counters": ([P], i),
        "pax_selftest_set_wait_limit": ([u64], i),
        "pax_shutdown": ([], None),
        "pax_version": ([], ctypes.c_char_p),
        "pax_sizeof_buffer": ([], sz),
        "pax_sizeof_gemm_desc": ([], sz),
    }
    for name, (args, res) in sigs.items():
        fn = getattr(L, name)
        fn.argtypes = args
        fn.restype = res


_LIB: ctypes.CDLL | None = None


def get() -> ctypes.CDLL:
    """The loaded library; raises LibraryNotBuilt if it has not been built."""
    global _LIB
    if _LIB is None:
        _LIB = load()
    return _LIB


def __getattr__(name):
    if name == "lib":
        return get()
    raise AttributeError(name)


def load() -> ctypes.CDLL:
    if not os.path.exists(LIB_PATH):
        raise LibraryNotBuilt(
            f"{LIB_PATH} is missing: build it with `python -m pax_b200.build` "
            "(nvcc, sm_100a). pax_b200 has no CPU fallback.")
    L = ctypes.CDLL(LIB_PATH)
    _declare(L)
    if L.pax_sizeof_buffer() != ctypes.sizeof(PaxBuffer):
        raise ImportError("pax_buffer_t layout mismatch between libpax_b200.so and the Python binding")
    if L.pax_sizeof_gemm_desc() != ctypes.sizeof(GemmDesc):
        raise ImportError("pax_gemm_desc_t layout mismatch between libpax_b200.so and the Python binding")
    return L

