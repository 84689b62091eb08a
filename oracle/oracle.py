"""ctypes front end to the CPU oracle (``oracle/liboracle.so``) and to the
reference's own CPU path built from its sources (``oracle/_ref/libpaxref.so``).

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).

What each function restates (reference file:line):
  gemm / gemm_f16      src/host_bridge.c:397-407 (cpu_gemm_ref; fp32 sequential
                       sum per element) on fp16 inputs widened exactly
                       (src/pax_kernel.fut:18-25)
  epilogue             src/rtx_gemm_epilogue.cu:7-10,76-80,176-233
  verify               src/host_bridge.c:422-445 (pax_verify_gemm)
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")
REF_LIB_PATH = os.path.join(HERE, "_ref", "libpaxref.so")
REF_WMMA_PATH = os.path.join(HERE, "_ref", "libpaxref_wmma.so")

EPI = {
    "none": 0, "bias": 1, "bias_gelu_tanh": 2, "bias_gelu_erf": 3,
    "residual_gelu_tanh": 4, "residual_gelu_erf": 5, "gelu_tanh": 6, "gelu_erf": 7,
    "residual": 8,
}

_lib = None
_ref = None


def build(ref: bool = False) -> None:
    """Build liboracle.so (and, with ref=True, the reference objects)."""
    subprocess.run(["make", "-s", "-C", HERE, "liboracle.so"], check=True)
    if ref:
        subprocess.run(["make", "-s", "-C", HERE, "ref"], check=True)


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = ctypes.CDLL(LIB_PATH)
        P = ctypes.c_void_p
        i64 = ctypes.c_int64
        L.oracle_f16_to_f32.argtypes = [ctypes.c_uint16]
        L.oracle_f16_to_f32.restype = ctypes.c_float
        L.oracle_f32_to_f16.argtypes = [ctypes.c_float]
        L.oracle_f32_to_f16.restype = ctypes.c_uint16
        L.oracle_f16_to_f32_array.argtypes = [P, P, i64]
        L.oracle_f32_to_f16_array.argtypes = [P, P, i64]
        L.oracle_cpu_gemm_ref.argtypes = [P, P, P, ctypes.c_int, ctypes.c_int, ctypes.c_int]
        L.oracle_gemm_f16.argtypes = [P, P, P, i64, i64, i64, i64, i64, P, ctypes.c_int]
        L.oracle_gelu_tanh.argtypes = [ctypes.c_float]
        L.oracle_gelu_tanh.restype = ctypes.c_float
        L.oracle_gelu_erf.argtypes = [ctypes.c_float]
        L.oracle_gelu_erf.restype = ctypes.c_float
        L.oracle_epilogue.argtypes = [P, i64, i64, ctypes.c_int, ctypes.c_float, P, P, ctypes.c_int, i64, P]
        L.oracle_verify.argtypes = [P, P, i64, ctypes.c_float, ctypes.POINTER(ctypes.c_float),
                                    ctypes.POINTER(ctypes.c_int64)]
        L.oracle_verify.restype = ctypes.c_int
        _lib = L
    return _lib


def ref_lib() -> ctypes.CDLL | None:
    """The reference's own cpu_gemm_ref / pax_verify_gemm, or None if not built."""
    global _ref
    if _ref is None and os.path.exists(REF_LIB_PATH):
        L = ctypes.CDLL(REF_LIB_PATH)
        P = ctypes.c_void_p
        L.paxref_cpu_gemm_ref.argtypes = [P, P, P, ctypes.c_int, ctypes.c_int, ctypes.c_int]
        L.paxref_verify_gemm.argtypes = [P, P, ctypes.c_int, ctypes.c_int, ctypes.c_float]
        L.paxref_verify_gemm.restype = ctypes.c_int
        _ref = L
    return _ref


def _ptr(a: np.ndarray | None) -> ctypes.c_void_p | None:
    return None if a is None else ctypes.c_void_p(a.ctypes.data)


def _u16(a: np.ndarray) -> np.ndarray:
    a = np.ascontiguousarray(a)
    if a.dtype == np.float16:
        return a.view(np.uint16)
    assert a.dtype == np.uint16, a.dtype
    return a


def f16_to_f32(h: np.ndarray) -> np.ndarray:
    h = _u16(h)
    out = np.empty(h.shape, np.float32)
    lib().oracle_f16_to_f32_array(_ptr(h), _ptr(out), h.size)
    return out


def f32_to_f16(x: np.ndarray) -> np.ndarray:
    """Round to nearest even; returns np.float16."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.shape, np.uint16)
    lib().oracle_f32_to_f16_array(_ptr(x), _ptr(out), x.size)
    return out.view(np.float16)


def cpu_gemm_ref(A: np.ndarray, B: np.ndarray) -> np.ndarray:
    """Literal restatement of the reference loop on fp32 inputs."""
    A = np.ascontiguousarray(A, dtype=np.float32)
    B = np.ascontiguousarray(B, dtype=np.float32)
    m, k = A.shape
    n = B.shape[1]
    C = np.empty((m, n), np.float32)
    lib().oracle_cpu_gemm_ref(_ptr(A), _ptr(B), _ptr(C), m, n, k)
    return C


def reference_cpu_gemm_ref(A: np.ndarray, B: np.ndarray) -> np.ndarray:
    """The reference's compiled cpu_gemm_ref (requires oracle/_ref)."""
    L = ref_lib()
    if L is None:
        raise FileNotFoundError(REF_LIB_PATH)
    A = np.ascontiguousarray(A, dtype=np.float32)
    B = np.ascontiguousarray(B, dtype=np.float32)
    m, k = A.shape
    n = B.shape[1]
    C = np.empty((m, n), np.float32)
    L.paxref_cpu_gemm_ref(_ptr(A), _ptr(B), _ptr(C), m, n, k)
    return C


def gemm_f16(A: np.ndarray, B: np.ndarray, rows: np.ndarray | None = None, nthreads: int = 0) -> np.ndarray:
    """fp32 accumulator of A.B for fp16 A [m][k], B [k][n] (row subset optional)."""
    A = _u16(A)
    B = _u16(B)
    m, k = A.shape
    n = B.shape[1]
    r = None if rows is None else np.ascontiguousarray(rows, dtype=np.int64)
    m_out = m if r is None else r.size
    C = np.empty((m_out, n), np.float32)
    nt = nthreads if nthreads > 0 else (os.cpu_count() or 1)
    lib().oracle_gemm_f16(_ptr(A), _ptr(B), _ptr(C), m_out, n, k, k, n, _ptr(r), nt)
    return C


def epilogue(C: np.ndarray, epi: str | int = "none", alpha: float = 1.0, bias: np.ndarray | None = None,
             residual: np.ndarray | None = None, rows: np.ndarray | None = None) -> np.ndarray:
    """Apply the epilogue in place to the fp32 accumulator C and return it."""
    e = EPI[epi] if isinstance(epi, str) else int(epi)
    m, n = C.shape
    b = None if bias is None else _u16(bias)
    res_f32 = 0
    res = None
    ld = n
    if residual is not None:
        if residual.dtype == np.float32:
            res = np.ascontiguousarray(residual)
            res_f32 = 1
        else:
            res = _u16(residual)
        ld = res.shape[1]
    r = None if rows is None else np.ascontiguousarray(rows, dtype=np.int64)
    lib().oracle_epilogue(_ptr(C), m, n, e, alpha, _ptr(b), _ptr(res), res_f32, ld, _ptr(r))
    return C


def gemm(A, B, epi="none", alpha=1.0, bias=None, residual=None, out_dtype=np.float32, rows=None,
         nthreads: int = 0) -> np.ndarray:
    """Full oracle: epilogue(A.B), output fp32 or fp16 (round to nearest even)."""
    C = gemm_f16(A, B, rows=rows, nthreads=nthreads)
    epilogue(C, epi, alpha, bias, residual, rows=rows)
    if np.dtype(out_dtype) == np.float16:
        return f32_to_f16(C)
    return C


def gelu_tanh(x: float) -> float:
    return lib().oracle_gelu_tanh(x)


def gelu_erf(x: float) -> float:
    return lib().oracle_gelu_erf(x)


def verify(C_gpu: np.ndarray, C_ref: np.ndarray, tol: float) -> tuple[bool, float, int]:
    """pax_verify_gemm semantics: (passed, max relative error, flat index)."""
    g = np.ascontiguousarray(C_gpu, dtype=np.float32)
    r = np.ascontiguousarray(C_ref, dtype=np.float32)
    me = ctypes.c_float()
    mi = ctypes.c_int64()
    ok = lib().oracle_verify(_ptr(g), _ptr(r), g.size, tol, ctypes.byref(me), ctypes.byref(mi))
    return bool(ok), float(me.value), int(mi.value)


def normwise_error(C_gpu: np.ndarray, C_ref: np.ndarray) -> float:
    """max|C - C_ref| / max|C_ref| (the north-star parity measure)."""
    g = np.asarray(C_gpu, dtype=np.float64)
    r = np.asarray(C_ref, dtype=np.float64)
    den = float(np.max(np.abs(r))) if r.size else 0.0
    num = float(np.max(np.abs(g - r))) if r.size else 0.0
    return num / den if den > 0 else num
