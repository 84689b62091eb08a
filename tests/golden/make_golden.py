"""Writes tests/golden/*.npz from the reference's own CPU path.

The reference (SNAPKITTYWEST/pax) ships no tests or fixtures; its only
verification code is cpu_gemm_ref and pax_verify_gemm in src/host_bridge.c
(:397-445).  oracle/Makefile compiles that file, unmodified, into
oracle/_ref/libpaxref.so; this script calls it on seeded fp16 inputs (widened
exactly to fp32, as the reference's callers do) and stores inputs and
outputs.  Run from the repository root in a tree where the reference is
present:

    make -C oracle ref && python tests/golden/make_golden.py
"""
from __future__ import annotations

import ctypes
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)
import oracle  # noqa: E402

OUT = os.path.dirname(os.path.abspath(__file__))
SEED = 0x5EED


def ref_gemm(A16: np.ndarray, B16: np.ndarray) -> np.ndarray:
    return oracle.reference_cpu_gemm_ref(A16.astype(np.float32), B16.astype(np.float32))


def ref_verify(g: np.ndarray, r: np.ndarray, tol: float) -> int:
    L = oracle.ref_lib()
    g = np.ascontiguousarray(g, np.float32)
    r = np.ascontiguousarray(r, np.float32)
    return int(L.paxref_verify_gemm(ctypes.c_void_p(g.ctypes.data), ctypes.c_void_p(r.ctypes.data),
                                    g.shape[0], g.shape[1], ctypes.c_float(tol)))


def main() -> None:
    if oracle.ref_lib() is None:
        raise SystemExit("oracle/_ref/libpaxref.so missing: run `make -C oracle ref` first")
    rng = np.random.default_rng(SEED)
    cases = {}
    # uniform[-1,1] inputs, the distribution of configs 1, 2 and 5
    for name, (m, n, k) in {"uniform_64": (64, 64, 64), "uniform_ragged": (17, 33, 45),
                            "uniform_tall": (130, 24, 96)}.items():
        A = rng.uniform(-1, 1, (m, k)).astype(np.float16)
        B = rng.uniform(-1, 1, (k, n)).astype(np.float16)
        cases[name] = (A, B)
    # N(0,1) x N(0,0.02), the distribution of configs 3 and 4
    A = rng.standard_normal((16, 128)).astype(np.float16)
    B = (rng.standard_normal((128, 256)) * 0.02).astype(np.float16)
    cases["normal_skinny"] = (A, B)
    # small integers: every product and partial sum is exact in fp32
    A = rng.integers(-3, 4, (48, 80)).astype(np.float16)
    B = rng.integers(-3, 4, (80, 40)).astype(np.float16)
    cases["int_kat"] = (A, B)
    # identity and permutation
    A = np.eye(32, dtype=np.float16)
    B = rng.uniform(-1, 1, (32, 48)).astype(np.float16)
    cases["identity"] = (A, B)
    P = np.eye(40, dtype=np.float16)[rng.permutation(40)]
    B = rng.uniform(-1, 1, (40, 24)).astype(np.float16)
    cases["permutation"] = (P, B)

    for name, (A, B) in cases.items():
        C = ref_gemm(A, B)
        np.savez(os.path.join(OUT, f"gemm_{name}.npz"), A=A, B=B, C=C)

    # pax_verify_gemm decisions on perturbed outputs
    A, B = cases["uniform_64"]
    C = ref_gemm(A, B)
    g_all = np.stack([C + np.float32(s) * np.random.default_rng(i).standard_normal(C.shape).astype(np.float32)
                      for i, s in enumerate((0.0, 1e-7, 1e-5, 1e-3, 1e-1))])
    dec = np.array([[ref_verify(g_all[i], C, t) for t in (1e-6, 1e-4, 1e-2, 1.0)] for i in range(5)], np.int32)
    np.savez(os.path.join(OUT, "verify_decisions.npz"), C_ref=C, C_gpu=g_all, tols=np.array([1e-6, 1e-4, 1e-2, 1.0],
             np.float32), decisions=dec)
    print("wrote", sorted(f for f in os.listdir(OUT) if f.endswith(".npz")))


if __name__ == "__main__":
    main()
