"""The C ABI (include/pax.h) on the host, without a GPU: exports, struct
layouts, argument checking, algorithm selection, and the host-side
verification functions the bridge mirrors from src/host_bridge.c."""
from __future__ import annotations

import ctypes
import os
import re
import subprocess

import numpy as np
import pytest

import oracle
import pax_b200
from pax_b200 import Algo, GemmDesc, PaxBuffer, lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "pax.h")


def declared_functions() -> list[str]:
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    names = re.findall(r"^[A-Za-z_][\w\s\*]*?\b(\w+)\s*\([^;{]*\)\s*;", src, flags=re.M)
    return sorted(set(n for n in names if n not in ("if", "while")))


def test_header_declares_the_reference_surface():
    names = set(declared_functions())
    for ref_name in ["pax_gemm_wmma_launch", "pax_gemm_ptx_launch", "pax_gemm_ptx_smem_bytes",
                     "pax_gemm_pipeline_launch", "pax_gemm_pipeline_smem_bytes", "pax_gemm_bias_gelu_launch",
                     "pax_gemm_residual_gelu_launch", "pax_gemm_scale_bias_gelu_launch",
                     "pax_gemm_tma_cluster_launch", "pax_gemm_tma_smem_bytes", "pax_validate_buffer",
                     "pax_alloc_device_1d", "pax_alloc_device_2d", "pax_alloc_host_1d", "pax_alloc_host_2d",
                     "pax_free_device", "pax_free_host", "pax_dispatch_wmma_gemm", "pax_dispatch_ptx_gemm",
                     "pax_dispatch_pipeline_gemm", "pax_dispatch_bias_gelu", "pax_dispatch_residual_gelu",
                     "cpu_gemm_ref", "pax_verify_gemm", "pax_bench_all"]:
        assert ref_name in names, ref_name


def test_library_exports_every_declared_symbol():
    out = subprocess.run(["nm", "-D", "--defined-only", pax_b200.LIB_PATH], capture_output=True, text=True,
                         check=True).stdout
    exported = set(line.split()[-1] for line in out.splitlines() if " T " in line)
    missing = [n for n in declared_functions() if n not in exported]
    assert not missing, missing
    for n in declared_functions():  # and ctypes can bind each of them
        getattr(lib, n)


def test_header_compiles_as_c(tmp_path):
    c = tmp_path / "use.c"
    c.write_text('#include "pax.h"\nint main(void){ pax_buffer_t b; (void)b; return (int)sizeof(pax_gemm_desc_t) > 0 ? 0 : 1; }\n')
    subprocess.run(["gcc", "-std=c99", "-I", os.path.join(ROOT, "include"), "-I", "/usr/local/cuda/include",
                    "-c", str(c), "-o", str(tmp_path / "use.o")], check=True)


C_CALLER = r"""
/* A C99 caller of the reference's host API, linked against this library. */
#define _POSIX_C_SOURCE 200112L
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include "pax.h"

int main(void) {
    int m = 3, n = 5, k = 4, i;
    float *a = NULL, *b = malloc(sizeof(float) * 20), *c = malloc(sizeof(float) * 15);
    float ref[15], acc = 0.0f;
    pax_buffer_t buf, pinned;
    pax_gemm_desc_t d;
    /* the descriptor below promises 64-byte alignment, as the reference's
       host allocations give */
    if (posix_memalign((void**)&a, 64, sizeof(float) * 12) != 0) return 10;
    if (!a || !b || !c) return 10;
    /* a caller-built descriptor, as the reference's users fill one */
    memset(&buf, 0, sizeof buf);
    buf.base = a;
    buf.elem_size = 4;
    buf.ndim = 2;
    buf.shape[0] = m;
    buf.shape[1] = k;
    buf.stride[0] = k;
    buf.stride[1] = 1;
    buf.alignment = 64;
    buf.ownership = PAX_HOST;
    if (!pax_validate_buffer(&buf)) return 11;
    buf.ndim = 4; /* more than three dimensions is invalid */
    if (pax_validate_buffer(&buf)) return 12;
    for (i = 0; i < m * k; ++i) a[i] = (float)(i % 7) - 3.0f;
    for (i = 0; i < k * n; ++i) b[i] = (float)(i % 5) - 2.0f;
    cpu_gemm_ref(a, b, c, m, n, k);
    for (i = 0; i < k; ++i) acc += a[i] * b[i * n]; /* C[0][0] by hand */
    if (c[0] != acc) return 13;
    memcpy(ref, c, sizeof ref);
    if (pax_verify_gemm(c, ref, m, n, 1e-3f) != 1) return 14;
    memset(&d, 0, sizeof d);
    d.M = -1;
    if (pax_gemm_ex(&d, 0) != PAX_ERR_INVALID || pax_last_error() != PAX_ERR_INVALID) return 15;
    if (pax_fp16_add_verified(0x3C00, 0x3C00) != 0x4000) return 16; /* 1 + 1 = 2 */
    if (strlen(pax_version()) == 0 || strlen(pax_status_string(PAX_OK)) == 0) return 17;
    /* pinned host memory needs the CUDA driver: without a GPU the helper
       reports the failure, as the reference's does */
    pinned = pax_alloc_host_2d(2, 2, 4, 0);
    if (pinned.base == NULL) {
        if (pax_last_error() != PAX_ERR_ALLOC) return 18;
    } else {
        pax_free_host(&pinned);
        if (pinned.base != NULL) return 19;
    }
    free(a);
    free(b);
    free(c);
    printf("c caller ok\n");
    return 0;
}
"""


def test_c_caller_links_and_runs(tmp_path):
    """The reference's own language: a C99 program using the host bridge's
    buffer helpers, cpu_gemm_ref, pax_verify_gemm, pax_gemm_ex's argument
    checks and a Lean-extraction symbol, linked with -lpax_b200."""
    c = tmp_path / "caller.c"
    c.write_text(C_CALLER)
    exe = tmp_path / "caller"
    libdir = os.path.join(ROOT, "pax_b200")
    subprocess.run(["gcc", "-std=c99", "-Wall", "-Werror", "-I", os.path.join(ROOT, "include"), "-I",
                    "/usr/local/cuda/include", str(c), "-o", str(exe), "-L", libdir, "-lpax_b200",
                    f"-Wl,-rpath,{libdir}"], check=True)
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=60)
    assert r.returncode == 0, (r.returncode, r.stdout, r.stderr)
    assert "c caller ok" in r.stdout


def test_struct_layouts_match():
    assert lib.pax_sizeof_buffer() == ctypes.sizeof(PaxBuffer) == 96
    assert lib.pax_sizeof_gemm_desc() == ctypes.sizeof(GemmDesc)


def _host_buffer(arr: np.ndarray) -> PaxBuffer:
    b = PaxBuffer()
    b.base = arr.ctypes.data
    b.elem_size = arr.itemsize
    b.ndim = arr.ndim
    for i in range(arr.ndim):
        b.shape[i] = arr.shape[i]
        b.stride[i] = arr.strides[i] // arr.itemsize
    b.alignment = 0
    return b


def test_validate_buffer_semantics():
    a = np.zeros((4, 8), np.float32)
    b = _host_buffer(a)
    assert lib.pax_validate_buffer(ctypes.byref(b)) == 1
    assert lib.pax_validate_buffer(None) == 0
    bad = _host_buffer(a)
    bad.base = None
    assert lib.pax_validate_buffer(ctypes.byref(bad)) == 0
    bad = _host_buffer(a)
    bad.ndim = 4
    assert lib.pax_validate_buffer(ctypes.byref(bad)) == 0
    bad = _host_buffer(a)
    bad.shape[1] = 0
    assert lib.pax_validate_buffer(ctypes.byref(bad)) == 0
    bad = _host_buffer(a)
    bad.stride[0] = -1
    assert lib.pax_validate_buffer(ctypes.byref(bad)) == 0
    bad = _host_buffer(a)
    bad.elem_size = 0
    assert lib.pax_validate_buffer(ctypes.byref(bad)) == 0
    odd = _host_buffer(a)
    odd.base = a.ctypes.data + 4
    odd.alignment = 8
    assert lib.pax_validate_buffer(ctypes.byref(odd)) == (1 if (a.ctypes.data + 4) % 8 == 0 else 0)


def test_cpu_gemm_ref_matches_reference_build(rng):
    A = rng.uniform(-1, 1, (33, 65)).astype(np.float16).astype(np.float32)
    B = rng.uniform(-1, 1, (65, 47)).astype(np.float16).astype(np.float32)
    C = np.empty((33, 47), np.float32)
    lib.cpu_gemm_ref(A.ctypes.data, B.ctypes.data, C.ctypes.data, 33, 47, 65)
    assert np.array_equal(C.view(np.uint32), oracle.cpu_gemm_ref(A, B).view(np.uint32))
    if oracle.ref_lib() is not None:
        assert np.array_equal(C.view(np.uint32), oracle.reference_cpu_gemm_ref(A, B).view(np.uint32))


def test_verify_gemm_matches_reference_decisions():
    d = np.load(os.path.join(ROOT, "tests", "golden", "verify_decisions.npz"))
    ref = np.ascontiguousarray(d["C_ref"])
    for i in range(d["C_gpu"].shape[0]):
        g = np.ascontiguousarray(d["C_gpu"][i])
        for j, tol in enumerate(d["tols"]):
            got = lib.pax_verify_gemm(g.ctypes.data, ref.ctypes.data, ref.shape[0], ref.shape[1], float(tol))
            assert got == d["decisions"][i, j]


def _desc(M=256, N=256, K=256, ptr=0x10000, **kw) -> GemmDesc:
    d = GemmDesc()
    d.A = d.B = d.C = ptr
    d.M, d.N, d.K = M, N, K
    d.alpha = 1.0
    d.c_dtype = kw.get("c_dtype", 1)
    d.epilogue = kw.get("epilogue", 0)
    d.bias = kw.get("bias", None)
    d.residual = kw.get("residual", None)
    d.lda = kw.get("lda", 0)
    return d


def test_gemm_ex_rejects_bad_arguments_before_touching_the_device():
    assert lib.pax_gemm_ex(None, None) == pax_b200.Status.INVALID
    d = _desc(M=-1)
    assert lib.pax_gemm_ex(ctypes.byref(d), None) == pax_b200.Status.INVALID
    d = _desc(epilogue=99)
    assert lib.pax_gemm_ex(ctypes.byref(d), None) == pax_b200.Status.INVALID
    d = _desc(epilogue=2)  # bias epilogue, NULL bias
    assert lib.pax_gemm_ex(ctypes.byref(d), None) == pax_b200.Status.INVALID
    d = _desc(epilogue=4)  # residual epilogue, NULL residual
    assert lib.pax_gemm_ex(ctypes.byref(d), None) == pax_b200.Status.INVALID
    d = _desc(lda=100)  # lda < K
    assert lib.pax_gemm_ex(ctypes.byref(d), None) == pax_b200.Status.INVALID
    d = _desc()
    d.C = None
    assert lib.pax_gemm_ex(ctypes.byref(d), None) == pax_b200.Status.INVALID
    assert lib.pax_last_error() == pax_b200.Status.INVALID
    d = _desc(M=0)  # empty output: nothing to do, no device needed
    assert lib.pax_gemm_ex(ctypes.byref(d), None) == pax_b200.Status.OK


def test_last_error_is_per_thread():
    """pax_last_error() is thread-local: a thread's failing call does not
    change the status another thread reads after its own successful call."""
    import threading

    barrier = threading.Barrier(8)
    results = {}

    def worker(i):
        bad = i % 2 == 0
        d = _desc(M=-1) if bad else _desc(M=0)  # M = 0: valid and empty, returns OK
        barrier.wait()  # all threads call at the same time
        for _ in range(200):
            st = lib.pax_gemm_ex(ctypes.byref(d), None)
            last = lib.pax_last_error()
            if st != last or st != (pax_b200.Status.INVALID if bad else pax_b200.Status.OK):
                results[i] = (st, last)
                return
        results[i] = "ok"

    threads = [threading.Thread(target=worker, args=(i,)) for i in range(8)]
    for t in threads:
        t.start()
    for t in threads:
        t.join(timeout=60)
    assert results == {i: "ok" for i in range(8)}


def test_algorithm_selection():
    sel = lambda d: Algo(lib.pax_gemm_select_algo(ctypes.byref(d)))  # noqa: E731
    assert sel(_desc(4096, 4096, 4096)) == Algo.TC
    assert sel(_desc(16, 16384, 4096)) == Algo.SKINNY
    assert sel(_desc(64, 16384, 4096)) == Algo.SKINNY
    assert sel(_desc(65, 16384, 4096)) == Algo.TC
    assert sel(_desc(128, 129, 256)) == Algo.SIMT      # fp16 row pitch not 16-byte aligned
    assert sel(_desc(128, 128, 100)) == Algo.SIMT      # K pitch 200 bytes
    assert sel(_desc(128, 128, 0)) == Algo.SIMT        # K == 0: epilogue of zero
    assert sel(_desc(128, 128, 128, ptr=0x10008)) == Algo.SIMT  # base not 16-byte aligned
    d = _desc(128, 132, 128, c_dtype=0)  # fp32 C pitch 528 B ok, but B pitch 264 B is not
    assert sel(d) == Algo.SIMT


def test_host_only_queries_without_a_device():
    """pax_gemm_pipeline_stages launches nothing; without a device it reports
    0 rather than failing, and bad descriptors also give 0."""
    assert lib.pax_gemm_pipeline_stages(ctypes.byref(_desc(4096, 4096, 4096))) == 0
    assert lib.pax_gemm_pipeline_stages(ctypes.byref(_desc(M=-1))) == 0


def test_replicated_and_batched_reject_bad_arguments():
    d = _desc(512, 512, 512)
    reps = (ctypes.c_void_p * 8)(*([0x1000] * 8))
    assert lib.pax_gemm_replicated_ex(ctypes.byref(d), reps, 8, None) == pax_b200.Status.INVALID  # > 7
    bad = (ctypes.c_void_p * 1)(0x1008)  # not 16-byte aligned
    assert lib.pax_gemm_replicated_ex(ctypes.byref(d), bad, 1, None) == pax_b200.Status.INVALID
    assert lib.pax_gemm_replicated_ex(ctypes.byref(d), None, 1, None) == pax_b200.Status.INVALID
    b = pax_b200._lib.GemmBatchedDesc()
    b.gemm = _desc(64, 64, 64)
    b.batch = 2
    b.stride_c = 64 * 64 - 1  # overlapping C items
    assert lib.pax_gemm_batched_ex(ctypes.byref(b), None) == pax_b200.Status.INVALID
    b.stride_c = 64 * 64
    b.stride_a = -8
    assert lib.pax_gemm_batched_ex(ctypes.byref(b), None) == pax_b200.Status.INVALID
    b.stride_a = 0
    b.batch = 0  # nothing to do
    assert lib.pax_gemm_batched_ex(ctypes.byref(b), None) == pax_b200.Status.OK


def test_ipc_helpers_reject_bad_arguments():
    h = pax_b200._lib.IpcHandle()
    assert lib.pax_ipc_export(None, ctypes.byref(h)) == pax_b200.Status.INVALID
    assert lib.pax_ipc_close(ctypes.c_void_p(0x1234)) == pax_b200.Status.INVALID  # never imported


def test_peer_barrier_rejects_bad_arguments():
    """pax_peer_barrier checks its arguments on the host, before any launch."""
    lib = pax_b200.lib
    P = ctypes.c_void_p
    own = P(0x10000)
    peers = (P * 8)(*[0x20000 + 0x1000 * i for i in range(8)])
    INVALID = pax_b200.Status.INVALID
    assert lib.pax_peer_barrier(own, peers, 8, 0, 1, 0, None) == INVALID  # more than 7 peers
    assert lib.pax_peer_barrier(own, peers, -1, 0, 1, 0, None) == INVALID
    assert lib.pax_peer_barrier(own, peers, 1, 2, 1, 0, None) == INVALID  # slot outside 2 ranks
    assert lib.pax_peer_barrier(own, peers, 1, -1, 1, 0, None) == INVALID
    assert lib.pax_peer_barrier(None, peers, 1, 0, 1, 0, None) == INVALID
    assert lib.pax_peer_barrier(P(0x10004), peers, 1, 0, 1, 0, None) == INVALID  # not 8-byte aligned
    assert lib.pax_peer_barrier(own, None, 1, 0, 1, 0, None) == INVALID
    bad = (P * 2)(0x20000, 0x20003)
    assert lib.pax_peer_barrier(own, bad, 2, 0, 1, 0, None) == INVALID
    assert lib.pax_peer_barrier(own, peers, 1, 0, 0, 0, None) == INVALID  # epoch 0
    assert lib.pax_last_error() == INVALID


def test_status_strings_and_version():
    for s in pax_b200.Status:
        assert lib.pax_status_string(int(s))
    assert b"sm_100a" in lib.pax_version()


def _probe_desc(M, N, K, c_dtype=pax_b200.DType.F32, algo=Algo.AUTO, aligned=True):
    d = GemmDesc()
    base = 0x10000 if aligned else 0x10002  # never dereferenced: host-only queries
    d.A, d.B, d.C = base, base, base
    d.M, d.N, d.K = M, N, K
    d.c_dtype = int(c_dtype)
    d.alpha = 1.0
    d.algo = int(algo)
    return d


def test_smem_queries_fit_the_part():
    for f in (lib.pax_gemm_ptx_smem_bytes, lib.pax_gemm_pipeline_smem_bytes, lib.pax_gemm_tma_smem_bytes):
        assert 0 < f() <= 232448


def test_smem_queries_report_the_kernel_the_launcher_runs():
    # The reference's *_smem_bytes give the dynamic shared memory of the
    # kernel its launcher runs (src/rtx_gemm_pipeline.cu:331-334,355-361).
    # The launchers here pick a kernel per problem; the queries answer for
    # the reference's default bench problem, 4096^3 with fp32 C.
    c2 = _probe_desc(4096, 4096, 4096)
    auto = lib.pax_gemm_smem_bytes(ctypes.byref(c2))
    assert auto > 0
    assert lib.pax_gemm_ptx_smem_bytes() == auto
    assert lib.pax_gemm_pipeline_smem_bytes() == auto
    pair = lib.pax_gemm_smem_bytes(ctypes.byref(_probe_desc(4096, 4096, 4096, algo=Algo.TC2)))
    assert lib.pax_gemm_tma_smem_bytes() == pair > 0
    # Other kernels need other amounts; the CUDA-core kernel's is static.
    skinny = lib.pax_gemm_smem_bytes(ctypes.byref(_probe_desc(16, 16384, 4096, c_dtype=pax_b200.DType.F16)))
    one_cta = lib.pax_gemm_smem_bytes(ctypes.byref(_probe_desc(1024, 1024, 1024, algo=Algo.TC)))
    assert 0 < skinny <= 232448 and 0 < one_cta <= 232448
    assert lib.pax_gemm_smem_bytes(ctypes.byref(_probe_desc(100, 100, 7, aligned=False))) == 0
    assert lib.pax_gemm_smem_bytes(None) == 0
    assert lib.pax_last_error() == pax_b200.Status.INVALID


def test_dispatch_rejects_invalid_buffers_without_gpu(capfd):
    a = np.zeros((4, 8), np.float16)
    good = _host_buffer(a)
    bad = _host_buffer(a)
    bad.base = None
    lib.pax_dispatch_wmma_gemm(ctypes.byref(bad), ctypes.byref(good), ctypes.byref(good), None)
    assert lib.pax_last_error() == pax_b200.Status.INVALID
    lib.pax_dispatch_bias_gelu(ctypes.byref(good), ctypes.byref(good), ctypes.byref(good), None, None)
    assert lib.pax_last_error() == pax_b200.Status.INVALID
    err = capfd.readouterr().err
    assert "[PAX]" in err and "NULL" in err
