"""CUDA kernels vs the oracle on seeded inputs, through the C ABI.

Every case runs libpax_b200.so (pax_gemm_ex or a reference-named launcher)
and compares with oracle.gemm: fp32-accumulated products of the same fp16
inputs with the reference's epilogue math.
"""
from __future__ import annotations

import ctypes
import glob
import os

import numpy as np
import pytest
import torch

import oracle
import pax_b200
from _helpers import check, inputs, run_gemm, to_dev

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def stream_ptr():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


class _DevArray:
    """Exposes a raw device pointer to torch via __cuda_array_interface__."""

    def __init__(self, ptr, shape, typestr):
        self.__cuda_array_interface__ = {"data": (int(ptr), False), "shape": tuple(shape), "typestr": typestr,
                                         "version": 3, "strides": None}


def dev_view(ptr, shape, dtype) -> torch.Tensor:
    typestr = {np.float16: "<f2", np.float32: "<f4"}[dtype]
    return torch.as_tensor(_DevArray(ptr, shape, typestr), device="cuda")


# ---------------------------------------------------------------- tcgen05 core
@pytest.mark.parametrize("bn", [256, 128])
@pytest.mark.parametrize("shape", [(128, 256, 64), (256, 512, 128), (384, 768, 1024)])
@pytest.mark.parametrize("out", [np.float32, np.float16])
def test_tc_plain(cuda, rng, monkeypatch, bn, shape, out):
    monkeypatch.setenv("PAX_TC_BN", str(bn))
    M, N, K = shape
    A, B = inputs(rng, M, N, K)
    got = run_gemm(A, B, cuda, out_dtype=out, algo="tc")
    check(got, oracle.gemm(A, B, out_dtype=out), out)


@pytest.mark.parametrize("shape", [(256, 256, 64), (512, 768, 512), (300, 520, 200), (128, 256, 128), (1000, 8, 8),
                                   (384, 264, 4104)])
@pytest.mark.parametrize("out", [np.float32, np.float16])
def test_tc2_cta_pair(cuda, rng, shape, out):
    """256 x 256 tiles on CTA pairs (tcgen05 cta_group::2), ragged edges
    included (rows of the odd CTA wholly outside C when M <= 128)."""
    M, N, K = shape
    A, B = inputs(rng, M, N, K)
    got = run_gemm(A, B, cuda, out_dtype=out, algo="tc2")
    check(got, oracle.gemm(A, B, out_dtype=out), out)


@pytest.mark.parametrize("shape", [(300, 520, 200), (129, 264, 72), (1000, 8, 8), (65, 1032, 136), (77, 40, 4104)])
@pytest.mark.parametrize("out", [np.float32, np.float16])
def test_tc_ragged_edges(cuda, rng, shape, out):
    M, N, K = shape
    A, B = inputs(rng, M, N, K)
    got = run_gemm(A, B, cuda, out_dtype=out, algo="tc")
    check(got, oracle.gemm(A, B, out_dtype=out), out)


EPIS = ["none", "bias", "bias_gelu_tanh", "bias_gelu_erf", "residual_gelu_tanh", "residual_gelu_erf", "gelu_tanh",
        "gelu_erf", "residual"]


@pytest.mark.parametrize("epi", EPIS)
@pytest.mark.parametrize("out", [np.float32, np.float16])
@pytest.mark.parametrize("res_dtype", [np.float32, np.float16])
@pytest.mark.parametrize("algo", ["tc", "tc2"])
def test_tc_epilogues(cuda, rng, epi, out, res_dtype, algo):
    if "residual" not in epi and res_dtype == np.float16:
        pytest.skip("residual dtype irrelevant")
    M, N, K = 256, 520, 320
    A, B = inputs(rng, M, N, K)
    bias = rng.standard_normal(N).astype(np.float16)
    res = rng.standard_normal((M, N)).astype(res_dtype)
    got = run_gemm(A, B, cuda, epi=epi, out_dtype=out, bias=bias if "bias" in epi else None,
                   residual=res if "residual" in epi else None, algo=algo)
    ref = oracle.gemm(A, B, epi=epi, bias=bias, residual=res, out_dtype=out)
    check(got, ref, out)


@pytest.mark.parametrize("algo", ["tc", "tc2", "skinny", "simt"])
def test_scale_bias_gelu(cuda, rng, algo):
    M = 48 if algo == "skinny" else 200
    A, B = inputs(rng, M, 264, 192)
    bias = rng.standard_normal(264).astype(np.float16)
    got = run_gemm(A, B, cuda, epi="bias_gelu_tanh", bias=bias, alpha=0.37, out_dtype=np.float32, algo=algo)
    check(got, oracle.gemm(A, B, epi="bias_gelu_tanh", bias=bias, alpha=0.37), np.float32)


# ---------------------------------------------------------------- skinny
@pytest.mark.parametrize("M", [1, 8, 16, 17, 33, 48, 64])
@pytest.mark.parametrize("NK", [(128, 64), (1000, 320), (4096, 4096), (384, 136)])
def test_skinny(cuda, rng, M, NK):
    N, K = NK
    A, B = inputs(rng, M, N, K, dist="normal")
    bias = rng.standard_normal(N).astype(np.float16)
    got = run_gemm(A, B, cuda, epi="bias", bias=bias, out_dtype=np.float16, algo="skinny")
    check(got, oracle.gemm(A, B, epi="bias", bias=bias, out_dtype=np.float16), np.float16)


@pytest.mark.parametrize("nt", [0, 128, 256])
@pytest.mark.parametrize("M,N,K", [(16, 16384, 4096), (1, 1000, 320), (33, 2048, 1088), (64, 768, 4096),
                                   (16, 520, 64), (16, 40960, 2048), (48, 16384, 4160), (16, 128, 4096)])
def test_skinny_layouts(cuda, rng, monkeypatch, nt, M, N, K):
    """Lockstep layout (nt=0: one CTA per (tile, interleaved K slice)) and the
    persistent stream-K layout with 128- and 256-column units, including
    ragged N, uneven K slices, tiles split between two or three CTAs and a
    single tile split over every SM."""
    monkeypatch.setenv("PAX_SKINNY_NT", str(nt))
    A, B = inputs(rng, M, N, K, dist="normal")
    bias = rng.standard_normal(N).astype(np.float16)
    got = run_gemm(A, B, cuda, epi="bias", bias=bias, out_dtype=np.float16, algo="skinny")
    check(got, oracle.gemm(A, B, epi="bias", bias=bias, out_dtype=np.float16), np.float16)


@pytest.mark.parametrize("epi", ["none", "bias_gelu_erf", "residual_gelu_tanh"])
@pytest.mark.parametrize("out", [np.float32, np.float16])
def test_skinny_epilogues(cuda, rng, epi, out):
    M, N, K = 16, 2048, 1024
    A, B = inputs(rng, M, N, K, dist="normal")
    bias = rng.standard_normal(N).astype(np.float16)
    res = rng.standard_normal((M, N)).astype(np.float16)
    got = run_gemm(A, B, cuda, epi=epi, bias=bias, residual=res, out_dtype=out, algo="skinny")
    check(got, oracle.gemm(A, B, epi=epi, bias=bias, residual=res, out_dtype=out), out)


@pytest.mark.parametrize("nt", ["128", "0"])
def test_skinny_stream_k_bit_exact_and_deterministic(cuda, rng, monkeypatch, nt):
    """Integer-valued inputs through split tiles (stream-K; lockstep with K
    slices at N = 4096): exact, and the same bits on every run (a tile's
    last contributor adds the others' partial sums in CTA order)."""
    monkeypatch.setenv("PAX_SKINNY_NT", nt)
    A = rng.integers(-3, 4, (16, 4096)).astype(np.float16)
    B = rng.integers(-3, 4, (4096, 16384 if nt == "128" else 4096)).astype(np.float16)
    exact = (A.astype(np.int64) @ B.astype(np.int64)).astype(np.float32)
    first = run_gemm(A, B, cuda, out_dtype=np.float32, algo="skinny")
    assert np.array_equal(first, exact)
    for _ in range(2):
        assert np.array_equal(run_gemm(A, B, cuda, out_dtype=np.float32, algo="skinny"), first)


def test_skinny_workspace_reuse_across_shapes(cuda, rng):
    """The per-stream workspace is reused by later calls with more column
    tiles (more counters) and larger partial-sum needs, and fewer again."""
    for M, N, K in [(16, 256, 4096), (16, 16384, 4096), (48, 2048, 1024), (16, 16384, 4096), (1, 128, 64)]:
        A, B = inputs(rng, M, N, K, dist="normal")
        got = run_gemm(A, B, cuda, out_dtype=np.float16, algo="skinny")
        check(got, oracle.gemm(A, B, out_dtype=np.float16), np.float16)


# ---------------------------------------------------------------- SIMT
@pytest.mark.parametrize("shape", [(1, 1, 1), (17, 17, 17), (127, 33, 129), (5, 300, 7), (64, 64, 0)])
@pytest.mark.parametrize("epi", ["none", "bias_gelu_tanh", "residual_gelu_erf"])
def test_simt_unaligned(cuda, rng, shape, epi):
    M, N, K = shape
    A, B = inputs(rng, M, N, K)
    bias = rng.standard_normal(N).astype(np.float16)
    res = rng.standard_normal((M, N)).astype(np.float32)
    got = run_gemm(A, B, cuda, epi=epi, bias=bias, residual=res, out_dtype=np.float32)
    assert pax_b200.select_algo(to_dev(A, cuda), to_dev(B, cuda),
                                torch.empty((M, N), dtype=torch.float32, device=cuda)) == pax_b200.Algo.SIMT
    check(got, oracle.gemm(A, B, epi=epi, bias=bias, residual=res), np.float32)


# ---------------------------------------------------------------- exactness
@pytest.mark.parametrize("algo,M", [("tc", 256), ("tc2", 384), ("skinny", 16), ("simt", 256)])
def test_integer_inputs_bit_exact(cuda, rng, algo, M):
    A = rng.integers(-3, 4, (M, 512)).astype(np.float16)
    B = rng.integers(-3, 4, (512, 384)).astype(np.float16)
    got = run_gemm(A, B, cuda, out_dtype=np.float32, algo=algo)
    exact = (A.astype(np.int64) @ B.astype(np.int64)).astype(np.float32)
    bad = np.argwhere(got != exact)
    assert bad.size == 0, (f"{len(bad)} mismatches, first {bad[:8].tolist()}, "
                           f"got {got[tuple(bad[0])]} want {exact[tuple(bad[0])]}")


GOLDEN = sorted(glob.glob(os.path.join(ROOT, "tests", "golden", "gemm_*.npz")))


@pytest.mark.parametrize("path", GOLDEN, ids=lambda p: os.path.basename(p)[5:-4])
def test_golden_through_reference_launcher(cuda, path):
    d = np.load(path)
    A, B, C = d["A"], d["B"], d["C"]
    M, K = A.shape
    N = B.shape[1]
    tA, tB = to_dev(A, cuda), to_dev(B, cuda)
    tC = torch.full((M, N), float("nan"), dtype=torch.float32, device=cuda)
    pax_b200.lib.pax_gemm_wmma_launch(tA.data_ptr(), tB.data_ptr(), tC.data_ptr(), M, N, K, stream_ptr())
    torch.cuda.synchronize()
    got = tC.cpu().numpy()
    name = os.path.basename(path)
    if any(s in name for s in ("int_kat", "identity", "permutation")):
        assert np.array_equal(got, C)
    else:
        check(got, C, np.float32)


def test_reference_wmma_kernel_agrees(cuda, rng):
    """The reference's own sm_86 WMMA kernel, compiled for sm_100a from its
    source (oracle/_ref), on a shape it handles (M, N multiples of 16, K of 8)."""
    path = oracle.REF_WMMA_PATH
    if not os.path.exists(path):
        pytest.skip("oracle/_ref/libpaxref_wmma.so not built")
    L = ctypes.CDLL(path)
    L.pax_gemm_wmma_launch.argtypes = [ctypes.c_void_p] * 3 + [ctypes.c_int] * 3 + [ctypes.c_void_p]
    M, N, K = 256, 384, 512
    A, B = inputs(rng, M, N, K)
    tA, tB = to_dev(A, cuda), to_dev(B, cuda)
    ref_out = torch.zeros((M, N), dtype=torch.float32, device=cuda)
    L.pax_gemm_wmma_launch(tA.data_ptr(), tB.data_ptr(), ref_out.data_ptr(), M, N, K, stream_ptr())
    ours = torch.zeros_like(ref_out)
    pax_b200.lib.pax_gemm_wmma_launch(tA.data_ptr(), tB.data_ptr(), ours.data_ptr(), M, N, K, stream_ptr())
    torch.cuda.synchronize()
    check(ours.cpu().numpy(), ref_out.cpu().numpy(), np.float32)


# ---------------------------------------------------------------- C ABI surface
def test_reference_named_launchers(cuda, rng):
    M, N, K = 256, 512, 256
    A, B = inputs(rng, M, N, K)
    bias = rng.standard_normal(N).astype(np.float16)
    res32 = rng.standard_normal((M, N)).astype(np.float32)
    res16 = res32.astype(np.float16)
    tA, tB, tb = to_dev(A, cuda), to_dev(B, cuda), to_dev(bias, cuda)
    tr32, tr16 = to_dev(res32, cuda), to_dev(res16, cuda)
    L = pax_b200.lib
    s = stream_ptr()
    c32 = lambda: torch.empty((M, N), dtype=torch.float32, device=cuda)  # noqa: E731
    c16 = lambda: torch.empty((M, N), dtype=torch.float16, device=cuda)  # noqa: E731
    cases = []
    for name in ("pax_gemm_wmma_launch", "pax_gemm_ptx_launch", "pax_gemm_pipeline_launch"):
        C = c32()
        getattr(L, name)(tA.data_ptr(), tB.data_ptr(), C.data_ptr(), M, N, K, s)
        cases.append((C, oracle.gemm(A, B), np.float32))
    C = c32()
    L.pax_gemm_tma_cluster_launch(tA.data_ptr(), tB.data_ptr(), C.data_ptr(), M, N, K, None, None, None, s)
    cases.append((C, oracle.gemm(A, B), np.float32))
    C = c32()
    L.pax_gemm_bias_gelu_launch(tA.data_ptr(), tB.data_ptr(), C.data_ptr(), M, N, K, tb.data_ptr(), s)
    cases.append((C, oracle.gemm(A, B, "bias_gelu_tanh", bias=bias), np.float32))
    C = c32()
    L.pax_gemm_residual_gelu_launch(tA.data_ptr(), tB.data_ptr(), C.data_ptr(), M, N, K, tr32.data_ptr(), s)
    cases.append((C, oracle.gemm(A, B, "residual_gelu_tanh", residual=res32), np.float32))
    C = c32()
    L.pax_gemm_scale_bias_gelu_launch(tA.data_ptr(), tB.data_ptr(), C.data_ptr(), M, N, K, 0.25, tb.data_ptr(), s)
    cases.append((C, oracle.gemm(A, B, "bias_gelu_tanh", alpha=0.25, bias=bias), np.float32))
    C = c16()
    L.pax_gemm_f16_launch(tA.data_ptr(), tB.data_ptr(), C.data_ptr(), M, N, K, s)
    cases.append((C, oracle.gemm(A, B, out_dtype=np.float16), np.float16))
    for name, epi in (("pax_gemm_bias_f16_launch", "bias"), ("pax_gemm_bias_gelu_f16_launch", "bias_gelu_tanh"),
                      ("pax_gemm_bias_gelu_erf_f16_launch", "bias_gelu_erf")):
        C = c16()
        getattr(L, name)(tA.data_ptr(), tB.data_ptr(), C.data_ptr(), M, N, K, tb.data_ptr(), s)
        cases.append((C, oracle.gemm(A, B, epi, bias=bias, out_dtype=np.float16), np.float16))
    for name, epi in (("pax_gemm_residual_gelu_f16_launch", "residual_gelu_tanh"),
                      ("pax_gemm_residual_gelu_erf_f16_launch", "residual_gelu_erf")):
        C = c16()
        getattr(L, name)(tA.data_ptr(), tB.data_ptr(), C.data_ptr(), M, N, K, tr16.data_ptr(), s)
        cases.append((C, oracle.gemm(A, B, epi, residual=res16, out_dtype=np.float16), np.float16))
    torch.cuda.synchronize()
    for C, ref, dt in cases:
        check(C.cpu().numpy(), ref, dt)
    assert L.pax_last_error() == 0


def test_dispatchers_with_library_buffers(cuda, rng):
    """pax_alloc_device_2d + pax_dispatch_* as a reference caller uses them."""
    L = pax_b200.lib
    M, N, K = 192, 256, 128
    A, B = inputs(rng, M, N, K)
    bias = rng.standard_normal(N).astype(np.float16)
    s = stream_ptr()
    bA = L.pax_alloc_device_2d(M, K, 2, s)
    bB = L.pax_alloc_device_2d(K, N, 2, s)
    bC = L.pax_alloc_device_2d(M, N, 4, s)
    bBias = L.pax_alloc_device_1d(N, 2, s)
    try:
        assert bA.base and bB.base and bC.base and bBias.base
        for buf, arr in ((bA, A), (bB, B), (bBias, bias)):
            dev_view(buf.base, arr.shape, np.float16).copy_(torch.from_numpy(arr))
        L.pax_dispatch_bias_gelu(ctypes.byref(bA), ctypes.byref(bB), ctypes.byref(bC), bBias.base, s)
        torch.cuda.synchronize()
        out = dev_view(bC.base, (M, N), np.float32).cpu().numpy()
        check(out, oracle.gemm(A, B, "bias_gelu_tanh", bias=bias), np.float32)
        L.pax_dispatch_pipeline_gemm(ctypes.byref(bA), ctypes.byref(bB), ctypes.byref(bC), s)
        torch.cuda.synchronize()
        out = dev_view(bC.base, (M, N), np.float32).cpu().numpy()
        check(out, oracle.gemm(A, B), np.float32)
        # fp16 C through the same dispatcher: elem_size 2 selects fp16 output
        bC16 = L.pax_alloc_device_2d(M, N, 2, s)
        try:
            L.pax_dispatch_wmma_gemm(ctypes.byref(bA), ctypes.byref(bB), ctypes.byref(bC16), s)
            torch.cuda.synchronize()
            out16 = dev_view(bC16.base, (M, N), np.float16).cpu().numpy()
            check(out16, oracle.gemm(A, B, out_dtype=np.float16), np.float16)
        finally:
            L.pax_free_device(ctypes.byref(bC16))
    finally:
        for b in (bA, bB, bC, bBias):
            L.pax_free_device(ctypes.byref(b))


def test_strided_operands(cuda, rng):
    """Row pitches larger than the row (sub-matrix views) are honoured."""
    M, N, K = 256, 384, 256
    bigA = rng.uniform(-1, 1, (M, K + 64)).astype(np.float16)
    bigB = rng.uniform(-1, 1, (K, N + 128)).astype(np.float16)
    tA = to_dev(bigA, cuda)[:, 32:32 + K]
    tB = to_dev(bigB, cuda)[:, 64:64 + N]
    outbig = torch.zeros((M, N + 64), dtype=torch.float16, device=cuda)
    C = outbig[:, :N]
    pax_b200.gemm(tA, tB, out=C)
    torch.cuda.synchronize()
    check(C.cpu().numpy(), oracle.gemm(bigA[:, 32:32 + K].copy(), bigB[:, 64:64 + N].copy(), out_dtype=np.float16),
          np.float16)
    assert (outbig[:, N:] == 0).all()


# ---------------------------------------------------------------- properties
def test_gelu_bound_on_device(cuda, rng):
    """|GeLU_tanh - GeLU_exact| <= 1e-3 |x| on the kernel's own fp32 values."""
    M, N, K = 256, 512, 512
    A, B = inputs(rng, M, N, K)
    bias = rng.standard_normal(N).astype(np.float16)
    x = run_gemm(A, B, cuda, epi="bias", bias=bias, out_dtype=np.float32)
    t = run_gemm(A, B, cuda, epi="bias_gelu_tanh", bias=bias, out_dtype=np.float32)
    e = run_gemm(A, B, cuda, epi="bias_gelu_erf", bias=bias, out_dtype=np.float32)
    assert (np.abs(t - e) <= 1e-3 * np.abs(x) + 1e-6).all()


@pytest.mark.parametrize("algo", ["tc", "tc2"])
def test_gelu_bound_on_device_fp16(cuda, rng, algo):
    """fp16 results (hardware tanh in the GeLU-tanh epilogue): the bound holds
    up to the fp16 rounding of the two outputs compared."""
    M, N, K = 512, 512, 512
    A, B = inputs(rng, M, N, K)
    bias = rng.standard_normal(N).astype(np.float16)
    x = run_gemm(A, B, cuda, epi="bias", bias=bias, out_dtype=np.float32, algo=algo)
    t = run_gemm(A, B, cuda, epi="bias_gelu_tanh", bias=bias, out_dtype=np.float16, algo=algo).astype(np.float32)
    e = run_gemm(A, B, cuda, epi="bias_gelu_erf", bias=bias, out_dtype=np.float16, algo=algo).astype(np.float32)
    assert (np.abs(t - e) <= 1e-3 * np.abs(x) + 2.0 ** -10 * (np.abs(t) + np.abs(e)) + 1e-6).all()


@pytest.mark.parametrize("algo,M", [("tc", 1024), ("tc2", 1024), ("skinny", 16)])
def test_deterministic(cuda, rng, algo, M):
    N, K = 4096, 2048
    A, B = inputs(rng, M, N, K)
    tA, tB = to_dev(A, cuda), to_dev(B, cuda)
    c1 = pax_b200.gemm(tA, tB, algo=algo)
    c2 = pax_b200.gemm(tA, tB, algo=algo)
    torch.cuda.synchronize()
    assert torch.equal(c1.view(torch.int16), c2.view(torch.int16))


def test_no_device_errors_recorded(cuda):
    assert pax_b200.device_error() == pax_b200.Status.OK


TAIL_SHAPES = [((4096, 4096, 512), "tc2"), ((4096, 4096, 512), "256"), ((4096, 4096, 512), "128"),
               ((1024, 1024, 1024), "128"), ((1024, 1024, 1024), "tc2"), ((2304, 1280, 200), "tc2"),
               ((300, 520, 136), "256"), ((2400, 1352, 72), "128"), ((4096, 4096, 512), "wide"),
               ((2304, 1280, 200), "wide"), ((300, 1040, 136), "wide"), ((9984, 3592, 64), "wide")]


def _force_tile(monkeypatch, algo):
    """'tc2' = CTA pair; 'wide' = CTA pair with 256 x 512 tiles; '128' /
    '256' = one-CTA tile width."""
    if algo == "tc2":
        return "tc2"
    if algo == "wide":
        monkeypatch.setenv("PAX_TC_SHAPE", "4")
        return "auto"
    monkeypatch.setenv("PAX_TC_BN", algo)
    return "tc"


@pytest.mark.parametrize("shape,algo", TAIL_SHAPES)
@pytest.mark.parametrize("epi", ["bias_gelu_tanh", "residual_gelu_erf"])
def test_tail_wave_halves(cuda, rng, monkeypatch, shape, algo, epi):
    """Tiles of the tail wave run as two column halves (MMA N = BN/2); the
    shapes leave a partial last wave, ragged edges and odd k-block counts."""
    algo = _force_tile(monkeypatch, algo)
    M, N, K = shape
    A, B = inputs(rng, M, N, K)
    bias = rng.standard_normal(N).astype(np.float16)
    res = rng.standard_normal((M, N)).astype(np.float16)
    for out in (np.float16, np.float32):
        got = run_gemm(A, B, cuda, epi=epi, bias=bias, residual=res, out_dtype=out, algo=algo)
        check(got, oracle.gemm(A, B, epi=epi, bias=bias, residual=res, out_dtype=out), out)


@pytest.mark.parametrize("algo", ["tc2", "wide", "256", "128"])
def test_tail_wave_halves_bit_exact_and_same_as_whole(cuda, rng, monkeypatch, algo):
    """Integer-valued inputs: every output exact, and identical with the
    tail halves switched off (PAX_TC_HALVES=0)."""
    algo = _force_tile(monkeypatch, algo)
    A = rng.integers(-3, 4, (768, 1024)).astype(np.float16)
    B = rng.integers(-3, 4, (1024, 1288)).astype(np.float16)
    exact = (A.astype(np.int64) @ B.astype(np.int64)).astype(np.float32)
    first = run_gemm(A, B, cuda, out_dtype=np.float32, algo=algo)
    assert np.array_equal(first, exact)
    monkeypatch.setenv("PAX_TC_HALVES", "0")
    assert np.array_equal(run_gemm(A, B, cuda, out_dtype=np.float32, algo=algo), first)


@pytest.mark.parametrize("epi", ["none", "bias", "bias_gelu_tanh", "bias_gelu_erf", "residual_gelu_tanh",
                                 "residual_gelu_erf"])
@pytest.mark.parametrize("out", [np.float16, np.float32])
@pytest.mark.parametrize("shape", [(512, 1024, 256), (1000, 1480, 328), (256, 512, 64)])
def test_wide_tile_epilogues(cuda, rng, monkeypatch, epi, out, shape):
    """The 256 x 512 CTA-pair tile: every epilogue, both output types, whole
    and ragged tiles."""
    monkeypatch.setenv("PAX_TC_SHAPE", "4")
    M, N, K = shape
    A, B = inputs(rng, M, N, K)
    bias = rng.standard_normal(N).astype(np.float16)
    res = rng.standard_normal((M, N)).astype(np.float16)
    got = run_gemm(A, B, cuda, epi=epi, bias=bias, residual=res, out_dtype=out)
    check(got, oracle.gemm(A, B, epi=epi, bias=bias, residual=res, out_dtype=out), out)


def test_lean_extraction_gemm_symbols(cuda, rng):
    """pax_gemm_*_verified (pax-lean4/PAX/Extraction.lean:32-56): 64-bit sizes,
    device pointers as integers, fp32 C, on the legacy default stream."""
    M, N, K = 320, 264, 200
    A, B = inputs(rng, M, N, K)
    bias = rng.standard_normal(N).astype(np.float16)
    res32 = rng.standard_normal((M, N)).astype(np.float32)
    tA, tB, tb, tr = to_dev(A, cuda), to_dev(B, cuda), to_dev(bias, cuda), to_dev(res32, cuda)
    L = pax_b200.lib
    torch.cuda.synchronize()
    outs = []
    for name in ("pax_gemm_wmma_verified", "pax_gemm_ptx_verified", "pax_gemm_pipeline3_verified"):
        C = torch.full((M, N), float("nan"), dtype=torch.float32, device=cuda)
        torch.cuda.synchronize()
        getattr(L, name)(M, N, K, tA.data_ptr(), tB.data_ptr(), C.data_ptr())
        outs.append((C, oracle.gemm(A, B)))
    C = torch.full((M, N), float("nan"), dtype=torch.float32, device=cuda)
    torch.cuda.synchronize()
    L.pax_gemm_bias_gelu_verified(M, N, K, tA.data_ptr(), tB.data_ptr(), C.data_ptr(), tb.data_ptr())
    outs.append((C, oracle.gemm(A, B, "bias_gelu_tanh", bias=bias)))
    C = torch.full((M, N), float("nan"), dtype=torch.float32, device=cuda)
    torch.cuda.synchronize()
    L.pax_gemm_residual_gelu_verified(M, N, K, tA.data_ptr(), tB.data_ptr(), C.data_ptr(), tr.data_ptr())
    outs.append((C, oracle.gemm(A, B, "residual_gelu_tanh", residual=res32)))
    torch.cuda.synchronize()
    assert pax_b200.last_error() == pax_b200.Status.OK
    for got, ref in outs:
        check(got.cpu().numpy(), ref, np.float32)


# ---------------------------------------------------------------- batched
def _batched_case(rng, nb, M, N, K, shared_b=False):
    A = rng.uniform(-1, 1, (nb, M, K)).astype(np.float16)
    B = rng.uniform(-1, 1, (K, N) if shared_b else (nb, K, N)).astype(np.float16)
    bias = rng.standard_normal((nb, N)).astype(np.float16)
    res = rng.standard_normal((nb, M, N)).astype(np.float16)
    return A, B, bias, res


@pytest.mark.parametrize("nb,M,N,K", [(3, 300, 520, 136), (4, 256, 512, 256), (2, 1000, 1480, 328), (5, 16, 1024, 512),
                                      (3, 40, 136, 72), (2, 17, 33, 31)])
@pytest.mark.parametrize("epi", ["none", "bias_gelu_tanh", "residual_gelu_erf"])
@pytest.mark.parametrize("out", [np.float16, np.float32])
def test_batched_gemm(cuda, rng, nb, M, N, K, epi, out):
    """pax_gemm_batched_ex: one tcgen05 launch over a 3-D tensor-map batch,
    or per-item launches for m <= 64 and unaligned shapes; per-item bias and
    residual."""
    A, B, bias, res = _batched_case(rng, nb, M, N, K)
    tA, tB, tb, tr = (to_dev(x, cuda) for x in (A, B, bias, res))
    td = torch.float16 if out == np.float16 else torch.float32
    C = pax_b200.gemm_batched(tA, tB, epilogue=epi, bias=tb if "bias" in epi else None,
                              residual=tr if "residual" in epi else None, out_dtype=td)
    got = C.cpu().numpy()
    for b in range(nb):
        ref = oracle.gemm(A[b], B[b], epi=epi, bias=bias[b], residual=res[b], out_dtype=out)
        check(got[b], ref, out)


def test_batched_shared_weights_and_padded_items(cuda, rng):
    """B shared by all items (stride 0), A items with padding between them
    (a slice of a taller tensor), C items with padding too."""
    nb, M, N, K = 3, 384, 640, 192
    A_big = rng.uniform(-1, 1, (nb, M + 8, K)).astype(np.float16)
    A = A_big[:, :M, :]
    _, B, bias, _ = _batched_case(rng, nb, M, N, K, shared_b=True)
    tA = to_dev(A_big, cuda)[:, :M, :]
    tB, tb = to_dev(B, cuda), to_dev(bias[0], cuda)
    C_big = torch.zeros((nb, M + 16, N), dtype=torch.float16, device=cuda)
    pax_b200.gemm_batched(tA, tB, epilogue="bias_gelu_tanh", bias=tb, out=C_big[:, :M, :])
    got = C_big.cpu().numpy()
    for b in range(nb):
        check(got[b, :M], oracle.gemm(A[b], B, epi="bias_gelu_tanh", bias=bias[0], out_dtype=np.float16), np.float16)
        assert not got[b, M:].any()  # padding rows untouched


@pytest.mark.parametrize("algo", ["tc2", "wide", "256", "128"])
def test_batched_bit_exact_every_tile_shape(cuda, rng, monkeypatch, algo):
    """Integer-valued inputs through each tile shape with batch items that
    split across waves (and a column-half tail): exact."""
    algo = _force_tile(monkeypatch, algo)
    nb, M, N, K = 5, 512, 1040, 256
    A = rng.integers(-3, 4, (nb, M, K)).astype(np.float16)
    B = rng.integers(-3, 4, (nb, K, N)).astype(np.float16)
    C = pax_b200.gemm_batched(to_dev(A, cuda), to_dev(B, cuda), out_dtype=torch.float32, algo=algo)
    exact = np.einsum("bmk,bkn->bmn", A.astype(np.int64), B.astype(np.int64)).astype(np.float32)
    assert np.array_equal(C.cpu().numpy(), exact)


def test_batched_rejects_overlapping_outputs(cuda):
    A = torch.zeros((2, 64, 64), dtype=torch.float16, device=cuda)
    B = torch.zeros((2, 64, 64), dtype=torch.float16, device=cuda)
    C = torch.zeros((64 * 64 + 64,), dtype=torch.float16, device=cuda)
    bad = C.as_strided((2, 64, 64), (64, 64, 1))  # item 1 starts one row after item 0
    with pytest.raises(pax_b200.PaxError):
        pax_b200.gemm_batched(A, B, out=bad)


@pytest.mark.parametrize("algo", ["tc2", "wide", "256", "128"])
@pytest.mark.parametrize("out", [np.float16, np.float32])
def test_replicated_output_to_local_buffers(cuda, rng, monkeypatch, algo, out):
    """pax_gemm_replicated_ex with replicas in this GPU's memory: every
    replica, with the same pitch as C (here a column slab of a wider buffer),
    holds exactly C; the bytes around the slab are untouched."""
    algo = _force_tile(monkeypatch, algo)
    M, N, K, W = 640, 520, 136, 1040
    A, B = inputs(rng, M, N, K)
    bias = rng.standard_normal(N).astype(np.float16)
    td = torch.float16 if out == np.float16 else torch.float32
    full = [torch.zeros((M, W), dtype=td, device=cuda) for _ in range(4)]
    C = full[0][:, 8:8 + N]
    reps = [f[:, 8:8 + N].data_ptr() for f in full[1:]]
    pax_b200.gemm(to_dev(A, cuda), to_dev(B, cuda), epilogue="bias_gelu_tanh", bias=to_dev(bias, cuda), out=C,
                  algo=algo, replicas=reps)
    ref = oracle.gemm(A, B, epi="bias_gelu_tanh", bias=bias, out_dtype=out)
    got = [f.cpu().numpy() for f in full]
    check(got[0][:, 8:8 + N], ref, out)
    for g in got[1:]:
        assert np.array_equal(g, got[0])


def test_replicated_output_rejects_skinny(cuda):
    A = torch.zeros((16, 256), dtype=torch.float16, device=cuda)
    B = torch.zeros((256, 512), dtype=torch.float16, device=cuda)
    C = torch.zeros((16, 512), dtype=torch.float16, device=cuda)
    R = torch.zeros((16, 512), dtype=torch.float16, device=cuda)
    with pytest.raises(pax_b200.PaxError):
        pax_b200.gemm(A, B, out=C, replicas=[R.data_ptr()])


# ------------------------------------------------ chained launches (PDL)
@pytest.mark.parametrize("m1,m2", [(512, 768), (16, 16), (512, 16), (16, 1024)])
def test_back_to_back_dependent_gemms(cuda, rng, m1, m2):
    """Kernels launched with programmatic dependent launch start their
    prologue while the previous kernel runs.  A chain where each GEMM reads
    the previous one's output (RAW), then overwrites a buffer the previous
    one read (WAR), queued without synchronisation, must match the oracle
    run step by step.  Shapes mix the skinny and tcgen05 kernels."""
    K0, N1, N2 = 256, 512, 384
    A0 = rng.uniform(-1, 1, (m1, K0)).astype(np.float16)
    B1 = (rng.uniform(-1, 1, (K0, N1)) / 8).astype(np.float16)
    B2 = (rng.uniform(-1, 1, (N1, N2)) / 8).astype(np.float16)
    B3 = (rng.uniform(-1, 1, (K0, N1)) / 8).astype(np.float16)
    tA0, tB1, tB2, tB3 = (to_dev(x, cuda) for x in (A0, B1, B2, B3))
    C1 = torch.empty((m1, N1), dtype=torch.float16, device=cuda)
    for _ in range(3):
        torch.cuda.synchronize()
        pax_b200.gemm(tA0, tB1, out=C1)                     # C1 = A0 B1
        C2 = pax_b200.gemm(C1[:m2] if m2 <= m1 else C1.repeat(1, 1)[:m2], tB2)  # reads C1 (RAW)
        pax_b200.gemm(tA0, tB3, out=C1)                     # overwrites C1 after C2 read it (WAR)
        torch.cuda.synchronize()
        ref1 = oracle.gemm(A0, B1, out_dtype=np.float16)
        ref2 = oracle.gemm(ref1[:m2], B2, out_dtype=np.float16)
        ref3 = oracle.gemm(A0, B3, out_dtype=np.float16)
        check(C2.cpu().numpy(), ref2, np.float16)
        check(C1.cpu().numpy(), ref3, np.float16)


def test_long_dependent_chain(cuda, rng):
    """Twelve GEMMs, each consuming the previous output, alternating the
    skinny (m = 16) and tcgen05 (m = 384) kernels through a residual."""
    N = 256
    Bs = [(rng.uniform(-1, 1, (N, N)) / 16).astype(np.float16) for _ in range(12)]
    X0 = rng.uniform(-1, 1, (384, N)).astype(np.float16)
    tB = [to_dev(b, cuda) for b in Bs]
    X = to_dev(X0, cuda)
    ref = X0
    torch.cuda.synchronize()
    for i in range(12):
        rows = 16 if i % 2 else 384
        Y = pax_b200.gemm(X[:rows], tB[i], epilogue="residual_gelu_tanh", residual=X[:rows])
        ref_y = oracle.gemm(ref[:rows], Bs[i], epi="residual_gelu_tanh", residual=ref[:rows], out_dtype=np.float16)
        if rows == 384:
            X, ref = Y, ref_y
        else:
            X = torch.cat([Y, X[16:]])
            ref = np.concatenate([ref_y, ref[16:]])
    torch.cuda.synchronize()
    check(X.cpu().numpy(), ref, np.float16)


@pytest.mark.parametrize("M,N,K", [(4096, 4096, 512), (4736, 4096, 256), (3000, 5000, 128), (1000, 1480, 328),
                                   (2304, 2560, 200), (520, 8200, 64)])
def test_planned_wide_tiling_bit_exact(cuda, rng, monkeypatch, M, N, K):
    """Wide tiles re-planned as mixed 512 / 384 / 256-column items (the
    host's per-pair work table): integer-valued inputs give exact results,
    identical to the round-robin schedule (PAX_TC_PLAN=0), ragged edges
    included."""
    monkeypatch.setenv("PAX_TC_SHAPE", "4")
    A = rng.integers(-3, 4, (M, K)).astype(np.float16)
    B = rng.integers(-3, 4, (K, N)).astype(np.float16)
    exact = (A.astype(np.int64) @ B.astype(np.int64)).astype(np.float32)
    planned = run_gemm(A, B, cuda, out_dtype=np.float32)
    assert np.array_equal(planned, exact)
    monkeypatch.setenv("PAX_TC_PLAN", "0")
    assert np.array_equal(run_gemm(A, B, cuda, out_dtype=np.float32), planned)


@pytest.mark.parametrize("epi", ["bias_gelu_tanh", "residual_gelu_erf"])
@pytest.mark.parametrize("out", [np.float16, np.float32])
def test_planned_wide_tiling_epilogues(cuda, rng, monkeypatch, epi, out):
    monkeypatch.setenv("PAX_TC_SHAPE", "4")
    M, N, K = 3000, 5000, 128
    A, B = inputs(rng, M, N, K)
    bias = rng.standard_normal(N).astype(np.float16)
    res = rng.standard_normal((M, N)).astype(np.float16)
    got = run_gemm(A, B, cuda, epi=epi, bias=bias, residual=res, out_dtype=out)
    check(got, oracle.gemm(A, B, epi=epi, bias=bias, residual=res, out_dtype=out), out)


@pytest.mark.parametrize("M", [16, 48])
def test_b_const_chain(cuda, rng, M):
    """PAX_GEMM_B_CONST (weights not written by the previous kernel): a chain
    of skinny GEMMs where each reads the previous output as A and its own
    constant B, launched back to back, matches the oracle step by step."""
    N = 512
    Bs = [(rng.uniform(-1, 1, (N, N)) / 16).astype(np.float16) for _ in range(6)]
    tB = [to_dev(b, cuda) for b in Bs]
    X0 = rng.uniform(-1, 1, (M, N)).astype(np.float16)
    X = to_dev(X0, cuda)
    ref = X0
    torch.cuda.synchronize()
    for i in range(6):
        X = pax_b200.gemm(X, tB[i], b_const=True)
        ref = oracle.gemm(ref, Bs[i], out_dtype=np.float16)
    torch.cuda.synchronize()
    check(X.cpu().numpy(), ref, np.float16)


@pytest.mark.parametrize("shared", ["none", "A", "B"])
@pytest.mark.parametrize("M", [1, 16, 64])
def test_batched_skinny_single_launch(cuda, rng, shared, M):
    """Batched m <= 64 problems in one skinny-kernel launch (whole (item,
    tile) units round-robin over the SMs): per-item bias and residual, and
    A or B shared by every item (stride 0)."""
    nb, N, K = 5, 640, 256
    A = rng.standard_normal((M, K) if shared == "A" else (nb, M, K)).astype(np.float16)
    B = (rng.standard_normal((K, N) if shared == "B" else (nb, K, N)) * 0.05).astype(np.float16)
    bias = rng.standard_normal((nb, N)).astype(np.float16)
    res = rng.standard_normal((nb, M, N)).astype(np.float16)
    C = pax_b200.gemm_batched(to_dev(A, cuda), to_dev(B, cuda), epilogue="residual_gelu_tanh",
                              residual=to_dev(res, cuda))
    got = C.cpu().numpy()
    C2 = pax_b200.gemm_batched(to_dev(A, cuda), to_dev(B, cuda), epilogue="bias", bias=to_dev(bias, cuda),
                               out_dtype=torch.float32)
    got2 = C2.cpu().numpy()
    for b in range(nb):
        a = A if shared == "A" else A[b]
        bb = B if shared == "B" else B[b]
        check(got[b], oracle.gemm(a, bb, epi="residual_gelu_tanh", residual=res[b], out_dtype=np.float16),
              np.float16)
        check(got2[b], oracle.gemm(a, bb, epi="bias", bias=bias[b], out_dtype=np.float32), np.float32)


@pytest.mark.parametrize("algo", ["tc2", "wide", "256", "128"])
def test_residual_staged_by_tma_matches_lane_loads(cuda, rng, monkeypatch, algo):
    """fp16 residual with fp16 C: residual chunks staged in shared memory by
    TMA give the same bits as per-lane global loads (PAX_TC_RES_TMA=0), with
    ragged edges and a residual that is a column slice of a wider tensor."""
    algo = _force_tile(monkeypatch, algo)
    M, N, K = 600, 1000, 264
    A, B = inputs(rng, M, N, K)
    wide = rng.standard_normal((M, N + 24)).astype(np.float16)
    tr = to_dev(wide, cuda)[:, 8:8 + N]
    res = wide[:, 8:8 + N]
    tA, tB = to_dev(A, cuda), to_dev(B, cuda)
    outs = []
    for flag in ("1", "0"):
        monkeypatch.setenv("PAX_TC_RES_TMA", flag)
        C = pax_b200.gemm(tA, tB, epilogue="residual_gelu_erf", residual=tr, out_dtype=torch.float16, algo=algo)
        outs.append(C.cpu().numpy())
    check(outs[0], oracle.gemm(A, B, epi="residual_gelu_erf", residual=res, out_dtype=np.float16), np.float16)
    assert np.array_equal(outs[0].view(np.uint16), outs[1].view(np.uint16))


def test_batched_shared_residual(cuda, rng):
    """One [M, N] residual shared by every batch item (stride 0)."""
    nb, M, N, K = 3, 384, 640, 192
    A, B, _, res = _batched_case(rng, nb, M, N, K)
    tA, tB, tr = to_dev(A, cuda), to_dev(B, cuda), to_dev(res[0], cuda)
    C = pax_b200.gemm_batched(tA, tB, epilogue="residual_gelu_tanh", residual=tr, out_dtype=torch.float16)
    got = C.cpu().numpy()
    for b in range(nb):
        check(got[b], oracle.gemm(A[b], B[b], epi="residual_gelu_tanh", residual=res[0], out_dtype=np.float16),
              np.float16)
