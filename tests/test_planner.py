"""Host-only checks of the wide tile's planned work lists (gemm_tc.cu,
wide_plan), through pax_selftest_wide_plan: for every planned shape, each
256-row block's columns [0, N) are covered by exactly one item, items do not
overlap, and the per-pair lists partition the items.  No GPU needed."""
from __future__ import annotations

import ctypes

import pytest

import pax_b200

WIDTH = {0: 512, 1: 384, 2: 256, 3: 128}


def _plan(M, N, K, units):
    lib = pax_b200.lib
    f = lib.pax_selftest_wide_plan
    f.argtypes = [ctypes.c_longlong] * 3 + [ctypes.c_int, ctypes.POINTER(ctypes.c_uint), ctypes.POINTER(ctypes.c_int),
                                            ctypes.c_int]
    f.restype = ctypes.c_int
    items = (ctypes.c_uint * 1024)()
    starts = (ctypes.c_int * (units + 1))()
    n = f(M, N, K, units, items, starts, 1024)
    return n, list(items[:max(n, 0)]), list(starts)


@pytest.mark.parametrize("M,N,K,units", [
    (4096, 4096, 4096, 74),     # C2: the planned headline shape
    (4736, 4096, 4096, 74),
    (4096, 4096, 1024, 74),
    (2048, 8192, 4096, 74),
    (8192, 4096, 4096, 74),
    (4096, 4000, 4096, 74),     # ragged N
    (3000, 6144, 2048, 70),     # ragged M, fewer pairs
    (4096, 4096, 4096, 66),
    (1024, 16384, 4096, 74),
])
def test_planned_items_cover_every_column_once(M, N, K, units):
    n, items, starts = _plan(M, N, K, units)
    if n == 0:
        pytest.skip("not planned: round-robin tiles")
    assert n > 0
    assert starts[0] == 0 and starts[units] == n
    assert all(a <= b for a, b in zip(starts, starts[1:]))
    rows = (M + 255) // 256
    cover = {r: [] for r in range(rows)}
    for it in items:
        row, col, w = it & 0xFFFF, ((it >> 16) & 0xFFF) * 128, WIDTH[(it >> 28) & 3]
        assert row < rows
        cover[row].append((col, col + w))
    for r, spans in cover.items():
        spans.sort()
        assert spans, f"row block {r} has no items"
        assert spans[0][0] == 0
        for (a0, a1), (b0, b1) in zip(spans, spans[1:]):
            assert a1 == b0, f"row block {r}: gap or overlap at {a1}/{b0}"
        assert spans[-1][1] >= N and spans[-1][1] - N < 256, f"row block {r} ends at {spans[-1][1]} for N={N}"


def test_headline_shape_is_planned():
    n, items, starts = _plan(4096, 4096, 4096, 74)
    assert n > 0
    per_unit = [starts[u + 1] - starts[u] for u in range(74)]
    assert max(per_unit) <= 3


def test_plan_hook_rejects_bad_arguments():
    lib = pax_b200.lib
    f = lib.pax_selftest_wide_plan
    f.argtypes = [ctypes.c_longlong] * 3 + [ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int]
    f.restype = ctypes.c_int
    buf = (ctypes.c_uint * 8)()
    st = (ctypes.c_int * 80)()
    assert f(0, 4096, 4096, 74, buf, st, 8) == -1
    assert f(4096, 4096, 4096, 74, None, st, 8) == -1
    assert f(4096, 4096, 4096, 74, buf, st, 8) == -1  # 8 items is too small for the C2 plan
