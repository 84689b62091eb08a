"""pax_fp16_{add,mul,fma}_verified (pax-lean4/PAX/Extraction.lean:58-84)
against an exact rational oracle: every operand is converted to a Fraction,
the operation is done exactly, and the result is rounded to the nearest
binary16 by searching the table of all finite binary16 values (ties to the
even bit pattern; |v| >= 65520 overflows).  The library computes the same
thing by integer bit arithmetic, so the two share no code.
"""
from __future__ import annotations

import bisect
import random
from fractions import Fraction

import pytest

import pax_b200

NAN = 0x7C01  # Float16.posNaN of the Lean model


def value(h: int):
    """binary16 bits -> ('nan'|'inf', sign) or Fraction (signed zeros as ('zero', sign))."""
    s = -1 if h >> 15 else 1
    e, m = (h >> 10) & 31, h & 1023
    if e == 31:
        return ("nan", s) if m else ("inf", s)
    if e == 0 and m == 0:
        return ("zero", s)
    if e == 0:
        return s * Fraction(m, 1 << 24)
    return s * Fraction(1024 + m, 1 << 10) * (Fraction(2) ** (e - 15))


POS = [value(h) for h in range(1, 0x7C00)]  # strictly increasing positive finite values


def round16(v: Fraction, zero_negative: bool = False) -> int:
    if v == 0:
        return 0x8000 if zero_negative else 0
    sign = 0x8000 if v < 0 else 0
    a = abs(v)
    if a >= 65520:
        return sign | 0x7C00
    i = bisect.bisect_left(POS, a)  # POS[i] >= a; bit pattern i + 1
    if i < len(POS) and POS[i] == a:
        return sign | (i + 1)
    lo = i  # bits of the value below (pattern i), or 0 for zero
    lo_v = POS[i - 1] if i > 0 else Fraction(0)
    hi = i + 1
    hi_v = POS[i] if i < len(POS) else None
    if hi_v is None:
        return sign | lo
    dl, dh = a - lo_v, hi_v - a
    if dl < dh or (dl == dh and lo % 2 == 0):
        return sign | lo
    return sign | hi


def ref_add(x: int, y: int) -> int:
    a, b = value(x), value(y)
    if (isinstance(a, tuple) and a[0] == "nan") or (isinstance(b, tuple) and b[0] == "nan"):
        return NAN
    ainf = isinstance(a, tuple) and a[0] == "inf"
    binf = isinstance(b, tuple) and b[0] == "inf"
    if ainf or binf:
        if ainf and binf and a[1] != b[1]:
            return NAN
        return x if ainf else y
    az = isinstance(a, tuple)
    bz = isinstance(b, tuple)
    if az and bz:
        return 0x8000 if (a[1] < 0 and b[1] < 0) else 0
    va = Fraction(0) if az else a
    vb = Fraction(0) if bz else b
    return round16(va + vb)


def ref_mul(x: int, y: int) -> int:
    a, b = value(x), value(y)
    kinds = [t[0] if isinstance(t, tuple) else "fin" for t in (a, b)]
    signs = [t[1] if isinstance(t, tuple) else (1 if t > 0 else -1) for t in (a, b)]
    neg = signs[0] != signs[1]
    if "nan" in kinds:
        return NAN
    if "inf" in kinds and "zero" in kinds:
        return NAN
    if "inf" in kinds:
        return (0x8000 if neg else 0) | 0x7C00
    if "zero" in kinds:
        return 0x8000 if neg else 0
    return round16(a * b)


def ref_fma(x: int, y: int, z: int) -> int:
    a, b, c = value(x), value(y), value(z)
    kinds = [t[0] if isinstance(t, tuple) else "fin" for t in (a, b, c)]
    signs = [t[1] if isinstance(t, tuple) else (1 if t > 0 else -1) for t in (a, b, c)]
    if "nan" in kinds:
        return NAN
    pneg = signs[0] != signs[1]
    if ("inf" in kinds[:2]) and ("zero" in kinds[:2]):
        return NAN
    pinf = "inf" in kinds[:2]
    if pinf or kinds[2] == "inf":
        if pinf and kinds[2] == "inf" and pneg != (signs[2] < 0):
            return NAN
        return ((0x8000 if pneg else 0) | 0x7C00) if pinf else z
    pzero = "zero" in kinds[:2]
    if pzero and kinds[2] == "zero":
        return 0x8000 if (pneg and signs[2] < 0) else 0
    if pzero:
        return z
    p = a * b
    if kinds[2] == "zero":
        return round16(p)
    return round16(p + c)


SPECIAL = [0x0000, 0x8000, 0x0001, 0x8001, 0x03FF, 0x0400, 0x3C00, 0xBC00, 0x3C01, 0x7BFF, 0xFBFF, 0x7C00, 0xFC00,
           0x7C01, 0x7E00, 0x6800, 0x6801, 0x5BFF, 0x0200, 0x1400, 0x3555, 0x7800, 0x77FF]


def lib():
    return pax_b200._lib.get()


def test_fp16_ops_special_values_exhaustive():
    L = lib()
    for x in SPECIAL:
        for y in SPECIAL:
            assert L.pax_fp16_add_verified(x, y) == ref_add(x, y), (hex(x), hex(y))
            assert L.pax_fp16_mul_verified(x, y) == ref_mul(x, y), (hex(x), hex(y))
            for z in SPECIAL[::3]:
                assert L.pax_fp16_fma_verified(x, y, z) == ref_fma(x, y, z), (hex(x), hex(y), hex(z))


@pytest.mark.parametrize("seed", [1, 2])
def test_fp16_ops_random_bit_patterns(seed):
    L = lib()
    r = random.Random(seed)
    for _ in range(6000):
        x, y, z = r.getrandbits(16), r.getrandbits(16), r.getrandbits(16)
        assert L.pax_fp16_add_verified(x, y) == ref_add(x, y), (hex(x), hex(y))
        assert L.pax_fp16_mul_verified(x, y) == ref_mul(x, y), (hex(x), hex(y))
        assert L.pax_fp16_fma_verified(x, y, z) == ref_fma(x, y, z), (hex(x), hex(y), hex(z))


def test_fp16_ops_close_operands_and_ties():
    """Cancellation, halfway cases and results near the subnormal and
    overflow boundaries, where rounding errors would show."""
    L = lib()
    r = random.Random(7)
    for _ in range(4000):
        e = r.randrange(0, 31)
        x = (r.getrandbits(1) << 15) | (e << 10) | r.getrandbits(10)
        y = x ^ 0x8000 ^ r.getrandbits(3)  # nearly the negation of x
        z = (e << 10) | r.getrandbits(10)
        assert L.pax_fp16_add_verified(x, y) == ref_add(x, y), (hex(x), hex(y))
        assert L.pax_fp16_fma_verified(x, 0x3C00, y) == ref_fma(x, 0x3C00, y)
        assert L.pax_fp16_fma_verified(x, z, y) == ref_fma(x, z, y), (hex(x), hex(z), hex(y))
    # 2048 + 1 is a tie between 2048 and 2050: even mantissa (2048) wins.
    assert L.pax_fp16_add_verified(0x6800, 0x3C00) == 0x6800
    # 65504 + 8 is below the overflow threshold, 65504 + 16 reaches it.
    assert L.pax_fp16_add_verified(0x7BFF, 0x4800) == 0x7BFF
    assert L.pax_fp16_add_verified(0x7BFF, 0x4C00) == 0x7C00
