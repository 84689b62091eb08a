// fp16_ops.cpp -- host IEEE-754 binary16 add / mul / fma with one
// round-to-nearest-even, the scalar operations PAX's Lean layer exports as
// pax_fp16_{add,mul,fma}_verified (pax-lean4/PAX/Extraction.lean:58-84,
// specified by Float16.add/mul/fma in pax-lean4/PAX/Float16.lean:99-125 and
// the RNE algorithm of pax-lean4/PAX/Float16_Rounding.lean:92-141).
//
// Every finite binary16 value is sig * 2^e with an 11-bit integer sig and
// e >= -24, so the exact sum, product and product-plus-addend are integers
// times a power of two that fit in 128 bits (the widest, an fma, needs 81).
// The exact value is then rounded once.
//
// Results follow IEEE 754-2019 for values, signed zeros, subnormals and
// overflow (|x| >= 65520 rounds to infinity).  A NaN result is the
// reference's encoding Float16.posNaN = 0x7C01.  Where the Lean
// specification's rational model cannot express IEEE behaviour, IEEE is
// followed:
//   - the sign of zero results, e.g. -0 * 3 = -0 and -0 + -0 = -0;
//   - infinities inside an fma;
//   - the overflow threshold, which is 65520, not 65504.
#include <stdint.h>

namespace {

constexpr uint16_t kNaN = 0x7C01;  // Float16.posNaN
constexpr uint16_t kInf = 0x7C00;

struct Dec {
    bool neg, nan, inf, zero;
    uint32_t sig;  // value = sig * 2^exp (finite, non-zero)
    int exp;
};

Dec decode(uint16_t h) {
    Dec d{};
    d.neg = (h >> 15) != 0;
    const uint32_t e = (h >> 10) & 31u, m = h & 1023u;
    if (e == 31) {
        d.nan = m != 0;
        d.inf = m == 0;
        return d;
    }
    if (e == 0) {
        d.zero = m == 0;
        d.sig = m;
        d.exp = -24;
    } else {
        d.sig = 1024u + m;
        d.exp = (int)e - 25;
    }
    return d;
}

int bit_length(unsigned __int128 v) {
    int n = 0;
    while (v) {
        v >>= 1;
        ++n;
    }
    return n;
}

// Round-to-nearest-even of the non-zero value mag * 2^exp (sign `neg`).
uint16_t round_half(bool neg, unsigned __int128 mag, int exp) {
    const uint16_t s = neg ? 0x8000u : 0u;
    const int p = bit_length(mag) - 1 + exp;  // value in [2^p, 2^(p+1))
    // Quantum of the result: 2^(p-10) for normals, 2^-24 below 2^-14.
    const int qexp = p >= -14 ? p - 10 : -24;
    const int shift = qexp - exp;  // bits of mag below the quantum
    unsigned __int128 q;
    if (shift <= 0) {
        q = mag << (-shift);
    } else if (shift >= 127) {
        q = 0;  // far below half a quantum (not reachable from binary16 inputs)
    } else {
        q = mag >> shift;
        const unsigned __int128 rem = mag & ((((unsigned __int128)1) << shift) - 1);
        const unsigned __int128 half = ((unsigned __int128)1) << (shift - 1);
        if (rem > half || (rem == half && (q & 1))) ++q;
    }
    if (p < -14) return (uint16_t)(s | (uint16_t)q);  // subnormal; q = 1024 is the smallest normal
    int E = p + 15;
    if (q == 2048) {  // the mantissa carried into the exponent
        q = 1024;
        ++E;
    }
    if (E >= 31) return (uint16_t)(s | kInf);
    return (uint16_t)(s | (uint16_t)(E << 10) | (uint16_t)(q - 1024));
}

// Exact signed sum of a*2^ea and b*2^eb (a, b signed magnitudes), rounded.
// zero_neg: sign of an exact zero result.
uint16_t sum_round(__int128 a, int ea, __int128 b, int eb, bool zero_neg) {
    const int e = ea < eb ? ea : eb;
    const __int128 v = a * (((__int128)1) << (ea - e)) + b * (((__int128)1) << (eb - e));
    if (v == 0) return zero_neg ? 0x8000u : 0u;
    return v < 0 ? round_half(true, (unsigned __int128)(-v), e) : round_half(false, (unsigned __int128)v, e);
}

__int128 signed_sig(const Dec& d) { return d.neg ? -(__int128)d.sig : (__int128)d.sig; }

}  // namespace

extern "C" {

uint16_t pax_fp16_add_verified(uint16_t x, uint16_t y) {
    const Dec a = decode(x), b = decode(y);
    if (a.nan || b.nan) return kNaN;
    if (a.inf || b.inf) {
        if (a.inf && b.inf && a.neg != b.neg) return kNaN;
        return a.inf ? x : y;
    }
    if (a.zero && b.zero) return (a.neg && b.neg) ? 0x8000u : 0u;
    if (a.zero) return y;
    if (b.zero) return x;
    // An exact zero from opposite operands is +0 under round-to-nearest.
    return sum_round(signed_sig(a), a.exp, signed_sig(b), b.exp, false);
}

uint16_t pax_fp16_mul_verified(uint16_t x, uint16_t y) {
    const Dec a = decode(x), b = decode(y);
    if (a.nan || b.nan) return kNaN;
    const bool neg = a.neg != b.neg;
    if ((a.inf && b.zero) || (a.zero && b.inf)) return kNaN;
    if (a.inf || b.inf) return (uint16_t)((neg ? 0x8000u : 0u) | kInf);
    if (a.zero || b.zero) return neg ? 0x8000u : 0u;
    return round_half(neg, (unsigned __int128)a.sig * b.sig, a.exp + b.exp);
}

uint16_t pax_fp16_fma_verified(uint16_t x, uint16_t y, uint16_t z) {
    const Dec a = decode(x), b = decode(y), c = decode(z);
    if (a.nan || b.nan || c.nan) return kNaN;
    const bool pneg = a.neg != b.neg;
    if ((a.inf && b.zero) || (a.zero && b.inf)) return kNaN;
    const bool pinf = a.inf || b.inf;
    if (pinf || c.inf) {
        if (pinf && c.inf && pneg != c.neg) return kNaN;
        return pinf ? (uint16_t)((pneg ? 0x8000u : 0u) | kInf) : z;
    }
    const bool pzero = a.zero || b.zero;
    if (pzero && c.zero) return (pneg && c.neg) ? 0x8000u : 0u;
    if (pzero) return z;
    const __int128 p = pneg ? -(__int128)((unsigned __int128)a.sig * b.sig) : (__int128)a.sig * b.sig;
    if (c.zero) return round_half(pneg, (unsigned __int128)(pneg ? -p : p), a.exp + b.exp);
    return sum_round(p, a.exp + b.exp, signed_sig(c), c.exp, false);
}

}  // extern "C"
