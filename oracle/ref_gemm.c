/*
 * ref_gemm.c -- CPU oracle for the pax_b200 GEMM path.
 *
 * TEST INFRASTRUCTURE ONLY.  Only tests/, __graft_entry__.smoke() and the
 * cpu_baseline leg of bench.py load this library, and only as the checker or
 * as the timed CPU baseline; no product code path calls it.
 *
 * Restates the reference's CPU verification path and the epilogue math:
 *   oracle_cpu_gemm_ref   src/host_bridge.c:397-407   i-j-l loop, fp32 acc
 *   oracle_verify         src/host_bridge.c:422-445   max |g-r|/(|r|+1e-8)
 *   oracle_gelu_tanh      src/rtx_gemm_epilogue.cu:76-80
 *   oracle_epilogue       src/rtx_gemm_epilogue.cu:7-10,176-233 with column
 *                         bias / element residual indexing as stated in
 *                         pax-lean4/PAX/Integration.lean:114-122
 *   fp16 widening         src/pax_kernel.fut:18-25 (f32(A)*f32(B), f32 sum)
 *
 * Parity is pinned by tests/golden (fixtures written by the reference's own
 * cpu_gemm_ref, compiled from its sources by oracle/Makefile into _ref/).
 * Build flags must match _ref's for bit-exact agreement: both use
 * -O3 -march=x86-64-v3 -ffp-contract=fast (fused multiply-add in the
 * accumulation, as gcc emits by default for the reference's -O3 build).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* ---------------------------------------------------------------- fp16 */

/* Exact fp16 -> fp32 widening (IEEE 754 binary16). */
float oracle_f16_to_f32(uint16_t h) {
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1Fu;
    uint32_t man = h & 0x3FFu;
    uint32_t bits;
    if (exp == 0x1Fu) {
        bits = sign | 0x7F800000u | (man << 13);
    } else if (exp != 0) {
        bits = sign | ((exp + 112u) << 23) | (man << 13);
    } else if (man == 0) {
        bits = sign;
    } else {
        /* subnormal: normalise */
        int e = -1;
        do {
            ++e;
            man <<= 1;
        } while ((man & 0x400u) == 0);
        man &= 0x3FFu;
        bits = sign | ((uint32_t)(112 - e) << 23) | (man << 13);
    }
    float f;
    memcpy(&f, &bits, sizeof f);
    return f;
}

/* fp32 -> fp16, round to nearest even, overflow to infinity, NaN kept quiet. */
uint16_t oracle_f32_to_f16(float f) {
    uint32_t x;
    memcpy(&x, &f, sizeof x);
    const uint16_t sign = (uint16_t)((x >> 16) & 0x8000u);
    const uint32_t ax = x & 0x7FFFFFFFu;
    if (ax >= 0x7F800000u) /* inf or nan */
        return (uint16_t)(sign | 0x7C00u | (ax > 0x7F800000u ? 0x200u : 0u));
    if (ax >= 0x477FF000u) /* rounds to >= 65520 -> inf */
        return (uint16_t)(sign | 0x7C00u);
    if (ax < 0x33000001u) /* < 2^-25 (half of the smallest subnormal) -> 0 */
        return sign;
    uint32_t exp = ax >> 23;
    uint32_t man = (ax & 0x7FFFFFu) | 0x800000u;
    int shift;
    if (exp < 113) { /* result is subnormal in fp16 */
        shift = (int)(126 - exp);  /* 14 + (113 - exp) - 1 */
    } else {
        shift = 13;
    }
    uint32_t keep = man >> shift;
    const uint32_t rem = man & ((1u << shift) - 1u);
    const uint32_t half = 1u << (shift - 1);
    if (rem > half || (rem == half && (keep & 1u))) ++keep;
    uint32_t out;
    if (exp < 113) {
        out = keep; /* may carry into the smallest normal: still correct */
    } else {
        out = ((exp - 112u) << 10) + (keep - 0x400u);
        /* keep - 0x400 may carry into the exponent: correct by construction */
    }
    return (uint16_t)(sign | out);
}

void oracle_f16_to_f32_array(const uint16_t* src, float* dst, int64_t n) {
    for (int64_t i = 0; i < n; ++i) dst[i] = oracle_f16_to_f32(src[i]);
}

void oracle_f32_to_f16_array(const float* src, uint16_t* dst, int64_t n) {
    for (int64_t i = 0; i < n; ++i) dst[i] = oracle_f32_to_f16(src[i]);
}

/* ---------------------------------------------------------------- GEMM */

/* Literal restatement of the reference loop: for each (i, j) a sequential
 * fp32 sum over l.  src/host_bridge.c:397-407. */
void oracle_cpu_gemm_ref(const float* A, const float* B, float* C, int m, int n, int k) {
    for (int i = 0; i < m; ++i) {
        for (int j = 0; j < n; ++j) {
            float acc = 0.f;
            for (int l = 0; l < k; ++l) acc += A[(size_t)i * k + l] * B[(size_t)l * n + j];
            C[(size_t)i * n + j] = acc;
        }
    }
}

/* Same per-element arithmetic as oracle_cpu_gemm_ref (each C[i][j] is the
 * sequential sum over l = 0..k-1 of A[i][l]*B[l][j], same contraction), but
 * the l loop runs outside the j loop so B is read row by row, and rows are
 * shared across threads.  Inputs are fp16, widened exactly.  `rows` (may be
 * NULL) selects which rows of A to compute: C row r holds A row rows[r]. */
void oracle_gemm_f16(const uint16_t* A, const uint16_t* B, float* C, int64_t m_out, int64_t n, int64_t k,
                     int64_t lda, int64_t ldb, const int64_t* rows, int nthreads) {
    float* Bf = (float*)malloc((size_t)k * (size_t)n * sizeof(float));
    if (!Bf) return;
#pragma omp parallel for schedule(static) num_threads(nthreads > 0 ? nthreads : 1) if (nthreads != 1)
    for (int64_t l = 0; l < k; ++l)
        for (int64_t j = 0; j < n; ++j) Bf[(size_t)l * n + j] = oracle_f16_to_f32(B[(size_t)l * ldb + j]);

#pragma omp parallel for schedule(dynamic, 1) num_threads(nthreads > 0 ? nthreads : 1) if (nthreads != 1)
    for (int64_t r = 0; r < m_out; ++r) {
        const int64_t i = rows ? rows[r] : r;
        float* c = C + (size_t)r * n;
        for (int64_t j = 0; j < n; ++j) c[j] = 0.f;
        for (int64_t l = 0; l < k; ++l) {
            const float a = oracle_f16_to_f32(A[(size_t)i * lda + l]);
            const float* b = Bf + (size_t)l * n;
            for (int64_t j = 0; j < n; ++j) c[j] += a * b[j];
        }
    }
    free(Bf);
}

/* ------------------------------------------------------------- epilogue */

float oracle_gelu_tanh(float x) {
    const float k_alpha = 0.7978845608028654f; /* sqrt(2/pi) */
    const float k_beta = 0.044715f;
    return 0.5f * x * (1.0f + tanhf(k_alpha * (x + k_beta * x * x * x)));
}

float oracle_gelu_erf(float x) { return 0.5f * x * (1.0f + erff(x * 0.70710678118654752f)); }

/* Epilogue selector values match pax_epilogue_t. */
enum {
    O_EPI_NONE = 0,
    O_EPI_BIAS = 1,
    O_EPI_BIAS_GELU_TANH = 2,
    O_EPI_BIAS_GELU_ERF = 3,
    O_EPI_RESIDUAL_GELU_TANH = 4,
    O_EPI_RESIDUAL_GELU_ERF = 5,
    O_EPI_GELU_TANH = 6,
    O_EPI_GELU_ERF = 7,
    O_EPI_RESIDUAL = 8
};

/* In place on C[m][n] (row r of C is row rows[r] of the full problem when
 * rows != NULL, for the residual lookup).  Order: scale, bias or residual,
 * GeLU.  bias: fp16 [n]; residual: fp32 or fp16 [*][ld_res]. */
void oracle_epilogue(float* C, int64_t m, int64_t n, int epi, float alpha, const uint16_t* bias,
                     const void* residual, int residual_f32, int64_t ld_res, const int64_t* rows) {
    const int has_bias = epi == O_EPI_BIAS || epi == O_EPI_BIAS_GELU_TANH || epi == O_EPI_BIAS_GELU_ERF;
    const int has_res = epi == O_EPI_RESIDUAL_GELU_TANH || epi == O_EPI_RESIDUAL_GELU_ERF || epi == O_EPI_RESIDUAL;
    const int gelu_t = epi == O_EPI_BIAS_GELU_TANH || epi == O_EPI_RESIDUAL_GELU_TANH || epi == O_EPI_GELU_TANH;
    const int gelu_e = epi == O_EPI_BIAS_GELU_ERF || epi == O_EPI_RESIDUAL_GELU_ERF || epi == O_EPI_GELU_ERF;
    for (int64_t r = 0; r < m; ++r) {
        const int64_t i = rows ? rows[r] : r;
        for (int64_t j = 0; j < n; ++j) {
            float v = C[(size_t)r * n + j];
            if (alpha != 1.0f) v = v * alpha;
            if (has_bias) v += oracle_f16_to_f32(bias[j]);
            if (has_res) {
                const size_t off = (size_t)i * ld_res + j;
                v += residual_f32 ? ((const float*)residual)[off] : oracle_f16_to_f32(((const uint16_t*)residual)[off]);
            }
            if (gelu_t) v = oracle_gelu_tanh(v);
            else if (gelu_e) v = oracle_gelu_erf(v);
            C[(size_t)r * n + j] = v;
        }
    }
}

/* --------------------------------------------------------------- checks */

/* pax_verify_gemm without the printing: returns 1 when
 * max_i |g-r|/(|r|+1e-8) <= tol.  src/host_bridge.c:422-445. */
int oracle_verify(const float* g, const float* r, int64_t count, float tol, float* max_err, int64_t* max_i) {
    float worst = 0.f;
    int64_t at = 0;
    for (int64_t i = 0; i < count; ++i) {
        const float e = fabsf(g[i] - r[i]) / (fabsf(r[i]) + 1e-8f);
        if (e > worst) {
            worst = e;
            at = i;
        }
    }
    if (max_err) *max_err = worst;
    if (max_i) *max_i = at;
    return worst <= tol;
}
