// epilogue.cuh -- element-wise epilogue shared by every GEMM kernel.
//
// Semantics follow the reference's fused epilogues
// (src/rtx_gemm_epilogue.cu:7-10 and the functor compositions at :176-233):
//   ScaleBiasGeLU(x) = GeLU(alpha*x + b[j])      scale, then bias, then GeLU
//   BiasGeLU(x)      = GeLU(x + b[j])            bias is indexed by column j
//   ResidualGeLU(x)  = GeLU(x + R[i][j])         residual indexed by (i, j)
// with the column/element indexing the reference states in its comments and
// in pax-lean4/PAX/Integration.lean:114-122 (its GPU functors mis-index
// fragments; the intended mapping is used here).
//
// GeLU variants:
//   tanh form, src/rtx_gemm_epilogue.cu:76-80:
//     0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3)))
//   exact form (no reference code; the definition PAX/GEMM.lean:150-152
//   bounds the tanh form against): 0.5 x (1 + erf(x / sqrt 2))
// Both call CUDA's tanhf / erff.
#pragma once

#include <cuda_fp16.h>
#include <stdint.h>

#include "params.h"
#include "sm100.cuh"

namespace pax {

__device__ __forceinline__ float gelu_tanh(float x) {
    const float k_alpha = 0.7978845608028654f;  // sqrt(2/pi)
    const float k_beta = 0.044715f;
    return 0.5f * x * (1.0f + tanhf(k_alpha * (x + k_beta * x * x * x)));
}

__device__ __forceinline__ float gelu_erf(float x) {
    return 0.5f * x * (1.0f + erff(x * 0.70710678118654752f));
}

// One output value: scale, then bias and/or residual, then GeLU.  `b` is the
// bias value and `r` the residual value (ignored unless their flag is set).
__device__ __forceinline__ float epi_scalar(float acc, float b, float r, int flags, float alpha) {
    float v = (flags & EPI_SCALE) ? acc * alpha : acc;
    if (flags & EPI_BIAS) v += b;
    if (flags & EPI_RES) v += r;
    if (flags & EPI_GELU_TANH) v = gelu_tanh(v);
    else if (flags & EPI_GELU_ERF) v = gelu_erf(v);
    return v;
}

// Unpack 8 fp16 (one uint4) to floats.
__device__ __forceinline__ void unpack_h8(const uint4& u, float* f) {
    const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        float2 t = __half22float2(h[i]);
        f[2 * i] = t.x;
        f[2 * i + 1] = t.y;
    }
}

// Residual values of one row chunk, fetched ahead of the TMEM read so that
// their global-memory latency overlaps it.  Holds n fp32 or n fp16 values
// (the fp16 case uses the first n/8 vectors).
template <int n>
struct ResChunk {
    uint4 u[n / 4];
};

template <int n>
__device__ __forceinline__ void res_prefetch(ResChunk<n>& rc, long long row, long long col0, long long M,
                                             long long N, const EpiParams& ep) {
    const int flags = ep.flags;
    if (!(flags & EPI_RES)) return;
#pragma unroll
    for (int i = 0; i < n / 4; ++i) rc.u[i] = make_uint4(0u, 0u, 0u, 0u);
    if (row >= M) return;
    const bool full = (flags & EPI_RES_VEC) && col0 + n <= N;
    if (flags & EPI_RES_F32) {
        const float* rp = static_cast<const float*>(ep.residual) + row * ep.ld_res + col0;
        if (full) {
#pragma unroll
            for (int i = 0; i < n / 4; ++i) rc.u[i] = ld_nc_v4(rp + 4 * i);
        } else {
#pragma unroll
            for (int i = 0; i < n / 4; ++i) {
                float x[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) x[e] = (col0 + 4 * i + e < N) ? rp[4 * i + e] : 0.f;
                rc.u[i] = make_uint4(__float_as_uint(x[0]), __float_as_uint(x[1]), __float_as_uint(x[2]),
                                     __float_as_uint(x[3]));
            }
        }
    } else {
        const __half* rp = static_cast<const __half*>(ep.residual) + row * ep.ld_res + col0;
        if (full) {
#pragma unroll
            for (int i = 0; i < n / 8; ++i) rc.u[i] = ld_nc_v4(rp + 8 * i);
        } else {
#pragma unroll
            for (int i = 0; i < n / 8; ++i) {
                uint32_t w[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const long long c = col0 + 8 * i + 2 * e;
                    const uint32_t lo = (c < N) ? __half_as_ushort(rp[8 * i + 2 * e]) : 0u;
                    const uint32_t hi = (c + 1 < N) ? __half_as_ushort(rp[8 * i + 2 * e + 1]) : 0u;
                    w[e] = lo | (hi << 16);
                }
                rc.u[i] = make_uint4(w[0], w[1], w[2], w[3]);
            }
        }
    }
}

// Apply the epilogue to n consecutive columns [col0, col0+n) of one row.
// Columns outside [0, N) get zero bias; the caller never stores them.
template <int n>
__device__ __forceinline__ void epi_apply_chunk(float (&v)[n], const ResChunk<n>& rc, long long col0,
                                                long long N, const EpiParams& ep) {
    const int flags = ep.flags;
    if ((flags & (EPI_BIAS | EPI_RES | EPI_SCALE | EPI_GELU_TANH | EPI_GELU_ERF)) == 0) return;
#pragma unroll
    for (int g = 0; g < n; g += 8) {
        float b[8];
        float r[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            b[e] = 0.f;
            r[e] = 0.f;
        }
        if (flags & EPI_BIAS) {
            if ((flags & EPI_BIAS_VEC) && col0 + g + 8 <= N) {
                unpack_h8(__ldg(reinterpret_cast<const uint4*>(ep.bias + col0 + g)), b);
            } else {
#pragma unroll
                for (int e = 0; e < 8; ++e)
                    if (col0 + g + e < N) b[e] = __half2float(ep.bias[col0 + g + e]);
            }
        }
        if (flags & EPI_RES) {
            if (flags & EPI_RES_F32) {
                const uint4 u0 = rc.u[g / 4], u1 = rc.u[g / 4 + 1];
                r[0] = __uint_as_float(u0.x); r[1] = __uint_as_float(u0.y);
                r[2] = __uint_as_float(u0.z); r[3] = __uint_as_float(u0.w);
                r[4] = __uint_as_float(u1.x); r[5] = __uint_as_float(u1.y);
                r[6] = __uint_as_float(u1.z); r[7] = __uint_as_float(u1.w);
            } else {
                unpack_h8(rc.u[g / 8], r);
            }
        }
#pragma unroll
        for (int e = 0; e < 8; ++e) v[g + e] = epi_scalar(v[g + e], b[e], r[e], flags, ep.alpha);
    }
}

}  // namespace pax
