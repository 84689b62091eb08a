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
// tanh: CUDA's tanhf, or the hardware tanh.approx.f32 for fp16 results;
// erf: Abramowitz & Stegun 7.1.28 (see gelu_erf).
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

// tanh form with the hardware tanh.approx.f32 (one transcendental-pipe op,
// relative error about 2^-11).  GeLU error <= 0.5|x| * 2^-11 ~ 2.4e-4 |x|,
// below the rounding of an fp16 result; used only when C is fp16.
__device__ __forceinline__ float tanh_hw(float x) {
    float y;
    asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
__device__ __forceinline__ float gelu_tanh_hw(float x) {
    const float k_alpha = 0.7978845608028654f;  // sqrt(2/pi)
    const float k_beta = 0.044715f;
    return 0.5f * x * (1.0f + tanh_hw(k_alpha * (x + k_beta * x * x * x)));
}

// Exact-form GeLU, 0.5 x (1 + erf(x / sqrt 2)), with erf from Abramowitz &
// Stegun, Handbook of Mathematical Functions (1964), formula 7.1.28
// (Hastings' rational approximation): for w >= 0
//   erf(w) = 1 - q,  q = (1 + a1 w + a2 w^2 + ... + a6 w^6)^-16,
// |error| <= 3e-7, and erf(-w) = -erf(w).  So 1 + erf(z) is 2 - q for
// z >= 0 and q itself for z < 0, with no cancellation in the negative tail.
// One reciprocal on the special-function unit and about a dozen FMA-pipe
// operations per value; the fp32 result is within about 1e-6 of the exact
// GeLU (checked against double-precision erf over |x| <= 20).
__device__ __forceinline__ float rcp_approx(float x) {
    float y;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
__device__ __forceinline__ float gelu_erf(float x) {
    const float z = x * 0.70710678118654752f;
    const float w = fabsf(z);
    float p = fmaf(w, 4.30638e-5f, 2.765672e-4f);
    p = fmaf(p, w, 1.520143e-4f);
    p = fmaf(p, w, 9.2705272e-3f);
    p = fmaf(p, w, 4.22820123e-2f);
    p = fmaf(p, w, 7.05230784e-2f);
    p = fmaf(p, w, 1.0f);
    p *= p;
    p *= p;
    p *= p;
    p *= p;                         // p^16 (inf for |z| above about 19: q = 0)
    const float q = rcp_approx(p);  // 1 - erf(w)
    return 0.5f * x * (z >= 0.f ? 2.0f - q : q);
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

// Residual values of one row chunk of n columns, fetched ahead of the TMEM
// read so that their global-memory latency overlaps it.  RES: 0 = none,
// 1 = fp16 residual (n/8 vectors), 2 = fp32 residual (n/4 vectors).
template <int n, int RES>
struct ResChunk {
    static constexpr int V = RES == 1 ? n / 8 : RES == 2 ? n / 4 : 1;
    uint4 u[V];
};

// The loads allocate in L1: each lane reads a 128-byte line of its row in
// two halves, one per 32-column sub-chunk, and the second half then comes
// from L1 (measured on C3: 1.64 GB of DRAM reads per launch, against 1.88 GB
// with L1::no_allocate, with or without an L2 evict-first hint).
template <int n, int RES>
__device__ __forceinline__ void res_prefetch(ResChunk<n, RES>& rc, long long row, long long col0, long long M,
                                             long long N, const EpiParams& ep) {
    if constexpr (RES == 0) {
        return;
    } else {
#pragma unroll
        for (int i = 0; i < ResChunk<n, RES>::V; ++i) rc.u[i] = make_uint4(0u, 0u, 0u, 0u);
        if (row >= M) return;
        const bool full = (ep.flags & EPI_RES_VEC) && col0 + n <= N;
        if constexpr (RES == 2) {
            const float* rp = static_cast<const float*>(ep.residual) + row * ep.ld_res + col0;
            if (full) {
#pragma unroll
                for (int i = 0; i < n / 4; ++i) rc.u[i] = ld_nc_v4_l1(rp + 4 * i);
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
                for (int i = 0; i < n / 8; ++i) rc.u[i] = ld_nc_v4_l1(rp + 8 * i);
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
}

// Bias of one output tile, 8 fp16 values per lane: lane l holds columns
// [tile_col0 + 8l, tile_col0 + 8l + 8).  Loaded once per tile, before the
// accumulator wait, and broadcast to the chunk loop by warp shuffles.
__device__ __forceinline__ uint4 bias_tile_load(long long tile_col0, int tile_cols, int lane, long long N,
                                                const EpiParams& ep) {
    uint4 b = make_uint4(0u, 0u, 0u, 0u);
    if (!(ep.flags & EPI_BIAS) || lane * 8 >= tile_cols) return b;
    const long long c = tile_col0 + lane * 8;
    if ((ep.flags & EPI_BIAS_VEC) && c + 8 <= N) return __ldg(reinterpret_cast<const uint4*>(ep.bias + c));
    uint32_t w[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        const uint32_t lo = (c + 2 * e < N) ? __half_as_ushort(ep.bias[c + 2 * e]) : 0u;
        const uint32_t hi = (c + 2 * e + 1 < N) ? __half_as_ushort(ep.bias[c + 2 * e + 1]) : 0u;
        w[e] = lo | (hi << 16);
    }
    return make_uint4(w[0], w[1], w[2], w[3]);
}

// Epilogue of one row chunk of n columns starting at tile column `tc` (a
// multiple of 8), in two phases so the caller can refill `rc` in between:
//   epi_linear: v = alpha*v (+ bias[j]) (+ R[i][j])
//   epi_gelu:   v = GeLU(v)     GELU: 0 none, 1 tanh (tanhf), 2 erf (gelu_erf), 3 tanh (tanh.approx)
// `bias8` is this lane's bias_tile_load value.
template <int n, int RES>
__device__ __forceinline__ void epi_linear(float (&v)[n], const ResChunk<n, RES>& rc, uint4 bias8, int tc,
                                           const EpiParams& ep) {
    const int flags = ep.flags;
    if (flags & EPI_SCALE) {
#pragma unroll
        for (int i = 0; i < n; ++i) v[i] *= ep.alpha;
    }
    if (flags & EPI_BIAS) {
#pragma unroll
        for (int g = 0; g < n; g += 8) {
            const int src = (tc + g) >> 3;
            uint4 u;
            u.x = __shfl_sync(0xffffffffu, bias8.x, src);
            u.y = __shfl_sync(0xffffffffu, bias8.y, src);
            u.z = __shfl_sync(0xffffffffu, bias8.z, src);
            u.w = __shfl_sync(0xffffffffu, bias8.w, src);
            float b[8];
            unpack_h8(u, b);
#pragma unroll
            for (int e = 0; e < 8; ++e) v[g + e] += b[e];
        }
    }
    if constexpr (RES == 2) {
#pragma unroll
        for (int i = 0; i < n / 4; ++i) {
            v[4 * i + 0] += __uint_as_float(rc.u[i].x);
            v[4 * i + 1] += __uint_as_float(rc.u[i].y);
            v[4 * i + 2] += __uint_as_float(rc.u[i].z);
            v[4 * i + 3] += __uint_as_float(rc.u[i].w);
        }
    } else if constexpr (RES == 1) {
#pragma unroll
        for (int i = 0; i < n / 8; ++i) {
            float r[8];
            unpack_h8(rc.u[i], r);
#pragma unroll
            for (int e = 0; e < 8; ++e) v[8 * i + e] += r[e];
        }
    }
}

template <int n, int GELU>
__device__ __forceinline__ void epi_gelu(float (&v)[n]) {
    if constexpr (GELU == 1) {
#pragma unroll
        for (int i = 0; i < n; ++i) v[i] = gelu_tanh(v[i]);
    } else if constexpr (GELU == 3) {
#pragma unroll
        for (int i = 0; i < n; ++i) v[i] = gelu_tanh_hw(v[i]);
    } else if constexpr (GELU == 2) {
#pragma unroll
        for (int i = 0; i < n; ++i) v[i] = gelu_erf(v[i]);
    }
}

}  // namespace pax
