// gemm_simt.cu -- CUDA-core GEMM for problems the TMA kernels cannot take.
//
// The tensor-memory-accelerator kernels need 16-byte aligned base pointers
// and row pitches (K and N multiples of 8 for fp16 rows).  The reference
// accepts any m, n, k (src/rtx_gemm_wmma.cu:52-74 guards every element), so
// the drop-in must too: ragged or misaligned problems, and K == 0, run here.
// Same epilogue semantics as the tensor-core kernels (epilogue.cuh).
//
// Also holds the bench-state fill kernel (counter-hash uniform fp16).
#include "internal.h"
#include "epilogue.cuh"

namespace pax {

struct SimtParams {
    const __half* A;
    const __half* B;
    void* C;
    long long M, N, K, lda, ldb, ldc;
    int c_f16;
    EpiParams epi;
};

// 64x64 output tile per CTA, 256 threads, 4x4 outputs per thread, k-step 16.
__global__ void __launch_bounds__(256) gemm_simt_kernel(const SimtParams p) {
    __shared__ float sA[16][64 + 1];  // [k][m]
    __shared__ float sB[16][64 + 1];  // [k][n]
    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
    const long long m0 = (long long)blockIdx.y * 64, n0 = (long long)blockIdx.x * 64;
    float acc[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;

    for (long long k0 = 0; k0 < p.K; k0 += 16) {
        for (int i = threadIdx.x; i < 64 * 16; i += 256) {
            const int mm = i >> 4, kk = i & 15;
            const long long gm = m0 + mm, gk = k0 + kk;
            sA[kk][mm] = (gm < p.M && gk < p.K) ? __half2float(p.A[gm * p.lda + gk]) : 0.f;
        }
        for (int i = threadIdx.x; i < 16 * 64; i += 256) {
            const int kk = i >> 6, nn = i & 63;
            const long long gk = k0 + kk, gn = n0 + nn;
            sB[kk][nn] = (gk < p.K && gn < p.N) ? __half2float(p.B[gk * p.ldb + gn]) : 0.f;
        }
        __syncthreads();
#pragma unroll
        for (int kk = 0; kk < 16; ++kk) {
            float a[4], b[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) a[i] = sA[kk][ty * 4 + i];
#pragma unroll
            for (int j = 0; j < 4; ++j) b[j] = sB[kk][tx * 4 + j];
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
        }
        __syncthreads();
    }

    const int flags = p.epi.flags;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const long long row = m0 + ty * 4 + i;
        if (row >= p.M) continue;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const long long col = n0 + tx * 4 + j;
            if (col >= p.N) continue;
            const float b = (flags & EPI_BIAS) ? __half2float(p.epi.bias[col]) : 0.f;
            float r = 0.f;
            if (flags & EPI_RES) {
                const long long off = row * p.epi.ld_res + col;
                r = (flags & EPI_RES_F32) ? static_cast<const float*>(p.epi.residual)[off]
                                          : __half2float(static_cast<const __half*>(p.epi.residual)[off]);
            }
            const float o = epi_scalar(acc[i][j], b, r, flags, p.epi.alpha);
            if (p.c_f16)
                static_cast<__half*>(p.C)[row * p.ldc + col] = __float2half_rn(o);
            else
                static_cast<float*>(p.C)[row * p.ldc + col] = o;
        }
    }
}

pax_status_t launch_simt(const Problem& pr, cudaStream_t stream) {
    SimtParams p;
    p.A = pr.A;
    p.B = pr.B;
    p.C = pr.C;
    p.M = pr.M;
    p.N = pr.N;
    p.K = pr.K;
    p.lda = pr.lda;
    p.ldb = pr.ldb;
    p.ldc = pr.ldc;
    p.c_f16 = pr.c_f16 ? 1 : 0;
    p.epi = pr.epi;
    const long long gx = (pr.N + 63) / 64, gy = (pr.M + 63) / 64;
    if (gx > 0x7fffffffLL || gy > 65535) return PAX_ERR_UNSUPPORTED;
    gemm_simt_kernel<<<dim3((unsigned)gx, (unsigned)gy), 256, 0, stream>>>(p);
    return cudaPeekAtLastError() == cudaSuccess ? PAX_OK : PAX_ERR_CUDA;
}

// splitmix64 finaliser: statistically independent values per (seed, index).
__device__ __forceinline__ unsigned long long mix64(unsigned long long x) {
    x += 0x9E3779B97F4A7C15ull;
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
    return x ^ (x >> 31);
}

__global__ void fill_uniform_f16_kernel(__half* p, long long n, unsigned long long seed, float lo, float hi) {
    const long long stride = (long long)gridDim.x * blockDim.x;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
        const unsigned long long h = mix64(seed * 0x100000001B3ull + (unsigned long long)i);
        const float u = (float)(h >> 40) * (1.0f / 16777216.0f);  // [0,1), 24 bits
        p[i] = __float2half_rn(lo + (hi - lo) * u);
    }
}

pax_status_t fill_uniform_f16(__half* p, long long n, unsigned long long seed, float lo, float hi,
                              cudaStream_t stream) {
    if (n <= 0) return PAX_OK;
    fill_uniform_f16_kernel<<<1184, 256, 0, stream>>>(p, n, seed, lo, hi);
    return cudaPeekAtLastError() == cudaSuccess ? PAX_OK : PAX_ERR_CUDA;
}

}  // namespace pax
