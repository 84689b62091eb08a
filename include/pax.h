/*
 * pax.h -- C ABI of the pax_b200 FP16 GEMM library (NVIDIA B200, sm_100a).
 *
 * Drop-in for the GEMM surface of PAX's host bridge (reference project
 * SNAPKITTYWEST/pax, file src/host_bridge.c).  Every entry point that the
 * reference declares or defines for the GEMM path keeps its name, argument
 * order, argument meaning and error behaviour; the citation next to each
 * declaration names the reference interface it replaces.  Entry points marked
 * "new" have no reference counterpart.
 *
 * Conventions shared by every launcher:
 *   A  [m][k] fp16, row-major (leading dimension k unless stated)
 *   B  [k][n] fp16, row-major (leading dimension n unless stated)
 *   C  [m][n] row-major, fp32 in the reference-named launchers, fp16 in the
 *      *_f16 twins
 *   All launches are asynchronous on the caller's stream.  Launchers never
 *   allocate caller-visible memory; the caller owns every buffer.
 *   Launchers return void, as in the reference; a failed argument check or
 *   launch prints "[PAX] ..." to stderr and is recorded for pax_last_error().
 *
 * This header is valid C99 and C++.
 */
#ifndef PAX_B200_PAX_H
#define PAX_B200_PAX_H

#include <stddef.h>
#include <stdint.h>
#include <cuda_runtime_api.h> /* cudaStream_t; C-compatible */

#ifdef __cplusplus
#include <cuda_fp16.h>
extern "C" {
#else
#ifndef PAX_HALF_DEFINED
#define PAX_HALF_DEFINED
/* Layout-compatible stand-in for CUDA's __half when compiling as C. */
typedef struct { unsigned short x; } __half;
#endif
#endif

/* ---------------------------------------------------------------------------
 * Buffer descriptor -- identical layout to the reference
 * (src/host_bridge.c:38-60).
 * ------------------------------------------------------------------------- */
typedef enum {
    PAX_HOST    = 0,
    PAX_DEVICE  = 1,
    PAX_UNIFIED = 2
} pax_ownership_t;

typedef struct {
    void*           base;
    size_t          elem_size;
    int64_t         shape[3];
    int64_t         stride[3];
    int             ndim;
    size_t          alignment;
    pax_ownership_t ownership;
    cudaStream_t    stream;
} pax_buffer_t;

/* ---------------------------------------------------------------------------
 * Status / epilogue / dtype enums (new).
 * ------------------------------------------------------------------------- */
typedef enum {
    PAX_OK              = 0,
    PAX_ERR_INVALID     = 1, /* NULL pointer, bad shape, bad stride */
    PAX_ERR_UNSUPPORTED = 2, /* forced algorithm cannot run this problem */
    PAX_ERR_CUDA        = 3, /* a CUDA runtime call failed */
    PAX_ERR_TIMEOUT     = 4, /* a device-side bounded wait expired */
    PAX_ERR_NO_DEVICE   = 5, /* no sm_100 device is current */
    PAX_ERR_ALLOC       = 6  /* workspace allocation failed */
} pax_status_t;

typedef enum {
    PAX_EPI_NONE               = 0, /* C = alpha*A.B                      */
    PAX_EPI_BIAS               = 1, /* C = alpha*A.B + bias[j]            */
    PAX_EPI_BIAS_GELU_TANH     = 2, /* C = gelu_tanh(alpha*A.B + bias[j]) */
    PAX_EPI_BIAS_GELU_ERF      = 3, /* C = gelu_erf(alpha*A.B + bias[j])  */
    PAX_EPI_RESIDUAL_GELU_TANH = 4, /* C = gelu_tanh(alpha*A.B + R[i][j]) */
    PAX_EPI_RESIDUAL_GELU_ERF  = 5, /* C = gelu_erf(alpha*A.B + R[i][j])  */
    PAX_EPI_GELU_TANH          = 6, /* C = gelu_tanh(alpha*A.B)           */
    PAX_EPI_GELU_ERF           = 7, /* C = gelu_erf(alpha*A.B)            */
    PAX_EPI_RESIDUAL           = 8  /* C = alpha*A.B + R[i][j]            */
} pax_epilogue_t;

typedef enum {
    PAX_DT_F32 = 0,
    PAX_DT_F16 = 1
} pax_dtype_t;

typedef enum {
    PAX_ALGO_AUTO   = 0, /* pick by shape and alignment                      */
    PAX_ALGO_TC     = 1, /* persistent tcgen05 kernel, one CTA per tile      */
    PAX_ALGO_TC2    = 2, /* persistent tcgen05 kernel, CTA pair per tile     */
    PAX_ALGO_SKINNY = 3, /* swap-AB stream-K tcgen05 kernel for small m      */
    PAX_ALGO_SIMT   = 4  /* CUDA-core kernel for TMA-unaligned problems      */
} pax_algo_t;

/* Hint bits ORed into pax_gemm_desc_t.algo (new; no counterpart in the
 * reference).  PAX_GEMM_B_CONST: B is not written by the kernel launched
 * just before on the same stream (typically weights).  The skinny kernel
 * then starts copying B into shared memory before that kernel has
 * finished; A and every write still wait for it.  Leave it unset when the
 * previous kernel may write B. */
#define PAX_GEMM_B_CONST 0x100

/* General GEMM descriptor (new).  Zero leading dimensions mean contiguous. */
typedef struct {
    const void*    A;        /* fp16 [M][lda]                              */
    const void*    B;        /* fp16 [K][ldb]                              */
    void*          C;        /* c_dtype [M][ldc]                           */
    int64_t        M, N, K;
    int64_t        lda, ldb, ldc;
    pax_dtype_t    c_dtype;
    pax_epilogue_t epilogue;
    float          alpha;    /* applied to A.B before bias/residual       */
    const void*    bias;     /* fp16 [N]      (BIAS* epilogues)           */
    const void*    residual; /* residual_dtype [M][ld_res] (RESIDUAL*)     */
    pax_dtype_t    residual_dtype;
    int64_t        ld_res;
    pax_algo_t     algo;
} pax_gemm_desc_t;

/* ---------------------------------------------------------------------------
 * Kernel launchers (reference-named, fp32 C).
 * ------------------------------------------------------------------------- */

/* replaces pax_gemm_wmma_launch, src/rtx_gemm_wmma.cu:107-112 (declared src/host_bridge.c:76-77) */
void pax_gemm_wmma_launch(const __half* A, const __half* B, float* C,
                          int m, int n, int k, cudaStream_t stream);

/* replaces pax_gemm_ptx_launch, src/rtx_gemm_ptx.cu:317-331 (declared src/host_bridge.c:80-81) */
void pax_gemm_ptx_launch(const __half* A, const __half* B, float* C,
                         int m, int n, int k, cudaStream_t stream);

/* replaces pax_gemm_ptx_smem_bytes, src/rtx_gemm_ptx.cu:308-312.  The
 * reference's launchers always run one kernel; these launchers pick a kernel
 * per problem, so this returns the dynamic shared memory of the kernel
 * pax_gemm_ptx_launch runs for the reference's default bench problem
 * (m = n = k = 4096, fp32 C; src/host_bridge.c:498-500) on the current
 * device.  pax_gemm_smem_bytes answers for any other problem. */
size_t pax_gemm_ptx_smem_bytes(void);

/* replaces pax_gemm_pipeline_launch, src/rtx_gemm_pipeline.cu:340-362 (declared src/host_bridge.c:85-87) */
void pax_gemm_pipeline_launch(const __half* A, const __half* B, float* C,
                              int m, int n, int k, cudaStream_t stream);

/* replaces pax_gemm_pipeline_smem_bytes, src/rtx_gemm_pipeline.cu:331-334:
 * as pax_gemm_ptx_smem_bytes, for pax_gemm_pipeline_launch. */
size_t pax_gemm_pipeline_smem_bytes(void);

/* replaces pax_gemm_bias_gelu_launch, src/rtx_gemm_epilogue.cu:375-392 (declared src/host_bridge.c:91-94).
 * C = gelu_tanh(A.B + bias[j]), bias fp16 [n]. */
void pax_gemm_bias_gelu_launch(const __half* A, const __half* B, float* C,
                               int m, int n, int k, const __half* bias,
                               cudaStream_t stream);

/* replaces pax_gemm_residual_gelu_launch, src/rtx_gemm_epilogue.cu:397-414 (declared src/host_bridge.c:95-98).
 * C = gelu_tanh(A.B + residual[i][j]), residual fp32 [m][n]. */
void pax_gemm_residual_gelu_launch(const __half* A, const __half* B, float* C,
                                   int m, int n, int k, const float* residual,
                                   cudaStream_t stream);

/* replaces pax_gemm_scale_bias_gelu_launch, src/rtx_gemm_epilogue.cu:418-436 (declared src/host_bridge.c:99-102).
 * C = gelu_tanh(alpha*A.B + bias[j]). */
void pax_gemm_scale_bias_gelu_launch(const __half* A, const __half* B, float* C,
                                     int m, int n, int k, float alpha,
                                     const __half* bias, cudaStream_t stream);

/* replaces pax_gemm_tma_cluster_launch, src/rtx_gemm_tma.cu:243-271.
 * C = A.B on the CTA-pair kernel.  The tensor-map arguments are accepted for
 * signature compatibility and ignored: tensor maps are built internally. */
void pax_gemm_tma_cluster_launch(const __half* A, const __half* B, float* C,
                                 int M, int N, int K,
                                 const void* tmap_A, const void* tmap_B,
                                 const void* tmap_C, cudaStream_t stream);

/* replaces pax_gemm_tma_smem_bytes, src/rtx_gemm_tma.cu:273-275: as
 * pax_gemm_ptx_smem_bytes, for pax_gemm_tma_cluster_launch (the CTA-pair
 * kernel). */
size_t pax_gemm_tma_smem_bytes(void);

/* ---------------------------------------------------------------------------
 * FP16-output twins (new; the reference writes fp32 C only).
 * ------------------------------------------------------------------------- */
void pax_gemm_f16_launch(const __half* A, const __half* B, __half* C,
                         int m, int n, int k, cudaStream_t stream);
void pax_gemm_bias_f16_launch(const __half* A, const __half* B, __half* C,
                              int m, int n, int k, const __half* bias,
                              cudaStream_t stream);
void pax_gemm_bias_gelu_f16_launch(const __half* A, const __half* B, __half* C,
                                   int m, int n, int k, const __half* bias,
                                   cudaStream_t stream);
void pax_gemm_bias_gelu_erf_f16_launch(const __half* A, const __half* B, __half* C,
                                       int m, int n, int k, const __half* bias,
                                       cudaStream_t stream);
void pax_gemm_residual_gelu_f16_launch(const __half* A, const __half* B, __half* C,
                                       int m, int n, int k, const __half* residual,
                                       cudaStream_t stream);
void pax_gemm_residual_gelu_erf_f16_launch(const __half* A, const __half* B, __half* C,
                                           int m, int n, int k, const __half* residual,
                                           cudaStream_t stream);

/* General entry point with status return (new). */
pax_status_t pax_gemm_ex(const pax_gemm_desc_t* desc, cudaStream_t stream);

/* Skinny GEMM (1 <= M <= 64) without any allocation.  No counterpart in the
 * reference.
 * For callers that cannot let a library allocate device memory: processes
 * whose GPU memory is owned by their own allocator (a framework's caching
 * allocator, a serving process that reserves memory at start-up) and loops
 * that cannot afford the device synchronisation of cudaMalloc/cudaFree.
 * Same kernel, epilogue and work layout as pax_gemm_ex with
 * PAX_ALGO_SKINNY (desc->algo is ignored): the lockstep layout when there
 * are no more 128-column tiles than SMs, else stream-K.  The split-K scratch
 * is a fixed 8 MiB array inside the library, held by every GPU that loads
 * it until the process exits.  Calls no cudaMalloc/cudaFree.  Problems whose
 * scratch need exceeds 8 MiB (stream-K above roughly m = 48 at 148 SMs)
 * return PAX_ERR_UNSUPPORTED with a message, before anything is launched.
 * The first call on a device (and the first after that device's CUDA
 * context was reset or re-created, or after pax_shutdown) looks up the
 * array's device address, so make it before any stream capture.  Nothing
 * in the array needs clearing between calls: the split-tile publication
 * flags hold a per-call 64-bit epoch.  Each device has its own
 * copy of the array, but all calls on one device share it: calls that
 * overlap on the GPU there (different streams without ordering between
 * them) race and give wrong results. */
pax_status_t pax_gemm_skinny_noalloc(const pax_gemm_desc_t* desc, cudaStream_t stream);

/* Batched GEMM (new; generalises the reference's Futhark entry
 * pax_batch_gemm, src/pax_kernel.fut:27-28,35, to strided items and every
 * epilogue): `batch` independent problems C_b = epi(alpha * A_b . B_b) of
 * the shape, leading dimensions and epilogue in `gemm`, whose pointers
 * address item 0.  Item b's operands start stride_* elements after item
 * b-1's.  A stride of 0 shares one A, B, bias or residual between all items;
 * C items must not overlap.  The tensor-core kernel runs a whole batch in one
 * launch; m <= 64 and TMA-unaligned problems run one launch per item. */
typedef struct {
    pax_gemm_desc_t gemm;
    int64_t batch;
    int64_t stride_a, stride_b, stride_c, stride_bias, stride_residual; /* elements */
} pax_gemm_batched_desc_t;
pax_status_t pax_gemm_batched_ex(const pax_gemm_batched_desc_t* desc, cudaStream_t stream);

/* Replicated output (new; the multi-GPU north star's "all-gather of C only
 * when the caller asks for a replicated output"): pax_gemm_ex, and the same
 * kernel also stores every finished tile of C to each of `n_replicas`
 * (0..7) further buffers of C's shape and pitch, typically the same region
 * of other GPUs' C buffers mapped with pax_ipc_import.  The copies travel
 * over NVLink while the kernel computes later tiles.  Each replica receives
 * complete, system-visible data once the kernel has finished; a reader on
 * another GPU must order its reads after that (pax_peer_barrier, or a
 * collective on the same streams).  The copies to the replicas are made
 * after each tile's local store, from the local C, so C itself must not be
 * written by anyone else while the kernel runs.  Tensor-core path only (m > 64, 16-byte aligned
 * rows): other problems return PAX_ERR_UNSUPPORTED. */
pax_status_t pax_gemm_replicated_ex(const pax_gemm_desc_t* desc, void* const* replicas, int n_replicas,
                                   cudaStream_t stream);

/* Rank barrier for replicated outputs, over NVLink peer memory (new; it
 * replaces a collective as the ordering around pax_gemm_replicated_ex).
 * `own` is this rank's array of n_peers + 1 64-bit flags in device memory,
 * zero when created; peers[i] are the other ranks' arrays, mapped with
 * pax_ipc_import; `slot` is this rank's index in every array.  One small
 * kernel on `stream`, after everything queued before it there, release-
 * stores `epoch` into slot `slot` of every peer's array, then waits until
 * every other slot of `own` holds at least `epoch`.  Work queued after it
 * therefore starts only when every rank has reached the barrier.  Epochs must
 * grow from call to call, the same sequence on every rank (nothing is ever
 * cleared).  A wait longer than timeout_ns (0: 10 s) gives up and records a
 * timeout that pax_device_error() returns as PAX_ERR_TIMEOUT. */
pax_status_t pax_peer_barrier(unsigned long long* own, unsigned long long* const* peers, int n_peers, int slot,
                              unsigned long long epoch, unsigned long long timeout_ns, cudaStream_t stream);

/* CUDA IPC handle of the allocation holding a device pointer, plus the
 * pointer's offset in it (new).  pax_ipc_import maps it in another process
 * (peer access enabled lazily) and returns the same address there;
 * pax_ipc_close unmaps. */
typedef struct {
    unsigned char handle[64];
    uint64_t offset;
} pax_ipc_handle_t;
pax_status_t pax_ipc_export(const void* device_ptr, pax_ipc_handle_t* out);
pax_status_t pax_ipc_import(const pax_ipc_handle_t* handle, void** device_ptr);
pax_status_t pax_ipc_close(void* device_ptr);

/* The algorithm pax_gemm_ex would run for desc with algo = PAX_ALGO_AUTO (new;
 * host-only, launches nothing). */
pax_algo_t pax_gemm_select_algo(const pax_gemm_desc_t* desc);

/* Shared-memory pipeline depth (TMA ring stages) of the kernel pax_gemm_ex
 * would launch for desc with algo = PAX_ALGO_AUTO on the current device; 0
 * for the CUDA-core kernel or without a device (new: no counterpart in the
 * reference; it lets a caller evaluate the reference's pipeline bound
 * throughput >= (1 - 1/STAGES) * min(compute, memory) for the kernel that
 * actually runs).  Host-only, launches nothing. */
int pax_gemm_pipeline_stages(const pax_gemm_desc_t* desc);

/* Dynamic shared memory, in bytes, of the kernel pax_gemm_ex would launch
 * for desc (desc->algo honoured; AUTO chosen as pax_gemm_ex chooses) on the
 * current device, 148 SMs assumed without one; 0 for the CUDA-core kernel,
 * whose shared memory is static (new: the per-problem form of the
 * reference's *_smem_bytes queries, src/rtx_gemm_pipeline.cu:331-334).
 * Host-only, launches nothing. */
size_t pax_gemm_smem_bytes(const pax_gemm_desc_t* desc);

/* ---- Lean-extraction symbols (pax-lean4/PAX/Extraction.lean:32-84) ----
 * The names and signatures PAX's Lean layer exports.  Sizes are 64-bit and
 * device pointers are passed as integers: A fp16 [M][K], B fp16 [K][N],
 * C fp32 [M][N], bias fp16 [N], residual fp32 [M][N].  The GEMMs run the
 * same kernels as pax_gemm_ex on the legacy default stream (asynchronous);
 * errors go to pax_last_error() and stderr, as for the launchers. */
void pax_gemm_wmma_verified(uint64_t M, uint64_t N, uint64_t K, uint64_t A, uint64_t B, uint64_t C);
void pax_gemm_ptx_verified(uint64_t M, uint64_t N, uint64_t K, uint64_t A, uint64_t B, uint64_t C);
void pax_gemm_pipeline3_verified(uint64_t M, uint64_t N, uint64_t K, uint64_t A, uint64_t B, uint64_t C);
void pax_gemm_bias_gelu_verified(uint64_t M, uint64_t N, uint64_t K, uint64_t A, uint64_t B, uint64_t C,
                                 uint64_t bias);
void pax_gemm_residual_gelu_verified(uint64_t M, uint64_t N, uint64_t K, uint64_t A, uint64_t B, uint64_t C,
                                     uint64_t residual);

/* IEEE-754 binary16 add, multiply and fused multiply-add with a single
 * round-to-nearest-even (host code; Extraction.lean:58-84 with
 * Float16.add/mul/fma of pax-lean4/PAX/Float16.lean:99-125).  NaN results
 * are 0x7C01, the Lean model's Float16.posNaN.  Signed zeros, infinities and
 * the overflow threshold (65520) follow IEEE 754. */
uint16_t pax_fp16_add_verified(uint16_t x, uint16_t y);
uint16_t pax_fp16_mul_verified(uint16_t x, uint16_t y);
uint16_t pax_fp16_fma_verified(uint16_t x, uint16_t y, uint16_t z);

/* ---------------------------------------------------------------------------
 * Host bridge (src/host_bridge.c).
 * ------------------------------------------------------------------------- */

/* replaces pax_validate_buffer, src/host_bridge.c:136-172.  1 = valid, 0 = not. */
int pax_validate_buffer(const pax_buffer_t* buf);

/* replace pax_alloc_device_1d/2d and pax_alloc_host_1d/2d, src/host_bridge.c:179-257.
 * On failure base == NULL. */
pax_buffer_t pax_alloc_device_1d(size_t nelems, size_t elem_size, cudaStream_t stream);
pax_buffer_t pax_alloc_device_2d(size_t rows, size_t cols, size_t elem_size, cudaStream_t stream);
pax_buffer_t pax_alloc_host_1d(size_t nelems, size_t elem_size, cudaStream_t stream);
pax_buffer_t pax_alloc_host_2d(size_t rows, size_t cols, size_t elem_size, cudaStream_t stream);

/* replace pax_free_device / pax_free_host, src/host_bridge.c:260-273 */
void pax_free_device(pax_buffer_t* buf);
void pax_free_host(pax_buffer_t* buf);

/* replace pax_dispatch_{wmma,ptx,pipeline}_gemm, src/host_bridge.c:312-348.
 * C->elem_size selects the output type: 4 = fp32 (reference), 2 = fp16.
 * Row strides (stride[0] of 2-D buffers) are honoured. */
void pax_dispatch_wmma_gemm(pax_buffer_t* A, pax_buffer_t* B, pax_buffer_t* C, cudaStream_t stream);
void pax_dispatch_ptx_gemm(pax_buffer_t* A, pax_buffer_t* B, pax_buffer_t* C, cudaStream_t stream);
void pax_dispatch_pipeline_gemm(pax_buffer_t* A, pax_buffer_t* B, pax_buffer_t* C, cudaStream_t stream);

/* replaces pax_dispatch_bias_gelu, src/host_bridge.c:351-366 */
void pax_dispatch_bias_gelu(pax_buffer_t* A, pax_buffer_t* B, pax_buffer_t* C,
                            const __half* bias, cudaStream_t stream);

/* replaces pax_dispatch_residual_gelu, src/host_bridge.c:369-386.  residual is
 * fp32 [m][n] as in the reference. */
void pax_dispatch_residual_gelu(pax_buffer_t* A, pax_buffer_t* B, pax_buffer_t* C,
                                const float* residual, cudaStream_t stream);

/* new: the dispatcher the reference declares a launcher for but never wires
 * (src/host_bridge.c:99-102). */
void pax_dispatch_scale_bias_gelu(pax_buffer_t* A, pax_buffer_t* B, pax_buffer_t* C,
                                  float alpha, const __half* bias, cudaStream_t stream);

/* replaces cpu_gemm_ref, src/host_bridge.c:397-407: naive fp32 GEMM on the
 * host, i-j-l loop, sequential accumulation.  Verification utility only; no
 * GPU entry point ever calls it. */
void cpu_gemm_ref(const float* A, const float* B, float* C, int m, int n, int k);

/* replaces pax_verify_gemm, src/host_bridge.c:422-445: max relative error
 * |g-r|/(|r|+1e-8) <= tol prints PASS and returns 1, else FAIL and 0. */
int pax_verify_gemm(const float* C_gpu, const float* C_ref, int m, int n, float tol);

/* replaces pax_bench_all, src/host_bridge.c:543-566: times every variant on
 * the state set by pax_bench_setup and prints ms/iter and TFLOP/s. */
void pax_bench_all(int iters);

/* new: the reference keeps its bench state in file-static globals
 * (src/host_bridge.c:487-500) with no setter; these allocate and release it. */
int  pax_bench_setup(int m, int n, int k, cudaStream_t stream);
void pax_bench_teardown(void);

/* ---------------------------------------------------------------------------
 * Status and lifetime (new).
 * ------------------------------------------------------------------------- */
pax_status_t pax_last_error(void);               /* thread-local, last call */
const char*  pax_status_string(pax_status_t s);
/* Reads and clears the device-side error word of the current device
 * (synchronises the device).  Returns PAX_ERR_TIMEOUT if a bounded wait in a
 * kernel expired since the last read, else PAX_OK. */
pax_status_t pax_device_error(void);
/* Self-test of the kernels' bounded waits (new; no counterpart in the
 * reference): launches one thread that waits on an mbarrier nothing arrives
 * on.  After the library's 2 s wait limit it records a timeout and ends; the
 * next pax_device_error() returns PAX_ERR_TIMEOUT and the CUDA context stays
 * usable.  For tests of the failure path; takes about 2 s of GPU time. */
pax_status_t pax_selftest_bounded_wait(cudaStream_t stream);
/* Test hook (new; no counterpart in the reference): writes into the skinny
 * kernel's split-tile publication flags of `stream`'s workspace (the current
 * device's) what launches that gave up on a timed-out wait leave behind.
 * The next skinny GEMM on that stream must still be correct.  Synchronises
 * `stream`.  PAX_ERR_INVALID if the stream has no workspace yet. */
pax_status_t pax_selftest_stale_counters(cudaStream_t stream);
/* Test hook (new; no counterpart in the reference): sets, on the current
 * device, the limit of the kernels' waits that a CTA may abandon, in
 * nanoseconds (0 restores the default 2 s; values below 1000 are
 * rejected).  With a limit of a few microseconds a real GEMM's waits run
 * out: the kernel takes its abort path (its issued TMA loads land, its
 * MMAs drain, TMEM is freed), records a timeout that pax_device_error()
 * reports, and ends.  The abort path's own waits keep the 2 s limit.
 * Synchronises the device.  For tests of the failure path only. */
pax_status_t pax_selftest_set_wait_limit(uint64_t ns);
/* Test hook (new; no counterpart in the reference; host only, launches
 * nothing): the work list the 256 x 512 CTA-pair tile would run for an
 * M x N x K problem on `units` pairs, when it is planned.  Writes
 * unit_start[0..units] and items[0..count), where item bits 0-15 are the
 * 256-row block, 16-27 the first column / 128 and 28-29 the width (0: 512,
 * 1: 384, 2: 256, 3: 128 columns); unit u runs items
 * [unit_start[u], unit_start[u+1]).  Returns count, 0 when the problem is not
 * planned (round-robin tiles), -1 on a bad argument or too small a buffer. */
int pax_selftest_wide_plan(long long M, long long N, long long K, int units, unsigned int* items, int* unit_start,
                           int max_items);

/* Frees the device memory this library allocated on its own: the skinny
 * kernel's per-stream workspaces and the planned tile tables of the wide
 * tensor-core tile.  Later calls allocate them again as needed.  Also
 * forgets the looked-up device address of pax_gemm_skinny_noalloc's array.
 * A workspace belongs to (device, stream handle) and, for
 * cudaStreamPerThread, to the calling host thread as well. */
void         pax_shutdown(void);
/* Library version string. */
const char*  pax_version(void);
/* sizeof(pax_buffer_t) and sizeof(pax_gemm_desc_t) as compiled into the
 * library, so that bindings can check their struct layouts. */
size_t       pax_sizeof_buffer(void);
size_t       pax_sizeof_gemm_desc(void);

#ifdef __cplusplus
} /* extern "C" */
#endif

#endif /* PAX_B200_PAX_H */
