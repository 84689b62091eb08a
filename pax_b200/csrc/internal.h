// internal.h -- host-side interface between the C-ABI layer (host_bridge.cpp)
// and the kernel translation units.  Not part of the public ABI.
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "../../include/pax.h"
#include "params.h"

namespace pax {

// A validated, normalised GEMM problem: C[M][ldc] = epi(A[M][lda] . B[K][ldb]).
struct Problem {
    const __half* A;
    const __half* B;
    void* C;
    long long M, N, K;
    long long lda, ldb, ldc;
    bool c_f16;
    EpiParams epi;
    // Batched problems: `batch` independent GEMMs; element strides between
    // consecutive items of A, B, C, bias and residual (0 = shared by all
    // items, allowed for A, B, bias and residual).
    long long batch = 1;
    long long sa = 0, sb = 0, sc = 0, sbias = 0, sres = 0;
    // Replicated output: C is also stored, by the same kernel, to these
    // buffers (same shape and pitch; usually peer GPUs' memory).
    void* const* replicas = nullptr;
    int n_replicas = 0;
    // PAX_GEMM_B_CONST: B is not written by the previous kernel in the stream.
    bool b_const = false;
};

// Per-device facts the launchers need (cached).
int device_sm_count(int dev);
int current_device();

// TMA-based kernels need 16-byte aligned bases and row pitches.
bool tma_compatible(const Problem& p);

// Launchers.  Each returns PAX_OK or an error status; none synchronises.
// Launch plan of the tcgen05 kernel.  shape: 128 or 256 = one CTA per
// 128 x shape output tile; 2 = CTA pair (cluster of two, cta_group::2) per
// 256 x 256 tile; 4 = CTA pair per 256 x 512 tile.  Tiles [0, full_items) are computed whole; the last
// tail_tiles tiles (the tail wave) as two column halves each.
// units = CTAs (or pairs) launched.
struct TcPlan {
    int shape = 128;
    int units = 0;
    int full_items = 0;
    int tail_tiles = 0;
    // Wide tile only: a host-planned per-unit list of mixed-width items
    // (null: the kernel's round-robin schedule of whole tiles and halves).
    const TcItemTable* table = nullptr;
    const int* table_dev = nullptr;  // its device copy (current device)
};
TcPlan tc_plan(const Problem& p, int shape, int dev, int sms, bool allow_halves, cudaStream_t stream);
pax_status_t launch_tc(const Problem& p, const TcPlan& plan, cudaStream_t stream);
pax_status_t launch_simt(const Problem& p, cudaStream_t stream);
// Skinny kernel, nt (128 or 256) output columns per work unit.  A tile split
// between CTAs is summed by its last contributor: the others each put their
// partial sum in their slot of `ws` (MP*nt fp32 per CTA) and set their entry
// of `flags` (one word per CTA) to the launch's epoch.  Nothing needs
// clearing between launches: a flag from an earlier launch, finished or
// aborted, holds an older epoch.  skinny_geometry gives the grid and both
// sizes; skinny_pick_nt the unit width.
int skinny_pick_nt(long long M, long long N, long long K, int sms);
int skinny_lockstep_slices(long long M, long long N, long long K, int sms);
void skinny_geometry(long long M, long long N, long long K, int sms, int nt, int* grid, size_t* ws_bytes,
                     size_t* flag_bytes);
// The layout pax_gemm_ex runs for a skinny problem: nt, grid, K slices
// (lockstep layout when > 0), and the workspace sizes.
struct SkinnyLayout {
    int nt = 128, grid = 1, slices = 0;
    size_t ws_bytes = 0, cnt_bytes = 0;  // partial sums, flags
};
// nt_force = 128 or 256 forces persistent stream-K with that unit width
// (PAX_SKINNY_NT).
SkinnyLayout skinny_layout(long long M, long long N, long long K, int sms, int nt_force);
int skinny_env_nt();
// Epoch of the most recent launch of the skinny kernel.
unsigned long long skinny_last_epoch();
// slices > 0 = the lockstep layout (nt 128, `grid` = tiles x slices CTAs,
// one per SM); 0: persistent stream-K, `grid` CTAs, each CTA's segments
// last to first (the head of its later tile first).
pax_status_t launch_skinny_ws(const Problem& p, int nt, int grid, float* ws, unsigned long long* flags,
                              cudaStream_t stream, int slices = 0);
// Forget the cached device address of the allocation-free path's scratch
// array (pax_shutdown).
void skinny_forget_scratch();

// Launch the GEMM kernels with programmatic stream serialization, so that a
// kernel's prologue overlaps the previous kernel in the stream (default on;
// PAX_PDL=0 turns it off).
bool pdl_enabled();
// Planned mixed-width tiling for the wide shape (default on; PAX_TC_PLAN=0
// turns it off).
bool tc_planning_enabled();
void tc_free_plans();
// Shared-memory pipeline depth (TMA ring stages) of each kernel variant.
int tc_stages(int shape);
int skinny_stages(long long M, int nt);
size_t skinny_smem_bytes(long long M, int nt);
// Dynamic shared memory of the tcgen05 kernel for a tile shape / output type.
size_t tc_smem_bytes(int shape, bool c_f16);
// Tile width of the one-CTA shape for a problem (128 or 256).
int tc_pick_bn(long long M, long long N, int sms);
// Tile shape pax_gemm_ex picks by itself: 128, 256 (one CTA), 2 (pair,
// 256 x 256) or 4 (pair, 256 x 512).
int tc_pick_shape(const Problem& p, int sms);
// Largest M the skinny kernel accepts.
constexpr long long kSkinnyMaxM = 64;

// Descriptor validation and status recording shared with the C-ABI layer
// (host_bridge.cpp): normalize_desc checks and normalises a descriptor,
// report_status records a status for pax_last_error() and prints msg.
pax_status_t normalize_desc(const pax_gemm_desc_t* d, Problem* p);
pax_status_t report_status(pax_status_t s, const char* msg);

// Read and clear the device error word of each kernel translation unit on
// the current device.
int read_clear_device_error_tc();
int read_clear_device_error_skinny();
int read_clear_device_error_peer();

// Rank barrier over peer memory (peer_sync.cu, pax_peer_barrier).
constexpr int kPeerMaxPeers = 7;
cudaError_t peer_barrier_launch(unsigned long long* own, unsigned long long* const* peers, int n_peers, int slot,
                                unsigned long long epoch, unsigned long long limit_ns, cudaStream_t stream);
// Set the limit of the kernels' abandonable waits on the current device
// (pax_selftest_set_wait_limit).
bool set_wait_limit_tc(unsigned long long ns);
bool set_wait_limit_skinny(unsigned long long ns);

// Fill a device fp16 buffer with a counter-hash uniform[lo,hi) pattern
// (bench state only).
pax_status_t fill_uniform_f16(__half* p, long long n, unsigned long long seed, float lo, float hi,
                              cudaStream_t stream);

}  // namespace pax
