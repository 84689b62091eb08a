// gemm_tc.cuh -- persistent, warp-specialised tcgen05 GEMM for sm_100a.
//
//   C[M][N] = epi(A[M][K] . B[K][N]),  A, B fp16 row-major, fp32 accumulate in
//   TMEM, C fp32 or fp16 row-major.
//
// Replaces the reference's sm_86 kernels on the GEMM path
// (src/rtx_gemm_wmma.cu:23-105, src/rtx_gemm_pipeline.cu:119-325,
// src/rtx_gemm_epilogue.cu:243-356); the epilogue semantics are those of
// src/rtx_gemm_epilogue.cu:176-233 (see epilogue.cuh).
//
// CTA layout (320 threads, one CTA per SM, or one CTA pair per two SMs with
// tcgen05 cta_group::2; persistent over work items):
//   warp 0      TMA producer: A 128x64 (K-major) and the item's B columns
//               in 64-column boxes (N-major; up to four adjacent boxes per
//               load when N is a multiple of 64) per k-block into a
//               STAGES-deep ring of 128B-swizzled shared-memory slots,
//               mbarrier full/empty pairs.
//   warp 1      MMA issuer (the pair leader): tcgen05.mma K=16, four k-steps
//               per stage, one MMA of N <= 256 per k-step (two for items
//               wider than 256 columns, sharing A); commits slot releases
//               and accumulator-ready.
//   warps 2..9  epilogue, two per TMEM lane quarter, each on half of the
//               item's columns: tcgen05.ld 32 lanes x 32 columns, bias /
//               residual / GeLU in registers, fp32->fp16, swizzled staging
//               in shared memory, TMA store (an fp16 residual is TMA-loaded
//               into that staging buffer first; replicated outputs are
//               copied to the replicas once the accumulator is handed
//               back).  With two accumulators, buffer i is handed back to
//               the MMA warp as soon as it is read, so the epilogue of one
//               item overlaps the main loop of the next.
// Work items: whole tiles and column halves of the tail wave in round-robin
// order, or (wide tiles) a host-planned per-pair list of 512 / 384 / 256
// column items.  Ragged M/N/K edges: TMA zero-fills out-of-range loads and
// clips stores.
//
// This header holds the kernel template and its launcher template; the
// gemm_tc_f16.cu / gemm_tc_f32.cu translation units instantiate them per
// output type, and gemm_tc.cu picks the tile shape.
#pragma once
#include "internal.h"
#include "sm100.cuh"
#include "epilogue.cuh"

#include <cudaTypedefs.h>
#include <stdlib.h>
#include <string.h>
#include <mutex>
#include <stdio.h>

namespace pax {

struct TcParams {
    int M, N, K;
    int tiles_m, tiles_n, num_tiles;
    int group_m;  // output tiles are visited in column-major groups of group_m tile rows
    int c_evict_first;  // store C with an L2 evict-first policy (C much larger than L2)
    int res_tma;        // fp16 residual, fp16 C: residual chunks staged by TMA (tmR)
    int zr;             // batched: the residual has one slice per item (else all share slice 0)
    int b_pairs;        // N % 64 == 0: B's 64-column boxes loaded two at a time (tmB2)
    int res_evict_first;  // TMA residual loads with an L2 evict-first policy
    // Work items: tiles [0, full_items) whole, then the last tail_tiles tiles
    // (the tail wave) as two column halves each, so
    // num_items = full_items + 2 * tail_tiles.
    int full_items, tail_tiles, num_items;
    // Batched launch: tiles of item b are [b * batch_tiles, (b + 1) * batch_tiles);
    // the tensor maps are 3-D with the item as z.  za / zb: whether A / B
    // have one slice per item (else all items share slice 0).  sbias / sres:
    // element strides of bias / residual between items.
    int batch_tiles, za, zb;
    long long sbias, sres;
    // Planned work list (device memory): plan[0 .. units] are the units'
    // first items, plan[units + 1 + k] item k (TcItemTable's packing).
    // Null: round-robin over num_items.
    const int* plan;
    EpiParams epi;
};

// Extra destinations of C (replicated output): tensor maps with C's shape
// and pitch over other buffers, typically other GPUs' memory mapped into
// this process.  Every finished chunk of C is stored to each of them too, so
// an all-gather of C happens inside the epilogue, overlapped with the MMAs of
// the next tiles.  Stores only: no TMA load ever reads another GPU here.
constexpr int kTcMaxReplicas = 7;
struct TcReplicas {
    CUtensorMap map[kTcMaxReplicas];
    int n;
};

// Output tile -> batch item, and the tile within it.
__device__ __forceinline__ int tile_batch(int t, const TcParams& p, int& tl) {
    const int b = t / p.batch_tiles;
    tl = t - b * p.batch_tiles;
    return b;
}

// Epilogue operands of batch item b.
__device__ __forceinline__ EpiParams epi_for(const TcParams& p, int b, bool res_f32) {
    EpiParams e = p.epi;
    if (e.bias) e.bias += (long long)b * p.sbias;
    if (e.residual)
        e.residual = static_cast<const char*>(e.residual) + (long long)b * p.sres * (res_f32 ? 4 : 2);
    return e;
}

// Work item -> output tile and column half: half = -1 for a whole tile, else
// 0 / 1 for the left / right BN/2 columns of a tail tile.
__device__ __forceinline__ void tc_item(int item, const TcParams& p, int& tile, int& half) {
    if (item < p.full_items) {
        tile = item;
        half = -1;
    } else {
        const int j = item - p.full_items;
        tile = p.full_items + (j >> 1);
        half = j & 1;
    }
}

// Tile configuration.  PAIR = false: one CTA computes a 128 x BN tile with
// tcgen05.mma.cta_group::1.  PAIR = true: a cluster of two CTAs computes a
// 256 x BN tile with tcgen05.mma.cta_group::2 issued by the even CTA; each
// CTA stages its own 128 rows of A and BN/2 columns of B, and holds its 128
// rows of the accumulator in its own TMEM.  A column-half item is the same
// with BN/2 accumulator columns (MMA N = BN/2).
// BN = 512 (pair only, "wide"): the pair computes a 256 x 512 tile as two
// N = 256 MMAs per k-step that share A, into one accumulator filling all 512
// TMEM columns (no second accumulator buffer).  Each CTA stages B columns
// [rank*128, +128) and [256 + rank*128, +128) of the tile.  Fewer staged
// bytes per MMA than the 256 x 256 tile; the epilogue is not overlapped with
// the next tile's MMAs.  Its column halves are single N = 256 MMAs.
template <int BN_, int STAGES_, typename OutT, bool PAIR_>
struct TcCfg {
    static constexpr bool PAIR = PAIR_;
    static constexpr bool WIDE = BN_ == 512;
    static constexpr int BM = 128;                       // rows per CTA
    static constexpr int BN = BN_;                       // accumulator columns (MMA N)
    static constexpr int BN_LOCAL = PAIR ? BN / 2 : BN;  // B columns staged per CTA
    static constexpr int TILE_M = PAIR ? 2 * BM : BM;    // rows per output tile
    static constexpr int BK = 64, STAGES = STAGES_;
    static constexpr uint32_t A_BYTES = BM * BK * 2;        // 16 KiB
    static constexpr uint32_t B_BYTES = BN_LOCAL * BK * 2;  // 16 / 32 KiB
    static constexpr uint32_t STAGE_BYTES = A_BYTES + B_BYTES;
    static constexpr int EPI_COLS = 128 / (int)sizeof(OutT);  // one 128-byte row per chunk
    // Epilogue: two warps per TMEM lane quarter, each owning half of the
    // item's columns (at least one 128-byte chunk), one staging buffer each.
    static constexpr int EPI_WARPS = 8;
    static constexpr int THREADS = 64 + 32 * EPI_WARPS;
    static constexpr uint32_t STG_BYTES = 32 * 128;            // per warp
    static constexpr uint32_t STG_TOTAL = EPI_WARPS * STG_BYTES;
    static constexpr int ACC_BUFS = WIDE ? 1 : 2;        // accumulator buffers in TMEM
    static constexpr uint32_t TMEM_COLS = ACC_BUFS * BN;
    // full[STAGES], empty[STAGES], tfull[2], tempty[2], drain, one per
    // epilogue warp for the reloads of its replica pushes, and (pair) the
    // non-leader's report of how many k-blocks it issued.
    static constexpr uint32_t NUM_BARS = 2 * STAGES + 6 + EPI_WARPS;
    static constexpr size_t SMEM_BYTES =
        1024 + (size_t)STAGES * STAGE_BYTES + STG_TOTAL + NUM_BARS * 8 + 16;
    static_assert(SMEM_BYTES <= 232448, "shared memory budget");
    static_assert(TMEM_COLS == 256 || TMEM_COLS == 512, "TMEM allocation must be a power of two");
    static_assert((BN_LOCAL / 2) % 64 == 0, "B (and a half of it) is staged in 64-column boxes");
    static_assert(!WIDE || PAIR, "the wide tile is a CTA-pair tile");
};

__device__ __forceinline__ void tile_coords(int t, const TcParams& p, int& mb, int& nb) {
    const int per_group = p.group_m * p.tiles_n;
    const int g = t / per_group;
    const int first_m = g * p.group_m;
    const int gm = min(p.tiles_m - first_m, p.group_m);
    const int r = t - g * per_group;
    mb = first_m + r % gm;
    nb = r / gm;
}

// One unit of work: output rows [mb * TILE_M, +TILE_M) of batch item bz,
// columns [col0, col0 + w).  w is the tile width, half of it (tail halves),
// or, from a planned table, 512 / 384 / 256 / 128 for CTA-pair tiles.
struct TcWork {
    int bz, mb, col0, w;
};

template <int BN>
__device__ __forceinline__ TcWork tc_work(int k, const TcParams& p, const unsigned int* items) {
    TcWork w;
    if (items != nullptr) {
        const unsigned int it = __ldg(items + k);
        const int code = (int)(it >> 28) & 3;
        w.bz = 0;
        w.mb = (int)(it & 0xFFFFu);
        w.col0 = (int)((it >> 16) & 0xFFFu) * 128;
        w.w = code == 0 ? 512 : code == 1 ? 384 : code == 2 ? 256 : 128;
    } else {
        int t, half, tl, nb;
        tc_item(k, p, t, half);
        w.bz = tile_batch(t, p, tl);
        tile_coords(tl, p, w.mb, nb);
        w.col0 = nb * BN + (half > 0 ? BN / 2 : 0);
        w.w = half < 0 ? BN : BN / 2;
    }
    return w;
}


// Wide pair tile, item of width w: the accumulator column holding item
// column ic.  CTA r stages item columns [r w/2, (r+1) w/2), the first n0/2
// of them for MMA 0 and the rest for MMA 1; each MMA's accumulator columns
// take CTA 0's share first, then CTA 1's.  Identity for w <= 256.
__device__ __forceinline__ int wide_tmem_col(int ic, int w) {
    const int n0 = w < 256 ? w : 256, h0 = n0 / 2, hw = w / 2, h1 = (w - n0) / 2;
    if (ic < h0) return ic;
    if (ic < hw) return n0 + (ic - h0);
    if (ic < hw + h0) return h0 + (ic - hw);
    return n0 + h1 + (ic - hw - h0);
}

template <int BN, int STAGES, typename OutT, int RES, int GELU, bool PAIR>
__global__ void __launch_bounds__(64 + 32 * 8, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ CUtensorMap tmC, const __grid_constant__ CUtensorMap tmR,
                   const __grid_constant__ CUtensorMap tmB2, const __grid_constant__ CUtensorMap tmB3,
                   const __grid_constant__ CUtensorMap tmB4, const TcParams p,
                   const __grid_constant__ TcReplicas reps) {
    using Cfg = TcCfg<BN, STAGES, OutT, PAIR>;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem =
        reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sA = smem;
    uint8_t* sB = sA + STAGES * Cfg::A_BYTES;
    uint8_t* sStg = sB + STAGES * Cfg::B_BYTES;
    uint64_t* bars = reinterpret_cast<uint64_t*>(sStg + Cfg::STG_TOTAL);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + Cfg::NUM_BARS);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    volatile uint32_t* issued_slot = tmem_slot + 2;  // pair: the non-leader's k-block count

    const uint32_t bar0 = smem_u32(bars);
    const uint32_t full0 = bar0;                     // [STAGES]
    const uint32_t empty0 = bar0 + 8u * STAGES;      // [STAGES]
    const uint32_t tfull0 = bar0 + 16u * STAGES;     // [2]
    const uint32_t tempty0 = tfull0 + 16u;           // [2]
    const uint32_t drain_bar = tempty0 + 16u;
    const uint32_t push0 = drain_bar + 8u;           // [EPI_WARPS]
    const uint32_t report_bar = push0 + 8u * Cfg::EPI_WARPS;

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    // Pair bookkeeping: rank within the CTA pair, index of the pair, number of pairs.
    const uint32_t rank = PAIR ? cluster_ctarank() : 0u;
    const int unit = PAIR ? (int)(blockIdx.x >> 1) : (int)blockIdx.x;
    const int units = PAIR ? (int)(gridDim.x >> 1) : (int)gridDim.x;
    const bool leader = rank == 0;
    // This unit's work items: a planned table's slice, or round-robin.
    const bool tabbed = p.plan != nullptr;
    const int k_begin = tabbed ? __ldg(p.plan + unit) : unit;
    const int k_end = tabbed ? __ldg(p.plan + unit + 1) : p.num_items;
    const int k_step = tabbed ? 1 : units;
    const unsigned int* items = tabbed ? reinterpret_cast<const unsigned int*>(p.plan + units + 1) : nullptr;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(full0 + 8u * s, 1);
            mbar_init(empty0 + 8u * s, 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(tfull0 + 8u * b, 1);
            // one arrive per epilogue warp (of both CTAs in pair mode)
            mbar_init(tempty0 + 8u * b, PAIR ? 2 * Cfg::EPI_WARPS : Cfg::EPI_WARPS);
        }
        mbar_init(drain_bar, 1);
        for (int w = 0; w < Cfg::EPI_WARPS; ++w) mbar_init(push0 + 8u * w, 1);
        mbar_init(report_bar, 1);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 0 && lane == 0) {
        tma_prefetch_desc(&tmA);
        tma_prefetch_desc(&tmB);
        tma_prefetch_desc(&tmC);
        if (p.res_tma) tma_prefetch_desc(&tmR);
        if (p.b_pairs) {
            tma_prefetch_desc(&tmB2);
            if constexpr (Cfg::WIDE) {
                tma_prefetch_desc(&tmB3);
                tma_prefetch_desc(&tmB4);
            }
        }
    }
    if (warp == 1) {
        tmem_alloc<PAIR ? 2 : 1>(smem_u32(tmem_slot), Cfg::TMEM_COLS);
        tmem_relinquish<PAIR ? 2 : 1>();
    }
    tc_fence_before();
    if constexpr (PAIR) {
        cluster_sync();  // barrier initialisation visible to the peer CTA
    } else {
        __syncthreads();
    }
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    const int num_kb = (p.K + Cfg::BK - 1) / Cfg::BK;
    // A following kernel launched with programmatic serialization may start
    // its prologue now; it waits for this grid before touching memory.
    if (threadIdx.x == 0) pdl_launch_dependents();

    if (warp == 0) {
        // ------------------------------------------------ TMA producer
        if (lane == 0) {
            pdl_wait();  // A and B may be written by the previous grid
            int stage = 0;
            uint32_t phase = 0;
            bool ok = true;
            uint32_t issued = 0, last_parity = 0;
            int total = 0;  // k-blocks issued by this CTA
            for (int k = k_begin; ok && k < k_end; k += k_step) {
                const TcWork wk = tc_work<BN>(k, p, items);
                const int za = p.za ? wk.bz : 0, zb = p.zb ? wk.bz : 0;
                // MMA 0 has N = n0, MMA 1 (items wider than 256 only) N = n1.
                // In pair mode each CTA supplies half of each MMA's B columns
                // (l0 / l1); alone, all of them.  Wide items: CTA r stages
                // the item's columns [r w/2, (r+1) w/2) in one piece, its first
                // l0 for MMA 0 and the next l1 for MMA 1, so one load can
                // bring them all; the epilogue maps accumulator columns back
                // to item columns (wide_tmem_col).  Otherwise CTA r stages
                // MMA 0's columns [r l0, (r+1) l0).
                const int n0 = wk.w < 256 ? wk.w : 256, n1 = Cfg::WIDE ? wk.w - n0 : 0;
                const int l0 = PAIR ? n0 / 2 : n0, l1 = PAIR ? n1 / 2 : n1;
                const int c0 = wk.col0 + (int)rank * (l0 + l1), c1 = c0 + l0;
                const int arow = wk.mb * Cfg::TILE_M + (int)rank * Cfg::BM;
                const uint32_t bytes = Cfg::A_BYTES + (uint32_t)(l0 + l1) * Cfg::BK * 2;
                for (int kb = 0; kb < num_kb; ++kb) {
                    if (!mbar_wait(empty0 + 8u * stage, phase ^ 1u, abort_flag)) {
                        ok = false;
                        break;
                    }
                    const uint32_t fb = full0 + 8u * stage;
                    const uint32_t adst = smem_u32(sA + stage * Cfg::A_BYTES);
                    const uint32_t bdst = smem_u32(sB + stage * Cfg::B_BYTES);
                    if constexpr (PAIR) {
                        // Both CTAs' loads complete on the leader's full barrier;
                        // the leader announces the bytes of both.
                        const uint32_t fb_leader = mapa_shared(fb, 0);
                        if (leader) mbar_arrive_expect_tx(fb, 2 * bytes);
                        tma_load_3d_pair(adst, &tmA, fb_leader, kb * Cfg::BK, arow, za);
                        // 64-column boxes: MMA 0's first, then MMA 1's; adjacent
                        // boxes in one load where B allows it.
                        if (Cfg::WIDE && p.b_pairs) {
                            // This CTA's l0 + l1 columns are adjacent: 1 to 4 boxes.
                            const int nb = (l0 + l1) / 64;
                            const CUtensorMap* m = nb == 4 ? &tmB4 : nb == 3 ? &tmB3 : nb == 2 ? &tmB2 : nullptr;
                            if (m != nullptr)
                                tma_load_4d_pair(bdst, m, fb_leader, 0, kb * Cfg::BK, c0 >> 6, zb);
                            else
                                tma_load_3d_pair(bdst, &tmB, fb_leader, c0, kb * Cfg::BK, zb);
                        } else {
                            int j = 0;
                            if (p.b_pairs)
                                for (; j + 2 <= l0 / 64; j += 2)
                                    tma_load_4d_pair(bdst + j * 8192, &tmB2, fb_leader, 0, kb * Cfg::BK, (c0 >> 6) + j,
                                                     zb);
                            for (; j < l0 / 64; ++j)
                                tma_load_3d_pair(bdst + j * 8192, &tmB, fb_leader, c0 + j * 64, kb * Cfg::BK, zb);
                            j = 0;
                            if (p.b_pairs)
                                for (; j + 2 <= l1 / 64; j += 2)
                                    tma_load_4d_pair(bdst + (l0 / 64 + j) * 8192, &tmB2, fb_leader, 0, kb * Cfg::BK,
                                                     (c1 >> 6) + j, zb);
                            for (; j < l1 / 64; ++j)
                                tma_load_3d_pair(bdst + (l0 / 64 + j) * 8192, &tmB, fb_leader, c1 + j * 64,
                                                 kb * Cfg::BK, zb);
                        }
                    } else {
                        mbar_arrive_expect_tx(fb, bytes);
                        tma_load_3d(adst, &tmA, fb, kb * Cfg::BK, arow, za);
                        int j = 0;
                        if (p.b_pairs)
                            for (; j + 2 <= l0 / 64; j += 2)
                                tma_load_4d(bdst + j * 8192, &tmB2, fb, 0, kb * Cfg::BK, (c0 >> 6) + j, zb);
                        for (; j < l0 / 64; ++j)
                            tma_load_3d(bdst + j * 8192, &tmB, fb, c0 + j * 64, kb * Cfg::BK, zb);
                        j = 0;
                        if (p.b_pairs)
                            for (; j + 2 <= l1 / 64; j += 2)
                                tma_load_4d(bdst + (l0 / 64 + j) * 8192, &tmB2, fb, 0, kb * Cfg::BK, (c1 >> 6) + j, zb);
                        for (; j < l1 / 64; ++j)
                            tma_load_3d(bdst + (l0 / 64 + j) * 8192, &tmB, fb, c1 + j * 64, kb * Cfg::BK, zb);
                    }
                    ++total;
                    issued |= 1u << stage;
                    last_parity = (last_parity & ~(1u << stage)) | (phase << stage);
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
            }
            if constexpr (PAIR) {
                // Every TMA load either CTA issued must land before the pair
                // tears down.  They all complete on the leader's full
                // barriers, so the non-leader reports how many k-blocks it
                // issued, and the leader settles the last phase of every
                // stage: a phase only one CTA contributed to is completed
                // for the other (its bytes cancelled, or the phase armed for
                // the non-leader's bytes alone), then waited for.  Both CTAs
                // issue the same k-block sequence, gated by the same slot
                // releases, so neither is more than STAGES k-blocks ahead.
                // After a normal run every phase has already completed.  The
                // non-leader leaves only at the final cluster barrier, after
                // these waits.
                if (!leader) {
                    st_shared_cluster_u32(smem_u32((const void*)issued_slot), 0, (uint32_t)total);
                    mbar_arrive_cluster(report_bar, 0);
                } else {
                    // The non-leader reports when its own loop ends, at the
                    // latest one abandonable wait later.
                    bool reported = mbar_wait<true>(report_bar, 0, nullptr);
                    if (!reported) reported = mbar_wait<true>(report_bar, 0, nullptr);
                    const int t_nl = reported ? (int)*issued_slot : total;
                    const int t_max = total > t_nl ? total : t_nl;
                    for (int s = 0; s < STAGES; ++s) {
                        if (t_max <= s) break;
                        const int i = s + ((t_max - 1 - s) / STAGES) * STAGES;  // last k-block on stage s
                        const bool mine = i < total, theirs = i < t_nl;
                        if (mine != theirs) {
                            const TcWork wk = tc_work<BN>(k_begin + (i / num_kb) * k_step, p, items);
                            const int n0 = wk.w < 256 ? wk.w : 256, n1 = Cfg::WIDE ? wk.w - n0 : 0;
                            const uint32_t half = Cfg::A_BYTES + (uint32_t)(n0 / 2 + n1 / 2) * Cfg::BK * 2;
                            if (mine)
                                mbar_complete_tx(full0 + 8u * s, half);  // the non-leader's half never comes
                            else
                                mbar_arrive_expect_tx(full0 + 8u * s, half);  // only the non-leader's half
                        }
                        mbar_wait(full0 + 8u * s, (uint32_t)(i / STAGES) & 1u, nullptr);
                    }
                }
            } else if (!ok) {
                // Abort: every TMA load issued must land before the CTA exits.
                for (int s = 0; s < STAGES; ++s)
                    if (issued & (1u << s)) mbar_wait(full0 + 8u * s, (last_parity >> s) & 1u, nullptr);
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------ MMA issuer (leader only in pair mode)
        if (lane == 0 && leader) {
            int stage = 0;
            uint32_t phase = 0;
            int acc = 0;
            uint32_t acc_phase = 0;
            bool ok = true;
            // Descriptors of stage 0, k-step 0; other stages / k-steps differ
            // only in the start-address field (address >> 4 in the low bits).
            const uint64_t adesc0 = umma_desc_sw128(smem_u32(sA), 16, 1024);
            const uint64_t bdesc0 = umma_desc_sw128(smem_u32(sB), 8192, 1024);
            for (int k = k_begin; ok && k < k_end; k += k_step) {
                const TcWork wk = tc_work<BN>(k, p, items);
                // MMA 0: item columns [0, n0); MMA 1 (items wider than 256):
                // [n0, w), its B boxes after MMA 0's in the stage.
                // Only wide-tile items have a second MMA: a compile-time zero
                // elsewhere keeps the MMA issue loop free of branches.
                const int n0 = wk.w < 256 ? wk.w : 256, n1 = Cfg::WIDE ? wk.w - n0 : 0;
                const uint32_t id0 = umma_idesc_f16(PAIR ? 256 : 128, n0, false, true);
                const uint32_t id1 = umma_idesc_f16(PAIR ? 256 : 128, n1 > 0 ? n1 : 16, false, true);
                const uint64_t b1 = (uint64_t)((((PAIR ? n0 / 2 : n0) / 64) * 8192) >> 4);
                // In pair mode the releases come from both CTAs' epilogues.
                if (!mbar_wait<PAIR>(tempty0 + 8u * acc, acc_phase ^ 1u, abort_flag)) break;
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + (uint32_t)(acc * BN);
                for (int kb = 0; kb < num_kb; ++kb) {
                    if (!mbar_wait(full0 + 8u * stage, phase, abort_flag)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint64_t as = adesc0 + (uint64_t)((stage * Cfg::A_BYTES) >> 4);
                    const uint64_t bs = bdesc0 + (uint64_t)((stage * Cfg::B_BYTES) >> 4);
                    // Straight-line MMA sequences: the one- or two-MMA choice is
                    // made once per stage, not between MMAs.
                    if (n1 > 0) {
#pragma unroll
                        for (int kk = 0; kk < Cfg::BK / 16; ++kk) {
                            const uint64_t ad = as + (uint64_t)((kk * 32) >> 4);    // +32 B along K
                            const uint64_t bd = bs + (uint64_t)((kk * 2048) >> 4);  // +16 rows of K
                            const uint32_t accum = (kb | kk) != 0 ? 1u : 0u;
                            if constexpr (PAIR) {
                                tc_mma_f16_pair(d_tmem, ad, bd, id0, accum);
                                tc_mma_f16_pair(d_tmem + (uint32_t)n0, ad, bd + b1, id1, accum);
                            } else {
                                tc_mma_f16(d_tmem, ad, bd, id0, accum);
                                tc_mma_f16(d_tmem + (uint32_t)n0, ad, bd + b1, id1, accum);
                            }
                        }
                    } else {
#pragma unroll
                        for (int kk = 0; kk < Cfg::BK / 16; ++kk) {
                            const uint64_t ad = as + (uint64_t)((kk * 32) >> 4);
                            const uint64_t bd = bs + (uint64_t)((kk * 2048) >> 4);
                            const uint32_t accum = (kb | kk) != 0 ? 1u : 0u;
                            if constexpr (PAIR)
                                tc_mma_f16_pair(d_tmem, ad, bd, id0, accum);
                            else
                                tc_mma_f16(d_tmem, ad, bd, id0, accum);
                        }
                    }
                    if constexpr (PAIR) {
                        tc_commit_pair(mapa_shared(empty0 + 8u * stage, 0));
                        tc_commit_pair(mapa_shared(empty0 + 8u * stage, 1));
                    } else {
                        tc_commit(empty0 + 8u * stage);
                    }
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
                if (!ok) break;
                if constexpr (PAIR) {
                    tc_commit_pair(mapa_shared(tfull0 + 8u * acc, 0));
                    tc_commit_pair(mapa_shared(tfull0 + 8u * acc, 1));
                } else {
                    tc_commit(tfull0 + 8u * acc);
                }
                if (++acc == Cfg::ACC_BUFS) {
                    acc = 0;
                    acc_phase ^= 1u;
                }
            }
            // No MMA may still be writing TMEM (or reading either CTA's shared
            // memory) when the pair tears down.
            if constexpr (PAIR)
                tc_commit_pair(mapa_shared(drain_bar, 0));
            else
                tc_commit(drain_bar);
            mbar_wait(drain_bar, 0, nullptr);
        }
    } else {
        // ------------------------------------------------ epilogue warps
        pdl_wait();  // bias, residual and C may belong to the previous grid
        constexpr int EC = Cfg::EPI_COLS;
        const int q = warp & 3;          // TMEM lane quarter this warp may read
        const int wh = (warp - 2) >> 2;  // which half of the item's columns
        uint8_t* sbuf = sStg + (warp - 2) * Cfg::STG_BYTES;
        // C much larger than L2 passes through it once.
        const uint64_t pol_stream = l2_evict_first_policy();
        // This warp's barrier for TMA loads into its staging buffer (residual
        // chunks, replica reloads); every lane tracks its phase.
        const uint32_t pbar = push0 + 8u * (uint32_t)(warp - 2);
        uint32_t push_phase = 0;
        // fp16 residual with fp16 C: each chunk's residual tile (32 rows x 64
        // columns, the output chunk's shape) is TMA-loaded into the staging
        // buffer, read from there and overwritten by the output chunk.  Whole
        // 128-byte rows, each fetched once, instead of one 64-byte half-row
        // per lane per 32-column sub-chunk.
        constexpr bool kResSmem = RES == 1 && sizeof(OutT) == 2;
        const bool res_tma = kResSmem && p.res_tma != 0;
        bool res_pending = false;  // a residual load is in flight (lane 0 issued it)
        const uint32_t sbuf_u32 = smem_u32(sbuf);
        auto load_residual = [&](int col, int row0_, int bz_) {
            if (lane == 0) {
                bulk_wait_read<0>();  // the buffer's last store has read it
                mbar_arrive_expect_tx(pbar, Cfg::STG_BYTES);
                if (p.res_evict_first)
                    tma_load_3d_hint(sbuf_u32, &tmR, pbar, col, row0_, bz_, pol_stream);
                else
                    tma_load_3d(sbuf_u32, &tmR, pbar, col, row0_, bz_);
            }
            res_pending = true;
        };
        int acc = 0;
        uint32_t acc_phase = 0;
        for (int k = k_begin; k < k_end; k += k_step) {
            const TcWork wk = tc_work<BN>(k, p, items);
            const int bz = wk.bz, mb = wk.mb;
            const EpiParams ep = epi_for(p, bz, RES == 2);
            // This warp's columns of the item: half of them, but at least one
            // 128-byte chunk (an item that narrow leaves the second warp of
            // the lane quarter without columns).
            const int width = wk.w;
            const bool two = width / 2 >= EC;
            const int wcols = two ? width / 2 : (wh == 0 ? width : 0);
            const int wcol = two ? wh * (width / 2) : 0;  // offset within the item
            const int row0 = mb * Cfg::TILE_M + (int)rank * Cfg::BM + q * 32;
            const long long row = (long long)row0 + lane;
            const long long tcol0 = (long long)wk.col0 + wcol;
            // Chunks wholly outside C (beyond N, or this warp's 32 rows beyond
            // M) are neither read nor stored.
            long long valid_cols = p.N - tcol0;
            if (valid_cols > wcols) valid_cols = wcols;
            if (valid_cols < 0) valid_cols = 0;
            const int nch = row0 < p.M ? (int)((valid_cols + EC - 1) / EC) : 0;
            // Operands that do not depend on the accumulator are fetched before
            // waiting for it: this warp's bias and the first residual chunk.
            const uint4 bias8 = bias_tile_load(tcol0, wcols, lane, p.N, ep);
            ResChunk<32, RES> rc;
            if (res_tma) {
                if (nch > 0) load_residual((int)tcol0, row0, p.zr ? bz : 0);
            } else if (wcols > 0) {
                res_prefetch<32, RES>(rc, row, tcol0, p.M, p.N, ep);
            }
            bool ok = mbar_wait(tfull0 + 8u * acc, acc_phase, abort_flag);
            ok = __all_sync(0xffffffffu, ok);
            if (!ok) break;
            tc_fence_after();
            const uint32_t t_row = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * BN);
            auto release_accumulator = [&]() {
                // Whole accumulator read: hand it back to the MMA warp (of the
                // pair leader).
                tc_fence_before();
                __syncwarp();
                if (lane == 0) {
                    if (PAIR && !leader)
                        mbar_arrive_cluster(tempty0 + 8u * acc, 0);
                    else
                        mbar_arrive(tempty0 + 8u * acc);
                }
            };
            if (nch == 0) release_accumulator();
            // Each chunk is one 128-byte output row per lane (EC columns), built
            // from 32-column sub-chunks: TMEM load, epilogue, GeLU, pack.  Only
            // 32 fp32 values are live at a time.
#pragma unroll 1
            for (int ci = 0; ci < nch; ++ci) {
                if (res_tma) {
                    // Every lane reads the tile, so every lane waits for it.
                    mbar_wait(pbar, push_phase, nullptr);
                    push_phase ^= 1u;
                    res_pending = false;
                }
                uint32_t w[32];  // packed output row
#pragma unroll
                for (int h = 0; h < EC / 32; ++h) {
                    const int c = ci * EC + 32 * h;
                    float v[32];
                    tmem_ld_32x32b_x32(t_row + (uint32_t)(Cfg::WIDE ? wide_tmem_col(wcol + c, width) : wcol + c), v);
                    tmem_wait_ld();
                    if (ci == nch - 1 && h == EC / 32 - 1) release_accumulator();
                    if constexpr (kResSmem) {
                        if (res_tma) {
                            // This lane's row, 16-byte granules 4h..4h+3 (128B swizzle).
#pragma unroll
                            for (int i = 0; i < 4; ++i)
                                rc.u[i] = ld_shared_v4(sbuf_u32 + (uint32_t)lane * 128u +
                                                       (uint32_t)(((4 * h + i) ^ (lane & 7)) << 4));
                        }
                    }
                    epi_linear<32, RES>(v, rc, bias8, c, ep);
                    // The residual registers are free again: start the next
                    // sub-chunk's loads, which then overlap the GeLU math below.
                    if constexpr (RES != 0) {
                        if (!res_tma && c + 32 < nch * EC)
                            res_prefetch<32, RES>(rc, row, tcol0 + c + 32, p.M, p.N, ep);
                    }
                    epi_gelu<32, GELU>(v);
#pragma unroll
                    for (int i = 0; i < 32 * (int)sizeof(OutT) / 4; ++i) {
                        if constexpr (sizeof(OutT) == 2)
                            w[16 * h + i] = pack_half2(v[2 * i], v[2 * i + 1]);
                        else
                            w[i] = __float_as_uint(v[i]);
                    }
                }
                // The staging buffer is free once this warp's previous store
                // has finished reading it.
                if (lane == 0) bulk_wait_read<0>();
                __syncwarp();
                const uint32_t srow = smem_u32(sbuf) + (uint32_t)lane * 128u;
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    // 128B swizzle: 16-byte chunk j of row r lives at chunk j ^ (r % 8).
                    st_shared_v4(srow + (uint32_t)((j ^ (lane & 7)) << 4), w[4 * j], w[4 * j + 1], w[4 * j + 2],
                                 w[4 * j + 3]);
                }
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) {
                    if (p.c_evict_first)
                        tma_store_3d_hint(&tmC, smem_u32(sbuf), (int)(tcol0 + ci * EC), row0, bz, pol_stream);
                    else
                        tma_store_3d(&tmC, smem_u32(sbuf), (int)(tcol0 + ci * EC), row0, bz);
                    bulk_commit();
                }
                if (res_tma && ci + 1 < nch) load_residual((int)(tcol0 + (ci + 1) * EC), row0, p.zr ? bz : 0);
            }
            // Replicas: once the accumulator is handed back, this warp copies
            // its finished chunks from the local C to every replica, one chunk
            // at a time through its staging buffer (TMA load from this GPU's
            // memory, then one TMA store per replica).  The pushes overlap the
            // next item's MMAs instead of holding up this epilogue; NVLink
            // bandwidth then limits only the last item's pushes.
            if (reps.n > 0 && nch > 0) {
                if (lane == 0) {
                    bulk_wait<0>();  // the local stores of this item are complete
#pragma unroll 1
                    for (int ci = 0; ci < nch; ++ci) {
                        const int col = (int)(tcol0 + ci * EC);
                        bulk_wait_read<0>();  // the previous chunk's pushes have read the buffer
                        mbar_arrive_expect_tx(pbar, Cfg::STG_BYTES);
                        tma_load_3d(smem_u32(sbuf), &tmC, pbar, col, row0, bz);
                        const bool landed = mbar_wait(pbar, push_phase, nullptr);
                        push_phase ^= 1u;
                        if (!landed) break;  // timed out: error recorded, the load has had 2 s
                        for (int d = 0; d < reps.n; ++d) tma_store_3d(&reps.map[d], smem_u32(sbuf), col, row0, bz);
                        bulk_commit();
                    }
                }
                push_phase = __shfl_sync(0xffffffffu, push_phase, 0);  // lane 0 waited for the reloads
                __syncwarp();
            }
            if (++acc == Cfg::ACC_BUFS) {
                acc = 0;
                acc_phase ^= 1u;
            }
        }
        if (lane == 0) {
            // A residual load issued before an abandoned accumulator wait
            // lands before the CTA leaves.
            if (res_pending) mbar_wait(pbar, push_phase, nullptr);
            bulk_wait<0>();
            // Stores to other GPUs are complete; make them visible system-wide
            // before the grid ends.
            if (reps.n > 0) __threadfence_system();
        }
        __syncwarp();
    }

    __syncwarp();
    tc_fence_before();
    if constexpr (PAIR) {
        cluster_sync();  // neither CTA leaves while the pair's MMAs or arrivals may touch it
    } else {
        __syncthreads();
    }
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc<PAIR ? 2 : 1>(tmem_base, Cfg::TMEM_COLS);
    }
}

// ======================================================================
// Host side
// ======================================================================

static PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

// 3-D tensor map of `depth` row-major matrices: `inner` contiguous elements
// per row, `outer` rows `pitch` bytes apart, matrices `zstride` bytes apart;
// box of box_inner x box_outer x 1, 128B swizzle.
static bool make_tmap(CUtensorMap* m, const void* base, CUtensorMapDataType dt, uint64_t inner, uint64_t outer,
                      uint64_t depth, uint64_t pitch_bytes, uint64_t zstride_bytes, uint32_t box_inner,
                      uint32_t box_outer) {
    auto enc = tensor_map_encoder();
    if (!enc) return false;
    cuuint64_t dims[3] = {inner, outer, depth};
    cuuint64_t strides[2] = {pitch_bytes, zstride_bytes};
    cuuint32_t box[3] = {box_inner, box_outer, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = enc(m, dt, 3, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                     CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

// Byte stride between batch items for a tensor map: the given element
// stride, or (single or shared slice) one whole matrix, which is never used
// to address anything but satisfies the encoder.
static uint64_t zstride(long long stride_elems, long long rows, long long pitch_bytes, int elem) {
    if (stride_elems > 0) return (uint64_t)stride_elems * (uint64_t)elem;
    const uint64_t whole = (uint64_t)rows * (uint64_t)pitch_bytes;
    return whole > 0 ? ((whole + 15) & ~uint64_t(15)) : 16;
}

template <int BN, int STAGES, typename OutT, int RES, int GELU, bool PAIR>
static pax_status_t launch_tc_impl(const Problem& pr, const TcPlan& plan, cudaStream_t stream) {
    using Cfg = TcCfg<BN, STAGES, OutT, PAIR>;
    if (plan.table && (!Cfg::WIDE || !plan.table_dev || plan.table->count <= 0 || pr.batch != 1))
        return PAX_ERR_INVALID;
    const bool f16 = sizeof(OutT) == 2;
    CUtensorMap tA, tB, tC;
    const bool za = pr.batch > 1 && pr.sa > 0, zb = pr.batch > 1 && pr.sb > 0;
    const int ce = f16 ? 2 : 4;
    if (!make_tmap(&tA, pr.A, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, pr.K, pr.M, za ? pr.batch : 1, pr.lda * 2,
                   zstride(za ? pr.sa : 0, pr.M, pr.lda * 2, 2), 64, 128))
        return PAX_ERR_CUDA;
    if (!make_tmap(&tB, pr.B, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, pr.N, pr.K, zb ? pr.batch : 1, pr.ldb * 2,
                   zstride(zb ? pr.sb : 0, pr.K, pr.ldb * 2, 2), 64, 64))
        return PAX_ERR_CUDA;
    if (!make_tmap(&tC, pr.C, f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, pr.N, pr.M,
                   pr.batch, pr.ldc * ce, zstride(pr.batch > 1 ? pr.sc : 0, pr.M, pr.ldc * ce, ce), Cfg::EPI_COLS,
                   32))
        return PAX_ERR_CUDA;
    // B as [batch][N/64][K][64]: two adjacent 64-column boxes per load.  Only
    // when N is a multiple of 64, so that a box is wholly inside B or wholly
    // outside it (zero-filled).  Otherwise tB2 is B's map, never read.
    // (The wide tile also loads 3 and 4 boxes at a time: tB3, tB4.)
    CUtensorMap tB2 = tB, tB3 = tB, tB4 = tB;
    int b_pairs = 0;
    if (pr.N % 64 == 0) {
        b_pairs = 1;
        if (const char* e = getenv("PAX_TC_BPAIRS")) b_pairs = atoi(e) != 0 ? 1 : 0;
        auto enc = tensor_map_encoder();
        auto make_b = [&](CUtensorMap* m, uint32_t boxes) {
            cuuint64_t dims[4] = {64, (cuuint64_t)pr.K, (cuuint64_t)(pr.N / 64), (cuuint64_t)(zb ? pr.batch : 1)};
            cuuint64_t strides[3] = {(cuuint64_t)(pr.ldb * 2), 128,
                                     (cuuint64_t)zstride(zb ? pr.sb : 0, pr.K, pr.ldb * 2, 2)};
            cuuint32_t box[4] = {64, 64, boxes, 1};
            cuuint32_t estr[4] = {1, 1, 1, 1};
            return enc != nullptr &&
                   enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, const_cast<void*>(static_cast<const void*>(pr.B)), dims,
                       strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                       CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
        };
        if (b_pairs && !(make_b(&tB2, 2) && (!Cfg::WIDE || (make_b(&tB3, 3) && make_b(&tB4, 4))))) {
            tB2 = tB3 = tB4 = tB;
            b_pairs = 0;
        }
    }
    // Residual tile map (fp16 residual, fp16 C, 16-byte aligned rows): same
    // box and swizzle as C's, so a residual chunk lands where its output
    // chunk is staged.  Otherwise tR is C's map, never read.
    CUtensorMap tR = tC;
    int res_tma = 0;
    const bool zr = pr.batch > 1 && pr.sres > 0;
    if (RES == 1 && f16 && (pr.epi.flags & EPI_RES_VEC) && (!zr || (pr.sres * 2) % 16 == 0)) {
        res_tma = 1;
        if (const char* e = getenv("PAX_TC_RES_TMA")) res_tma = atoi(e) != 0 ? 1 : 0;
        if (res_tma && !make_tmap(&tR, pr.epi.residual, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, pr.N, pr.M,
                                  zr ? pr.batch : 1, pr.epi.ld_res * 2,
                                  zstride(zr ? pr.sres : 0, pr.M, pr.epi.ld_res * 2, 2), Cfg::EPI_COLS, 32))
            return PAX_ERR_CUDA;
    }
    TcReplicas reps;
    memset(&reps, 0, sizeof(reps));
    if (pr.n_replicas < 0 || pr.n_replicas > kTcMaxReplicas) return PAX_ERR_INVALID;
    reps.n = pr.n_replicas;
    for (int d = 0; d < reps.n; ++d)
        if (!make_tmap(&reps.map[d], pr.replicas[d], f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32,
                       pr.N, pr.M, pr.batch, pr.ldc * ce, zstride(pr.batch > 1 ? pr.sc : 0, pr.M, pr.ldc * ce, ce),
                       Cfg::EPI_COLS, 32))
            return PAX_ERR_CUDA;

    TcParams p;
    p.M = (int)pr.M;
    p.N = (int)pr.N;
    p.K = (int)pr.K;
    p.tiles_m = (int)((pr.M + Cfg::TILE_M - 1) / Cfg::TILE_M);
    p.tiles_n = (int)((pr.N + BN - 1) / BN);
    p.batch_tiles = p.tiles_m * p.tiles_n;
    const long long all_tiles = (long long)p.batch_tiles * pr.batch;
    if (all_tiles > 0x7fffffffLL) return PAX_ERR_UNSUPPORTED;
    p.num_tiles = (int)all_tiles;
    p.za = za ? 1 : 0;
    p.zb = zb ? 1 : 0;
    p.sbias = pr.batch > 1 ? pr.sbias : 0;
    p.sres = pr.batch > 1 ? pr.sres : 0;
    p.plan = plan.table ? plan.table_dev : nullptr;
    // Tiles run in column-major groups of group_m tile rows.  Per k-step the
    // U tiles in flight fetch group_m A slices and U / group_m B slices, so
    // the DRAM traffic of large-K problems is least near
    // sqrt(U * tile_n / tile_m), about 8 to 12 here.  Measured, 16 is best
    // for every shape: C5 (256 x 512) 1182 against 1049 TF/s with 8; C3
    // (256 x 256, residual) 1.72 ms and 2.16 GB of DRAM traffic against
    // 1.78 ms and 2.86 GB with 8, and 3.9 GB with 32.
    p.group_m = 16;
    if (const char* g = getenv("PAX_TC_GROUP")) {
        const int v = atoi(g);
        if (v >= 1 && v <= 1024) p.group_m = v;
    }
    // C written once and much larger than L2 would push A and B out of it:
    // store it with an evict-first policy (PAX_TC_C_EVICT=0/1 forces).
    const long long c_bytes = pr.M * pr.N * (long long)ce * pr.batch;
    p.c_evict_first = c_bytes > (64LL << 20) ? 1 : 0;
    if (const char* e = getenv("PAX_TC_C_EVICT")) p.c_evict_first = atoi(e) != 0 ? 1 : 0;
    p.res_tma = res_tma;
    // The residual is read once: with C (same size) it would otherwise push
    // A and B out of L2.
    p.res_evict_first = p.c_evict_first;
    if (const char* e = getenv("PAX_TC_RES_EVICT")) p.res_evict_first = atoi(e) != 0 ? 1 : 0;
    p.b_pairs = b_pairs;
    p.zr = zr ? 1 : 0;
    p.full_items = plan.full_items;
    p.tail_tiles = plan.tail_tiles;
    p.num_items = plan.full_items + 2 * plan.tail_tiles;
    p.epi = pr.epi;
    if (p.num_tiles != plan.full_items + plan.tail_tiles) return PAX_ERR_INVALID;

    auto kern = gemm_tc_kernel<BN, STAGES, OutT, RES, GELU, PAIR>;
    // Attribute is per device; setting it again is cheap and idempotent.
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)Cfg::SMEM_BYTES) != cudaSuccess)
        return PAX_ERR_CUDA;
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = PAIR ? 2 : 1;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.blockDim = dim3(Cfg::THREADS);
    cfg.dynamicSmemBytes = Cfg::SMEM_BYTES;
    cfg.stream = stream;
    cfg.attrs = attr;
    cfg.numAttrs = PAIR ? 2 : 1;
    cfg.gridDim = dim3(PAIR ? 2 * plan.units : plan.units);
    if (cudaLaunchKernelEx(&cfg, kern, tA, tB, tC, tR, tB2, tB3, tB4, p, reps) != cudaSuccess) return PAX_ERR_CUDA;
    return cudaPeekAtLastError() == cudaSuccess ? PAX_OK : PAX_ERR_CUDA;
}

// Resident CTA pairs of the pair kernel on device `dev` (SMs pair up within
// a GPC, so this can be below SMs / 2).
template <typename OutT>
static int tc_pair_units_typed(int dev, int sms) {
    static int cache[64] = {0};
    int& v = cache[dev & 63];
    if (v == 0) {
        using Cfg = TcCfg<256, 6, OutT, true>;
        auto kern = gemm_tc_kernel<256, 6, OutT, 0, 0, true>;
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)Cfg::SMEM_BYTES);
        cudaLaunchConfig_t cfg = {};
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = 2;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.blockDim = dim3(Cfg::THREADS);
        cfg.dynamicSmemBytes = Cfg::SMEM_BYTES;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        cfg.gridDim = dim3(sms & ~1);
        int n = 0;
        if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess || n <= 0) {
            cudaGetLastError();
            n = sms / 2;
        }
        v = n;
    }
    return v;
}

constexpr int kStages256 = 4;
constexpr int kStages128 = 6;
constexpr int kStagesPair = 6;
constexpr int kStagesWide = 4;

// Residual type and GeLU form are compile-time parameters so that each
// instantiation carries only the epilogue code it runs.
template <int BN, int STAGES, typename OutT, int GELU, bool PAIR>
static pax_status_t launch_tc_gelu(const Problem& p, const TcPlan& plan, cudaStream_t stream) {
    if (!(p.epi.flags & EPI_RES)) return launch_tc_impl<BN, STAGES, OutT, 0, GELU, PAIR>(p, plan, stream);
    if (p.epi.flags & EPI_RES_F32) return launch_tc_impl<BN, STAGES, OutT, 2, GELU, PAIR>(p, plan, stream);
    return launch_tc_impl<BN, STAGES, OutT, 1, GELU, PAIR>(p, plan, stream);
}

template <int BN, int STAGES, typename OutT, bool PAIR>
static pax_status_t launch_tc_res(const Problem& p, const TcPlan& plan, cudaStream_t stream) {
    // GeLU-tanh uses the hardware tanh when the result is rounded to fp16
    // anyway, and tanhf for fp32 results.
    if (p.epi.flags & EPI_GELU_TANH)
        return launch_tc_gelu<BN, STAGES, OutT, sizeof(OutT) == 2 ? 3 : 1, PAIR>(p, plan, stream);
    if (p.epi.flags & EPI_GELU_ERF) return launch_tc_gelu<BN, STAGES, OutT, 2, PAIR>(p, plan, stream);
    return launch_tc_gelu<BN, STAGES, OutT, 0, PAIR>(p, plan, stream);
}

// plan.shape: 128 / 256 = one CTA per 128 x shape tile; 2 = CTA pair, 256 x 256
// tile; 4 = CTA pair, 256 x 512 tile.
template <typename OutT>
static pax_status_t launch_tc_typed(const Problem& p, const TcPlan& plan, cudaStream_t stream) {
    if (plan.shape == 4) return launch_tc_res<512, kStagesWide, OutT, true>(p, plan, stream);
    if (plan.shape == 2) return launch_tc_res<256, kStagesPair, OutT, true>(p, plan, stream);
    if (plan.shape == 256) return launch_tc_res<256, kStages256, OutT, false>(p, plan, stream);
    return launch_tc_res<128, kStages128, OutT, false>(p, plan, stream);
}

static int read_clear_device_error_this_unit() {
    int v = 0, z = 0;
    if (cudaMemcpyFromSymbol(&v, g_pax_device_error, sizeof(int)) != cudaSuccess) return -1;
    if (v) cudaMemcpyToSymbol(g_pax_device_error, &z, sizeof(int));
    return v;
}

static bool set_wait_limit_this_unit(unsigned long long ns) {
    return cudaMemcpyToSymbol(g_pax_wait_limit_ns, &ns, sizeof(ns)) == cudaSuccess;
}

}  // namespace pax
