// gemm_skinny.cu -- swap-AB tcgen05 GEMM for small M (decode shapes).
//
//   C[M][N] = epi(A[M][K] . B[K][N]), M <= 64.  The reference has no separate
//   skinny path: its kernels tile M by 128 and would leave most of every tile
//   empty (src/rtx_gemm_epilogue.cu:362-366).  Here the product is computed
//   transposed, C^T = B^T . A^T, so N supplies the 128-row MMA dimension and
//   M (padded to MP, a multiple of 16) the MMA N dimension:
//     MMA A operand: B^T tile, 128 n x BK k, read N-major straight from B.
//     MMA B operand: A tile, MP rows x BK k, K-major.
//   Two work layouts over the (column tiles x k-blocks) units:
//     lockstep: one CTA per (tile, K slice), the slices of a tile
//       interleaved by k-block, so all CTAs stream the same k-rows of B
//       together (the default while tiles fit the SMs);
//     stream-K: equal contiguous unit ranges, one per persistent CTA, each
//       visited last to first.
//   A column tile split between CTAs is finished by the contributor that
//   computes its last K part: every other contributor writes its fp32
//   partial sum to its own workspace slot and release-stores this launch's
//   epoch into its flag; the finisher waits for those flags (bounded) and
//   adds the partial sums in CTA order, so the result does not depend on
//   timing and nothing needs clearing between launches.
//
// Warp roles as in gemm_tc.cu: warp 0 TMA, warp 1 MMA + TMEM, warps 2..5
// epilogue.
#include "internal.h"
#include "sm100.cuh"
#include "epilogue.cuh"

#include <cudaTypedefs.h>
#include <atomic>
#include <mutex>
#include <stdio.h>
#include <stdlib.h>
#include <vector>

namespace pax {

struct SkinnyParams {
    int M, N, K;
    int num_tiles;  // ceil(N / NT)
    int kblocks;    // ceil(K / 64)
    long long work; // num_tiles * kblocks
    int grid;       // number of CTAs (<= work)
    int slices;     // lockstep layout: K slices per tile (CTA = tile * slices + slice); 0 = stream-K
    int korder;     // stream-K: the CTA's segments last to first (always set there; see sk_next_seg)
    // Lockstep layout with one slice per tile only: CTAs in groups of
    // rot_group start their k loop at different k-blocks (group g at
    // g * kblocks / groups, wrapping around), so that fewer CTAs read the same
    // k-block of A at the same time.  0 = every CTA starts at k-block 0.
    int rot_group;
    int b_early;    // B may be copied to shared memory before the previous grid ends
    // Batched launch (rr = 1): `batch` items of num_tiles tiles each; CTA c
    // takes whole tiles c, c + grid, ... of all items (no K split).  Tile t
    // is tile t % num_tiles of item t / num_tiles; the tensor maps are 3-D
    // with the item as z (za / zb: A / B have one slice per item, else the
    // items share slice 0).  sc, sbias, sres: element strides between items.
    int rr, batch, za, zb;
    long long sc, sbias, sres;
    float* ws;      // [grid][MP][NT] fp32 partial sums, one slot per CTA
    // [grid] publication flags: CTA c sets flags[c] to this launch's epoch
    // once its partial sum is in its slot.  A flag left by an earlier launch
    // (finished or aborted) holds an older epoch, so nothing needs clearing
    // between launches.
    unsigned long long* flags;
    unsigned long long epoch;  // this launch's epoch, never 0 (64 bits: never wraps in practice)
    __half* c16;    // exactly one of c16 / c32 is set
    float* c32;
    long long ldc;
    EpiParams epi;
};

// MP: M padded to a multiple of 16 (the MMA N).  NT: output columns per work
// unit, NT/128 MMAs of M = 128 per k-step.  Wider units make each k-row of B
// a longer contiguous DRAM burst (NT * 2 bytes).  BK: k-rows per ring slot
// (a "k-block"), 64 or 128.  With 128 every slot holds two 64-wide k-steps'
// worth: half the TMA instructions, barrier operations and MMA commits per
// byte of B (on C4 the MMA issue and release of a slot cost about 12 % of
// the streaming rate with 64).
template <int MP_, int NT_, int BK_>
struct SkCfg {
    static constexpr int MP = MP_, NT = NT_, BK = BK_;
    static constexpr int NSUB = NT / 128;
    static constexpr uint32_t B_COL_BYTES = BK * 128;  // one 64-column box: BK rows of 128 bytes
    static constexpr uint32_t B_BYTES = NT * BK * 2;   // NT/64 boxes of 64n x BK k
    static constexpr uint32_t A_HALF_BYTES = MP * 128; // MP rows of 64 k (128 bytes)
    static constexpr uint32_t A_BYTES = MP * BK * 2;   // BK/64 such boxes
    static constexpr uint32_t STAGE_BYTES = B_BYTES + A_BYTES;
    static constexpr int STAGES = (225 * 1024) / STAGE_BYTES;
    static constexpr uint32_t ACC_COLS = NSUB * MP;  // one accumulator: NSUB blocks of MP columns
    static constexpr uint32_t TMEM_COLS =
        (2 * ACC_COLS <= 32) ? 32 : (2 * ACC_COLS <= 64) ? 64 : (2 * ACC_COLS <= 128) ? 128 : (2 * ACC_COLS <= 256) ? 256 : 512;
    static constexpr uint32_t ACC_STRIDE = TMEM_COLS / 2;  // column offset of accumulator 1
    static constexpr uint32_t NUM_BARS = 2 * STAGES + 5;
    static constexpr size_t SMEM_BYTES = 1024 + (size_t)STAGES * STAGE_BYTES + NUM_BARS * 8 + 16;
    static constexpr uint32_t IDESC = umma_idesc_f16(128, MP, /*a_mn*/ true, /*b_mn*/ false);
    static_assert(SMEM_BYTES <= 232448, "shared memory budget");
    static_assert(STAGES >= 3, "at least three stages in flight");
    static_assert(A_HALF_BYTES % 1024 == 0, "A boxes must keep 1024-byte swizzle alignment");
    static_assert(BK == 64 || BK == 128, "k-block of 64 or 128");
    static_assert(2 * ACC_COLS <= 512, "two accumulators must fit in TMEM");
};

__device__ __forceinline__ long long sk_unit_begin(long long c, const SkinnyParams& p) {
    return c * p.work / p.grid;
}
// CTA whose unit range contains unit x.
__device__ __forceinline__ int sk_owner(long long x, const SkinnyParams& p) {
    return (int)(((x + 1) * p.grid + p.work - 1) / p.work - 1);
}

// One accumulation segment of a CTA: nk k-blocks kb0, kb0 + kstep, ... of
// column tile `tile`.
struct SkSeg {
    int tile, kb0, kstep, nk;
};

// Segments of this CTA in order; `cursor` starts at sk_cursor0().
//   stream-K: the CTA's contiguous unit range [ub, ue), cut at tile edges,
//             first to last; with korder, last to first.  A range shorter
//             than a tile then starts with the head (k-blocks 0..) of its
//             second tile and ends with the tail of its first, so every CTA
//             reads within (tile k-blocks - range length) k-rows of the same
//             place in B at any time.
//   lockstep: one segment, slice s = blockIdx.x % slices of tile
//             blockIdx.x / slices takes k-blocks s, s + slices, ..., so all
//             CTAs advance through the same k-rows of B together.
__device__ __forceinline__ long long sk_cursor0(const SkinnyParams& p) {
    if (p.rr) return blockIdx.x;
    if (p.slices > 0) return 0;
    return p.korder ? sk_unit_begin(blockIdx.x + 1, p) : sk_unit_begin(blockIdx.x, p);
}
__device__ __forceinline__ bool sk_next_seg(const SkinnyParams& p, long long& cursor, SkSeg& sg) {
    const int KB = p.kblocks;
    if (p.rr) {
        if (cursor >= (long long)p.batch * p.num_tiles) return false;
        sg.tile = (int)cursor;
        sg.kb0 = 0;
        sg.kstep = 1;
        sg.nk = KB;
        cursor += p.grid;
        return true;
    }
    if (p.slices > 0) {
        if (cursor != 0) return false;
        cursor = 1;
        const int sl = (int)blockIdx.x % p.slices;
        sg.tile = (int)blockIdx.x / p.slices;
        sg.kb0 = sl;
        sg.kstep = p.slices;
        sg.nk = sl < KB ? (KB - sl + p.slices - 1) / p.slices : 0;
        return sg.nk > 0;
    }
    if (p.korder) {
        const long long ub = sk_unit_begin(blockIdx.x, p);
        if (cursor <= ub) return false;
        sg.tile = (int)((cursor - 1) / KB);
        const long long seg_begin = max(ub, (long long)sg.tile * KB);
        sg.kb0 = (int)(seg_begin - (long long)sg.tile * KB);
        sg.kstep = 1;
        sg.nk = (int)(cursor - seg_begin);
        cursor = seg_begin;
        return true;
    }
    const long long ue = sk_unit_begin(blockIdx.x + 1, p);
    if (cursor >= ue) return false;
    sg.tile = (int)(cursor / KB);
    const long long seg_end = min(ue, (long long)(sg.tile + 1) * KB);
    sg.kb0 = (int)(cursor - (long long)sg.tile * KB);
    sg.kstep = 1;
    sg.nk = (int)(seg_end - cursor);
    cursor = seg_end;
    return true;
}

// One output value of the generic epilogue (scale, bias, residual R[off],
// GeLU), kept out of line: see the output loop of gemm_skinny_kernel.
__device__ __noinline__ float sk_epi_value(float acc, float b, int flags, float alpha, const void* residual,
                                           long long off) {
    float r = 0.f;
    if (flags & EPI_RES)
        r = (flags & EPI_RES_F32) ? static_cast<const float*>(residual)[off]
                                  : __half2float(static_cast<const __half*>(residual)[off]);
    return epi_scalar(acc, b, r, flags, alpha);
}

// First k-block of this CTA's rotated k loop (0 without rotation); always
// in [0, kblocks).
__device__ __forceinline__ int sk_rotation(const SkinnyParams& p) {
    if (p.rot_group <= 0) return 0;
    const int groups = (p.grid + p.rot_group - 1) / p.rot_group;
    return (int)(((long long)((int)blockIdx.x / p.rot_group) * p.kblocks) / groups);
}
// k-block of step j of segment sg.  With a rotation (one segment covering
// every k-block, kb0 = 0, kstep = 1) the sequence wraps: every k-block is
// still visited exactly once.
__device__ __forceinline__ int sk_kblock(const SkinnyParams& p, const SkSeg& sg, int j, int rot) {
    int kb = sg.kb0 + j * sg.kstep;
    kb += rot;
    if (kb >= p.kblocks) kb -= p.kblocks;
    return kb;
}

template <int MP, int NT, int BK>
__global__ void __launch_bounds__(192, 1)
    gemm_skinny_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                       const SkinnyParams p) {
    using Cfg = SkCfg<MP, NT, BK>;
    constexpr int STAGES = Cfg::STAGES;
    constexpr int NSUB = Cfg::NSUB;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem =
        reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sB = smem;                              // [STAGES][B_BYTES]
    uint8_t* sA = sB + STAGES * Cfg::B_BYTES;        // [STAGES][A_BYTES]
    uint64_t* bars = reinterpret_cast<uint64_t*>(sA + STAGES * Cfg::A_BYTES);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + Cfg::NUM_BARS);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const uint32_t bar0 = smem_u32(bars);
    const uint32_t full0 = bar0;
    const uint32_t empty0 = bar0 + 8u * STAGES;
    const uint32_t tfull0 = bar0 + 16u * STAGES;
    const uint32_t tempty0 = tfull0 + 16u;
    const uint32_t drain_bar = tempty0 + 16u;

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    // Producer state (thread 0, the TMA producer of warp 0), kept across the
    // barrier below: the producer issues the first k-block's loads before
    // it, right after initialising the barriers, so that the first bytes are
    // on their way while the other warps still set up.  Only one: a whole
    // ring's worth of loads issued at once by every CTA completes later, k-block
    // by k-block, than loads issued as the ring drains (measured on B200:
    // first k-block 3.6 us after kernel start with one, 6.0 us with twelve).
    int p_stage = 0;
    uint32_t p_phase = 0, p_issued = 0, p_last_parity = 0;
    long long p_cur = 0;
    SkSeg p_sg = {0, 0, 1, 0};
    bool p_has_seg = false;
    int p_j = 0;  // next k-block of the current segment

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(full0 + 8u * s, 1);
            mbar_init(empty0 + 8u * s, 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(tfull0 + 8u * b, 1);
            mbar_init(tempty0 + 8u * b, 4);
        }
        mbar_init(drain_bar, 1);
        *abort_flag = 0;
        fence_mbar_init();
        tma_prefetch_desc(&tmA);
        tma_prefetch_desc(&tmB);
        const int rot0 = sk_rotation(p);
        p_cur = sk_cursor0(p);
        p_has_seg = sk_next_seg(p, p_cur, p_sg);
        // The first segment's first k-block (its slot is free).  With b_early
        // the whole first ring of B is copied before the previous grid ends,
        // so A follows for all of it.
        const int nfill = !p_has_seg ? 0 : p.b_early ? (p_sg.nk < STAGES ? p_sg.nk : STAGES) : 1;
        const int bz0 = p_sg.tile / p.num_tiles, tl0 = p_sg.tile - bz0 * p.num_tiles;
        const int za0 = p.za ? bz0 : 0, zb0 = p.zb ? bz0 : 0;
        if (p.b_early) {
            // Before waiting for the previous grid (the caller promised it
            // does not write B), B of those k-blocks is copied into their
            // slots now.  Each slot's barrier expects B's bytes without
            // arriving, so it completes only after A, issued after the wait,
            // lands too.
            for (int jj = 0; jj < nfill; ++jj) {
                const int kb = sk_kblock(p, p_sg, jj, rot0);
                const uint32_t fb = full0 + 8u * jj;
                mbar_expect_tx(fb, Cfg::B_BYTES);
                const uint32_t bdst = smem_u32(sB + jj * Cfg::B_BYTES);
#pragma unroll
                for (int b = 0; b < NT / 64; ++b)
                    tma_load_3d(bdst + b * Cfg::B_COL_BYTES, &tmB, fb, tl0 * NT + b * 64, kb * BK, zb0);
            }
        }
        pdl_wait();  // A and B may be written by the previous grid
        for (int jj = 0; jj < nfill; ++jj) {
            const int kb = sk_kblock(p, p_sg, jj, rot0);
            const uint32_t fb = full0 + 8u * jj;
            if (p.b_early) {
                mbar_arrive_expect_tx(fb, Cfg::A_BYTES);
            } else {
                mbar_arrive_expect_tx(fb, Cfg::STAGE_BYTES);
                const uint32_t bdst = smem_u32(sB + jj * Cfg::B_BYTES);
                // All NT/64 boxes of this k-block together: NT*2 contiguous
                // bytes of every k-row of B.
#pragma unroll
                for (int b = 0; b < NT / 64; ++b)
                    tma_load_3d(bdst + b * Cfg::B_COL_BYTES, &tmB, fb, tl0 * NT + b * 64, kb * BK, zb0);
            }
#pragma unroll
            for (int h = 0; h < BK / 64; ++h)
                tma_load_3d(smem_u32(sA + jj * Cfg::A_BYTES + h * Cfg::A_HALF_BYTES), &tmA, fb, kb * BK + h * 64, 0,
                            za0);
        }
        p_issued = (1u << nfill) - 1u;  // all at phase 0
        p_j = nfill;
        p_stage = nfill == STAGES ? 0 : nfill;
        p_phase = nfill == STAGES ? 1u : 0u;
    }
    if (warp == 1) {
        tmem_alloc<1>(smem_u32(tmem_slot), Cfg::TMEM_COLS);
        tmem_relinquish<1>();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    const int KB = p.kblocks;
    const int rot = sk_rotation(p);  // first k-block of this CTA's k loop
    // A following kernel launched with programmatic serialization may start
    // its prologue now; it waits for this grid before touching memory.
    if (threadIdx.x == 0) pdl_launch_dependents();

    if (warp == 0) {
        if (lane == 0) {
            // The rest of the loads, from where the first ring stopped.
            bool ok = true;
            while (ok && p_has_seg) {
                const int bz = p_sg.tile / p.num_tiles, tile = p_sg.tile - bz * p.num_tiles;
                const int za = p.za ? bz : 0, zb = p.zb ? bz : 0;
                for (; p_j < p_sg.nk; ++p_j) {
                    const int kb = sk_kblock(p, p_sg, p_j, rot);
                    if (!mbar_wait(empty0 + 8u * p_stage, p_phase ^ 1u, abort_flag)) {
                        ok = false;
                        break;
                    }
                    const uint32_t fb = full0 + 8u * p_stage;
                    mbar_arrive_expect_tx(fb, Cfg::STAGE_BYTES);
                    const uint32_t bdst = smem_u32(sB + p_stage * Cfg::B_BYTES);
#pragma unroll
                    for (int b = 0; b < NT / 64; ++b)
                        tma_load_3d(bdst + b * Cfg::B_COL_BYTES, &tmB, fb, tile * NT + b * 64, kb * BK, zb);
#pragma unroll
                    for (int h = 0; h < BK / 64; ++h)
                        tma_load_3d(smem_u32(sA + p_stage * Cfg::A_BYTES + h * Cfg::A_HALF_BYTES), &tmA, fb,
                                    kb * BK + h * 64, 0, za);
                    p_issued |= 1u << p_stage;
                    p_last_parity = (p_last_parity & ~(1u << p_stage)) | (p_phase << p_stage);
                    if (++p_stage == STAGES) {
                        p_stage = 0;
                        p_phase ^= 1u;
                    }
                }
                if (!ok) break;
                p_has_seg = sk_next_seg(p, p_cur, p_sg);
                p_j = 0;
            }
            if (!ok)
                for (int s = 0; s < STAGES; ++s)
                    if (p_issued & (1u << s)) mbar_wait(full0 + 8u * s, (p_last_parity >> s) & 1u, nullptr);
        }
    } else if (warp == 1) {
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            int acc = 0;
            uint32_t acc_phase = 0;
            bool ok = true;
            long long cur = sk_cursor0(p);
            SkSeg sg;
            const uint64_t bdesc0 = umma_desc_sw128(smem_u32(sB), Cfg::B_COL_BYTES, 1024);  // B^T, N-major
            const uint64_t adesc0 = umma_desc_sw128(smem_u32(sA), 16, 1024);    // A, K-major
            while (ok && sk_next_seg(p, cur, sg)) {
                if (!mbar_wait(tempty0 + 8u * acc, acc_phase ^ 1u, abort_flag)) break;
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + (uint32_t)acc * Cfg::ACC_STRIDE;
                for (int v = 0; v < sg.nk; ++v) {
                    if (!mbar_wait(full0 + 8u * stage, phase, abort_flag)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint64_t bs = bdesc0 + (uint64_t)((stage * Cfg::B_BYTES) >> 4);
                    const uint64_t as = adesc0 + (uint64_t)((stage * Cfg::A_BYTES) >> 4);
#pragma unroll
                    for (int kk = 0; kk < BK / 16; ++kk) {
#pragma unroll
                        for (int sb = 0; sb < NSUB; ++sb) {
                            // B^T: sub-tile sb is column boxes 2sb, 2sb+1; k-step
                            // kk is 16 k-rows further in.  A: 64-k box kk/4,
                            // 32 bytes further per k-step within it.
                            const uint64_t ad =
                                bs + (uint64_t)((sb * 2 * Cfg::B_COL_BYTES + kk * 2048) >> 4);
                            const uint64_t bd =
                                as + (uint64_t)(((kk / 4) * Cfg::A_HALF_BYTES + (kk % 4) * 32) >> 4);
                            tc_mma_f16(d_tmem + (uint32_t)(sb * MP), ad, bd, Cfg::IDESC,
                                       (v != 0 || kk != 0) ? 1u : 0u);
                        }
                    }
                    tc_commit(empty0 + 8u * stage);
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
                if (!ok) break;
                tc_commit(tfull0 + 8u * acc);
                if (++acc == 2) {
                    acc = 0;
                    acc_phase ^= 1u;
                }
            }
            tc_commit(drain_bar);
            mbar_wait(drain_bar, 0, nullptr);
        }
    } else {
        pdl_wait();  // bias, residual, C and the workspace may belong to the previous grid
        const int q = warp & 3;
        const int et = threadIdx.x - 64;  // 0..127 among epilogue threads
        const int n_local = q * 32 + lane;
        const int first_tile = p.slices > 0 ? 0 : (int)(sk_unit_begin(blockIdx.x, p) / KB);
        int acc = 0;
        uint32_t acc_phase = 0;
        long long cur = sk_cursor0(p);
        SkSeg sg;
        while (sk_next_seg(p, cur, sg)) {
            const int tile = sg.tile;  // global tile (item * num_tiles + tile) in batched launches
            // This thread's bias values, loaded before the accumulator wait so
            // that their latency is hidden behind it.
            float bpre[NSUB];
            {
                const int bz = tile / p.num_tiles, tl = tile - bz * p.num_tiles;
                const __half* bias = (p.epi.flags & EPI_BIAS) ? p.epi.bias + (long long)bz * p.sbias : nullptr;
#pragma unroll
                for (int sb = 0; sb < NSUB; ++sb) {
                    const long long n = (long long)tl * NT + sb * 128 + n_local;
                    bpre[sb] = (bias != nullptr && n < p.N) ? __half2float(bias[n]) : 0.f;
                }
            }
            // All four epilogue warps take the same branch (they meet at named
            // barriers below), so the wait outcome is AND-reduced across them.
            const bool ok = named_barrier_and<1, 128>(mbar_wait(tfull0 + 8u * acc, acc_phase, abort_flag));
            if (!ok) break;
            tc_fence_after();
            float v[NSUB][MP];
            const uint32_t t_row = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)acc * Cfg::ACC_STRIDE;
#pragma unroll
            for (int sb = 0; sb < NSUB; ++sb)
#pragma unroll
                for (int j = 0; j < MP / 16; ++j) tmem_ld_32x32b_x16(t_row + (uint32_t)(sb * MP + 16 * j), v[sb] + 16 * j);
            tmem_wait_ld();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(tempty0 + 8u * acc);
            if (++acc == 2) {
                acc = 0;
                acc_phase ^= 1u;
            }

            const bool whole = p.slices > 0 ? p.slices == 1 : (sg.kb0 == 0 && sg.nk == KB);
            bool do_out = whole;
            if (!whole) {
                // A split tile: contributors c_first..c_last.  The last one
                // (the tile's last K slice; in stream-K the CTA holding the
                // tile's tail, which it computes last) adds the others'
                // partial sums to its own, in CTA order, and writes C.  The
                // others publish theirs: the partial sum to their slot, then
                // their flag.  In stream-K a CTA publishes only the first
                // segment it computes (the head of its later tile), so one
                // slot per CTA suffices, and the tail owner finds the head
                // long published.
                int c_first, c_last;
                if (p.slices > 0) {
                    c_first = tile * p.slices;
                    c_last = c_first + min(p.slices, KB) - 1;
                } else {
                    c_first = sk_owner((long long)tile * KB, p);
                    c_last = sk_owner((long long)(tile + 1) * KB - 1, p);
                }
                if ((int)blockIdx.x != c_last) {
                    float* wp = p.ws + (size_t)blockIdx.x * (size_t)(MP * NT);
#pragma unroll
                    for (int sb = 0; sb < NSUB; ++sb)
#pragma unroll
                        for (int m = 0; m < MP; ++m) __stcg(wp + m * NT + sb * 128 + n_local, v[sb][m]);
                    // Every epilogue thread's stores precede the release.
                    asm volatile("bar.sync 1, 128;" ::: "memory");
                    if (et == 0) st_release_gpu(p.flags + blockIdx.x, p.epoch);
                    do_out = false;
                } else {
                    float acc[NSUB][MP];
#pragma unroll
                    for (int sb = 0; sb < NSUB; ++sb)
#pragma unroll
                        for (int m = 0; m < MP; ++m) acc[sb][m] = 0.f;
                    // The epilogue threads wait (bounded) for the other
                    // contributors' flags in parallel, one each; the barrier
                    // then orders every thread's loads after those acquires.
                    bool mine = true;
                    for (int i = et; i < c_last - c_first; i += 128)
                        mine = mine && wait_flag(p.flags + c_first + i, p.epoch, abort_flag);
                    const bool got = named_barrier_and<1, 128>(mine);
                    if (got) {
                        for (int c = c_first; c < c_last; ++c) {
                            const float* rp = p.ws + (size_t)c * (size_t)(MP * NT);
#pragma unroll
                            for (int sb = 0; sb < NSUB; ++sb)
#pragma unroll
                                for (int m = 0; m < MP; ++m) acc[sb][m] += __ldcg(rp + m * NT + sb * 128 + n_local);
                        }
                    }
                    if (!got) break;
#pragma unroll
                    for (int sb = 0; sb < NSUB; ++sb)
#pragma unroll
                        for (int m = 0; m < MP; ++m) v[sb][m] = acc[sb][m] + v[sb][m];
                    do_out = true;
                }
            }
            if (do_out) {
                const int flags = p.epi.flags;
                // Batch item of this tile (0 unless batched) and its operands.
                const int bz = tile / p.num_tiles, tl = tile - bz * p.num_tiles;
                const long long res_off = (long long)bz * p.sres;
                __half* c16 = p.c16 ? p.c16 + (long long)bz * p.sc : nullptr;
                float* c32 = p.c32 ? p.c32 + (long long)bz * p.sc : nullptr;
                // This code runs once per tile, from a cold instruction cache,
                // unrolled over the MP rows.  fp16 output with at most a bias
                // (the decode case) is straight-line code; every other
                // epilogue calls one out-of-line copy per value, so that the
                // unrolled rows do not each carry the residual and GeLU code.
                const bool has_bias = (flags & EPI_BIAS) != 0;
                const bool lean = c16 != nullptr && (flags & (EPI_RES | EPI_GELU_TANH | EPI_GELU_ERF | EPI_SCALE)) == 0;
#pragma unroll
                for (int sb = 0; sb < NSUB; ++sb) {
                    const long long n = (long long)tl * NT + sb * 128 + n_local;
                    if (n >= p.N) continue;
                    const float b = bpre[sb];
                    if (lean) {
#pragma unroll
                        for (int m = 0; m < MP; ++m)
                            if (m < p.M) c16[(long long)m * p.ldc + n] = __float2half_rn(has_bias ? v[sb][m] + b : v[sb][m]);
                    } else {
#pragma unroll
                        for (int m = 0; m < MP; ++m) {
                            if (m < p.M) {
                                const float o = sk_epi_value(v[sb][m], b, flags, p.epi.alpha, p.epi.residual,
                                                             res_off + (long long)m * p.epi.ld_res + n);
                                if (c16)
                                    c16[(long long)m * p.ldc + n] = __float2half_rn(o);
                                else
                                    c32[(long long)m * p.ldc + n] = o;
                            }
                        }
                    }
                }
            }
        }
    }

    __syncwarp();
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc<1>(tmem_base, Cfg::TMEM_COLS);
    }
}

// ======================================================================
// Host side
// ======================================================================

static PFN_cuTensorMapEncodeTiled_v12000 sk_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &ptr, 12000, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
    });
    return fn;
}

// 3-D map of `depth` row-major fp16 matrices `zstride` bytes apart (depth 1
// for a single problem; the stride then only has to satisfy the encoder).
static bool sk_tmap(CUtensorMap* m, const void* base, uint64_t inner, uint64_t outer, uint64_t pitch_bytes,
                    uint64_t depth, uint64_t zstride, uint32_t box_inner, uint32_t box_outer) {
    auto enc = sk_encoder();
    if (!enc) return false;
    if (zstride == 0) zstride = ((outer * pitch_bytes) + 15) & ~uint64_t(15);
    cuuint64_t dims[3] = {inner, outer, depth};
    cuuint64_t strides[2] = {pitch_bytes, zstride};
    cuuint32_t box[3] = {box_inner, box_outer, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    return enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int skinny_mp(long long M) { return (int)((M + 15) / 16) * 16; }

// k-rows per ring slot: 128 for 128-column units with m <= 32 (five or six
// slots of 36-40 KB), else 64 (the wider slots would leave too few).
int skinny_bk(long long M, int nt) { return (nt == 128 && skinny_mp(M) <= 32) ? 128 : 64; }

int skinny_stages(long long M, int nt) {
    const int mp = skinny_mp(M);
    if (nt == 256)
        return mp == 16 ? SkCfg<16, 256, 64>::STAGES : mp == 32 ? SkCfg<32, 256, 64>::STAGES
                         : mp == 48 ? SkCfg<48, 256, 64>::STAGES : SkCfg<64, 256, 64>::STAGES;
    return mp == 16 ? SkCfg<16, 128, 128>::STAGES : mp == 32 ? SkCfg<32, 128, 128>::STAGES
                     : mp == 48 ? SkCfg<48, 128, 64>::STAGES : SkCfg<64, 128, 64>::STAGES;
}

int skinny_pick_nt(long long M, long long N, long long K, int sms) {
    const long long kb = (K + 63) / 64;
    (void)M;
    // 256-column units when every SM still gets at least four units to
    // balance; the lockstep layout below always uses 128.
    if (((N + 255) / 256) * kb >= 4LL * sms) return 256;
    return 128;
}

// Lockstep layout: one CTA per (128-column tile, K slice), at most one CTA
// per SM, slices interleaved by k-block.  Every SM then streams the same
// number of bytes of B, the same k-rows at the same time, and a tile is
// split only when there are SMs to spare for it.  Returns the number of K
// slices (floor(SMs / tiles), at least 1), or 0 when there are more tiles
// than SMs (persistent stream-K balances those better).
int skinny_lockstep_slices(long long M, long long N, long long K, int sms) {
    const long long tiles = (N + 127) / 128;
    const long long bk = skinny_bk(M, 128);
    const long long kb = (K + bk - 1) / bk;
    if (tiles > sms) return 0;
    long long s = sms / tiles;
    if (s > kb) s = kb;
    return (int)(s < 1 ? 1 : s);
}

void skinny_geometry(long long M, long long N, long long K, int sms, int nt, int* grid, size_t* ws_bytes,
                     size_t* flag_bytes) {
    const long long tiles = (N + nt - 1) / nt;
    const long long bk = skinny_bk(M, nt);
    const long long work = tiles * ((K + bk - 1) / bk);
    long long g = sms;
    if (g > work) g = work;
    if (g < 1) g = 1;
    *grid = (int)g;
    *ws_bytes = (size_t)g * (size_t)skinny_mp(M) * (size_t)nt * sizeof(float);  // one slot per CTA
    *flag_bytes = (size_t)g * sizeof(unsigned long long);
}

// Read on every call, like the other layout switches, so that a process
// can compare layouts.
int skinny_env_nt() {
    const char* e = getenv("PAX_SKINNY_NT");
    return e ? atoi(e) : 0;
}


// Lockstep layout when there are no more column tiles than SMs; otherwise
// persistent stream-K, one CTA per SM.  nt_force = 128 or 256 forces the
// persistent layout with that unit width.
SkinnyLayout skinny_layout(long long M, long long N, long long K, int sms, int nt_force) {
    SkinnyLayout L;
    int nt = nt_force;
    L.slices = (nt == 0) ? skinny_lockstep_slices(M, N, K, sms) : 0;
    if (L.slices > 0) nt = 128;
    if (nt != 128 && nt != 256) nt = skinny_pick_nt(M, N, K, sms);
    L.nt = nt;
    skinny_geometry(M, N, K, sms, nt, &L.grid, &L.ws_bytes, &L.cnt_bytes);
    if (L.slices > 0) {
        const size_t per_cta = L.ws_bytes / (size_t)L.grid;
        L.grid = (int)(((N + 127) / 128) * L.slices);
        L.ws_bytes = per_cta * (size_t)L.grid;
        L.cnt_bytes = (size_t)L.grid * sizeof(unsigned long long);
        // One slice per tile splits nothing: no partial sums, no flags.
        if (L.slices == 1) L.ws_bytes = L.cnt_bytes = 0;
    }
    return L;
}

size_t skinny_smem_bytes(long long M, int nt) {
    const int mp = skinny_mp(M);
    if (nt == 256)
        return mp == 16 ? SkCfg<16, 256, 64>::SMEM_BYTES : mp == 32 ? SkCfg<32, 256, 64>::SMEM_BYTES
                        : mp == 48 ? SkCfg<48, 256, 64>::SMEM_BYTES : SkCfg<64, 256, 64>::SMEM_BYTES;
    return mp == 16 ? SkCfg<16, 128, 128>::SMEM_BYTES : mp == 32 ? SkCfg<32, 128, 128>::SMEM_BYTES
                    : mp == 48 ? SkCfg<48, 128, 64>::SMEM_BYTES : SkCfg<64, 128, 64>::SMEM_BYTES;
}

// Epoch of the next launch (never 0).
static std::atomic<unsigned long long> g_skinny_epoch{0};
static unsigned long long next_epoch() {
    unsigned long long e = ++g_skinny_epoch;
    while (e == 0) e = ++g_skinny_epoch;
    return e;
}
unsigned long long skinny_last_epoch() { return g_skinny_epoch.load(); }

int skinny_rotation_group();

template <int MP, int NT, int BK>
static pax_status_t launch_skinny_impl(const Problem& pr, int grid, int slices, float* ws,
                                       unsigned long long* flags, cudaStream_t stream) {
    using Cfg = SkCfg<MP, NT, BK>;
    CUtensorMap tA, tB;
    const bool batched = pr.batch > 1;
    const bool za = batched && pr.sa > 0, zb = batched && pr.sb > 0;
    if (!sk_tmap(&tA, pr.A, pr.K, pr.M, pr.lda * 2, za ? pr.batch : 1, za ? pr.sa * 2 : 0, 64, MP))
        return PAX_ERR_CUDA;
    if (!sk_tmap(&tB, pr.B, pr.N, pr.K, pr.ldb * 2, zb ? pr.batch : 1, zb ? pr.sb * 2 : 0, 64, BK))
        return PAX_ERR_CUDA;
    SkinnyParams p;
    p.M = (int)pr.M;
    p.N = (int)pr.N;
    p.K = (int)pr.K;
    p.num_tiles = (int)((pr.N + NT - 1) / NT);
    p.kblocks = (int)((pr.K + BK - 1) / BK);
    p.work = (long long)p.num_tiles * p.kblocks;
    p.grid = grid;
    p.slices = slices;
    // Stream-K visits each CTA's segments last to first: the head of its
    // later tile, which it publishes, comes first, and the tail of its
    // earlier tile, where it is the reducer, last.
    p.korder = slices == 0 ? 1 : 0;
    // A rotation keeps each slice's k-blocks a whole lap only with one slice
    // per tile, outside batched launches.
    p.rot_group = (slices == 1 && !batched) ? skinny_rotation_group() : 0;
    p.b_early = (pr.b_const && pdl_enabled()) ? 1 : 0;
    p.ws = ws;
    p.flags = flags;
    p.epoch = next_epoch();
    p.c16 = pr.c_f16 ? static_cast<__half*>(pr.C) : nullptr;
    p.c32 = pr.c_f16 ? nullptr : static_cast<float*>(pr.C);
    p.ldc = pr.ldc;
    p.epi = pr.epi;
    p.rr = batched ? 1 : 0;
    p.batch = batched ? (int)pr.batch : 1;
    p.za = za ? 1 : 0;
    p.zb = zb ? 1 : 0;
    p.sc = batched ? pr.sc : 0;
    p.sbias = batched ? pr.sbias : 0;
    p.sres = batched ? pr.sres : 0;
    if (batched) {
        // Whole tiles round-robin over the CTAs: no workspace, no K split.
        if (slices != 0 || grid < 1 || (long long)grid > (long long)p.batch * p.num_tiles ||
            (long long)p.batch * p.num_tiles > 0x7fffffffLL)
            return PAX_ERR_INVALID;
    } else if (grid < 1 || grid > p.work) {
        return PAX_ERR_INVALID;
    }
    if (slices > 0 && slices * p.num_tiles != grid) return PAX_ERR_INVALID;
    auto kern = gemm_skinny_kernel<MP, NT, BK>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)Cfg::SMEM_BYTES) != cudaSuccess)
        return PAX_ERR_CUDA;
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(192);
    cfg.dynamicSmemBytes = Cfg::SMEM_BYTES;
    cfg.stream = stream;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaLaunchKernelEx(&cfg, kern, tA, tB, p) != cudaSuccess) return PAX_ERR_CUDA;
    return cudaPeekAtLastError() == cudaSuccess ? PAX_OK : PAX_ERR_CUDA;
}

template <int NT>
static pax_status_t launch_skinny_nt(const Problem& p, int grid, int slices, float* ws,
                                     unsigned long long* flags, cudaStream_t stream) {
    switch (skinny_mp(p.M)) {
        case 16: return launch_skinny_impl<16, NT, NT == 128 ? 128 : 64>(p, grid, slices, ws, flags, stream);
        case 32: return launch_skinny_impl<32, NT, NT == 128 ? 128 : 64>(p, grid, slices, ws, flags, stream);
        case 48: return launch_skinny_impl<48, NT, 64>(p, grid, slices, ws, flags, stream);
        default: return launch_skinny_impl<64, NT, 64>(p, grid, slices, ws, flags, stream);
    }
}

// PAX_SKINNY_ROT=g: in the lockstep layout, CTAs in groups of g start their
// k loop at different k-blocks (0, the default, starts every CTA at 0).
int skinny_rotation_group() {
    static const int g = [] {
        const char* v = getenv("PAX_SKINNY_ROT");
        const int x = v ? atoi(v) : 0;
        return x > 0 ? x : 0;
    }();
    return g;
}

// nt: 128 or 256 output columns per unit.  slices > 0: lockstep layout (nt
// 128, grid = tiles x slices); 0: persistent stream-K over `grid` CTAs.
pax_status_t launch_skinny_ws(const Problem& p, int nt, int grid, float* ws, unsigned long long* flags,
                              cudaStream_t stream, int slices) {
    if (p.M < 1 || p.M > kSkinnyMaxM || p.N > 0x7fffffffLL || p.K > 0x7fffffffLL) return PAX_ERR_UNSUPPORTED;
    if (slices > 0) return launch_skinny_nt<128>(p, grid, slices, ws, flags, stream);
    if (nt == 256) return launch_skinny_nt<256>(p, grid, 0, ws, flags, stream);
    return launch_skinny_nt<128>(p, grid, 0, ws, flags, stream);
}

// Self-test of the bounded waits (pax_selftest_bounded_wait): one thread
// waits on an mbarrier that nothing arrives on.  mbar_wait gives up after
// kWaitTimeoutNs, records PAX_DEVERR_TIMEOUT in this unit's error word and
// returns false; the kernel then ends normally and the context stays usable.
__global__ void selftest_wait_kernel() {
    __shared__ __align__(8) uint64_t bar;
    __shared__ int abort_flag;
    if (threadIdx.x == 0) {
        abort_flag = 0;
        mbar_init(smem_u32(&bar), 1);
        fence_mbar_init();
        (void)mbar_wait(smem_u32(&bar), 0, reinterpret_cast<volatile int*>(&abort_flag));
    }
}

pax_status_t launch_selftest_wait(cudaStream_t stream) {
    selftest_wait_kernel<<<1, 32, 0, stream>>>();
    return cudaPeekAtLastError() == cudaSuccess ? PAX_OK : PAX_ERR_CUDA;
}

bool set_wait_limit_skinny(unsigned long long ns) {
    return cudaMemcpyToSymbol(g_pax_wait_limit_ns, &ns, sizeof(ns)) == cudaSuccess;
}

int read_clear_device_error_skinny() {
    int v = 0, z = 0;
    if (cudaMemcpyFromSymbol(&v, g_pax_device_error, sizeof(int)) != cudaSuccess) return -1;
    if (v) cudaMemcpyToSymbol(g_pax_device_error, &z, sizeof(int));
    return v;
}

// ----------------------------------------------------------------------
// Allocation-free variant (pax_gemm_skinny_noalloc).
//
// Some callers cannot let a library call cudaMalloc: processes whose device
// memory is owned by their own allocator (a framework's caching allocator,
// or a serving process that reserves the GPU's memory at start-up and treats
// any later allocation as a failure), and latency-critical loops where the
// implicit device synchronisation of cudaMalloc/cudaFree is not acceptable.
// For them the skinny kernel's scratch (per-CTA publication flags followed
// by the fp32 partial sums) lives in this fixed array instead of the
// per-stream workspace.  Every GPU that loads the library holds it until the
// process exits.
constexpr size_t kNoAllocScratchBytes = size_t(8) << 20;  // 8 MiB per device
static __device__ __align__(256) unsigned char g_skinny_scratch[kNoAllocScratchBytes];

// Device address of g_skinny_scratch, looked up once per device and CUDA
// context (the host symbol is only a handle; passing it to a kernel would be
// wrong).  The entry is keyed by the context as well as the device: after
// the primary context is reset or released and created again, the module
// may load at another address, and the next call looks the address up
// again.  pax_shutdown forgets every entry.
using CtxGetCurrentFn = CUresult (*)(CUcontext*);
static CtxGetCurrentFn ctx_get_current() {
    static CtxGetCurrentFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPointByVersion("cuCtxGetCurrent", &f, 4000, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<CtxGetCurrentFn>(f);
    });
    return fn;
}

struct ScratchEntry {
    int dev;
    CUcontext ctx;
    void* addr;
};
static std::mutex g_scratch_mu;
static std::vector<ScratchEntry> g_scratch_addr;

static pax_status_t scratch_address(int dev, void** out) {
    CtxGetCurrentFn get = ctx_get_current();
    CUcontext ctx = nullptr;
    if (!get || get(&ctx) != CUDA_SUCCESS || ctx == nullptr) return PAX_ERR_CUDA;
    std::lock_guard<std::mutex> lk(g_scratch_mu);
    for (const ScratchEntry& e : g_scratch_addr)
        if (e.dev == dev && e.ctx == ctx) {
            *out = e.addr;
            return PAX_OK;
        }
    void* ptr = nullptr;
    if (cudaGetSymbolAddress(&ptr, g_skinny_scratch) != cudaSuccess || ptr == nullptr) {
        cudaGetLastError();
        return PAX_ERR_CUDA;
    }
    // A context this device no longer uses cannot come back: drop its entry.
    for (size_t i = 0; i < g_scratch_addr.size(); ++i)
        if (g_scratch_addr[i].dev == dev) {
            g_scratch_addr.erase(g_scratch_addr.begin() + (long)i);
            break;
        }
    g_scratch_addr.push_back({dev, ctx, ptr});
    *out = ptr;
    return PAX_OK;
}

void skinny_forget_scratch() {
    std::lock_guard<std::mutex> lk(g_scratch_mu);
    g_scratch_addr.clear();
}

}  // namespace pax

extern "C" pax_status_t pax_selftest_bounded_wait(cudaStream_t stream) {
    const pax_status_t st = pax::launch_selftest_wait(stream);
    return pax::report_status(st, st == PAX_OK ? "" : "pax_selftest_bounded_wait: launch failed");
}

extern "C" pax_status_t pax_gemm_skinny_noalloc(const pax_gemm_desc_t* desc, cudaStream_t stream) {
    using namespace pax;
    Problem p;
    pax_status_t st = normalize_desc(desc, &p);
    if (st != PAX_OK) return st;
    if (p.M == 0 || p.N == 0) return report_status(PAX_OK, "");
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return report_status(PAX_ERR_CUDA, "pax_gemm_skinny_noalloc: no device");
    int major = 0, sms = 0;
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (major != 10) return report_status(PAX_ERR_NO_DEVICE, "pax_gemm_skinny_noalloc: needs an sm_100 device");
    if (p.M > kSkinnyMaxM || !tma_compatible(p))
        return report_status(PAX_ERR_UNSUPPORTED,
                             "pax_gemm_skinny_noalloc: needs 1 <= m <= 64, k >= 1 and 16-byte aligned rows");
    // The layout pax_gemm_ex would run (lockstep for up to one column tile
    // per SM, else stream-K), so that both entry points take the same time.
    const SkinnyLayout L = skinny_layout(p.M, p.N, p.K, sms, skinny_env_nt());
    const size_t cnt_pad = (L.cnt_bytes + 255) & ~size_t(255);
    if (cnt_pad + L.ws_bytes > kNoAllocScratchBytes) {
        char msg[160];
        snprintf(msg, sizeof msg,
                 "pax_gemm_skinny_noalloc: problem needs %zu bytes of scratch, above the fixed %zu-byte limit",
                 cnt_pad + L.ws_bytes, kNoAllocScratchBytes);
        return report_status(PAX_ERR_UNSUPPORTED, msg);
    }
    void* scratch = nullptr;
    if (scratch_address(dev, &scratch) != PAX_OK)
        return report_status(PAX_ERR_CUDA, "pax_gemm_skinny_noalloc: cudaGetSymbolAddress failed");
    // The array keeps whatever the previous call left.  Nothing in it has to
    // start at zero: a publication flag counts only when it holds this
    // launch's epoch (a 64-bit number no earlier launch in this process
    // used), and a partial sum is read only after its flag.
    st = launch_skinny_ws(p, L.nt, L.grid, reinterpret_cast<float*>(static_cast<char*>(scratch) + cnt_pad),
                          static_cast<unsigned long long*>(scratch), stream, L.slices);
    if (st != PAX_OK) return report_status(st, "pax_gemm_skinny_noalloc: launch failed");
    return report_status(PAX_OK, "");
}
