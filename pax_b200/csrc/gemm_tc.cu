// gemm_tc.cu -- tile-shape choice and dispatch for the tcgen05 GEMM
// (kernel in gemm_tc.cuh, instantiated in gemm_tc_f16.cu / gemm_tc_f32.cu).
#include "internal.h"
#include "gemm_tc.cuh"

namespace pax {

pax_status_t launch_tc_f16(const Problem& p, const TcPlan& plan, cudaStream_t stream);
pax_status_t launch_tc_f32(const Problem& p, const TcPlan& plan, cudaStream_t stream);
int tc_pair_units_f16(int dev, int sms);
int read_clear_device_error_tc_f16();
int read_clear_device_error_tc_f32();

int tc_stages(int shape) {
    return shape == 4 ? kStagesWide : shape == 2 ? kStagesPair : shape == 256 ? kStages256 : kStages128;
}

size_t tc_smem_bytes(int shape, bool c_f16) {
    if (shape == 4)
        return c_f16 ? TcCfg<512, kStagesWide, __half, true>::SMEM_BYTES
                     : TcCfg<512, kStagesWide, float, true>::SMEM_BYTES;
    if (shape == 2)
        return c_f16 ? TcCfg<256, kStagesPair, __half, true>::SMEM_BYTES
                     : TcCfg<256, kStagesPair, float, true>::SMEM_BYTES;
    if (shape == 256)
        return c_f16 ? TcCfg<256, kStages256, __half, false>::SMEM_BYTES
                     : TcCfg<256, kStages256, float, false>::SMEM_BYTES;
    return c_f16 ? TcCfg<128, kStages128, __half, false>::SMEM_BYTES : TcCfg<128, kStages128, float, false>::SMEM_BYTES;
}

int tc_pick_bn(long long M, long long N, int sms) {
    const long long tm = (M + 127) / 128;
    const long long t256 = tm * ((N + 255) / 256);
    const long long t128 = tm * ((N + 127) / 128);
    // Wide tiles halve A re-reads from shared memory; fall back to 128-wide
    // tiles when 256-wide ones would leave most SMs idle.
    if (t256 >= sms || t128 == t256) return 256;
    return 128;
}

// Tile shape by a wave-count cost model.  Time ~ rounds x (time of one
// tile on its SM or pair); time unit: one 128 x 256 x K tile on one SM at
// the one-CTA kernel's rate.  Relative mainloop throughputs measured on
// B200 (4096^3 and 8192^3): 128 x 128 = 0.67, CTA pair 256 x 256 = 1.10,
// wide pair 256 x 512 = 1.32.  The wide tile has a single accumulator, so
// its epilogue is not hidden behind the next tile: it adds a per-tile term
// that grows with the epilogue's work and shrinks with K (fitted: 0.03 of a
// unit at K = 4096 for bias / tanh-GeLU, 0.43 with residual and erf-GeLU).
// Tail waves of at most half the units run as column halves.
static double tc_rounds(long long tiles, long long units) {
    const long long full = tiles / units, rem = tiles % units;
    if (rem == 0) return (double)full;
    return (double)full + (2 * rem <= units ? 0.5 : 1.0);
}

int tc_pick_shape(const Problem& p, int sms) {
    const long long pairs = sms / 2;  // resident pairs are refined at launch (tc_pair_units)
    const long long M = p.M, N = p.N;
    // Batch items add tile rows (the model only counts tiles).
    const long long tm = (M + 127) / 128 * p.batch, tm2 = (M + 255) / 256 * p.batch;
    const double t256 = tc_rounds(tm * ((N + 255) / 256), sms);
    const double t128 = tc_rounds(tm * ((N + 127) / 128), sms) * 0.5 / 0.67;
    const double tpair = tc_rounds(tm2 * ((N + 255) / 256), pairs) / 1.10;
    const int f = p.epi.flags;
    const double epi = 0.03 + ((f & EPI_RES) ? 0.2 : 0.0) + ((f & EPI_GELU_ERF) ? 0.2 : 0.0);
    const double kscale = 4096.0 / (double)(p.K > 64 ? p.K : 64);
    const double twide = tc_rounds(tm2 * ((N + 511) / 512), pairs) * (2.0 / 1.32 + epi * kscale);
    double best = t256;
    int shape = 256;
    if (t128 < best) { best = t128; shape = 128; }
    if (tpair <= best) { best = tpair; shape = 2; }
    if (twide < best) { best = twide; shape = 4; }
    return shape;
}

TcPlan tc_plan(const Problem& p, int shape, int dev, int sms, bool allow_halves) {
    TcPlan plan;
    plan.shape = (shape == 2 || shape == 4 || shape == 256) ? shape : 128;
    const bool pair = plan.shape == 2 || plan.shape == 4;
    const long long tile_m = pair ? 256 : 128;
    const long long tile_n = plan.shape == 4 ? 512 : plan.shape == 128 ? 128 : 256;
    const long long tiles = ((p.M + tile_m - 1) / tile_m) * ((p.N + tile_n - 1) / tile_n) * p.batch;
    const long long max_units = pair ? tc_pair_units_f16(dev, sms) : sms;
    // The tail wave: tiles left after whole waves.  When at most half the
    // units would be busy on them, each is cut into two column halves, so
    // the tail takes about half the time of a wave.
    const long long rem = tiles >= max_units ? tiles % max_units : tiles;
    const bool halves = allow_halves && rem > 0 && 2 * rem <= max_units;
    plan.tail_tiles = halves ? (int)rem : 0;
    plan.full_items = (int)(tiles - plan.tail_tiles);
    const long long items = plan.full_items + 2LL * plan.tail_tiles;
    plan.units = (int)(items < max_units ? items : max_units);
    return plan;
}

pax_status_t launch_tc(const Problem& p, const TcPlan& plan, cudaStream_t stream) {
    if (p.M > 0x7fffffffLL || p.N > 0x7fffffffLL || p.K > 0x7fffffffLL) return PAX_ERR_UNSUPPORTED;
    return p.c_f16 ? launch_tc_f16(p, plan, stream) : launch_tc_f32(p, plan, stream);
}

int read_clear_device_error_tc() {
    const int a = read_clear_device_error_tc_f16();
    const int b = read_clear_device_error_tc_f32();
    if (a < 0 || b < 0) return -1;
    return a | b;
}

}  // namespace pax
