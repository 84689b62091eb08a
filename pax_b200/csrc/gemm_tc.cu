// gemm_tc.cu -- tile-shape choice and dispatch for the tcgen05 GEMM
// (kernel in gemm_tc.cuh, instantiated in gemm_tc_f16.cu / gemm_tc_f32.cu).
#include "internal.h"

#include <algorithm>
#include <map>
#include <memory>
#include <mutex>
#include <string.h>
#include <vector>
#include "gemm_tc.cuh"

namespace pax {

pax_status_t launch_tc_f16(const Problem& p, const TcPlan& plan, cudaStream_t stream);
pax_status_t launch_tc_f32(const Problem& p, const TcPlan& plan, cudaStream_t stream);
int tc_pair_units_f16(int dev, int sms);
int read_clear_device_error_tc_f16();
int read_clear_device_error_tc_f32();
bool set_wait_limit_tc_f16(unsigned long long ns);
bool set_wait_limit_tc_f32(unsigned long long ns);

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

double tc_wide_rounds(long long M, long long N, long long K, int units);

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
    const double wrounds =
        p.batch == 1 ? tc_wide_rounds(M, N, p.K, (int)pairs) : tc_rounds(tm2 * ((N + 511) / 512), pairs);
    const double twide = wrounds * (2.0 / 1.32 + epi * kscale);
    double best = t256;
    int shape = 256;
    if (t128 < best) { best = t128; shape = 128; }
    if (tpair <= best) { best = tpair; shape = 2; }
    if (twide < best) { best = twide; shape = 4; }
    return shape;
}

// ------------------------------------------------------------ tile planner
// For the wide CTA-pair shape, a problem with few tiles per pair loses up to
// a whole round to quantization: 4096^2 is 128 tiles of 256 x 512 on 74
// pairs, so 54 pairs run two tiles and 20 run one.  The planner re-tiles
// each 256-row block with items 512, 384 or 256 columns wide and assigns them
// to pairs longest first.  For 4096^2: 7 blocks of 8 x 512 and 9 blocks of
// 2 x 512 + 8 x 384 give every pair one 512 and (almost) every pair one 384
// item, 1.75 tile-times instead of 2.
//
// Item cost, in 256 x 512 item-times at this K: width / 512 over the width's
// relative efficiency (512: 1, 384: 0.96, 256: 0.83, from the measured rates
// of the wide and 256 x 256 tiles), plus an exposed per-item epilogue of
// 0.04 x 4096 / K.
namespace {

double item_cost(int w, long long K) {
    const double eff = w == 512 ? 1.0 : w == 384 ? 0.96 : 0.83;
    return (double)w / 512.0 / eff + 0.04 * 4096.0 / (double)(K > 64 ? K : 64);
}

struct RowPattern {
    int n512, n384, n256;
};

// Longest-processing-time assignment of `widths` to `units`; returns the
// makespan and, when `out` is given, fills the per-unit lists.
double lpt(std::vector<std::pair<int, int>> items /* (width, index) */, int units, long long K,
           std::vector<std::vector<int>>* out) {
    std::stable_sort(items.begin(), items.end(), [](const auto& a, const auto& b) { return a.first > b.first; });
    std::vector<double> load((size_t)units, 0.0);
    if (out) out->assign((size_t)units, {});
    for (const auto& it : items) {
        int best = 0;
        for (int u = 1; u < units; ++u)
            if (load[(size_t)u] < load[(size_t)best]) best = u;
        load[(size_t)best] += item_cost(it.first, K);
        if (out) (*out)[(size_t)best].push_back(it.second);
    }
    double m = 0;
    for (double l : load) m = l > m ? l : m;
    return m;
}

struct PlanKey {
    long long M, N, K;
    int units;
    bool operator<(const PlanKey& o) const {
        if (M != o.M) return M < o.M;
        if (N != o.N) return N < o.N;
        if (K != o.K) return K < o.K;
        return units < o.units;
    }
};
std::mutex g_plan_mu;
std::map<PlanKey, std::unique_ptr<TcItemTable>> g_plans;  // null entry: no better plan
std::map<PlanKey, double> g_plan_rounds;                 // planned makespan in whole-tile times

// Planned table for a wide-shape problem, or null when the round-robin
// schedule (whole tiles, column-half tail) is as good.
const TcItemTable* wide_plan(long long M, long long N, long long K, int units) {
    const long long R = (M + 255) / 256;
    const long long tiles = R * ((N + 511) / 512);
    if (units < 2 || units > TcItemTable::kMaxUnits || tiles > 8LL * units || N > (4096LL * 128) ||
        R > 0xFFFF)
        return nullptr;
    const PlanKey key{M, N, K, units};
    std::lock_guard<std::mutex> lk(g_plan_mu);
    auto hit = g_plans.find(key);
    if (hit != g_plans.end()) return hit->second.get();

    // The round-robin schedule's makespan in the same cost model.
    double base;
    {
        const long long full = tiles / units, rem = tiles % units;
        base = (double)full * item_cost(512, K);
        if (rem > 0) base += (2 * rem <= units) ? item_cost(256, K) : item_cost(512, K);
    }
    // Column patterns of one row block: a 512s, b 384s, c <= 3 256s, covering
    // N with less than 256 columns to spare.
    std::vector<RowPattern> pats;
    for (int a = 0; 512LL * a <= N + 511; ++a)
        for (int b = 0; 512LL * a + 384LL * b <= N + 383; ++b) {
            const long long rest = N - 512LL * a - 384LL * b;
            const int c = rest > 0 ? (int)((rest + 255) / 256) : 0;
            if (c > 3 || 512LL * a + 384LL * b + 256LL * c - N >= 256) continue;
            pats.push_back({a, b, c});
        }
    auto items_of = [&](const RowPattern& q, int row, std::vector<std::pair<int, int>>& items,
                        std::vector<unsigned int>& packed) {
        int col = 0;
        auto add = [&](int w, unsigned int code) {
            items.emplace_back(w, (int)packed.size());
            packed.push_back((unsigned int)row | ((unsigned int)(col / 128) << 16) | (code << 28));
            col += w;
        };
        for (int i = 0; i < q.n512; ++i) add(512, 0u);
        for (int i = 0; i < q.n384; ++i) add(384, 1u);
        for (int i = 0; i < q.n256; ++i) add(256, 2u);
    };
    double best = base * 0.97;  // a plan must beat round-robin by 3 %
    int bp = -1, bq = -1;
    long long br = 0;
    for (size_t ip = 0; ip < pats.size(); ++ip)
        for (size_t iq = ip; iq < pats.size(); ++iq)
            for (long long r = (ip == iq ? 0 : 1); r <= (ip == iq ? 0 : R - 1); ++r) {
                std::vector<std::pair<int, int>> items;
                std::vector<unsigned int> packed;
                for (long long row = 0; row < R; ++row)
                    items_of(row < R - r ? pats[ip] : pats[iq], (int)row, items, packed);
                if ((long long)items.size() > TcItemTable::kMaxItems) continue;
                const double m = lpt(items, units, K, nullptr);
                if (m < best) {
                    best = m;
                    bp = (int)ip;
                    bq = (int)iq;
                    br = r;
                }
            }
    if (bp < 0) {
        g_plans[key] = nullptr;
        return nullptr;
    }
    g_plan_rounds[key] = best / item_cost(512, K);
    std::vector<std::pair<int, int>> items;
    std::vector<unsigned int> packed;
    for (long long row = 0; row < R; ++row) items_of(row < R - br ? pats[(size_t)bp] : pats[(size_t)bq], (int)row, items, packed);
    std::vector<std::vector<int>> per_unit;
    lpt(items, units, K, &per_unit);
    auto t = std::make_unique<TcItemTable>();
    memset(t.get(), 0, sizeof(TcItemTable));
    int n = 0;
    for (int u = 0; u < units; ++u) {
        t->unit_start[u] = n;
        for (int idx : per_unit[(size_t)u]) t->item[n++] = packed[(size_t)idx];
    }
    t->unit_start[units] = n;
    t->count = n;
    const TcItemTable* ret = t.get();
    g_plans[key] = std::move(t);
    return ret;
}

// Device copy of a plan for `dev`: [unit_start 0..units][items], uploaded
// once (synchronously, never while the stream is captured) and kept until the process
// exits.  Null if the upload fails, in which case the launch runs without a
// plan.
std::map<std::pair<const TcItemTable*, int>, int*> g_plan_dev;

const int* plan_on_device(const TcItemTable* t, int dev, int units, cudaStream_t stream) {
    std::lock_guard<std::mutex> lk(g_plan_mu);
    auto it = g_plan_dev.find({t, dev});
    if (it != g_plan_dev.end()) return it->second;
    std::vector<int> host((size_t)units + 1 + (size_t)t->count);
    for (int u = 0; u <= units; ++u) host[(size_t)u] = t->unit_start[u];
    for (int k = 0; k < t->count; ++k) host[(size_t)units + 1 + (size_t)k] = (int)t->item[k];
    int* d = nullptr;
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    // No allocation while `stream` is being captured: run unplanned instead.
    if (cudaStreamIsCapturing(stream, &cs) != cudaSuccess || cs != cudaStreamCaptureStatusNone) {
        cudaGetLastError();
        return nullptr;
    }
    if (cudaMalloc(&d, host.size() * sizeof(int)) != cudaSuccess) {
        cudaGetLastError();
        return nullptr;
    }
    if (cudaMemcpy(d, host.data(), host.size() * sizeof(int), cudaMemcpyHostToDevice) != cudaSuccess) {
        cudaGetLastError();
        cudaFree(d);
        return nullptr;
    }
    g_plan_dev[{t, dev}] = d;
    return d;
}

}  // namespace

// Frees the planned tables' device copies (pax_shutdown).
void tc_free_plans() {
    std::lock_guard<std::mutex> lk(g_plan_mu);
    for (auto& kv : g_plan_dev) {
        int prev = 0;
        cudaGetDevice(&prev);
        cudaSetDevice(kv.first.second);
        cudaFree(kv.second);
        cudaSetDevice(prev);
    }
    g_plan_dev.clear();
    cudaGetLastError();
}

// Whole-tile rounds the wide shape takes for this problem on `units` pairs:
// the planner's makespan when it plans, else the round-robin count.
double tc_wide_rounds(long long M, long long N, long long K, int units) {
    const long long tiles = ((M + 255) / 256) * ((N + 511) / 512);
    if (tc_planning_enabled() && wide_plan(M, N, K, units)) {
        std::lock_guard<std::mutex> lk(g_plan_mu);
        auto it = g_plan_rounds.find(PlanKey{M, N, K, units});
        if (it != g_plan_rounds.end()) return it->second;
    }
    return tc_rounds(tiles, units);
}

TcPlan tc_plan(const Problem& p, int shape, int dev, int sms, bool allow_halves, cudaStream_t stream) {
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
    // Wide tiles: a planned mix of item widths when it beats round-robin.
    if (plan.shape == 4 && p.batch == 1 && allow_halves && tc_planning_enabled()) {
        const TcItemTable* t = wide_plan(p.M, p.N, p.K, (int)max_units);
        const int* d = t ? plan_on_device(t, dev, (int)max_units, stream) : nullptr;
        if (t && d) {
            plan.table = t;
            plan.table_dev = d;
            plan.units = (int)max_units;
        }
    }
    return plan;
}

pax_status_t launch_tc(const Problem& p, const TcPlan& plan, cudaStream_t stream) {
    if (p.M > 0x7fffffffLL || p.N > 0x7fffffffLL || p.K > 0x7fffffffLL) return PAX_ERR_UNSUPPORTED;
    return p.c_f16 ? launch_tc_f16(p, plan, stream) : launch_tc_f32(p, plan, stream);
}

bool set_wait_limit_tc(unsigned long long ns) {
    const bool a = set_wait_limit_tc_f16(ns);
    const bool b = set_wait_limit_tc_f32(ns);
    return a && b;
}

int read_clear_device_error_tc() {
    const int a = read_clear_device_error_tc_f16();
    const int b = read_clear_device_error_tc_f32();
    if (a < 0 || b < 0) return -1;
    return a | b;
}

}  // namespace pax

// Host-only test hook: the planned work list of the wide tile (see wide_plan).
extern "C" int pax_selftest_wide_plan(long long M, long long N, long long K, int units, unsigned int* items,
                                      int* unit_start, int max_items) {
    if (M <= 0 || N <= 0 || K <= 0 || units < 1 || !items || !unit_start || max_items < 0) return -1;
    const pax::TcItemTable* t = pax::wide_plan(M, N, K, units);
    if (t == nullptr) return 0;
    if (t->count > max_items) return -1;
    for (int u = 0; u <= units; ++u) unit_start[u] = t->unit_start[u];
    for (int i = 0; i < t->count; ++i) items[i] = t->item[i];
    return t->count;
}
