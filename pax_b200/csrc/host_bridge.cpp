// host_bridge.cpp -- the C ABI (include/pax.h) over the sm_100a kernels.
//
// Mirrors the GEMM surface of the reference's host bridge (src/host_bridge.c):
// buffer descriptor helpers (:136-273), per-variant dispatchers (:311-386),
// the CPU verification GEMM and checker (:397-445) and the bench harness
// (:452-566), plus the kernel launchers the bridge declares (:75-102).
// Argument checks print "[PAX] ..." to stderr and return, as the reference
// does; every entry point also records a status for pax_last_error().
#include <cuda_runtime.h>
#include <cuda_fp16.h>

#include <math.h>
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <map>
#include <cuda.h>
#include <mutex>
#include <thread>
#include <vector>
#include <utility>

#include "../../include/pax.h"
#include "internal.h"

namespace pax {

static thread_local pax_status_t t_last = PAX_OK;

static pax_status_t set_status(pax_status_t s) {
    t_last = s;
    return s;
}

static pax_status_t fail(pax_status_t s, const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    fprintf(stderr, "[PAX] ");
    vfprintf(stderr, fmt, ap);
    fprintf(stderr, "\n");
    va_end(ap);
    return set_status(s);
}

// ------------------------------------------------------------ devices
struct DevInfo {
    int sms = 0;
    int major = 0;
    int minor = 0;
    bool known = false;
};
static std::mutex g_dev_mu;
static std::map<int, DevInfo> g_dev;

static DevInfo device_info(int dev) {
    std::lock_guard<std::mutex> lk(g_dev_mu);
    DevInfo& d = g_dev[dev];
    if (!d.known) {
        cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev);
        cudaDeviceGetAttribute(&d.major, cudaDevAttrComputeCapabilityMajor, dev);
        cudaDeviceGetAttribute(&d.minor, cudaDevAttrComputeCapabilityMinor, dev);
        d.known = true;
    }
    return d;
}

int current_device() {
    int dev = 0;
    cudaGetDevice(&dev);
    return dev;
}

int device_sm_count(int dev) { return device_info(dev).sms; }

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

bool tma_compatible(const Problem& p) {
    const long long csz = p.c_f16 ? 2 : 4;
    // Batch strides address whole matrices through the 3-D tensor maps.
    const bool batch_ok = p.batch <= 1 || ((p.sa * 2) % 16 == 0 && (p.sb * 2) % 16 == 0 && (p.sc * csz) % 16 == 0 &&
                                           p.sa < (1LL << 38) && p.sb < (1LL << 38) && p.sc < (1LL << 37));
    return p.K >= 1 && aligned16(p.A) && aligned16(p.B) && aligned16(p.C) && (p.lda * 2) % 16 == 0 &&
           (p.ldb * 2) % 16 == 0 && (p.ldc * csz) % 16 == 0 && p.M < (1LL << 31) && p.N < (1LL << 31) &&
           p.K < (1LL << 31) && batch_ok;
}

// Item b of a batched problem as a single problem.
static Problem batch_item(const Problem& p, long long b) {
    Problem q = p;
    q.batch = 1;
    q.sa = q.sb = q.sc = q.sbias = q.sres = 0;
    q.A = p.A + b * p.sa;
    q.B = p.B + b * p.sb;
    q.C = static_cast<char*>(p.C) + b * p.sc * (p.c_f16 ? 2 : 4);
    if (p.epi.bias) q.epi.bias = p.epi.bias + b * p.sbias;
    if (p.epi.residual)
        q.epi.residual = static_cast<const char*>(p.epi.residual) + b * p.sres * ((p.epi.flags & EPI_RES_F32) ? 4 : 2);
    return q;
}

// --------------------------------------------------------- workspaces
// Split-K scratch of the skinny kernel, one buffer per stream so that
// launches on different streams never share one.  Layout:
// [per-CTA publication flags: cnt_cap bytes][partial sums: ws_cap bytes].
// Nothing in it needs clearing between launches: a flag counts only when it
// holds the current launch's epoch, and a flag that an earlier launch left
// behind (finished, or aborted after a timed-out wait) holds an older one.
// Growing either region reallocates the buffer.
//
// The key is (device, stream handle, thread).  The thread part is used only
// for cudaStreamPerThread: that one handle value names a different stream in
// every host thread, and two threads must not share a buffer for it.
struct Workspace {
    void* ptr = nullptr;
    size_t cnt_cap = 0;
    size_t ws_cap = 0;
};
struct WsKey {
    int dev;
    uintptr_t stream;
    std::thread::id thread;
    bool operator<(const WsKey& o) const {
        if (dev != o.dev) return dev < o.dev;
        if (stream != o.stream) return stream < o.stream;
        return thread < o.thread;
    }
};
static std::mutex g_ws_mu;
static std::map<WsKey, Workspace> g_ws;

static WsKey ws_key(int dev, cudaStream_t s) {
    return {dev, reinterpret_cast<uintptr_t>(s),
            s == cudaStreamPerThread ? std::this_thread::get_id() : std::thread::id()};
}

static pax_status_t get_workspace(int dev, cudaStream_t s, size_t cnt_need, size_t ws_need,
                                  unsigned long long** flags, float** partials) {
    std::lock_guard<std::mutex> lk(g_ws_mu);
    Workspace& w = g_ws[ws_key(dev, s)];
    if (w.cnt_cap < cnt_need || w.ws_cap < ws_need) {
        const size_t cnt_cap = w.cnt_cap > cnt_need ? w.cnt_cap : cnt_need;
        const size_t ws_cap = w.ws_cap > ws_need ? w.ws_cap : ws_need;
        if (w.ptr) {
            cudaStreamSynchronize(s);
            cudaFree(w.ptr);
            w = Workspace();
        }
        if (cudaMalloc(&w.ptr, cnt_cap + ws_cap) != cudaSuccess) {
            w = Workspace();
            return PAX_ERR_ALLOC;
        }
        if (cudaMemsetAsync(w.ptr, 0, cnt_cap + ws_cap, s) != cudaSuccess) {
            // Counters of unknown value must never be used: drop the buffer.
            cudaFree(w.ptr);
            w = Workspace();
            return PAX_ERR_CUDA;
        }
        w.cnt_cap = cnt_cap;
        w.ws_cap = ws_cap;
    }
    *flags = static_cast<unsigned long long*>(w.ptr);
    *partials = reinterpret_cast<float*>(static_cast<char*>(w.ptr) + w.cnt_cap);
    return PAX_OK;
}

// Test hook (pax_selftest_stale_counters): write into the publication
// flags of this stream's workspace what launches that gave up on a
// timed-out wait leave behind: flags holding the latest launch epoch, and
// older ones.
static pax_status_t poison_workspace_counters(int dev, cudaStream_t s) {
    std::lock_guard<std::mutex> lk(g_ws_mu);
    auto it = g_ws.find(ws_key(dev, s));
    if (it == g_ws.end() || !it->second.ptr) return PAX_ERR_INVALID;
    const size_t n = it->second.cnt_cap / sizeof(unsigned long long);
    std::vector<unsigned long long> v(n);
    const unsigned long long last = skinny_last_epoch();
    for (size_t i = 0; i < n; ++i) v[i] = (i % 2 == 0 || last < 2) ? last : last - 1;
    if (cudaStreamSynchronize(s) != cudaSuccess ||
        cudaMemcpy(it->second.ptr, v.data(), n * sizeof(unsigned long long), cudaMemcpyHostToDevice) != cudaSuccess)
        return PAX_ERR_CUDA;
    return PAX_OK;
}

static void free_workspaces() {
    std::lock_guard<std::mutex> lk(g_ws_mu);
    int prev = current_device();
    for (auto& kv : g_ws) {
        if (kv.second.ptr) {
            cudaSetDevice(kv.first.dev);
            cudaDeviceSynchronize();
            cudaFree(kv.second.ptr);
        }
    }
    g_ws.clear();
    cudaSetDevice(prev);
}

// ------------------------------------------------------------ problems
static int epilogue_flags(pax_epilogue_t e, pax_dtype_t res_dt, float alpha) {
    int f = 0;
    switch (e) {
        case PAX_EPI_NONE: break;
        case PAX_EPI_BIAS: f = EPI_BIAS; break;
        case PAX_EPI_BIAS_GELU_TANH: f = EPI_BIAS | EPI_GELU_TANH; break;
        case PAX_EPI_BIAS_GELU_ERF: f = EPI_BIAS | EPI_GELU_ERF; break;
        case PAX_EPI_RESIDUAL_GELU_TANH: f = EPI_RES | EPI_GELU_TANH; break;
        case PAX_EPI_RESIDUAL_GELU_ERF: f = EPI_RES | EPI_GELU_ERF; break;
        case PAX_EPI_GELU_TANH: f = EPI_GELU_TANH; break;
        case PAX_EPI_GELU_ERF: f = EPI_GELU_ERF; break;
        case PAX_EPI_RESIDUAL: f = EPI_RES; break;
        default: return -1;
    }
    if ((f & EPI_RES) && res_dt == PAX_DT_F32) f |= EPI_RES_F32;
    if (alpha != 1.0f) f |= EPI_SCALE;
    return f;
}

// The algorithm field without its hint bits.
static pax_algo_t algo_of(const pax_gemm_desc_t* d) { return static_cast<pax_algo_t>((int)d->algo & 0xFF); }

static pax_status_t normalize(const pax_gemm_desc_t* d, Problem* p) {
    if (!d) return fail(PAX_ERR_INVALID, "pax_gemm_ex: NULL descriptor");
    p->b_const = ((int)d->algo & PAX_GEMM_B_CONST) != 0;
    if (d->M < 0 || d->N < 0 || d->K < 0)
        return fail(PAX_ERR_INVALID, "pax_gemm_ex: negative shape m=%lld n=%lld k=%lld", (long long)d->M,
                    (long long)d->N, (long long)d->K);
    if (d->c_dtype != PAX_DT_F32 && d->c_dtype != PAX_DT_F16)
        return fail(PAX_ERR_INVALID, "pax_gemm_ex: bad output dtype %d", (int)d->c_dtype);
    const int flags = epilogue_flags(d->epilogue, d->residual_dtype, d->alpha);
    if (flags < 0) return fail(PAX_ERR_INVALID, "pax_gemm_ex: bad epilogue %d", (int)d->epilogue);
    p->A = static_cast<const __half*>(d->A);
    p->B = static_cast<const __half*>(d->B);
    p->C = d->C;
    p->M = d->M;
    p->N = d->N;
    p->K = d->K;
    p->lda = d->lda ? d->lda : d->K;
    p->ldb = d->ldb ? d->ldb : d->N;
    p->ldc = d->ldc ? d->ldc : d->N;
    p->c_f16 = d->c_dtype == PAX_DT_F16;
    p->epi.bias = static_cast<const __half*>(d->bias);
    p->epi.residual = d->residual;
    p->epi.ld_res = d->ld_res ? d->ld_res : d->N;
    p->epi.alpha = d->alpha;
    p->epi.flags = flags;
    if (p->M == 0 || p->N == 0) return PAX_OK;  // nothing to write
    if (!p->C) return fail(PAX_ERR_INVALID, "pax_gemm_ex: NULL C");
    if (p->K > 0 && (!p->A || !p->B)) return fail(PAX_ERR_INVALID, "pax_gemm_ex: NULL A or B");
    if ((flags & EPI_BIAS) && !p->epi.bias) return fail(PAX_ERR_INVALID, "pax_gemm_ex: NULL bias");
    if ((flags & EPI_RES) && !p->epi.residual) return fail(PAX_ERR_INVALID, "pax_gemm_ex: NULL residual");
    if ((flags & EPI_RES) && d->residual_dtype != PAX_DT_F32 && d->residual_dtype != PAX_DT_F16)
        return fail(PAX_ERR_INVALID, "pax_gemm_ex: bad residual dtype %d", (int)d->residual_dtype);
    if (p->lda < p->K || p->ldb < p->N || p->ldc < p->N || ((flags & EPI_RES) && p->epi.ld_res < p->N))
        return fail(PAX_ERR_INVALID, "pax_gemm_ex: leading dimension smaller than the row length");
    if (aligned16(p->epi.bias)) p->epi.flags |= EPI_BIAS_VEC;
    const long long rsz = (flags & EPI_RES_F32) ? 4 : 2;
    if ((flags & EPI_RES) && aligned16(p->epi.residual) && (p->epi.ld_res * rsz) % 16 == 0)
        p->epi.flags |= EPI_RES_VEC;
    return PAX_OK;
}

// Internal entry points for other translation units (internal.h).
pax_status_t normalize_desc(const pax_gemm_desc_t* d, Problem* p) { return normalize(d, p); }
pax_status_t report_status(pax_status_t s, const char* msg) {
    if (s == PAX_OK) return set_status(s);
    return fail(s, "%s", msg);
}

static pax_algo_t select_algo(const Problem& p) {
    if (!tma_compatible(p)) return PAX_ALGO_SIMT;
    if (p.M <= kSkinnyMaxM) return PAX_ALGO_SKINNY;
    return PAX_ALGO_TC;
}

static int env_int(const char* name, int dflt) {
    const char* v = getenv(name);
    return v ? atoi(v) : dflt;
}

bool pdl_enabled() {
    static const bool on = env_int("PAX_PDL", 1) != 0;
    return on;
}

bool tc_planning_enabled() { return env_int("PAX_TC_PLAN", 1) != 0; }

// The kernel a problem runs on: `algo` as requested (AUTO: chosen here) and,
// for the tensor-core kernel, its tile shape (128 or 256: one CTA per
// 128 x shape tile; 2: CTA pair per 256 x 256; 4: CTA pair per 256 x 512).
// PAX_TC_SHAPE forces a shape for AUTO; PAX_TC_BN a one-CTA tile width.
static void choose_kernel(const Problem& p, int sms, pax_algo_t* algo, int* shape) {
    *shape = 0;
    if (*algo == PAX_ALGO_AUTO) {
        *algo = select_algo(p);
        if (*algo == PAX_ALGO_TC) {
            *shape = tc_pick_shape(p, sms);
            const int forced = env_int("PAX_TC_SHAPE", 0);
            if (forced == 2 || forced == 4 || forced == 128 || forced == 256) *shape = forced;
            if (*shape == 2 || *shape == 4) *algo = PAX_ALGO_TC2;
        }
    }
    if (*algo == PAX_ALGO_TC2) {
        if (*shape != 4) *shape = 2;
    } else if (*algo == PAX_ALGO_TC && *shape != 128 && *shape != 256) {
        *shape = env_int("PAX_TC_BN", 0);
        if (*shape != 128 && *shape != 256) *shape = tc_pick_bn(p.M, p.N, sms);
    }
}

// Dynamic shared memory of the kernel a problem runs on (0 for the CUDA-core
// kernel, whose shared memory is static).
static size_t kernel_smem_bytes(const Problem& p, pax_algo_t algo, int sms) {
    int shape = 0;
    choose_kernel(p, sms, &algo, &shape);
    if (algo == PAX_ALGO_TC || algo == PAX_ALGO_TC2) return tc_smem_bytes(shape, p.c_f16);
    if (algo == PAX_ALGO_SKINNY && p.M <= kSkinnyMaxM)
        return skinny_smem_bytes(p.M, p.batch > 1 ? 128
                                                  : skinny_layout(p.M, p.N, p.K, sms, skinny_env_nt()).nt);
    return 0;
}

static pax_status_t run(const Problem& p, pax_algo_t algo, cudaStream_t s) {
    if (p.M == 0 || p.N == 0 || p.batch == 0) return PAX_OK;
    const int dev = current_device();
    const DevInfo di = device_info(dev);
    if (di.major != 10) return fail(PAX_ERR_NO_DEVICE, "device %d is sm_%d%d; this library needs sm_100", dev,
                                    di.major, di.minor);
    int shape = 0;  // tensor-core tile shape
    choose_kernel(p, di.sms, &algo, &shape);
    pax_status_t st;
    if (p.n_replicas > 0 && algo != PAX_ALGO_TC && algo != PAX_ALGO_TC2)
        return fail(PAX_ERR_UNSUPPORTED, "replicated output needs the tensor-core path (m > %lld, 16-byte aligned rows)",
                    kSkinnyMaxM);
    // The tensor-core kernels take a whole batch in one launch (3-D tensor
    // maps); the skinny kernel as whole (item, tile) units round-robin over
    // the SMs.  The CUDA-core kernel runs one launch per item.
    if (p.batch > 1 && algo == PAX_ALGO_SKINNY) {
        if (!tma_compatible(p) || p.M > kSkinnyMaxM)
            return fail(PAX_ERR_UNSUPPORTED, "skinny path needs m <= %lld and 16-byte aligned rows", kSkinnyMaxM);
        const long long units = p.batch * ((p.N + 127) / 128);
        const int grid = (int)(units < di.sms ? units : di.sms);
        st = launch_skinny_ws(p, 128, grid, nullptr, nullptr, s, 0);
        if (st != PAX_OK) return fail(st, "launch failed: %s", cudaGetErrorString(cudaGetLastError()));
        return set_status(PAX_OK);
    }
    if (p.batch > 1 && algo == PAX_ALGO_SIMT) {
        for (long long b = 0; b < p.batch; ++b) {
            st = run(batch_item(p, b), algo, s);
            if (st != PAX_OK) return st;
        }
        return set_status(PAX_OK);
    }
    switch (algo) {
        case PAX_ALGO_TC:
        case PAX_ALGO_TC2: {
            if (!tma_compatible(p)) return fail(PAX_ERR_UNSUPPORTED, "tensor-core path needs 16-byte aligned rows");
            // The tail wave's tiles run as column halves (PAX_TC_HALVES=0
            // turns that off for comparisons).
            const TcPlan plan = tc_plan(p, shape, dev, di.sms, env_int("PAX_TC_HALVES", 1) != 0, s);
            st = launch_tc(p, plan, s);
            break;
        }
        case PAX_ALGO_SKINNY: {
            if (!tma_compatible(p) || p.M > kSkinnyMaxM)
                return fail(PAX_ERR_UNSUPPORTED, "skinny path needs m <= %lld and 16-byte aligned rows",
                            kSkinnyMaxM);
            // Lockstep layout when there are no more column tiles than SMs;
            // otherwise persistent stream-K, one CTA per SM.
            // PAX_SKINNY_NT=128|256 forces the persistent layout.
            const SkinnyLayout L = skinny_layout(p.M, p.N, p.K, di.sms, skinny_env_nt());
            const size_t cnt_pad = (L.cnt_bytes + 255) & ~size_t(255);
            unsigned long long* flags = nullptr;
            float* partials = nullptr;
            st = get_workspace(dev, s, cnt_pad, L.ws_bytes, &flags, &partials);
            if (st != PAX_OK)
                return fail(st, "skinny workspace allocation failed (%zu bytes)", cnt_pad + L.ws_bytes);
            st = launch_skinny_ws(p, L.nt, L.grid, partials, flags, s, L.slices);
            break;
        }
        case PAX_ALGO_SIMT: st = launch_simt(p, s); break;
        default: return fail(PAX_ERR_INVALID, "unknown algorithm %d", (int)algo);
    }
    if (st != PAX_OK) return fail(st, "launch failed: %s", cudaGetErrorString(cudaGetLastError()));
    return set_status(PAX_OK);
}

static pax_status_t gemm_simple(const void* A, const void* B, void* C, int m, int n, int k, pax_dtype_t cdt,
                                pax_epilogue_t epi, float alpha, const void* bias, const void* residual,
                                pax_dtype_t rdt, cudaStream_t s, const char* who) {
    if (m < 0 || n < 0 || k < 0) return fail(PAX_ERR_INVALID, "%s: negative shape m=%d n=%d k=%d", who, m, n, k);
    pax_gemm_desc_t d;
    memset(&d, 0, sizeof(d));
    d.A = A;
    d.B = B;
    d.C = C;
    d.M = m;
    d.N = n;
    d.K = k;
    d.c_dtype = cdt;
    d.epilogue = epi;
    d.alpha = alpha;
    d.bias = bias;
    d.residual = residual;
    d.residual_dtype = rdt;
    d.algo = PAX_ALGO_AUTO;
    return pax_gemm_ex(&d, s);
}

}  // namespace pax

using namespace pax;

extern "C" {

// ================================================================ status
const char* pax_version(void) { return "pax_b200 0.1.0 (sm_100a)"; }

pax_status_t pax_last_error(void) { return t_last; }

const char* pax_status_string(pax_status_t s) {
    switch (s) {
        case PAX_OK: return "ok";
        case PAX_ERR_INVALID: return "invalid argument";
        case PAX_ERR_UNSUPPORTED: return "unsupported problem for the requested algorithm";
        case PAX_ERR_CUDA: return "CUDA error";
        case PAX_ERR_TIMEOUT: return "device-side wait timed out";
        case PAX_ERR_NO_DEVICE: return "no sm_100 device";
        case PAX_ERR_ALLOC: return "workspace allocation failed";
    }
    return "unknown status";
}

pax_status_t pax_device_error(void) {
    if (cudaDeviceSynchronize() != cudaSuccess) return set_status(PAX_ERR_CUDA);
    const int a = read_clear_device_error_tc();
    const int b = read_clear_device_error_skinny();
    const int c = read_clear_device_error_peer();
    if (a < 0 || b < 0 || c < 0) return set_status(PAX_ERR_CUDA);
    return set_status((a | b | c) ? PAX_ERR_TIMEOUT : PAX_OK);
}

void pax_shutdown(void) {
    free_workspaces();
    tc_free_plans();
    skinny_forget_scratch();
}

pax_status_t pax_selftest_set_wait_limit(uint64_t ns) {
    // 0 restores the default.  Below a microsecond every launch would give up.
    const unsigned long long v = ns == 0 ? 2000000000ull : (unsigned long long)ns;
    if (v < 1000ull) return fail(PAX_ERR_INVALID, "pax_selftest_set_wait_limit: %llu ns is below 1 us", v);
    if (cudaDeviceSynchronize() != cudaSuccess) return fail(PAX_ERR_CUDA, "pax_selftest_set_wait_limit: device error");
    if (!set_wait_limit_tc(v) || !set_wait_limit_skinny(v))
        return fail(PAX_ERR_CUDA, "pax_selftest_set_wait_limit: copy to the device failed");
    return set_status(PAX_OK);
}

pax_status_t pax_selftest_stale_counters(cudaStream_t stream) {
    const pax_status_t st = poison_workspace_counters(current_device(), stream);
    if (st == PAX_ERR_INVALID) return fail(st, "pax_selftest_stale_counters: no skinny workspace on this stream");
    if (st != PAX_OK) return fail(st, "pax_selftest_stale_counters: copy failed");
    return set_status(PAX_OK);
}

size_t pax_sizeof_buffer(void) { return sizeof(pax_buffer_t); }
size_t pax_sizeof_gemm_desc(void) { return sizeof(pax_gemm_desc_t); }

// ================================================================ general
pax_status_t pax_gemm_ex(const pax_gemm_desc_t* desc, cudaStream_t stream) {
    Problem p;
    pax_status_t st = normalize(desc, &p);
    if (st != PAX_OK) return st;
    return run(p, algo_of(desc), stream);
}

pax_status_t pax_gemm_replicated_ex(const pax_gemm_desc_t* desc, void* const* replicas, int n_replicas,
                                   cudaStream_t stream) {
    Problem p;
    pax_status_t st = normalize(desc, &p);
    if (st != PAX_OK) return st;
    if (n_replicas < 0 || n_replicas > 7 || (n_replicas > 0 && !replicas))
        return fail(PAX_ERR_INVALID, "pax_gemm_replicated_ex: %d replicas (0..7 allowed)", n_replicas);
    for (int i = 0; i < n_replicas; ++i)
        if (!replicas[i] || !aligned16(replicas[i]))
            return fail(PAX_ERR_INVALID, "pax_gemm_replicated_ex: replica %d is NULL or not 16-byte aligned", i);
    p.replicas = replicas;
    p.n_replicas = n_replicas;
    return run(p, algo_of(desc), stream);
}

pax_status_t pax_peer_barrier(unsigned long long* own, unsigned long long* const* peers, int n_peers, int slot,
                              unsigned long long epoch, unsigned long long timeout_ns, cudaStream_t stream) {
    if (n_peers < 0 || n_peers > kPeerMaxPeers)
        return fail(PAX_ERR_INVALID, "pax_peer_barrier: %d peers (0..%d allowed)", n_peers, kPeerMaxPeers);
    if (slot < 0 || slot > n_peers)
        return fail(PAX_ERR_INVALID, "pax_peer_barrier: slot %d outside the %d ranks", slot, n_peers + 1);
    if (!own || (reinterpret_cast<uintptr_t>(own) & 7u) || (n_peers > 0 && !peers))
        return fail(PAX_ERR_INVALID, "pax_peer_barrier: own flags NULL or not 8-byte aligned");
    for (int i = 0; i < n_peers; ++i)
        if (!peers[i] || (reinterpret_cast<uintptr_t>(peers[i]) & 7u))
            return fail(PAX_ERR_INVALID, "pax_peer_barrier: peer %d flags NULL or not 8-byte aligned", i);
    if (epoch == 0) return fail(PAX_ERR_INVALID, "pax_peer_barrier: epoch 0 (flags start at 0)");
    const unsigned long long limit = timeout_ns ? timeout_ns : 10000000000ull;
    if (peer_barrier_launch(own, peers, n_peers, slot, epoch, limit, stream) != cudaSuccess)
        return fail(PAX_ERR_CUDA, "pax_peer_barrier: launch failed");
    return set_status(PAX_OK);
}

// ------------------------------------------------------------- CUDA IPC
// Handles that let each rank map the others' C buffers for
// pax_gemm_replicated_ex.  A handle names the whole allocation that holds
// the pointer plus the pointer's offset in it, so buffers carved out of a
// larger allocation (a framework's caching allocator) can be shared.
static std::mutex g_ipc_mu;
static std::vector<std::pair<void*, void*>> g_ipc_open;  // (pointer returned, mapped base)

static CUresult mem_range(CUdeviceptr* base, size_t* size, CUdeviceptr ptr) {
    using Fn = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);
    static Fn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPointByVersion("cuMemGetAddressRange", &f, 3020, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<Fn>(f);
    });
    return fn ? fn(base, size, ptr) : CUDA_ERROR_NOT_SUPPORTED;
}

pax_status_t pax_ipc_export(const void* device_ptr, pax_ipc_handle_t* out) {
    if (!device_ptr || !out) return fail(PAX_ERR_INVALID, "pax_ipc_export: NULL argument");
    CUdeviceptr base = 0;
    size_t size = 0;
    if (mem_range(&base, &size, (CUdeviceptr)(uintptr_t)device_ptr) != CUDA_SUCCESS)
        return fail(PAX_ERR_CUDA, "pax_ipc_export: pointer is not device memory of this process");
    cudaIpcMemHandle_t h;
    if (cudaIpcGetMemHandle(&h, reinterpret_cast<void*>((uintptr_t)base)) != cudaSuccess) {
        cudaGetLastError();
        return fail(PAX_ERR_CUDA, "pax_ipc_export: cudaIpcGetMemHandle failed");
    }
    static_assert(sizeof(h) == sizeof(out->handle), "IPC handle size");
    memcpy(out->handle, &h, sizeof(h));
    out->offset = (uint64_t)((uintptr_t)device_ptr - (uintptr_t)base);
    return set_status(PAX_OK);
}

pax_status_t pax_ipc_import(const pax_ipc_handle_t* handle, void** device_ptr) {
    if (!handle || !device_ptr) return fail(PAX_ERR_INVALID, "pax_ipc_import: NULL argument");
    cudaIpcMemHandle_t h;
    memcpy(&h, handle->handle, sizeof(h));
    void* base = nullptr;
    if (cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
        cudaGetLastError();
        return fail(PAX_ERR_CUDA, "pax_ipc_import: cudaIpcOpenMemHandle failed");
    }
    *device_ptr = static_cast<char*>(base) + handle->offset;
    std::lock_guard<std::mutex> lk(g_ipc_mu);
    g_ipc_open.emplace_back(*device_ptr, base);
    return set_status(PAX_OK);
}

pax_status_t pax_ipc_close(void* device_ptr) {
    void* base = nullptr;
    {
        std::lock_guard<std::mutex> lk(g_ipc_mu);
        for (size_t i = 0; i < g_ipc_open.size(); ++i)
            if (g_ipc_open[i].first == device_ptr) {
                base = g_ipc_open[i].second;
                g_ipc_open.erase(g_ipc_open.begin() + (long)i);
                break;
            }
    }
    if (!base) return fail(PAX_ERR_INVALID, "pax_ipc_close: pointer was not imported");
    if (cudaIpcCloseMemHandle(base) != cudaSuccess) {
        cudaGetLastError();
        return fail(PAX_ERR_CUDA, "pax_ipc_close: cudaIpcCloseMemHandle failed");
    }
    return set_status(PAX_OK);
}

pax_status_t pax_gemm_batched_ex(const pax_gemm_batched_desc_t* desc, cudaStream_t stream) {
    if (!desc) return fail(PAX_ERR_INVALID, "pax_gemm_batched_ex: NULL descriptor");
    Problem p;
    pax_status_t st = normalize(&desc->gemm, &p);
    if (st != PAX_OK) return st;
    const long long nb = desc->batch;
    if (nb < 0 || desc->stride_a < 0 || desc->stride_b < 0 || desc->stride_c < 0 || desc->stride_bias < 0 ||
        desc->stride_residual < 0)
        return fail(PAX_ERR_INVALID, "pax_gemm_batched_ex: negative batch or stride");
    p.batch = nb;
    if (nb > 1) {
        p.sa = desc->stride_a;
        p.sb = desc->stride_b;
        p.sc = desc->stride_c;
        p.sbias = desc->stride_bias;
        p.sres = desc->stride_residual;
        // Items of C must not overlap: every row of item b ends before item
        // b + 1 begins.
        if (p.M > 0 && p.N > 0 && p.sc < (p.M - 1) * p.ldc + p.N)
            return fail(PAX_ERR_INVALID, "pax_gemm_batched_ex: stride_c %lld overlaps consecutive C items",
                        (long long)p.sc);
        // Vector epilogue loads need every item's bias / residual aligned.
        if ((p.sbias * 2) % 16 != 0) p.epi.flags &= ~EPI_BIAS_VEC;
        const long long rsz = (p.epi.flags & EPI_RES_F32) ? 4 : 2;
        if ((p.sres * rsz) % 16 != 0) p.epi.flags &= ~EPI_RES_VEC;
    }
    return run(p, algo_of(&desc->gemm), stream);
}

pax_algo_t pax_gemm_select_algo(const pax_gemm_desc_t* desc) {
    Problem p;
    if (normalize(desc, &p) != PAX_OK) return PAX_ALGO_AUTO;
    set_status(PAX_OK);
    pax_algo_t a = select_algo(p);
    // With a device present, report the tensor-core tile shape as well: the
    // kernel pax_gemm_ex would launch (CTA pair or not), shape switches
    // included.
    int dev = 0, sms = 0;
    if (a == PAX_ALGO_TC && cudaGetDevice(&dev) == cudaSuccess &&
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess && sms > 0) {
        pax_algo_t b = PAX_ALGO_AUTO;
        int shape = 0;
        choose_kernel(p, sms, &b, &shape);
        a = b;
    }
    cudaGetLastError();  // no device here is not an error of this call
    return a;
}

int pax_gemm_pipeline_stages(const pax_gemm_desc_t* desc) {
    Problem p;
    if (normalize(desc, &p) != PAX_OK) return 0;
    set_status(PAX_OK);
    int dev = 0, sms = 0;
    if (cudaGetDevice(&dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0) {
        cudaGetLastError();
        return 0;
    }
    // The same choices as run() makes for PAX_ALGO_AUTO.
    pax_algo_t a = PAX_ALGO_AUTO;
    int shape = 0;
    choose_kernel(p, sms, &a, &shape);
    if (a == PAX_ALGO_TC || a == PAX_ALGO_TC2) return tc_stages(shape);
    if (a == PAX_ALGO_SKINNY)
        return skinny_stages(p.M, skinny_layout(p.M, p.N, p.K, sms, skinny_env_nt()).nt);
    return 0;  // CUDA-core kernel: no TMA ring
}

// ================================================ Lean-extraction symbols
// pax-lean4/PAX/Extraction.lean:32-56 exports these names with 64-bit sizes
// and device pointers passed as integers; C is fp32 [M][N], bias fp16 [N],
// residual fp32 [M][N].  They run the same kernels as pax_gemm_ex on the
// legacy default stream and report errors as the launchers do.
static void gemm_verified(uint64_t M, uint64_t N, uint64_t K, uint64_t A, uint64_t B, uint64_t C,
                          pax_epilogue_t epi, uint64_t extra, const char* who) {
    if (M > (uint64_t)INT64_MAX || N > (uint64_t)INT64_MAX || K > (uint64_t)INT64_MAX) {
        fail(PAX_ERR_INVALID, "%s: size above 2^63", who);
        return;
    }
    pax_gemm_desc_t d;
    memset(&d, 0, sizeof(d));
    d.A = reinterpret_cast<const void*>((uintptr_t)A);
    d.B = reinterpret_cast<const void*>((uintptr_t)B);
    d.C = reinterpret_cast<void*>((uintptr_t)C);
    d.M = (int64_t)M;
    d.N = (int64_t)N;
    d.K = (int64_t)K;
    d.c_dtype = PAX_DT_F32;
    d.epilogue = epi;
    d.alpha = 1.f;
    if (epi == PAX_EPI_BIAS_GELU_TANH) d.bias = reinterpret_cast<const void*>((uintptr_t)extra);
    if (epi == PAX_EPI_RESIDUAL_GELU_TANH) d.residual = reinterpret_cast<const void*>((uintptr_t)extra);
    d.residual_dtype = PAX_DT_F32;
    d.algo = PAX_ALGO_AUTO;
    pax_gemm_ex(&d, 0);
}

void pax_gemm_wmma_verified(uint64_t M, uint64_t N, uint64_t K, uint64_t A, uint64_t B, uint64_t C) {
    gemm_verified(M, N, K, A, B, C, PAX_EPI_NONE, 0, "pax_gemm_wmma_verified");
}
void pax_gemm_ptx_verified(uint64_t M, uint64_t N, uint64_t K, uint64_t A, uint64_t B, uint64_t C) {
    gemm_verified(M, N, K, A, B, C, PAX_EPI_NONE, 0, "pax_gemm_ptx_verified");
}
void pax_gemm_pipeline3_verified(uint64_t M, uint64_t N, uint64_t K, uint64_t A, uint64_t B, uint64_t C) {
    gemm_verified(M, N, K, A, B, C, PAX_EPI_NONE, 0, "pax_gemm_pipeline3_verified");
}
void pax_gemm_bias_gelu_verified(uint64_t M, uint64_t N, uint64_t K, uint64_t A, uint64_t B, uint64_t C,
                                 uint64_t bias) {
    gemm_verified(M, N, K, A, B, C, PAX_EPI_BIAS_GELU_TANH, bias, "pax_gemm_bias_gelu_verified");
}
void pax_gemm_residual_gelu_verified(uint64_t M, uint64_t N, uint64_t K, uint64_t A, uint64_t B, uint64_t C,
                                     uint64_t residual) {
    gemm_verified(M, N, K, A, B, C, PAX_EPI_RESIDUAL_GELU_TANH, residual, "pax_gemm_residual_gelu_verified");
}

// ======================================================= reference launchers
void pax_gemm_wmma_launch(const __half* A, const __half* B, float* C, int m, int n, int k, cudaStream_t s) {
    gemm_simple(A, B, C, m, n, k, PAX_DT_F32, PAX_EPI_NONE, 1.f, nullptr, nullptr, PAX_DT_F32, s,
                "pax_gemm_wmma_launch");
}
void pax_gemm_ptx_launch(const __half* A, const __half* B, float* C, int m, int n, int k, cudaStream_t s) {
    gemm_simple(A, B, C, m, n, k, PAX_DT_F32, PAX_EPI_NONE, 1.f, nullptr, nullptr, PAX_DT_F32, s,
                "pax_gemm_ptx_launch");
}
void pax_gemm_pipeline_launch(const __half* A, const __half* B, float* C, int m, int n, int k, cudaStream_t s) {
    gemm_simple(A, B, C, m, n, k, PAX_DT_F32, PAX_EPI_NONE, 1.f, nullptr, nullptr, PAX_DT_F32, s,
                "pax_gemm_pipeline_launch");
}
// The reference's *_smem_bytes report the shared memory of the one kernel
// their launcher always runs (src/rtx_gemm_pipeline.cu:331-334,355-361).
// Here the launcher picks a kernel per problem, so these report the dynamic
// shared memory of the kernel the launcher runs for the reference's default
// bench problem, m = n = k = 4096 with fp32 C (src/host_bridge.c:498-500),
// on the current device (148 SMs when there is none).
static size_t launcher_smem_bytes(pax_algo_t algo) {
    Problem p{};
    // Any 16-byte aligned pointers: only the shape and alignment matter.
    alignas(16) static const __half probe_operand[8] = {};
    alignas(16) static float probe_c[4];
    p.A = probe_operand;
    p.B = probe_operand;
    p.C = probe_c;
    p.M = p.N = p.K = 4096;
    p.lda = p.ldb = p.ldc = 4096;
    p.c_f16 = false;
    p.epi.alpha = 1.f;
    p.epi.flags = 0;
    int dev = 0, sms = 0;
    if (cudaGetDevice(&dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0)
        sms = 148;
    cudaGetLastError();
    set_status(PAX_OK);
    return kernel_smem_bytes(p, algo, sms);
}

size_t pax_gemm_ptx_smem_bytes(void) { return launcher_smem_bytes(PAX_ALGO_AUTO); }
size_t pax_gemm_pipeline_smem_bytes(void) { return launcher_smem_bytes(PAX_ALGO_AUTO); }
size_t pax_gemm_tma_smem_bytes(void) { return launcher_smem_bytes(PAX_ALGO_TC2); }

size_t pax_gemm_smem_bytes(const pax_gemm_desc_t* desc) {
    Problem p;
    if (normalize(desc, &p) != PAX_OK) return 0;
    set_status(PAX_OK);
    int dev = 0, sms = 0;
    if (cudaGetDevice(&dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0)
        sms = 148;
    cudaGetLastError();
    return kernel_smem_bytes(p, algo_of(desc), sms);
}

void pax_gemm_bias_gelu_launch(const __half* A, const __half* B, float* C, int m, int n, int k,
                               const __half* bias, cudaStream_t s) {
    gemm_simple(A, B, C, m, n, k, PAX_DT_F32, PAX_EPI_BIAS_GELU_TANH, 1.f, bias, nullptr, PAX_DT_F32, s,
                "pax_gemm_bias_gelu_launch");
}
void pax_gemm_residual_gelu_launch(const __half* A, const __half* B, float* C, int m, int n, int k,
                                   const float* residual, cudaStream_t s) {
    gemm_simple(A, B, C, m, n, k, PAX_DT_F32, PAX_EPI_RESIDUAL_GELU_TANH, 1.f, nullptr, residual, PAX_DT_F32, s,
                "pax_gemm_residual_gelu_launch");
}
void pax_gemm_scale_bias_gelu_launch(const __half* A, const __half* B, float* C, int m, int n, int k,
                                     float alpha, const __half* bias, cudaStream_t s) {
    gemm_simple(A, B, C, m, n, k, PAX_DT_F32, PAX_EPI_BIAS_GELU_TANH, alpha, bias, nullptr, PAX_DT_F32, s,
                "pax_gemm_scale_bias_gelu_launch");
}
void pax_gemm_tma_cluster_launch(const __half* A, const __half* B, float* C, int M, int N, int K,
                                 const void* tmap_A, const void* tmap_B, const void* tmap_C, cudaStream_t s) {
    (void)tmap_A;
    (void)tmap_B;
    (void)tmap_C;
    if (M < 0 || N < 0 || K < 0) {
        fail(PAX_ERR_INVALID, "pax_gemm_tma_cluster_launch: negative shape");
        return;
    }
    pax_gemm_desc_t d;
    memset(&d, 0, sizeof(d));
    d.A = A;
    d.B = B;
    d.C = C;
    d.M = M;
    d.N = N;
    d.K = K;
    d.c_dtype = PAX_DT_F32;
    d.epilogue = PAX_EPI_NONE;
    d.alpha = 1.f;
    d.algo = PAX_ALGO_TC2;
    Problem p;
    if (normalize(&d, &p) != PAX_OK) return;
    // Problems the tensor-core path cannot take still get an answer.
    run(p, tma_compatible(p) ? PAX_ALGO_TC2 : PAX_ALGO_SIMT, s);
}

// ================================================================ fp16 twins
void pax_gemm_f16_launch(const __half* A, const __half* B, __half* C, int m, int n, int k, cudaStream_t s) {
    gemm_simple(A, B, C, m, n, k, PAX_DT_F16, PAX_EPI_NONE, 1.f, nullptr, nullptr, PAX_DT_F16, s,
                "pax_gemm_f16_launch");
}
void pax_gemm_bias_f16_launch(const __half* A, const __half* B, __half* C, int m, int n, int k,
                              const __half* bias, cudaStream_t s) {
    gemm_simple(A, B, C, m, n, k, PAX_DT_F16, PAX_EPI_BIAS, 1.f, bias, nullptr, PAX_DT_F16, s,
                "pax_gemm_bias_f16_launch");
}
void pax_gemm_bias_gelu_f16_launch(const __half* A, const __half* B, __half* C, int m, int n, int k,
                                   const __half* bias, cudaStream_t s) {
    gemm_simple(A, B, C, m, n, k, PAX_DT_F16, PAX_EPI_BIAS_GELU_TANH, 1.f, bias, nullptr, PAX_DT_F16, s,
                "pax_gemm_bias_gelu_f16_launch");
}
void pax_gemm_bias_gelu_erf_f16_launch(const __half* A, const __half* B, __half* C, int m, int n, int k,
                                       const __half* bias, cudaStream_t s) {
    gemm_simple(A, B, C, m, n, k, PAX_DT_F16, PAX_EPI_BIAS_GELU_ERF, 1.f, bias, nullptr, PAX_DT_F16, s,
                "pax_gemm_bias_gelu_erf_f16_launch");
}
void pax_gemm_residual_gelu_f16_launch(const __half* A, const __half* B, __half* C, int m, int n, int k,
                                       const __half* residual, cudaStream_t s) {
    gemm_simple(A, B, C, m, n, k, PAX_DT_F16, PAX_EPI_RESIDUAL_GELU_TANH, 1.f, nullptr, residual, PAX_DT_F16, s,
                "pax_gemm_residual_gelu_f16_launch");
}
void pax_gemm_residual_gelu_erf_f16_launch(const __half* A, const __half* B, __half* C, int m, int n, int k,
                                           const __half* residual, cudaStream_t s) {
    gemm_simple(A, B, C, m, n, k, PAX_DT_F16, PAX_EPI_RESIDUAL_GELU_ERF, 1.f, nullptr, residual, PAX_DT_F16, s,
                "pax_gemm_residual_gelu_erf_f16_launch");
}

// ================================================================ buffers
int pax_validate_buffer(const pax_buffer_t* buf) {
    if (!buf) {
        fail(PAX_ERR_INVALID, "validate_buffer: NULL descriptor");
        return 0;
    }
    if (!buf->base) {
        fail(PAX_ERR_INVALID, "validate_buffer: NULL base pointer");
        return 0;
    }
    if (buf->elem_size == 0) {
        fail(PAX_ERR_INVALID, "validate_buffer: elem_size == 0");
        return 0;
    }
    if (buf->ndim < 1 || buf->ndim > 3) {
        fail(PAX_ERR_INVALID, "validate_buffer: ndim=%d out of [1,3]", buf->ndim);
        return 0;
    }
    for (int d = 0; d < buf->ndim; ++d) {
        if (buf->shape[d] <= 0) {
            fail(PAX_ERR_INVALID, "validate_buffer: shape[%d]=%lld <= 0", d, (long long)buf->shape[d]);
            return 0;
        }
        if (buf->stride[d] <= 0) {
            fail(PAX_ERR_INVALID, "validate_buffer: stride[%d]=%lld <= 0", d, (long long)buf->stride[d]);
            return 0;
        }
    }
    if (buf->alignment && (reinterpret_cast<uintptr_t>(buf->base) % buf->alignment != 0)) {
        fail(PAX_ERR_INVALID, "validate_buffer: base %p not aligned to %zu", buf->base, buf->alignment);
        return 0;
    }
    set_status(PAX_OK);
    return 1;
}

static pax_buffer_t make_buffer(int ndim, size_t d0, size_t d1, size_t elem, size_t align, pax_ownership_t own,
                                cudaStream_t s) {
    pax_buffer_t b;
    memset(&b, 0, sizeof(b));
    b.elem_size = elem;
    b.ndim = ndim;
    b.shape[0] = (int64_t)d0;
    if (ndim == 1) {
        b.stride[0] = 1;
    } else {
        b.shape[1] = (int64_t)d1;
        b.stride[0] = (int64_t)d1;
        b.stride[1] = 1;
    }
    b.alignment = align;
    b.ownership = own;
    b.stream = s;
    return b;
}

pax_buffer_t pax_alloc_device_1d(size_t nelems, size_t elem_size, cudaStream_t stream) {
    pax_buffer_t b = make_buffer(1, nelems, 0, elem_size, 256, PAX_DEVICE, stream);
    if (cudaMalloc(&b.base, nelems * elem_size) != cudaSuccess) {
        fail(PAX_ERR_ALLOC, "pax_alloc_device_1d: cudaMalloc failed (%zu bytes)", nelems * elem_size);
        b.base = nullptr;
    } else {
        set_status(PAX_OK);
    }
    return b;
}

pax_buffer_t pax_alloc_device_2d(size_t rows, size_t cols, size_t elem_size, cudaStream_t stream) {
    pax_buffer_t b = make_buffer(2, rows, cols, elem_size, 256, PAX_DEVICE, stream);
    if (cudaMalloc(&b.base, rows * cols * elem_size) != cudaSuccess) {
        fail(PAX_ERR_ALLOC, "pax_alloc_device_2d: cudaMalloc failed (%zu bytes)", rows * cols * elem_size);
        b.base = nullptr;
    } else {
        set_status(PAX_OK);
    }
    return b;
}

pax_buffer_t pax_alloc_host_1d(size_t nelems, size_t elem_size, cudaStream_t stream) {
    pax_buffer_t b = make_buffer(1, nelems, 0, elem_size, 64, PAX_HOST, stream);
    if (cudaMallocHost(&b.base, nelems * elem_size) != cudaSuccess) {
        fail(PAX_ERR_ALLOC, "pax_alloc_host_1d: cudaMallocHost failed");
        b.base = nullptr;
    } else {
        set_status(PAX_OK);
    }
    return b;
}

pax_buffer_t pax_alloc_host_2d(size_t rows, size_t cols, size_t elem_size, cudaStream_t stream) {
    pax_buffer_t b = make_buffer(2, rows, cols, elem_size, 64, PAX_HOST, stream);
    if (cudaMallocHost(&b.base, rows * cols * elem_size) != cudaSuccess) {
        fail(PAX_ERR_ALLOC, "pax_alloc_host_2d: cudaMallocHost failed");
        b.base = nullptr;
    } else {
        set_status(PAX_OK);
    }
    return b;
}

void pax_free_device(pax_buffer_t* buf) {
    if (buf && buf->base) {
        cudaFree(buf->base);
        buf->base = nullptr;
    }
}

void pax_free_host(pax_buffer_t* buf) {
    if (buf && buf->base) {
        cudaFreeHost(buf->base);
        buf->base = nullptr;
    }
}

// ============================================================ dispatchers
// The reference reads m = A.shape[0], k = A.shape[1], n = B.shape[1] and
// ignores strides (src/host_bridge.c:317-321); row strides are honoured here.
static bool buffers_to_desc(pax_buffer_t* A, pax_buffer_t* B, pax_buffer_t* C, pax_gemm_desc_t* d,
                            const char* who) {
    if (!pax_validate_buffer(A) || !pax_validate_buffer(B) || !pax_validate_buffer(C)) return false;
    memset(d, 0, sizeof(*d));
    d->A = A->base;
    d->B = B->base;
    d->C = C->base;
    d->M = A->shape[0];
    d->K = A->shape[1];
    d->N = B->shape[1];
    d->lda = (A->ndim >= 2 && A->stride[1] == 1) ? A->stride[0] : 0;
    d->ldb = (B->ndim >= 2 && B->stride[1] == 1) ? B->stride[0] : 0;
    d->ldc = (C->ndim >= 2 && C->stride[1] == 1) ? C->stride[0] : 0;
    if (C->elem_size == 4) {
        d->c_dtype = PAX_DT_F32;
    } else if (C->elem_size == 2) {
        d->c_dtype = PAX_DT_F16;
    } else {
        fail(PAX_ERR_INVALID, "%s: C elem_size %zu is neither 4 (fp32) nor 2 (fp16)", who, C->elem_size);
        return false;
    }
    if (A->elem_size != 2 || B->elem_size != 2) {
        fail(PAX_ERR_INVALID, "%s: A and B must be fp16 (elem_size 2)", who);
        return false;
    }
    d->alpha = 1.f;
    d->algo = PAX_ALGO_AUTO;
    return true;
}

static void dispatch_plain(pax_buffer_t* A, pax_buffer_t* B, pax_buffer_t* C, cudaStream_t s, const char* who) {
    pax_gemm_desc_t d;
    if (!buffers_to_desc(A, B, C, &d, who)) return;
    d.epilogue = PAX_EPI_NONE;
    pax_gemm_ex(&d, s);
}

void pax_dispatch_wmma_gemm(pax_buffer_t* A, pax_buffer_t* B, pax_buffer_t* C, cudaStream_t s) {
    dispatch_plain(A, B, C, s, "pax_dispatch_wmma_gemm");
}
void pax_dispatch_ptx_gemm(pax_buffer_t* A, pax_buffer_t* B, pax_buffer_t* C, cudaStream_t s) {
    dispatch_plain(A, B, C, s, "pax_dispatch_ptx_gemm");
}
void pax_dispatch_pipeline_gemm(pax_buffer_t* A, pax_buffer_t* B, pax_buffer_t* C, cudaStream_t s) {
    dispatch_plain(A, B, C, s, "pax_dispatch_pipeline_gemm");
}

void pax_dispatch_bias_gelu(pax_buffer_t* A, pax_buffer_t* B, pax_buffer_t* C, const __half* bias,
                            cudaStream_t s) {
    pax_gemm_desc_t d;
    if (!buffers_to_desc(A, B, C, &d, "pax_dispatch_bias_gelu")) return;
    if (!bias) {
        fail(PAX_ERR_INVALID, "pax_dispatch_bias_gelu: NULL bias");
        return;
    }
    d.epilogue = PAX_EPI_BIAS_GELU_TANH;
    d.bias = bias;
    pax_gemm_ex(&d, s);
}

void pax_dispatch_residual_gelu(pax_buffer_t* A, pax_buffer_t* B, pax_buffer_t* C, const float* residual,
                                cudaStream_t s) {
    pax_gemm_desc_t d;
    if (!buffers_to_desc(A, B, C, &d, "pax_dispatch_residual_gelu")) return;
    if (!residual) {
        fail(PAX_ERR_INVALID, "pax_dispatch_residual_gelu: NULL residual");
        return;
    }
    d.epilogue = PAX_EPI_RESIDUAL_GELU_TANH;
    d.residual = residual;
    d.residual_dtype = PAX_DT_F32;
    pax_gemm_ex(&d, s);
}

void pax_dispatch_scale_bias_gelu(pax_buffer_t* A, pax_buffer_t* B, pax_buffer_t* C, float alpha,
                                  const __half* bias, cudaStream_t s) {
    pax_gemm_desc_t d;
    if (!buffers_to_desc(A, B, C, &d, "pax_dispatch_scale_bias_gelu")) return;
    if (!bias) {
        fail(PAX_ERR_INVALID, "pax_dispatch_scale_bias_gelu: NULL bias");
        return;
    }
    d.epilogue = PAX_EPI_BIAS_GELU_TANH;
    d.alpha = alpha;
    d.bias = bias;
    pax_gemm_ex(&d, s);
}

// ============================================================ verification
void cpu_gemm_ref(const float* A, const float* B, float* C, int m, int n, int k) {
    for (int i = 0; i < m; ++i) {
        const float* a = A + (size_t)i * k;
        for (int j = 0; j < n; ++j) {
            float s = 0.f;
            for (int l = 0; l < k; ++l) s += a[l] * B[(size_t)l * n + j];
            C[(size_t)i * n + j] = s;
        }
    }
}

int pax_verify_gemm(const float* C_gpu, const float* C_ref, int m, int n, float tol) {
    float worst = 0.f;
    long long at = 0;
    const long long total = (long long)m * n;
    for (long long i = 0; i < total; ++i) {
        const float e = fabsf(C_gpu[i] - C_ref[i]) / (fabsf(C_ref[i]) + 1e-8f);
        if (e > worst) {
            worst = e;
            at = i;
        }
    }
    if (worst <= tol) {
        printf("[PAX] PASS  max_rel_err = %.6e  (tol = %.6e)\n", (double)worst, (double)tol);
        return 1;
    }
    printf("[PAX] FAIL  max_rel_err = %.6e  (tol = %.6e)  at index %lld  gpu=%.6f  ref=%.6f\n", (double)worst,
           (double)tol, at, (double)C_gpu[at], (double)C_ref[at]);
    return 0;
}

// ================================================================ bench
static struct {
    bool ready = false;
    int m = 0, n = 0, k = 0;
    cudaStream_t stream = nullptr;
    __half *A = nullptr, *B = nullptr, *bias = nullptr, *res16 = nullptr, *C16 = nullptr;
    float *C32 = nullptr, *res32 = nullptr;
} g_bench;

void pax_bench_teardown(void) {
    cudaFree(g_bench.A);
    cudaFree(g_bench.B);
    cudaFree(g_bench.bias);
    cudaFree(g_bench.res16);
    cudaFree(g_bench.C16);
    cudaFree(g_bench.C32);
    cudaFree(g_bench.res32);
    g_bench.A = g_bench.B = g_bench.bias = g_bench.res16 = g_bench.C16 = nullptr;
    g_bench.C32 = g_bench.res32 = nullptr;
    g_bench.ready = false;
}

int pax_bench_setup(int m, int n, int k, cudaStream_t stream) {
    pax_bench_teardown();
    if (m <= 0 || n <= 0 || k <= 0) {
        fail(PAX_ERR_INVALID, "pax_bench_setup: bad shape");
        return 0;
    }
    const size_t mk = (size_t)m * k, kn = (size_t)k * n, mn = (size_t)m * n;
    bool ok = cudaMalloc(&g_bench.A, mk * 2) == cudaSuccess && cudaMalloc(&g_bench.B, kn * 2) == cudaSuccess &&
              cudaMalloc(&g_bench.bias, (size_t)n * 2) == cudaSuccess &&
              cudaMalloc(&g_bench.res16, mn * 2) == cudaSuccess && cudaMalloc(&g_bench.C16, mn * 2) == cudaSuccess &&
              cudaMalloc(&g_bench.C32, mn * 4) == cudaSuccess && cudaMalloc(&g_bench.res32, mn * 4) == cudaSuccess;
    if (!ok) {
        pax_bench_teardown();
        fail(PAX_ERR_ALLOC, "pax_bench_setup: allocation failed");
        return 0;
    }
    fill_uniform_f16(g_bench.A, (long long)mk, 1, -1.f, 1.f, stream);
    fill_uniform_f16(g_bench.B, (long long)kn, 2, -1.f, 1.f, stream);
    fill_uniform_f16(g_bench.bias, n, 3, -1.f, 1.f, stream);
    fill_uniform_f16(g_bench.res16, (long long)mn, 4, -1.f, 1.f, stream);
    cudaMemsetAsync(g_bench.res32, 0, mn * 4, stream);
    g_bench.m = m;
    g_bench.n = n;
    g_bench.k = k;
    g_bench.stream = stream;
    g_bench.ready = cudaStreamSynchronize(stream) == cudaSuccess;
    return g_bench.ready ? 1 : 0;
}

typedef void (*bench_fn)(cudaStream_t);

static void b_wmma(cudaStream_t s) {
    pax_gemm_wmma_launch(g_bench.A, g_bench.B, g_bench.C32, g_bench.m, g_bench.n, g_bench.k, s);
}
static void b_ptx(cudaStream_t s) {
    pax_gemm_ptx_launch(g_bench.A, g_bench.B, g_bench.C32, g_bench.m, g_bench.n, g_bench.k, s);
}
static void b_pipe(cudaStream_t s) {
    pax_gemm_pipeline_launch(g_bench.A, g_bench.B, g_bench.C32, g_bench.m, g_bench.n, g_bench.k, s);
}
static void b_bias_gelu(cudaStream_t s) {
    pax_gemm_bias_gelu_launch(g_bench.A, g_bench.B, g_bench.C32, g_bench.m, g_bench.n, g_bench.k, g_bench.bias, s);
}
static void b_res_gelu(cudaStream_t s) {
    pax_gemm_residual_gelu_launch(g_bench.A, g_bench.B, g_bench.C32, g_bench.m, g_bench.n, g_bench.k,
                                  g_bench.res32, s);
}
static void b_bias_gelu_f16(cudaStream_t s) {
    pax_gemm_bias_gelu_f16_launch(g_bench.A, g_bench.B, g_bench.C16, g_bench.m, g_bench.n, g_bench.k, g_bench.bias,
                                  s);
}
static void b_res_gelu_erf_f16(cudaStream_t s) {
    pax_gemm_residual_gelu_erf_f16_launch(g_bench.A, g_bench.B, g_bench.C16, g_bench.m, g_bench.n, g_bench.k,
                                          g_bench.res16, s);
}

static double time_variant(bench_fn fn, int iters, cudaStream_t s) {
    cudaEvent_t e0, e1;
    cudaEventCreate(&e0);
    cudaEventCreate(&e1);
    fn(s);  // warm-up
    cudaStreamSynchronize(s);
    cudaEventRecord(e0, s);
    for (int i = 0; i < iters; ++i) fn(s);
    cudaEventRecord(e1, s);
    cudaEventSynchronize(e1);
    float ms = 0.f;
    cudaEventElapsedTime(&ms, e0, e1);
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    return (double)ms / (iters > 0 ? iters : 1);
}

void pax_bench_all(int iters) {
    if (!g_bench.ready) {
        fail(PAX_ERR_INVALID, "pax_bench_all: call pax_bench_setup first");
        return;
    }
    printf("\n[PAX] Benchmark  m=%d  n=%d  k=%d  iters=%d\n", g_bench.m, g_bench.n, g_bench.k, iters);
    printf("%-28s  %10s  %10s\n", "Kernel", "ms/iter", "TFLOPS");
    const double flops = 2.0 * g_bench.m * (double)g_bench.n * (double)g_bench.k;
    struct {
        const char* name;
        bench_fn fn;
    } variants[] = {
        {"wmma", b_wmma},         {"ptx", b_ptx},
        {"pipeline", b_pipe},     {"bias_gelu", b_bias_gelu},
        {"residual_gelu", b_res_gelu}, {"bias_gelu_f16", b_bias_gelu_f16},
        {"residual_gelu_erf_f16", b_res_gelu_erf_f16},
    };
    for (auto& v : variants) {
        const double ms = time_variant(v.fn, iters, g_bench.stream);
        printf("%-28s  %10.4f  %10.3f\n", v.name, ms, flops / (ms * 1e9));
    }
    printf("\n");
    // The table goes out now, not at exit, when stdout is a pipe or a file.
    fflush(stdout);
}

}  // extern "C"
