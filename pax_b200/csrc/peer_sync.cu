// peer_sync.cu -- rank barrier over NVLink peer memory, for replicated
// outputs (pax_gemm_replicated_ex).
//
// Every rank owns an array of `world` 64-bit flags in its own device memory
// and maps the other ranks' arrays (CUDA IPC).  One barrier is one small
// kernel on the caller's stream, which starts only when everything queued
// before it on that stream has finished:
//   * one thread per peer makes this rank's earlier writes visible system-wide
//     and release-stores the barrier's epoch into its own slot of that peer's
//     array;
//   * one thread per other rank waits, with acquire loads at system scope,
//     until that rank's slot of this rank's array holds the epoch (or a later
//     one).
// Epochs grow from barrier to barrier, the same sequence on every rank, so
// nothing is ever cleared: a rank can run at most one barrier ahead, and its
// later epoch satisfies the ">=" of the barrier its peers are still in.
// Every wait is bounded; on expiry the kernel records PAX_DEVERR_TIMEOUT in
// this translation unit's error word and ends, so a missing peer costs the
// timeout, never a hung GPU.
#include "internal.h"
#include "sm100.cuh"

namespace pax {

struct PeerFlagPtrs {
    unsigned long long* peer[kPeerMaxPeers];
};

__device__ __forceinline__ void st_release_sys(unsigned long long* p, unsigned long long v) {
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

__global__ void __launch_bounds__(32, 1)
    peer_barrier_kernel(const PeerFlagPtrs peers, const unsigned long long* own, int n_peers, int slot,
                        unsigned long long epoch, unsigned long long limit_ns) {
    const int t = threadIdx.x;
    if (t < n_peers) {
        __threadfence_system();
        st_release_sys(peers.peer[t] + slot, epoch);
    }
    // Thread t waits for rank t (every rank but this one).
    if (t <= n_peers && t != slot) {
        const unsigned long long t0 = globaltimer_ns();
        while (ld_acquire_sys(own + t) < epoch) {
            if (globaltimer_ns() - t0 > limit_ns) {
                atomicOr(&g_pax_device_error, PAX_DEVERR_TIMEOUT);
                break;
            }
            __nanosleep(128);
        }
    }
    __syncwarp();
    if (t == 0) __threadfence_system();
}

cudaError_t peer_barrier_launch(unsigned long long* own, unsigned long long* const* peers, int n_peers, int slot,
                                unsigned long long epoch, unsigned long long limit_ns, cudaStream_t stream) {
    PeerFlagPtrs pf;
    for (int i = 0; i < kPeerMaxPeers; ++i) pf.peer[i] = i < n_peers ? peers[i] : nullptr;
    peer_barrier_kernel<<<1, 32, 0, stream>>>(pf, own, n_peers, slot, epoch, limit_ns);
    return cudaGetLastError();
}

int read_clear_device_error_peer() {
    int v = 0, z = 0;
    if (cudaMemcpyFromSymbol(&v, g_pax_device_error, sizeof(int)) != cudaSuccess) return -1;
    if (v) cudaMemcpyToSymbol(g_pax_device_error, &z, sizeof(int));
    return v;
}

}  // namespace pax
