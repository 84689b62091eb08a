// params.h -- epilogue parameter block shared by host code and kernels.
// Plain C++ (no device code) so the C-ABI layer can build it.
#pragma once

#include <cuda_fp16.h>

namespace pax {

enum EpiFlags : int {
    EPI_BIAS      = 1 << 0,  // add fp16 bias[j]
    EPI_RES       = 1 << 1,  // add residual R[i][j]
    EPI_RES_F32   = 1 << 2,  // residual is fp32 (else fp16)
    EPI_GELU_TANH = 1 << 3,
    EPI_GELU_ERF  = 1 << 4,
    EPI_SCALE     = 1 << 5,  // multiply by alpha first
    EPI_BIAS_VEC  = 1 << 6,  // bias pointer 16-byte aligned (vector loads allowed)
    EPI_RES_VEC   = 1 << 7   // residual base and row pitch 16-byte aligned
};

struct EpiParams {
    const __half* bias;     // [N]
    const void* residual;   // [M][ld_res]
    long long ld_res;       // elements
    float alpha;
    int flags;
};

// Host-planned work list of the tcgen05 kernel: the items of unit u (a CTA
// or CTA pair) are item[unit_start[u] .. unit_start[u + 1]).  An item packs
// its 256-row block (bits 0-15), its first column / 128 (bits 16-27) and its
// width code (bits 28-29: 512, 384, 256, 128 columns).  count = 0: no table,
// the kernel's own round-robin schedule.  The kernel reads a device copy
// (unit_start then item, as ints) through TcParams::plan.
struct TcItemTable {
    static constexpr int kMaxUnits = 160;
    static constexpr int kMaxItems = 640;
    int count;
    int unit_start[kMaxUnits + 1];
    unsigned int item[kMaxItems];
};

}  // namespace pax
