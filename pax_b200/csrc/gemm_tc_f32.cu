// gemm_tc_f32.cu -- instantiates the tcgen05 GEMM (gemm_tc.cuh) for fp32 C.
#include "gemm_tc.cuh"

namespace pax {

pax_status_t launch_tc_f32(const Problem& p, const TcPlan& plan, cudaStream_t stream) {
    return launch_tc_typed<float>(p, plan, stream);
}

int tc_pair_units_f32(int dev, int sms) { return tc_pair_units_typed<float>(dev, sms); }

int read_clear_device_error_tc_f32() { return read_clear_device_error_this_unit(); }

bool set_wait_limit_tc_f32(unsigned long long ns) { return set_wait_limit_this_unit(ns); }

}  // namespace pax
