// gemm_tc_f16.cu -- instantiates the tcgen05 GEMM (gemm_tc.cuh) for fp16 C.
#include "gemm_tc.cuh"

namespace pax {

pax_status_t launch_tc_f16(const Problem& p, const TcPlan& plan, cudaStream_t stream) {
    return launch_tc_typed<__half>(p, plan, stream);
}

int tc_pair_units_f16(int dev, int sms) { return tc_pair_units_typed<__half>(dev, sms); }

int read_clear_device_error_tc_f16() { return read_clear_device_error_this_unit(); }

bool set_wait_limit_tc_f16(unsigned long long ns) { return set_wait_limit_this_unit(ns); }

}  // namespace pax
