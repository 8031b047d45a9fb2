// Single-launch decode step kernels, bf16 instantiations.
#include "m3_step_impl.cuh"

namespace m3 {

cudaError_t launch_mimo_step_bf16(StepParams &sp, cudaStream_t stream) { return launch_step_d<__nv_bfloat16>(sp, stream); }
cudaError_t launch_siso_step_bf16(StepParams &sp, cudaStream_t stream) {
  return launch_siso_step_d<__nv_bfloat16>(sp, stream);
}

int step_bf16_device_error(bool reset) { return device_error_of_this_unit(reset); }

}  // namespace m3
