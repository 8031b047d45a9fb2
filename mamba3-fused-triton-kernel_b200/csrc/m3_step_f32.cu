// Single-launch decode step kernels, f32 instantiations.
#include "m3_step_impl.cuh"

namespace m3 {

cudaError_t launch_mimo_step_f32(StepParams &sp, cudaStream_t stream) { return launch_step_d<float>(sp, stream); }
cudaError_t launch_siso_step_f32(StepParams &sp, cudaStream_t stream) {
  return launch_siso_step_d<float>(sp, stream);
}

int step_f32_device_error(bool reset) { return device_error_of_this_unit(reset); }

}  // namespace m3
