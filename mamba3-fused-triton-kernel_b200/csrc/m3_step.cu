// Host side of the single-launch decode step: the projection tile choice
// and the dtype dispatch (kernels in m3_step_f32.cu / m3_step_bf16.cu, code
// in m3_step_impl.cuh).
#include "m3_step.cuh"

namespace m3 {

int step_gemm_cfg(int M, int N, int K, int grid) {
  int best = -1;
  long long best_cost = 0;
  for (int c = 0; c < kStepGemmCfgs; ++c) {
    const int KS = kCfgKS[c], KW = kCfgKW[c], KC = KW * KS;
    if ((long long)KW * (KS - 1) >= K) continue;  // a K slice would be empty
    const long long tiles = (long long)((M + kStepTileRows - 1) / kStepTileRows) * ((N + 64 / KS - 1) / (64 / KS));
    const long long rounds = (tiles + grid - 1) / grid;
    const long long chunks = (K + KC - 1) / KC;
    // per chunk: load latency (~8 units of 32 k) plus a warp's 32-k units
    const long long cost = rounds * chunks * (8 + KW / 32);
    if (best < 0 || cost < best_cost) {
      best_cost = cost;
      best = c;
    }
  }
  return best < 0 ? 0 : best;
}

cudaError_t launch_mimo_step(StepParams &sp, cudaStream_t stream) {
  return sp.kp.par_dt == M3_BF16 ? launch_mimo_step_bf16(sp, stream) : launch_mimo_step_f32(sp, stream);
}

cudaError_t launch_siso_step(StepParams &sp, cudaStream_t stream) {
  return sp.kp.par_dt == M3_BF16 ? launch_siso_step_bf16(sp, stream) : launch_siso_step_f32(sp, stream);
}

int step_device_error(bool reset) {
  const int a = step_f32_device_error(reset), b = step_bf16_device_error(reset);
  return a < 0 || b < 0 ? -1 : a | b;
}

}  // namespace m3
