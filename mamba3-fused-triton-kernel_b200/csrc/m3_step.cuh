// Parameter block and host interface of the single-launch decode step
// (m3_step.cu).
#pragma once

#include "m3_kernels.cuh"

namespace m3 {

// Projection tile configurations: KS K-slices across the CTA's 8 warps
// (tile columns 64 / KS), KW k per warp and chunk (a chunk spans KW * KS).
constexpr int kStepGemmCfgs = 4;
constexpr int kStepTileRows = 16;  // output rows of a projection tile
constexpr int kCfgKS[kStepGemmCfgs] = {1, 1, 2, 4};
constexpr int kCfgKW[kStepGemmCfgs] = {128, 256, 128, 128};
// Shared floats of a projection tile: the chunk's 16 A rows and the K-slice
// partial sums.
__host__ __device__ constexpr int step_gemm_smem_floats(int ks, int kw) {
  return kStepTileRows * kw * ks + (ks - 1) * (8 / ks) * 32 * 4;
}
// Grid-barrier words at the start of the workspace: a base word and an
// arrival counter kStepBarStride u32 (128 bytes) after it.
constexpr int kStepBarStride = 32;
constexpr int kStepBarBytes = 256;
constexpr int kStepMaxPrefetch = 16;

// C[M, N] = A[M, K] W[N, K]^T, elements of the step's dtype.
struct StepGemm {
  const void *A; int64_t lda;
  const void *W; int64_t ldw;
  void *C; int64_t ldc;
  int M, N, K;
};

struct StepParams {
  KParams kp;              // decode phase: zx and y point into the workspace
  StepGemm g_in, g_out;    // the two projections
  int cfg_in, cfg_out;     // their tile configurations (set by the launcher)
  int rows_per_item, n_items;  // decode-phase work split (set by the launcher)
  unsigned *bar;           // grid-barrier words at the start of the workspace
  int n_prefetch;          // L2 prefetch ranges (16-byte aligned, sizes % 16 == 0)
  const void *pf_ptr[kStepMaxPrefetch];
  int64_t pf_bytes[kStepMaxPrefetch];
  int pf_first[kStepMaxPrefetch + 1];  // prefix sums of the ranges' 4 KB chunks
};

// Tile configuration the launcher picks for one projection on `grid` CTAs.
int step_gemm_cfg(int M, int N, int K, int grid);
// Enqueue the step kernel (cooperative launch).  Fills the launcher fields.
cudaError_t launch_mimo_step(StepParams &sp, cudaStream_t stream);
cudaError_t launch_mimo_step_f32(StepParams &sp, cudaStream_t stream);
cudaError_t launch_mimo_step_bf16(StepParams &sp, cudaStream_t stream);
// The SISO single-launch step (phase 2: one (batch row, head) tile per item).
cudaError_t launch_siso_step(StepParams &sp, cudaStream_t stream);
cudaError_t launch_siso_step_f32(StepParams &sp, cudaStream_t stream);
cudaError_t launch_siso_step_bf16(StepParams &sp, cudaStream_t stream);
int step_device_error(bool reset);
// The checks of m3_mimo_step without the launch (M3_OK when it would launch;
// *empty when the batch has no rows).
int step_validate(const m3_dims *d, const m3_step_args *a, bool *empty);
int step_f32_device_error(bool reset);
int step_bf16_device_error(bool reset);

}  // namespace m3
