// Launchers of the MIMO decode kernels (see m3_kernels.cuh).
#include "m3_kernels.cuh"

namespace m3 {

namespace {

template <int BD, int R, bool FULL>
cudaError_t launch_t(const KParams &kp, cudaStream_t stream) {
  const int ngrp = (kp.H + kp.heads_per_cta - 1) / kp.heads_per_cta;
  const unsigned grid = (unsigned)((int64_t)kp.B * ngrp);
  const size_t smem = FULL ? (size_t)2 * R * BD * sizeof(float) : 0;
  mimo_decode_kernel<BD, R, FULL><<<grid, kp.heads_per_cta * 32, smem, stream>>>(kp);
  return cudaGetLastError();
}

template <int BD, bool FULL>
cudaError_t launch_r(const KParams &kp, cudaStream_t stream) {
  switch (kp.R) {
    case 1: return launch_t<BD, 1, FULL>(kp, stream);
    case 2: return launch_t<BD, 2, FULL>(kp, stream);
    case 4: return launch_t<BD, 4, FULL>(kp, stream);
    case 8: return launch_t<BD, 8, FULL>(kp, stream);
    default: return cudaErrorInvalidValue;
  }
}

template <bool FULL>
cudaError_t launch_bd(const KParams &kp, cudaStream_t stream) {
  if (kp.D <= 16) return launch_r<16, FULL>(kp, stream);
  if (kp.D <= 32) return launch_r<32, FULL>(kp, stream);
  if (kp.D <= 64) return launch_r<64, FULL>(kp, stream);
  if (kp.D <= 128) return launch_r<128, FULL>(kp, stream);
  return launch_r<256, FULL>(kp, stream);
}

}  // namespace

int mimo_heads_per_cta(int H) { return H < 8 ? H : 8; }

cudaError_t launch_mimo(const KParams &kp, bool full, cudaStream_t stream) {
  return full ? launch_bd<true>(kp, stream) : launch_bd<false>(kp, stream);
}

}  // namespace m3
