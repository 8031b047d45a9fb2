// Launchers of the SISO decode kernels (see m3_kernels.cuh).
#include "m3_kernels.cuh"

namespace m3 {

namespace {

template <int BD>
int siso_warps(int P) {
  using Sh = SisoShape<BD>;
  const int rows_per_warp = Sh::RPW * Sh::RPT;  // rows one warp covers per iteration
  int w = (P + rows_per_warp - 1) / rows_per_warp;
  return w < 2 ? 2 : (w > 16 ? 16 : w);
}

template <int BD, bool FULL>
cudaError_t launch_t(const KParams &kp, cudaStream_t stream) {
  const int threads = siso_warps<BD>(kp.P) * 32;
  const size_t smem = (size_t)(2 * BD + 2 * kp.P) * sizeof(float);
  const unsigned grid = (unsigned)((int64_t)kp.B * kp.H);
  siso_decode_kernel<BD, FULL><<<grid, threads, smem, stream>>>(kp);
  return cudaGetLastError();
}

template <bool FULL>
cudaError_t launch_bd(const KParams &kp, cudaStream_t stream) {
  if (kp.D <= 16) return launch_t<16, FULL>(kp, stream);
  if (kp.D <= 32) return launch_t<32, FULL>(kp, stream);
  if (kp.D <= 64) return launch_t<64, FULL>(kp, stream);
  if (kp.D <= 128) return launch_t<128, FULL>(kp, stream);
  return launch_t<256, FULL>(kp, stream);
}

}  // namespace

int siso_block_threads(int D, int P) {
  if (D <= 16) return siso_warps<16>(P) * 32;
  if (D <= 32) return siso_warps<32>(P) * 32;
  if (D <= 64) return siso_warps<64>(P) * 32;
  if (D <= 128) return siso_warps<128>(P) * 32;
  return siso_warps<256>(P) * 32;
}

cudaError_t launch_siso(const KParams &kp, bool full, cudaStream_t stream) {
  return full ? launch_bd<true>(kp, stream) : launch_bd<false>(kp, stream);
}

}  // namespace m3
