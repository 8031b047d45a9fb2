// MIMO decode kernels.
//
// mimo_row_kernel (full-step fused): the row algorithm of m3_mimo_row.cuh,
// one CTA per (group of 8 heads, run of consecutive batch rows); each thread
// issues all of a row's independent loads before using any of them, and four
// CTAs share an SM so that their rows hide each other's latency.
// mimo_decode_kernel (m3_kernels.cuh) serves everything else: the
// state-update-only entry points and shapes the row kernel does not take
// (head counts that are not a multiple of 8, headdim > 128, mixed dtypes).
#include "m3_async.cuh"
#include "m3_kernels.cuh"
#include "m3_mimo_row.cuh"

namespace m3 {

namespace {

using row::kRowWarps;
using row::row_block_floats;

// The standalone full-step kernel: one CTA per (head group, run of rows).
// PRE: per-head parameters held in registers across the CTA's rows (wider
// state rows, 2 CTAs per SM with twice the registers); otherwise re-read per
// row through the read-only cache (4 CTAs per SM).
template <int BD, int R, typename T, int KP, bool PRE>
__global__ void __launch_bounds__(kRowWarps * 32, PRE ? 2 : 4) mimo_row_kernel(const KParams p, const int rows_per_cta) {
  extern __shared__ __align__(16) float smem[];
  const int ngrp = p.H / kRowWarps;
  const int grp = blockIdx.x % ngrp;
  const int b0 = (blockIdx.x / ngrp) * rows_per_cta;
  const int b1 = min(p.B, b0 + rows_per_cta);
  row::mimo_row_block<BD, R, T, KP, false, PRE>(p, grp, b0, b1, smem, [] {
    pdl_wait();
    pdl_trigger();
  });
}

int num_sms() { return sm_count_current(); }

bool aligned(const void *p, unsigned a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; }

// Whether the row kernel can take this call: whole groups of 8 heads, one
// dtype for the in_proj output and the parameters, vector-aligned state
// and parameter rows, and headdim <= 32 * KP.
bool row_eligible(const KParams &kp, int es, int VW) {
  if (kp.zx_dt != kp.par_dt) return false;
  if (kp.H % kRowWarps != 0 || kp.P > 128) return false;
  if (!aligned(kp.h, 16) || !aligned(kp.bx, 16) || !aligned(kp.bB, VW * es) || !aligned(kp.bC, VW * es)) return false;
  if ((kp.D * es) % (VW * es) != 0) return false;
  return true;
}

template <int BD, int R, typename T, int KP>
cudaError_t launch_row_kp(const KParams &kp, cudaStream_t stream) {
  auto kern = mimo_row_kernel<BD, R, T, KP, (BD >= 128)>;
  const size_t smem = 2 * (size_t)row_block_floats(R, BD, kp.A) * sizeof(float);
  static LaunchCache cache;
  if (cudaError_t e = ensure_smem_optin(cache, kern, 96 * 1024); e != cudaSuccess) return e;
  int per_sm = 0;
  if (occupancy_per_sm(cache, kern, kRowWarps * 32, smem, &per_sm) != cudaSuccess || per_sm < 1) per_sm = 1;
  const int ngrp = kp.H / kRowWarps;
  const int slots = num_sms() * per_sm;
  const int64_t items = (int64_t)kp.B * ngrp;
  int rows = (int)((items + slots - 1) / slots);
  if (rows < 1) rows = 1;
  const int64_t grid = (int64_t)ngrp * ((kp.B + rows - 1) / rows);
  return launch_pdl(kern, dim3((unsigned)grid), dim3(kRowWarps * 32), smem, stream, kp, rows);
}

template <int BD, int R, typename T>
cudaError_t launch_row(const KParams &kp, cudaStream_t stream, bool *taken) {
  *taken = false;
  if (!row_eligible(kp, sizeof(T), MimoShape<BD>::VW)) return cudaSuccess;
  *taken = true;
  if (kp.P <= 32) return launch_row_kp<BD, R, T, 1>(kp, stream);
  if (kp.P <= 64) return launch_row_kp<BD, R, T, 2>(kp, stream);
  return launch_row_kp<BD, R, T, 4>(kp, stream);
}

template <int BD, int R>
cudaError_t launch_full_t(const KParams &kp, cudaStream_t stream) {
  bool taken = false;
  if (BD >= 64) {
    cudaError_t e = launch_mimo_stream(kp, stream, &taken);
    if (e != cudaSuccess || taken) return e;
  }
  cudaError_t e = kp.zx_dt == M3_BF16 ? launch_row<BD, R, __nv_bfloat16>(kp, stream, &taken)
                                      : launch_row<BD, R, float>(kp, stream, &taken);
  if (e != cudaSuccess || taken) return e;
  // generic path
  const int ngrp = (kp.H + kp.heads_per_cta - 1) / kp.heads_per_cta;
  const unsigned grid = (unsigned)((int64_t)kp.B * ngrp);
  const size_t smem = (size_t)2 * R * BD * sizeof(float);
  return launch_pdl(mimo_decode_kernel<BD, R, true>, dim3(grid), dim3(kp.heads_per_cta * 32), smem, stream, kp);
}

template <int BD, int R>
cudaError_t launch_ssm_t(const KParams &kp, cudaStream_t stream) {
  const int ngrp = (kp.H + kp.heads_per_cta - 1) / kp.heads_per_cta;
  const unsigned grid = (unsigned)((int64_t)kp.B * ngrp);
  return launch_pdl(mimo_decode_kernel<BD, R, false>, dim3(grid), dim3(kp.heads_per_cta * 32), 0, stream, kp);
}

template <int BD>
cudaError_t launch_r(const KParams &kp, bool full, cudaStream_t stream) {
  switch (kp.R) {
    case 1: return full ? launch_full_t<BD, 1>(kp, stream) : launch_ssm_t<BD, 1>(kp, stream);
    case 2: return full ? launch_full_t<BD, 2>(kp, stream) : launch_ssm_t<BD, 2>(kp, stream);
    case 4: return full ? launch_full_t<BD, 4>(kp, stream) : launch_ssm_t<BD, 4>(kp, stream);
    case 8: return full ? launch_full_t<BD, 8>(kp, stream) : launch_ssm_t<BD, 8>(kp, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace

int mimo_heads_per_cta(int H) { return H < 8 ? H : 8; }

cudaError_t launch_mimo(const KParams &kp, bool full, cudaStream_t stream) {
  if (kp.D <= 16) return launch_r<16>(kp, full, stream);
  if (kp.D <= 32) return launch_r<32>(kp, full, stream);
  if (kp.D <= 64) return launch_r<64>(kp, full, stream);
  if (kp.D <= 128) return launch_r<128>(kp, full, stream);
  return launch_r<256>(kp, full, stream);
}

int mimo_device_error(bool reset) { return device_error_of_this_unit(reset); }

}  // namespace m3
