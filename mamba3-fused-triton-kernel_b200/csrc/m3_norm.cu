// Residual add + RMSNorm between the blocks of a Mamba-3 stack.
//
// A residual block is x <- x + mixer(RMSNorm(x)) (src/models/mamba3.py:
// 412-421, RMSNorm :26-36).  Decoding a stack alternates the mixer step with
//     x_next  = x + o                     (in x's dtype, like torch's add)
//     xn_next = RMSNorm_next(x_next)      (fp32 math, result in x's dtype)
// which this kernel does in one pass over the (B, d_model) activations: one
// CTA per batch row, the row held in registers between the two halves.
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "m3_kernels.cuh"

namespace m3 {

namespace {

constexpr int kNormThreads = 256;
constexpr int kNormMaxPerThread = 32;  // d_model <= 8192

template <typename T> __device__ __forceinline__ float ld_t(const T *p, int64_t i);
template <> __device__ __forceinline__ float ld_t<float>(const float *p, int64_t i) { return p[i]; }
template <> __device__ __forceinline__ float ld_t<__nv_bfloat16>(const __nv_bfloat16 *p, int64_t i) {
  return __bfloat162float(p[i]);
}
template <typename T> __device__ __forceinline__ float round_t(float v);
template <> __device__ __forceinline__ float round_t<float>(float v) { return v; }
template <> __device__ __forceinline__ float round_t<__nv_bfloat16>(float v) {
  return __bfloat162float(__float2bfloat16_rn(v));
}
template <typename T> __device__ __forceinline__ void st_t(T *p, int64_t i, float v);
template <> __device__ __forceinline__ void st_t<float>(float *p, int64_t i, float v) { p[i] = v; }
template <> __device__ __forceinline__ void st_t<__nv_bfloat16>(__nv_bfloat16 *p, int64_t i, float v) {
  p[i] = __float2bfloat16_rn(v);
}

// x_out = x (+ o); xn = x_out / sqrt(mean(x_out^2) + eps) * w, with w in
// fp32 (the stack's norm weights are created fp32, src/models/mamba3.py:417).
template <typename T>
__global__ void __launch_bounds__(kNormThreads) residual_rmsnorm_kernel(const T *x, const T *o, const float *w,
                                                                        T *x_out, T *xn, int N, int64_t ldx,
                                                                        int64_t ldo, int64_t ldxo, int64_t ldn,
                                                                        float eps) {
  __shared__ float red[kNormThreads / 32];
  const int row = blockIdx.x, tid = threadIdx.x;
  float v[kNormMaxPerThread];
  pdl_wait();
  pdl_trigger();
  float ss = 0.f;
#pragma unroll
  for (int q = 0; q < kNormMaxPerThread; ++q) {
    const int c = tid + q * kNormThreads;
    v[q] = 0.f;
    if (c < N) {
      float a = ld_t(x, (int64_t)row * ldx + c);
      if (o != nullptr) a = round_t<T>(a + ld_t(o, (int64_t)row * ldo + c));
      v[q] = a;
      if (x_out != nullptr) st_t(x_out, (int64_t)row * ldxo + c, a);
      ss += a * a;
    }
  }
  if (xn == nullptr) return;
  ss = group_sum<32>(ss);
  if ((tid & 31) == 0) red[tid >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int i = 0; i < kNormThreads / 32; ++i) tot += red[i];
  const float rms = sqrtf(tot / (float)N + eps);
#pragma unroll
  for (int q = 0; q < kNormMaxPerThread; ++q) {
    const int c = tid + q * kNormThreads;
    if (c < N) st_t(xn, (int64_t)row * ldn + c, v[q] / rms * w[c]);
  }
}

}  // namespace

cudaError_t launch_residual_rmsnorm(int dtype, const void *x, const void *o, const float *w, void *x_out, void *xn,
                                    int M, int N, int64_t ldx, int64_t ldo, int64_t ldxo, int64_t ldn, float eps,
                                    cudaStream_t stream) {
  if (dtype == M3_BF16)
    return launch_pdl(residual_rmsnorm_kernel<__nv_bfloat16>, dim3(M), dim3(kNormThreads), 0, stream,
                      static_cast<const __nv_bfloat16 *>(x), static_cast<const __nv_bfloat16 *>(o), w,
                      static_cast<__nv_bfloat16 *>(x_out), static_cast<__nv_bfloat16 *>(xn), N, ldx, ldo, ldxo, ldn,
                      eps);
  return launch_pdl(residual_rmsnorm_kernel<float>, dim3(M), dim3(kNormThreads), 0, stream,
                    static_cast<const float *>(x), static_cast<const float *>(o), w, static_cast<float *>(x_out),
                    static_cast<float *>(xn), N, ldx, ldo, ldxo, ldn, eps);
}

int residual_rmsnorm_max_width() { return kNormThreads * kNormMaxPerThread; }

}  // namespace m3
