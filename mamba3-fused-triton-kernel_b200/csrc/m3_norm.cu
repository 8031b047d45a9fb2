// Residual add + RMSNorm between the blocks of a Mamba-3 stack.
//
// A residual block is x <- x + mixer(RMSNorm(x)) (src/models/mamba3.py:
// 412-421, RMSNorm :26-36).  Decoding a stack alternates the mixer step with
//     x_next  = x + o                     (in x's dtype, like torch's add)
//     xn_next = RMSNorm_next(x_next)      (fp32 math, result in x's dtype)
// which this kernel does in one pass over the (B, d_model) activations: one
// CTA per batch row, the row held in registers between the two halves
// (16-byte vector accesses when the rows are aligned, else element-wise).
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

// The same on 16-byte vectors: each thread owns up to CH chunks of VEC
// consecutive elements (VEC = 16 / sizeof(T)), so a row of d_model 2048 in
// bf16 is one load of x, one of o and one store of each output per thread.
template <typename T> struct Vec16;
template <> struct Vec16<float> {
  static constexpr int N = 4;
  __device__ static void load(const float *p, float (&v)[4]) {
    const float4 t = *reinterpret_cast<const float4 *>(p);
    v[0] = t.x; v[1] = t.y; v[2] = t.z; v[3] = t.w;
  }
  __device__ static void store(float *p, const float (&v)[4]) {
    *reinterpret_cast<float4 *>(p) = make_float4(v[0], v[1], v[2], v[3]);
  }
};
template <> struct Vec16<__nv_bfloat16> {
  static constexpr int N = 8;
  __device__ static void load(const __nv_bfloat16 *p, float (&v)[8]) {
    const uint4 t = *reinterpret_cast<const uint4 *>(p);
    const uint32_t u[4] = {t.x, t.y, t.z, t.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&u[i]));
      v[2 * i] = f.x;
      v[2 * i + 1] = f.y;
    }
  }
  __device__ static void store(__nv_bfloat16 *p, const float (&v)[8]) {
    uint4 t;
    uint32_t *u = reinterpret_cast<uint32_t *>(&t);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const __nv_bfloat162 b = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
      u[i] = *reinterpret_cast<const uint32_t *>(&b);
    }
    *reinterpret_cast<uint4 *>(p) = t;
  }
};

template <typename T, int CH>
__global__ void __launch_bounds__(kNormThreads) residual_rmsnorm_vec_kernel(const T *x, const T *o, const float *w,
                                                                            T *x_out, T *xn, int N, int64_t ldx,
                                                                            int64_t ldo, int64_t ldxo, int64_t ldn,
                                                                            float eps) {
  constexpr int VEC = Vec16<T>::N;
  __shared__ float red[kNormThreads / 32];
  const int row = blockIdx.x, tid = threadIdx.x;
  float v[CH][VEC];
  pdl_wait();
  pdl_trigger();
  float ss = 0.f;
#pragma unroll
  for (int q = 0; q < CH; ++q) {
    const int c = (tid + q * kNormThreads) * VEC;
    if (c < N) {
      Vec16<T>::load(x + (int64_t)row * ldx + c, v[q]);
      if (o != nullptr) {
        float b[VEC];
        Vec16<T>::load(o + (int64_t)row * ldo + c, b);
#pragma unroll
        for (int e = 0; e < VEC; ++e) v[q][e] = round_t<T>(v[q][e] + b[e]);
      }
      if (x_out != nullptr) Vec16<T>::store(x_out + (int64_t)row * ldxo + c, v[q]);
#pragma unroll
      for (int e = 0; e < VEC; ++e) ss += v[q][e] * v[q][e];
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
  for (int q = 0; q < CH; ++q) {
    const int c = (tid + q * kNormThreads) * VEC;
    if (c < N) {
      float wv[VEC], r[VEC];
#pragma unroll
      for (int e = 0; e < VEC; e += 4) {
        const float4 t = *reinterpret_cast<const float4 *>(w + c + e);
        wv[e] = t.x; wv[e + 1] = t.y; wv[e + 2] = t.z; wv[e + 3] = t.w;
      }
#pragma unroll
      for (int e = 0; e < VEC; ++e) r[e] = v[q][e] / rms * wv[e];
      Vec16<T>::store(xn + (int64_t)row * ldn + c, r);
    }
  }
}

bool vec_ok(const void *p, int64_t ld, int es) {
  return p == nullptr || ((reinterpret_cast<uintptr_t>(p) & 15) == 0 && (ld * es) % 16 == 0);
}

template <typename T>
cudaError_t launch_vec(const T *x, const T *o, const float *w, T *x_out, T *xn, int M, int N, int64_t ldx,
                       int64_t ldo, int64_t ldxo, int64_t ldn, float eps, cudaStream_t stream) {
  const int per = kNormThreads * Vec16<T>::N;  // elements per chunk round
  const int ch = (N + per - 1) / per;
  if (ch <= 1)
    return launch_pdl(residual_rmsnorm_vec_kernel<T, 1>, dim3(M), dim3(kNormThreads), 0, stream, x, o, w, x_out, xn,
                      N, ldx, ldo, ldxo, ldn, eps);
  if (ch <= 2)
    return launch_pdl(residual_rmsnorm_vec_kernel<T, 2>, dim3(M), dim3(kNormThreads), 0, stream, x, o, w, x_out, xn,
                      N, ldx, ldo, ldxo, ldn, eps);
  if (ch <= 4)
    return launch_pdl(residual_rmsnorm_vec_kernel<T, 4>, dim3(M), dim3(kNormThreads), 0, stream, x, o, w, x_out, xn,
                      N, ldx, ldo, ldxo, ldn, eps);
  return launch_pdl(residual_rmsnorm_vec_kernel<T, 8>, dim3(M), dim3(kNormThreads), 0, stream, x, o, w, x_out, xn, N,
                    ldx, ldo, ldxo, ldn, eps);
}

}  // namespace

cudaError_t launch_residual_rmsnorm(int dtype, const void *x, const void *o, const float *w, void *x_out, void *xn,
                                    int M, int N, int64_t ldx, int64_t ldo, int64_t ldxo, int64_t ldn, float eps,
                                    cudaStream_t stream) {
  const int es = dtype == M3_BF16 ? 2 : 4;
  if (N % (16 / es) == 0 && vec_ok(x, ldx, es) && vec_ok(o, ldo, es) && vec_ok(x_out, ldxo, es) &&
      vec_ok(xn, ldn, es) && vec_ok(w, 0, 4)) {
    if (dtype == M3_BF16)
      return launch_vec(static_cast<const __nv_bfloat16 *>(x), static_cast<const __nv_bfloat16 *>(o), w,
                        static_cast<__nv_bfloat16 *>(x_out), static_cast<__nv_bfloat16 *>(xn), M, N, ldx, ldo, ldxo,
                        ldn, eps, stream);
    return launch_vec(static_cast<const float *>(x), static_cast<const float *>(o), w, static_cast<float *>(x_out),
                      static_cast<float *>(xn), M, N, ldx, ldo, ldxo, ldn, eps, stream);
  }
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
