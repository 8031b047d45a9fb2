// Small-batch fp32 linear layer for the decode step's projections:
//   C[m, n] = sum_k A[m, k] * W[n, k]      (A: M x K, W: N x K, both K-contiguous)
// i.e. nn.Linear(x) = x @ W^T without bias, for M (the batch) up to a few
// hundred rows.  At these sizes the GEMM is latency-bound, not FLOP-bound:
// one CTA owns 16 output rows x 16 output columns; its 16 A rows of a K
// chunk are staged in shared memory, each warp keeps the K-slices of its two
// W rows in registers (lane l holds k = 4l + 128t), every load of a chunk is
// issued before any is used, and the 32 partial sums of a warp (16 rows x 2
// columns) are combined across lanes with one transpose-butterfly (31
// shuffles) after which lane l owns output l.  Summation is in fp32.
//
// For 1-8 rows and K of 512-2048 the layer is a stream of its weight:
// gemv_kernel gives a CTA 8 (at 8 batch rows: 4) weight rows whose K range
// its 8 warps split (a lane's 16-byte loads of all of them issued before
// the dependency wait, so every weight byte of the launch can be in flight
// at once), stages the batch rows in shared memory, reduces each warp's
// rows x MR partial sums with one transpose-butterfly and adds the warps'
// in warp order.
#include <cuda_runtime.h>
#include <stdint.h>

#include "m3_kernels.cuh"

namespace m3 {

namespace {

constexpr int kLinWarps = 8;            // 2 output columns per warp
constexpr int kLinRows = 16;            // output rows per CTA
constexpr int kLinCols = 2 * kLinWarps;  // output columns per CTA

__device__ __forceinline__ float4 ldg4(const float *p) { return __ldg(reinterpret_cast<const float4 *>(p)); }

// Sum each of the 32 values over the warp; afterwards lane l holds the total
// of v[l] (halving exchange at offsets 16, 8, 4, 2, 1).
__device__ __forceinline__ float warp_transpose_sum32(float (&v)[32]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int lvl = 0; lvl < 5; ++lvl) {
    const int off = 16 >> lvl;
    const int half = 16 >> lvl;  // live values after this level
    const bool upper = (lane & off) != 0;
#pragma unroll
    for (int q = 0; q < half; ++q) {
      const float send = upper ? v[q] : v[q + half];
      const float keep = upper ? v[q + half] : v[q];
      v[q] = keep + __shfl_xor_sync(kFullMask, send, off);
    }
  }
  return v[0];
}

// KT float4 per lane per W row and chunk: a chunk spans KT * 128 columns.
template <int KT>
__global__ void __launch_bounds__(kLinWarps * 32) linear_small_m_kernel(const float *__restrict__ A, int64_t lda,
                                                                        const float *__restrict__ W, int64_t ldw,
                                                                        float *__restrict__ C, int64_t ldc, int M,
                                                                        int N, int K) {
  constexpr int KC = KT * 128;
  __shared__ __align__(16) float4 As[kLinRows * KT * 32];  // [16 rows][KC / 4]

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int m0 = blockIdx.y * kLinRows;
  const int n0 = blockIdx.x * kLinCols + 2 * warp;
  const int mrows = min(kLinRows, M - m0);

  float acc[32];  // acc[j * 16 + i]: row m0 + i, column n0 + j
#pragma unroll
  for (int q = 0; q < 32; ++q) acc[q] = 0.f;

  for (int kc = 0; kc < K; kc += KC) {
    float4 w[2][KT];
#pragma unroll
    for (int j = 0; j < 2; ++j)
#pragma unroll
      for (int t = 0; t < KT; ++t) {
        const int k = kc + 4 * lane + 128 * t;
        w[j][t] = (n0 + j < N && k < K) ? ldg4(W + (int64_t)(n0 + j) * ldw + k) : make_float4(0.f, 0.f, 0.f, 0.f);
      }
    if (kc == 0) {  // the weights are in flight; A is produced by the preceding kernel
      pdl_wait();
      pdl_trigger();
    }
    for (int v = tid; v < kLinRows * KT * 32; v += kLinWarps * 32) {
      const int i = v / (KT * 32), k = kc + (v - i * (KT * 32)) * 4;
      As[v] = (i < mrows && k < K) ? ldg4(A + (int64_t)(m0 + i) * lda + k) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    __syncthreads();
#pragma unroll
    for (int i = 0; i < kLinRows; ++i) {
#pragma unroll
      for (int t = 0; t < KT; ++t) {
        const float4 a = As[i * (KT * 32) + lane + 32 * t];
        acc[i] += a.x * w[0][t].x + a.y * w[0][t].y + a.z * w[0][t].z + a.w * w[0][t].w;
        acc[16 + i] += a.x * w[1][t].x + a.y * w[1][t].y + a.z * w[1][t].z + a.w * w[1][t].w;
      }
    }
    __syncthreads();
  }
  const float v = warp_transpose_sum32(acc);
  const int i = lane & 15, j = lane >> 4;
  if (i < mrows && n0 + j < N) C[(int64_t)(m0 + i) * ldc + n0 + j] = v;
}

// Sum each of V values (V a power of two <= 32) over the warp: afterwards
// lane l holds the total of v[l >> (5 - log2 V)] (halving exchanges at
// offsets 16, 8, ... while values remain, then butterflies on the last).
template <int V>
__device__ __forceinline__ float warp_transpose_sum(float (&v)[V]) {
  const int lane = threadIdx.x & 31;
  int off = 16;
#pragma unroll
  for (int half = V / 2; half >= 1; half >>= 1, off >>= 1) {
    const bool upper = (lane & off) != 0;
#pragma unroll
    for (int q = 0; q < half; ++q) {
      const float send = upper ? v[q] : v[q + half];
      const float keep = upper ? v[q + half] : v[q];
      v[q] = keep + __shfl_xor_sync(kFullMask, send, off);
    }
  }
  for (; off >= 1; off >>= 1) v[0] += __shfl_xor_sync(kFullMask, v[0], off);
  return v[0];
}

constexpr int kGemvWarps = 8;
constexpr int kGemvMaxRows = 8;  // batch rows

// Weight rows per CTA for MR batch rows: rows x MR <= 32 partial sums per lane.
template <int MR> constexpr int gemv_rows() { return MR <= 4 ? 8 : 32 / MR; }

// C[m, n] for m < M <= MR and the CTA's weight rows: warp w takes columns
// [w CPL 128, (w + 1) CPL 128) of all of them (lane l: k = 4l + 128t), the
// batch rows staged in shared memory; each warp's rows x MR partial sums
// go through one transpose-butterfly and the 8 warps' are added in warp
// order.
template <int MR, int CPL>
__global__ void __launch_bounds__(kGemvWarps * 32) gemv_kernel(const float *__restrict__ A, int64_t lda,
                                                               const float *__restrict__ W, int64_t ldw,
                                                               float *__restrict__ C, int64_t ldc, int M, int N,
                                                               int K) {
  constexpr int RPC = gemv_rows<MR>();
  constexpr int V = RPC * MR;  // partial sums per lane
  static_assert(V == 8 || V == 16 || V == 32, "transpose-butterfly width");
  constexpr int LV = V == 8 ? 3 : V == 16 ? 4 : 5;
  extern __shared__ __align__(16) float4 xs[];  // [M][K / 4]
  __shared__ float part[kGemvWarps][V];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int n0 = blockIdx.x * RPC;
  const int k4n = K >> 2;
  float4 w[RPC][CPL];
#pragma unroll
  for (int r = 0; r < RPC; ++r)
#pragma unroll
    for (int t = 0; t < CPL; ++t) {
      const int k = (warp * CPL + t) * 128 + 4 * lane;
      w[r][t] = (n0 + r < N && k < K) ? ldg4(W + (int64_t)(n0 + r) * ldw + k) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
  pdl_wait();  // the weights are constant and already requested; the batch rows are the preceding kernel's
  pdl_trigger();
  for (int v = tid; v < M * k4n; v += kGemvWarps * 32) {
    const int m = v / k4n, k4 = v - m * k4n;
    xs[v] = ldg4(A + (int64_t)m * lda + 4 * k4);
  }
  __syncthreads();
  float acc[V];
#pragma unroll
  for (int j = 0; j < V; ++j) acc[j] = 0.f;
#pragma unroll
  for (int t = 0; t < CPL; ++t) {
    const int k = (warp * CPL + t) * 128 + 4 * lane;
    if (k < K) {
#pragma unroll
      for (int m = 0; m < MR; ++m) {
        const float4 a = m < M ? xs[m * k4n + (k >> 2)] : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int r = 0; r < RPC; ++r)
          acc[r * MR + m] += a.x * w[r][t].x + a.y * w[r][t].y + a.z * w[r][t].z + a.w * w[r][t].w;
      }
    }
  }
  const float v = warp_transpose_sum<V>(acc);
  if ((lane & ((32 >> LV) - 1)) == 0) part[warp][lane >> (5 - LV)] = v;
  __syncthreads();
  if (tid < V) {
    float s = 0.f;
#pragma unroll
    for (int q = 0; q < kGemvWarps; ++q) s += part[q][tid];
    const int r = tid / MR, m = tid - r * MR;
    if (n0 + r < N && m < M) C[(int64_t)m * ldc + n0 + r] = s;
  }
}

template <int MR, int CPL>
cudaError_t launch_gemv(const float *A, int64_t lda, const float *W, int64_t ldw, float *C, int64_t ldc, int M, int N,
                        int K, cudaStream_t stream) {
  constexpr int rows = gemv_rows<MR>();
  const size_t smem = (size_t)M * K * sizeof(float);  // at most 8 x 2048 x 4 = 64 KB
  auto kern = gemv_kernel<MR, CPL>;
  static LaunchCache cache;
  if (smem > 48 * 1024)
    if (cudaError_t e = ensure_smem_optin(cache, kern, 64 * 1024); e != cudaSuccess) return e;
  return launch_pdl(kern, dim3((unsigned)((N + rows - 1) / rows)), dim3(kGemvWarps * 32), smem, stream, A, lda, W,
                    ldw, C, ldc, M, N, K);
}

template <int MR>
cudaError_t launch_gemv_m(const float *A, int64_t lda, const float *W, int64_t ldw, float *C, int64_t ldc, int M,
                          int N, int K, cudaStream_t stream) {
  if (K <= kGemvWarps * 128) return launch_gemv<MR, 1>(A, lda, W, ldw, C, ldc, M, N, K, stream);
  return launch_gemv<MR, 2>(A, lda, W, ldw, C, ldc, M, N, K, stream);
}

template <int KT>
cudaError_t launch_kt(const float *A, int64_t lda, const float *W, int64_t ldw, float *C, int64_t ldc, int M, int N,
                      int K, cudaStream_t stream) {
  const dim3 grid((unsigned)((N + kLinCols - 1) / kLinCols), (unsigned)((M + kLinRows - 1) / kLinRows));
  return launch_pdl(linear_small_m_kernel<KT>, grid, dim3(kLinWarps * 32), 0, stream, A, lda, W, ldw, C, ldc, M, N,
                    K);
}

}  // namespace

cudaError_t launch_linear_small_m(const float *A, int64_t lda, const float *W, int64_t ldw, float *C, int64_t ldc,
                                  int M, int N, int K, cudaStream_t stream) {
  if (K >= 512 && K <= 2 * kGemvWarps * 128 && M <= kGemvMaxRows) {
    if (M == 1) return launch_gemv_m<1>(A, lda, W, ldw, C, ldc, M, N, K, stream);
    if (M == 2) return launch_gemv_m<2>(A, lda, W, ldw, C, ldc, M, N, K, stream);
    if (M <= 4) return launch_gemv_m<4>(A, lda, W, ldw, C, ldc, M, N, K, stream);
    return launch_gemv_m<8>(A, lda, W, ldw, C, ldc, M, N, K, stream);
  }
  if (K <= 128) return launch_kt<1>(A, lda, W, ldw, C, ldc, M, N, K, stream);
  if (K <= 256) return launch_kt<2>(A, lda, W, ldw, C, ldc, M, N, K, stream);
  if (K <= 384) return launch_kt<3>(A, lda, W, ldw, C, ldc, M, N, K, stream);
  return launch_kt<4>(A, lda, W, ldw, C, ldc, M, N, K, stream);
}

}  // namespace m3
