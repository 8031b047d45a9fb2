// Single-launch MIMO decode step: in_proj GEMM -> fused decode -> out_proj
// GEMM in one persistent kernel.
//
// Included by m3_step_f32.cu and m3_step_bf16.cu (one instantiation set per
// dtype, compiled in parallel); m3_step.cu holds the host-side dispatch.
//
// The three-launch step (src/models/inference.py:476-559: in_proj, the
// fused Triton kernel, out_proj) moves a few megabytes per step at the
// batch sizes of decoding, so its time is the latency of three dependent
// kernels, each of which starts with a cold DRAM round trip.  Here one
// cooperative grid (every CTA resident) runs the three phases separated by
// two grid-wide barriers:
//
//   0  every CTA asks L2 to prefetch its share of everything the later
//      phases read from DRAM (out_proj weight, carried state, per-head
//      parameters, the rest of in_proj's weight), so those reads overlap
//      phase 1 and later phases only wait on L2;
//   1  zx = u @ W_in^T into the workspace (fp32 FMA tiles, below);
//   2  the MIMO row algorithm (m3_mimo_row.cuh) on zx, writing the gated
//      output y into the workspace and the carried state in place;
//   3  out = y @ W_out^T.
//
// Projection tiles.  A CTA computes 16 rows x TC columns of C = A W^T.  Its
// 8 warps form 8/KS column groups of 4 columns times KS slices of the K
// range; a lane holds the K-slices (4 consecutive k per 128) of its warp's
// 4 W rows in registers, the tile's 16 A rows of the current K chunk sit in
// shared memory, and each lane accumulates all 64 (row, column) partial
// sums of its k values.  One 64-value transpose-butterfly then leaves lane l
// with 2 finished sums, and the KS slices are added in slice order through
// shared memory.  The per-output summation order is fixed by (KS, TK), so
// results are deterministic.  (KS, TK) is chosen per projection on the host
// from the tile count and the grid size.
//
// Grid barriers count arrivals on a counter in the workspace that is never
// reset (see grid_barrier).  Each barrier wait sits inside the next phase,
// after the loads that do not depend on the previous phase (carried state,
// parameters, weights) have been issued.  Every spin is bounded: a wait
// that gives up records M3_DEVERR_TIMEOUT and the CTA carries on (its
// accesses stay in bounds; the launch's results are then undefined).
#pragma once

#include "m3_async.cuh"
#include "m3_kernels.cuh"
#include "m3_mimo_row.cuh"
#include "m3_step.cuh"

namespace m3 {

namespace {

using row::kRowWarps;
using row::row_block_floats;

constexpr int kStepThreads = kRowWarps * 32;
constexpr int kTileRows = kStepTileRows;
constexpr int kPrefetchChunk = 4096;

__device__ __forceinline__ void st_out(float *p, float v) { *p = v; }
__device__ __forceinline__ void st_out(__nv_bfloat16 *p, float v) { *p = __float2bfloat16_rn(v); }

// ---------------------------------------------------------------------------
// projection tiles (tensor cores)
// ---------------------------------------------------------------------------
//
// C[M, N] = A[M, K] W[N, K]^T on mma.sync tiles: fp32 operands as three
// TF32 products (A_lo W_hi + A_hi W_lo + A_hi W_hi, each operand split into
// a TF32 head and the TF32 rounding of its remainder, so the result carries
// fp32-level error), bf16 operands as one bf16 product; fp32 accumulation.
// A CTA computes 16 rows x TC columns; warp w covers the 8 columns
// n0 + 8 (w / KS) over K slice w % KS of every chunk, and the KS slices are
// added in slice order through shared memory (deterministic).  Per 16-wide
// k unit, lane (g = lane / 4, t = lane % 4) supplies k = 4t .. 4t + 3 of A
// rows g and g + 8 and of W row n0 + g; the MMA's k slots receive a fixed
// permutation of those k (the same for A and W), which leaves every product
// and the sum unchanged and lets each lane read its k values with one
// vector load.  The chunk's 16 A rows are staged in shared memory (fp32:
// split into head / remainder planes once, for all warps); each warp's W
// values go straight to registers.  Independent accumulators (k-unit parity
// x product) keep the MMA dependency chains short; they are added in a
// fixed order at the end.

__device__ __forceinline__ uint32_t tf32_rna(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return r;
}

// D += A B for one m16n8k8 TF32 / m16n8k16 bf16 fragment set.
__device__ __forceinline__ void mma_tf32(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void mma_bf16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Four consecutive elements: fp32 as float4, bf16 as 4 x 16 bits (uint2),
// through the read-only path (data constant for the whole launch) or L2
// only (data written earlier in this launch).
template <typename T> struct Quad;
template <> struct Quad<float> { using V = float4; };
template <> struct Quad<__nv_bfloat16> { using V = uint2; };

template <bool COHERENT, typename T>
__device__ __forceinline__ typename Quad<T>::V ldq(const T *p) {
  using V = typename Quad<T>::V;
  if constexpr (COHERENT) return __ldcg(reinterpret_cast<const V *>(p));
  else return __ldg(reinterpret_cast<const V *>(p));
}
template <typename T> __device__ __forceinline__ typename Quad<T>::V zero_quad();
template <> __device__ __forceinline__ float4 zero_quad<float>() { return make_float4(0.f, 0.f, 0.f, 0.f); }
template <> __device__ __forceinline__ uint2 zero_quad<__nv_bfloat16>() { return make_uint2(0u, 0u); }

// All tiles of C assigned to this CTA (tile t to CTA t mod gridDim.x).
// K, lda, ldw multiples of 4; A/W 16-byte (f32) or 8-byte (bf16) aligned.
// `pre()` runs once, by every thread, after the first tile's weights have
// been requested and before A is read (A may be produced by other CTAs up
// to that point).
template <typename T, int KS, int U, bool ACOH, typename Pre>
__device__ __noinline__ void gemm_tiles(const StepGemm g, Pre pre) {
  extern __shared__ __align__(16) float smem[];  // the kernel's dynamic shared memory
  constexpr bool F32 = sizeof(T) == 4;
  using Q = typename Quad<T>::V;
  constexpr int NCG = 8 / KS;                      // column groups of 8
  constexpr int TC = 8 * NCG;                      // tile columns
  constexpr int KW = 16 * U;                       // k per warp and chunk
  constexpr int KC = KW * KS;                      // k per chunk
  constexpr int KC4 = KC / 4;
  constexpr int AST = step_a_stride(F32, KC);      // A row stride in shared memory (32- or 16-bit words)
  uint32_t *Ahi = reinterpret_cast<uint32_t *>(smem);  // f32: TF32 heads [16][AST]
  uint32_t *Alo = Ahi + kTileRows * AST;                // f32: TF32 remainders [16][AST]
  uint16_t *Ab = reinterpret_cast<uint16_t *>(smem);   // bf16: [16][AST]
  float *red = smem + step_a_floats(F32, KC);          // [KS - 1][NCG][32][4]

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int gq = lane >> 2, tq = lane & 3;
  const int cg = warp / KS, ks = warp - cg * KS;
  const T *A = static_cast<const T *>(g.A);
  const T *W = static_cast<const T *>(g.W);
  T *C = static_cast<T *>(g.C);
  const int mt = (g.M + kTileRows - 1) / kTileRows;
  const int ntiles = mt * ((g.N + TC - 1) / TC);
  if ((int)blockIdx.x >= ntiles) pre();

  for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
    const int m0 = (tile % mt) * kTileRows;
    const int n0 = (tile / mt) * TC + 8 * cg;  // this warp's 8 columns
    const int nw = n0 + gq;                    // the W row this lane reads
    constexpr int NACC = F32 ? 6 : 4;
    float da[NACC][4];
#pragma unroll
    for (int a = 0; a < NACC; ++a)
#pragma unroll
      for (int e = 0; e < 4; ++e) da[a][e] = 0.f;

    for (int kc = 0; kc < g.K; kc += KC) {
      Q w[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int k = kc + ks * KW + 16 * u + 4 * tq;
        w[u] = (nw < g.N && k < g.K) ? ldq<false>(W + (int64_t)nw * g.ldw + k) : zero_quad<T>();
      }
      if (tile == (int)blockIdx.x && kc == 0) pre();
      // every A load of the chunk is in flight before the first is stored
      constexpr int NLD = kTileRows * KC4 / kStepThreads;
      Q av[NLD];
#pragma unroll
      for (int q = 0; q < NLD; ++q) {
        const int v = tid + q * kStepThreads;
        const int i = v / KC4, k = kc + 4 * (v - i * KC4);
        av[q] = (m0 + i < g.M && k < g.K) ? ldq<ACOH>(A + (int64_t)(m0 + i) * g.lda + k) : zero_quad<T>();
      }
#pragma unroll
      for (int q = 0; q < NLD; ++q) {
        const int v = tid + q * kStepThreads;
        const int i = v / KC4, k4 = v - i * KC4;
        if constexpr (F32) {
          const float4 x = av[q];
          uint4 hi, lo;
          hi.x = tf32_rna(x.x); lo.x = tf32_rna(x.x - __uint_as_float(hi.x));
          hi.y = tf32_rna(x.y); lo.y = tf32_rna(x.y - __uint_as_float(hi.y));
          hi.z = tf32_rna(x.z); lo.z = tf32_rna(x.z - __uint_as_float(hi.z));
          hi.w = tf32_rna(x.w); lo.w = tf32_rna(x.w - __uint_as_float(hi.w));
          *reinterpret_cast<uint4 *>(Ahi + i * AST + 4 * k4) = hi;
          *reinterpret_cast<uint4 *>(Alo + i * AST + 4 * k4) = lo;
        } else {
          *reinterpret_cast<uint2 *>(Ab + i * AST + 4 * k4) = av[q];
        }
      }
      __syncthreads();
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int kl = ks * KW + 16 * u + 4 * tq;
        if constexpr (F32) {
          const uint4 h0 = *reinterpret_cast<const uint4 *>(Ahi + gq * AST + kl);
          const uint4 h1 = *reinterpret_cast<const uint4 *>(Ahi + (gq + 8) * AST + kl);
          const uint4 l0 = *reinterpret_cast<const uint4 *>(Alo + gq * AST + kl);
          const uint4 l1 = *reinterpret_cast<const uint4 *>(Alo + (gq + 8) * AST + kl);
          const float4 x = w[u];
          const uint32_t wh0 = tf32_rna(x.x), wh1 = tf32_rna(x.y), wh2 = tf32_rna(x.z), wh3 = tf32_rna(x.w);
          const uint32_t wl0 = tf32_rna(x.x - __uint_as_float(wh0)), wl1 = tf32_rna(x.y - __uint_as_float(wh1));
          const uint32_t wl2 = tf32_rna(x.z - __uint_as_float(wh2)), wl3 = tf32_rna(x.w - __uint_as_float(wh3));
          // k step 0: slots t / t + 4 <- k 4t / 4t + 1; step 1: <- 4t + 2 / 4t + 3
          float(&d0)[4] = da[3 * (u & 1) + 0];
          float(&d1)[4] = da[3 * (u & 1) + 1];
          float(&d2)[4] = da[3 * (u & 1) + 2];
          mma_tf32(d0, l0.x, l1.x, l0.y, l1.y, wh0, wh1);
          mma_tf32(d1, h0.x, h1.x, h0.y, h1.y, wl0, wl1);
          mma_tf32(d2, h0.x, h1.x, h0.y, h1.y, wh0, wh1);
          mma_tf32(d0, l0.z, l1.z, l0.w, l1.w, wh2, wh3);
          mma_tf32(d1, h0.z, h1.z, h0.w, h1.w, wl2, wl3);
          mma_tf32(d2, h0.z, h1.z, h0.w, h1.w, wh2, wh3);
        } else {
          // k pairs (2t, 2t + 1) <- (4t, 4t + 1), (2t + 8, 2t + 9) <- (4t + 2, 4t + 3)
          const uint2 r0 = *reinterpret_cast<const uint2 *>(Ab + gq * AST + kl);
          const uint2 r1 = *reinterpret_cast<const uint2 *>(Ab + (gq + 8) * AST + kl);
          const uint2 x = w[u];
          mma_bf16(da[u & 3], r0.x, r1.x, r0.y, r1.y, x.x, x.y);
        }
      }
      __syncthreads();
    }
    // small products first: (lo.hi + hi.lo) of both parities, then hi.hi
    float d[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      if constexpr (F32) d[e] = ((da[0][e] + da[3][e]) + (da[1][e] + da[4][e])) + (da[2][e] + da[5][e]);
      else d[e] = (da[0][e] + da[1][e]) + (da[2][e] + da[3][e]);
    }
    // d: rows m0 + gq (d[0], d[1]) and m0 + gq + 8 (d[2], d[3]), columns n0 + 2tq, n0 + 2tq + 1
    if constexpr (KS > 1) {
      if (ks > 0) {
#pragma unroll
        for (int e = 0; e < 4; ++e) red[(((ks - 1) * NCG + cg) * 32 + lane) * 4 + e] = d[e];
      }
      __syncthreads();
      if (ks == 0) {
#pragma unroll
        for (int s = 1; s < KS; ++s)
#pragma unroll
          for (int e = 0; e < 4; ++e) d[e] += red[(((s - 1) * NCG + cg) * 32 + lane) * 4 + e];
      }
    }
    if (ks == 0) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int m = m0 + gq + (e >> 1) * 8, n = n0 + 2 * tq + (e & 1);
        if (m < g.M && n < g.N) st_out(C + (int64_t)m * g.ldc + n, d[e]);
      }
    }
  }
}

// ---------------------------------------------------------------------------
// L2 prefetch and grid barriers
// ---------------------------------------------------------------------------

__device__ __forceinline__ void prefetch_l2(const void *p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// The ranges are cut into 4 KB chunks (chunk prefix sums from the host);
// chunk c is issued by thread c / gridDim.x of CTA c % gridDim.x, so every
// SM's copy engine gets a few.  Starts and sizes are multiples of 16 bytes.
__device__ __forceinline__ void prefetch_ranges(const StepParams &sp) {
  const int c = threadIdx.x * gridDim.x + blockIdx.x;
  if (c >= sp.pf_first[sp.n_prefetch]) return;
  int r = 0;
  while (c >= sp.pf_first[r + 1]) ++r;
  const int64_t off = (int64_t)(c - sp.pf_first[r]) * kPrefetchChunk;
  const int64_t left = sp.pf_bytes[r] - off;
  prefetch_l2(static_cast<const char *>(sp.pf_ptr[r]) + off, left < kPrefetchChunk ? (uint32_t)left : kPrefetchChunk);
}

__device__ __forceinline__ unsigned ld_relaxed(const unsigned *p) {
  unsigned v;
  asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void red_release_add(unsigned *p, unsigned v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void fence_acq_rel_gpu() { asm volatile("fence.acq_rel.gpu;" ::: "memory"); }

// Grid barriers.  The workspace holds a base word and one arrival counter
// (on its own 128-byte line); neither is ever reset.  A CTA arrives by
// adding 1 to the counter (release), and barrier j of a launch completes
// when the counter reaches base + j * grid (u32 arithmetic, compared through
// the signed difference), so a wait can end late but never early; the
// relaxed polls are followed by an acquire fence, so every write made before
// any CTA's arrival is visible afterwards.  After the last barrier CTA 0
// advances the base by 2 * grid for the next launch on the workspace (every
// CTA reads it before arriving).  A wait gives up after a bounded spin and
// records M3_DEVERR_TIMEOUT; the counter then no longer matches the base,
// later launches time out as well (never pass early), and the workspace has
// to be zeroed again.
__device__ bool grid_barrier(unsigned *ws, unsigned target, int *s_flag) {
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned *ctr = ws + kStepBarStride;
    red_release_add(ctr, 1u);
    int ok = 0;
    for (long long i = 0; i < kSpinLimit; ++i) {
      if ((int)(ld_relaxed(ctr) - target) >= 0) {
        ok = 1;
        break;
      }
    }
    fence_acq_rel_gpu();
    if (!ok) atomicOr(&g_device_error, M3_DEVERR_TIMEOUT);
    *s_flag = ok;
  }
  __syncthreads();
  return *s_flag != 0;
}

template <typename T, bool ACOH, typename Pre>
__device__ __forceinline__ void gemm_phase(int cfg, const StepGemm &g, Pre pre) {
  static_assert(kStepGemmCfgs == 5, "one case per configuration");
  switch (cfg) {
    case 0: gemm_tiles<T, kCfgKS[0], kCfgU[0], ACOH>(g, pre); break;
    case 1: gemm_tiles<T, kCfgKS[1], kCfgU[1], ACOH>(g, pre); break;
    case 2: gemm_tiles<T, kCfgKS[2], kCfgU[2], ACOH>(g, pre); break;
    case 3: gemm_tiles<T, kCfgKS[3], kCfgU[3], ACOH>(g, pre); break;
    default: gemm_tiles<T, kCfgKS[4], kCfgU[4], ACOH>(g, pre); break;
  }
}

struct NoPre {
  __device__ void operator()() const {}
};

// Grid barrier `j` as a pre() hook: waits once, records the outcome.
struct BarrierPre {
  unsigned *bar;
  unsigned target;
  int *s_flag;
  bool *ok;
  __device__ void operator()() const { *ok = grid_barrier(bar, target, s_flag) && *ok; }
};

// ---------------------------------------------------------------------------
// the step kernel
// ---------------------------------------------------------------------------

template <int BD, int R, typename T, int KP>
__global__ void __launch_bounds__(kStepThreads, 2) mimo_step_kernel(const StepParams sp) {
  extern __shared__ __align__(16) float smem[];
  __shared__ int s_flag;
  const KParams &p = sp.kp;
  unsigned base = 0;
  if (threadIdx.x == 0) base = ld_relaxed(sp.bar);

  prefetch_ranges(sp);

  gemm_phase<T, false>(sp.cfg_in, sp.g_in, NoPre{});

  // barrier 1 inside the first item, once its parameters and carried state
  // are in flight (a CTA without items waits after the loop)
  bool ok = true, waited = false;
  const BarrierPre bar1{sp.bar, base + gridDim.x, &s_flag, &ok};
  const int ngrp = p.H / kRowWarps;
  for (int item = blockIdx.x; item < sp.n_items; item += gridDim.x) {
    const int grp = item % ngrp;
    const int b0 = (item / ngrp) * sp.rows_per_item;
    const int b1 = min(p.B, b0 + sp.rows_per_item);
    row::mimo_row_block<BD, R, T, KP, true, true>(p, grp, b0, b1, smem, [&] {
      if (!waited) bar1();
      waited = true;
    });
    __syncthreads();  // the next item reuses the shared work blocks
  }
  if (!waited) bar1();

  // barrier 2 inside the first out_proj tile, once its weights are in flight
  gemm_phase<T, true>(sp.cfg_out, sp.g_out, BarrierPre{sp.bar, base + 2 * gridDim.x, &s_flag, &ok});
  if (blockIdx.x == 0 && threadIdx.x == 0) sp.bar[0] = base + 2 * gridDim.x;
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------

int num_sms_current() {
  static int cached[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (cached[dev] == 0) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    cached[dev] = n > 0 ? n : 148;
  }
  return cached[dev];
}

size_t step_smem_bytes(int R, int BD, int A, bool f32) {
  int f = 2 * row_block_floats(R, BD, A);
  for (int c = 0; c < kStepGemmCfgs; ++c) {
    const int g = step_gemm_smem_floats(f32, kCfgKS[c], kCfgU[c]);
    f = g > f ? g : f;
  }
  return (size_t)f * sizeof(float);
}

template <int BD, int R, typename T, int KP>
cudaError_t launch_step_t(StepParams &sp, cudaStream_t stream) {
  auto kern = mimo_step_kernel<BD, R, T, KP>;
  const size_t smem = step_smem_bytes(R, BD, sp.kp.A, sizeof(T) == 4);
  static int attr_dev[64] = {0};  // 1 + device once the attribute is set
  static int per_sm_dev[64] = {0};
  static size_t smem_dev[64] = {0};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (attr_dev[dev] == 0) {
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 96 * 1024);
    if (e != cudaSuccess) return e;
    attr_dev[dev] = 1;
  }
  if (smem_dev[dev] != smem || per_sm_dev[dev] == 0) {
    int per_sm = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kStepThreads, smem);
    if (e != cudaSuccess) return e;
    if (per_sm < 1) return cudaErrorInvalidConfiguration;
    per_sm_dev[dev] = per_sm > 2 ? 2 : per_sm;
    smem_dev[dev] = smem;
  }
  const int grid = num_sms_current() * per_sm_dev[dev];

  // phase-2 work items: (head group, run of rows), about one per CTA
  const int ngrp = sp.kp.H / kRowWarps;
  const int64_t rows_total = (int64_t)sp.kp.B * ngrp;
  int rows = (int)((rows_total + grid - 1) / grid);
  if (rows < 1) rows = 1;
  sp.rows_per_item = rows;
  sp.n_items = ngrp * ((sp.kp.B + rows - 1) / rows);
  sp.cfg_in = step_gemm_cfg(sp.g_in.M, sp.g_in.N, sp.g_in.K, grid);
  sp.cfg_out = step_gemm_cfg(sp.g_out.M, sp.g_out.N, sp.g_out.K, grid);

  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3(kStepThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, kern, sp);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

template <int BD, int R, typename T>
cudaError_t launch_step_p(StepParams &sp, cudaStream_t stream) {
  if (sp.kp.P <= 32) return launch_step_t<BD, R, T, 1>(sp, stream);
  if (sp.kp.P <= 64) return launch_step_t<BD, R, T, 2>(sp, stream);
  return launch_step_t<BD, R, T, 4>(sp, stream);
}

template <int BD, typename T>
cudaError_t launch_step_r(StepParams &sp, cudaStream_t stream) {
  switch (sp.kp.R) {
    case 1: return launch_step_p<BD, 1, T>(sp, stream);
    case 2: return launch_step_p<BD, 2, T>(sp, stream);
    case 4: return launch_step_p<BD, 4, T>(sp, stream);
    case 8: return launch_step_p<BD, 8, T>(sp, stream);
    default: return cudaErrorInvalidValue;
  }
}

// d_state <= 32 runs the 32-wide instantiation (the row code masks columns
// >= d_state).
template <typename T>
cudaError_t launch_step_d(StepParams &sp, cudaStream_t stream) {
  if (sp.kp.D <= 32) return launch_step_r<32, T>(sp, stream);
  if (sp.kp.D <= 64) return launch_step_r<64, T>(sp, stream);
  return launch_step_r<128, T>(sp, stream);
}

}  // namespace
}  // namespace m3
