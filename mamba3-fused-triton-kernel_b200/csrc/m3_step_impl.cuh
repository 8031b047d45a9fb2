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
#include "m3_siso_tile.cuh"
#include "m3_step.cuh"

namespace m3 {

namespace {

using row::kRowWarps;
using row::row_block_floats;

constexpr int kStepThreads = kRowWarps * 32;
constexpr int kTileRows = kStepTileRows;
constexpr int kPrefetchChunk = 4096;


// ---------------------------------------------------------------------------
// loads
// ---------------------------------------------------------------------------

__device__ __forceinline__ float4 bf16x4_to_f4(uint2 t) {
  const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&t.x));
  const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&t.y));
  return make_float4(a.x, a.y, b.x, b.y);
}
// Four consecutive elements through the read-only path (data constant for
// the whole launch) or L2 only (data written earlier in this launch).
template <bool COHERENT>
__device__ __forceinline__ float4 ld4(const float *p) {
  if constexpr (COHERENT) return __ldcg(reinterpret_cast<const float4 *>(p));
  else return __ldg(reinterpret_cast<const float4 *>(p));
}
template <bool COHERENT>
__device__ __forceinline__ float4 ld4(const __nv_bfloat16 *p) {
  if constexpr (COHERENT) return bf16x4_to_f4(__ldcg(reinterpret_cast<const uint2 *>(p)));
  else return bf16x4_to_f4(__ldg(reinterpret_cast<const uint2 *>(p)));
}

__device__ __forceinline__ void st_out(float *p, float v) { *p = v; }
__device__ __forceinline__ void st_out(__nv_bfloat16 *p, float v) { *p = __float2bfloat16_rn(v); }

// ---------------------------------------------------------------------------
// projection tiles
// ---------------------------------------------------------------------------

// Sum each of the 32 values over the 8 lanes of each aligned lane octet
// (offsets 4, 2, 1, halving exchanges); afterwards the lane at position q
// of its octet holds the totals of values 4q .. 4q + 3 in v[0 .. 3].
__device__ __forceinline__ void octet_transpose_sum(float (&v)[32]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int lvl = 0; lvl < 3; ++lvl) {
    const int off = 4 >> lvl;
    const int half = 16 >> lvl;
    const bool upper = (lane & off) != 0;
#pragma unroll
    for (int q = 0; q < half; ++q) {
      const float send = upper ? v[q] : v[q + half];
      const float keep = upper ? v[q + half] : v[q];
      v[q] = keep + __shfl_xor_sync(kFullMask, send, off);
    }
  }
}

// All tiles of C[M, N] = A[M, K] W[N, K]^T assigned to this CTA (tile t to
// CTA t mod gridDim.x).  A CTA computes 16 rows x (64 / KS) columns: warp w
// covers the 8 columns n0 + 8 (w / KS) over K slice w % KS of every chunk
// (KW k per warp and chunk).  Lane (p = lane / 8, q = lane % 8) holds the
// weights of columns 2p, 2p + 1 for k = 4q + 32t in registers, reads the
// chunk's A rows from shared memory (lanes with the same q read the same
// address: a broadcast) and accumulates 16 rows x 2 columns; one 3-level
// transpose-sum over each lane octet finishes the 32 sums, and the KS
// slices are added in slice order through shared memory.  The summation
// order is fixed by (KS, KW), so results are deterministic.  K, lda, ldw
// multiples of 4; A/W 16-byte (f32) or 8-byte (bf16) aligned.  `pre()` runs
// once, by every thread, after the first tile's weights have been
// requested and before A is read (A may be produced by other CTAs up to
// that point).
template <typename T, int KS, int KW, bool ACOH, typename Pre>
__device__ __noinline__ void gemm_tiles(const StepGemm g, Pre pre) {
  extern __shared__ __align__(16) float smem[];  // the kernel's dynamic shared memory
  constexpr int NCG = 8 / KS;    // column groups of 8
  constexpr int TC = 8 * NCG;    // tile columns
  constexpr int KC = KW * KS;    // k per chunk
  constexpr int KC4 = KC / 4;
  constexpr int NT = KW / 32;    // float4 of each weight row per lane and chunk
  float4 *As = reinterpret_cast<float4 *>(smem);  // [16][KC / 4]
  float *red = smem + kTileRows * KC;              // [KS - 1][NCG][32][4]

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int cp = lane >> 3, kq = lane & 7;
  const int cg = warp / KS, ks = warp - cg * KS;
  const T *A = static_cast<const T *>(g.A);
  const T *W = static_cast<const T *>(g.W);
  T *C = static_cast<T *>(g.C);
  const int mt = (g.M + kTileRows - 1) / kTileRows;
  const int ntiles = mt * ((g.N + TC - 1) / TC);
  if ((int)blockIdx.x >= ntiles) pre();

  for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
    const int m0 = (tile % mt) * kTileRows;
    const int nc = (tile / mt) * TC + 8 * cg + 2 * cp;  // this lane's first column
    float acc[32];  // acc[j * 16 + i]: row m0 + i, column nc + j
#pragma unroll
    for (int q = 0; q < 32; ++q) acc[q] = 0.f;

    for (int kc = 0; kc < g.K; kc += KC) {
      float4 w[2][NT];
#pragma unroll
      for (int j = 0; j < 2; ++j)
#pragma unroll
        for (int t = 0; t < NT; ++t) {
          const int k = kc + ks * KW + 32 * t + 4 * kq;
          w[j][t] = (nc + j < g.N && k < g.K) ? ld4<false>(W + (int64_t)(nc + j) * g.ldw + k)
                                               : make_float4(0.f, 0.f, 0.f, 0.f);
        }
      if (tile == (int)blockIdx.x && kc == 0) pre();
      // every A load of the chunk is in flight before the first is stored
      constexpr int NLD = kTileRows * KC4 / kStepThreads;
      float4 av[NLD];
#pragma unroll
      for (int q = 0; q < NLD; ++q) {
        const int v = tid + q * kStepThreads;
        const int i = v / KC4, k = kc + 4 * (v - i * KC4);
        av[q] = (m0 + i < g.M && k < g.K) ? ld4<ACOH>(A + (int64_t)(m0 + i) * g.lda + k)
                                           : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int q = 0; q < NLD; ++q) As[tid + q * kStepThreads] = av[q];
      __syncthreads();
#pragma unroll
      for (int i = 0; i < kTileRows; ++i) {
#pragma unroll
        for (int t = 0; t < NT; ++t) {
          const float4 a = As[i * KC4 + (ks * KW + 32 * t) / 4 + kq];
#pragma unroll
          for (int j = 0; j < 2; ++j) {
            float &c = acc[j * 16 + i];
            c = fmaf(a.x, w[j][t].x, c);
            c = fmaf(a.y, w[j][t].y, c);
            c = fmaf(a.z, w[j][t].z, c);
            c = fmaf(a.w, w[j][t].w, c);
          }
        }
      }
      __syncthreads();
    }
    octet_transpose_sum(acc);  // lane (p, q): column nc + (q >> 2), rows 4 (q & 3) + {0 .. 3}
    if constexpr (KS > 1) {
      if (ks > 0) {
#pragma unroll
        for (int e = 0; e < 4; ++e) red[(((ks - 1) * NCG + cg) * 32 + lane) * 4 + e] = acc[e];
      }
      __syncthreads();
      if (ks == 0) {
#pragma unroll
        for (int s2 = 1; s2 < KS; ++s2)
#pragma unroll
          for (int e = 0; e < 4; ++e) acc[e] += red[(((s2 - 1) * NCG + cg) * 32 + lane) * 4 + e];
      }
    }
    if (ks == 0) {
      const int n = nc + (kq >> 2);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int m = m0 + 4 * (kq & 3) + e;
        if (m < g.M && n < g.N) st_out(C + (int64_t)m * g.ldc + n, acc[e]);
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
  static_assert(kStepGemmCfgs == 4, "one case per configuration");
  switch (cfg) {
    case 0: gemm_tiles<T, kCfgKS[0], kCfgKW[0], ACOH>(g, pre); break;
    case 1: gemm_tiles<T, kCfgKS[1], kCfgKW[1], ACOH>(g, pre); break;
    case 2: gemm_tiles<T, kCfgKS[2], kCfgKW[2], ACOH>(g, pre); break;
    default: gemm_tiles<T, kCfgKS[3], kCfgKW[3], ACOH>(g, pre); break;
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
// the SISO step kernel
// ---------------------------------------------------------------------------

// The SISO update of one (batch row, head) tile, whose parameters are in q:
// state rows of S lanes with FPL float4 columns each (SisoShape), h and Bx
// read from L2 (prefetched in phase 0) and written back, y_p = sum_d
// C[d] h[p, d] + D x_p gated by silu(z_p) -- the streamed SISO kernel's
// arithmetic, operation for operation (src/kernels/utils.py:73-102).
template <int BD>
__device__ void siso_tile_update(const KParams &p, const ParBlock &q, int b, int hh, int t) {
  using Sh = SisoShape<BD>;
  constexpr int S = Sh::S, FPL = Sh::FPL, RPW = Sh::RPW;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int j = lane % S, slot = warp * RPW + lane / S, nslots = (int)(blockDim.x / 32) * RPW;
  const int P = p.P, G = p.D / 4;
  const Coef cf = {q.sS[kDecay], q.sS[kDT], q.sS[kOmt], q.sS[kHtr]};
  const float dskip = q.sS[kDskip];
  float *hg = p.h + (size_t)t * P * p.D;
  float *bg = p.bx + (size_t)t * P * p.D;
  const int64_t ybase = (int64_t)b * p.y_sb + (int64_t)hh * p.y_sh;
  for (int rb = 0; rb < P; rb += nslots) {
    const int row = rb + slot;
    const bool rok = row < P;
    const float xp = rok ? q.sX[row] : 0.f;
    float part = 0.f;
#pragma unroll
    for (int f = 0; f < FPL; ++f) {
      const int col = j + S * f;
      if (rok && col < G) {
        const int o = row * G + col;
        const float4 ho = ld_state4(hg + (size_t)o * 4);
        const float4 bo = ld_state4(bg + (size_t)o * 4);
        const float4 Bq = reinterpret_cast<const float4 *>(q.sB)[col];
        const float4 Cq = reinterpret_cast<const float4 *>(q.sC)[col];
        float4 bn, hn;
        bn.x = xp * Bq.x; bn.y = xp * Bq.y; bn.z = xp * Bq.z; bn.w = xp * Bq.w;
        hn.x = trap_update(cf, bn.x, bo.x, ho.x);
        hn.y = trap_update(cf, bn.y, bo.y, ho.y);
        hn.z = trap_update(cf, bn.z, bo.z, ho.z);
        hn.w = trap_update(cf, bn.w, bo.w, ho.w);
        part += Cq.x * hn.x;
        part += Cq.y * hn.y;
        part += Cq.z * hn.z;
        part += Cq.w * hn.w;
        st_state4(hg + (size_t)o * 4, hn);
        st_state4(bg + (size_t)o * 4, bn);
      }
    }
    part = group_sum<S>(part);
    if (j == 0 && rok) st_any(p.y, ybase + (int64_t)row * p.y_sp, (part + dskip * xp) * q.sG[row], p.y_dt);
  }
}

// The single-launch step of a SISO layer: phase 1 in_proj, grid barrier,
// phase 2 one (batch row, head) tile per work item (its parameters, then its
// P x D state), grid barrier, phase 3 out_proj.  A tile is never split over
// CTAs: its accumulated angles are read and rewritten by the one CTA.
template <int BD, typename T>
__global__ void __launch_bounds__(kStepThreads, 2) siso_step_kernel(const StepParams sp) {
  extern __shared__ __align__(16) float smem[];
  __shared__ int s_flag;
  const KParams &p = sp.kp;
  unsigned base = 0;
  if (threadIdx.x == 0) base = ld_relaxed(sp.bar);

  prefetch_ranges(sp);

  gemm_phase<T, false>(sp.cfg_in, sp.g_in, NoPre{});

  bool ok = grid_barrier(sp.bar, base + gridDim.x, &s_flag);
  const ParBlock q = par_block<BD>(reinterpret_cast<unsigned char *>(smem), p);
  for (int i = threadIdx.x; i < p.H; i += blockDim.x) {
    q.dtb[i] = ld_any(p.dt_bias, i, p.par_dt);
    q.dsk[i] = ld_any(p.Dp, i, p.par_dt);
  }
  for (int i = threadIdx.x; i < p.D; i += blockDim.x) {
    q.wB[i] = ld_any(p.wB, i, p.par_dt);
    q.wC[i] = ld_any(p.wC, i, p.par_dt);
  }
  __syncthreads();
  const int ntiles = p.B * p.H;
  for (int t = blockIdx.x; t < ntiles; t += gridDim.x) {
    const int b = t / p.H, hh = t - b * p.H;
    tile_params_global<BD, true>(p, q, b, hh, t);
    __syncthreads();
    siso_tile_update<BD>(p, q, b, hh, t);
    __syncthreads();  // the next tile reuses the parameter block
  }

  // barrier 2 inside the first out_proj tile, once its weights are in flight
  gemm_phase<T, true>(sp.cfg_out, sp.g_out, BarrierPre{sp.bar, base + 2 * gridDim.x, &s_flag, &ok});
  if (blockIdx.x == 0 && threadIdx.x == 0) sp.bar[0] = base + 2 * gridDim.x;
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------

int num_sms_current() { return sm_count_current(); }

size_t step_smem_bytes(int R, int BD, int A) {
  int f = 2 * row_block_floats(R, BD, A);
  for (int c = 0; c < kStepGemmCfgs; ++c) {
    const int g = step_gemm_smem_floats(kCfgKS[c], kCfgKW[c]);
    f = g > f ? g : f;
  }
  return (size_t)f * sizeof(float);
}

template <int BD, int R, typename T, int KP>
cudaError_t launch_step_t(StepParams &sp, cudaStream_t stream) {
  auto kern = mimo_step_kernel<BD, R, T, KP>;
  const size_t smem = step_smem_bytes(R, BD, sp.kp.A);
  static LaunchCache cache;
  cudaError_t e = ensure_smem_optin(cache, kern, 96 * 1024);
  if (e != cudaSuccess) return e;
  int per_sm = 0;
  e = occupancy_per_sm(cache, kern, kStepThreads, smem, &per_sm);
  if (e != cudaSuccess) return e;
  if (per_sm < 1) return cudaErrorInvalidConfiguration;
  if (per_sm > 2) per_sm = 2;
  const int grid = num_sms_current() * per_sm;

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

size_t siso_step_smem_bytes(int BD, int P, int H) {
  int f = 2 * BD + 2 * P + kNScalar + 2 * BD + 2 * H;
  for (int c = 0; c < kStepGemmCfgs; ++c) {
    const int g = step_gemm_smem_floats(kCfgKS[c], kCfgKW[c]);
    f = g > f ? g : f;
  }
  return (size_t)f * sizeof(float);
}

template <int BD, typename T>
cudaError_t launch_siso_step_t(StepParams &sp, cudaStream_t stream) {
  auto kern = siso_step_kernel<BD, T>;
  const size_t smem = siso_step_smem_bytes(BD, sp.kp.P, sp.kp.H);
  if (smem > 200 * 1024) return cudaErrorInvalidValue;
  static LaunchCache cache;
  cudaError_t e = ensure_smem_optin(cache, kern, 200 * 1024);
  if (e != cudaSuccess) return e;
  int per_sm = 0;
  e = occupancy_per_sm(cache, kern, kStepThreads, smem, &per_sm);
  if (e != cudaSuccess) return e;
  if (per_sm < 1) return cudaErrorInvalidConfiguration;
  if (per_sm > 2) per_sm = 2;
  const int grid = num_sms_current() * per_sm;
  sp.rows_per_item = 1;
  sp.n_items = sp.kp.B * sp.kp.H;
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

template <typename T>
cudaError_t launch_siso_step_d(StepParams &sp, cudaStream_t stream) {
  if (sp.kp.D <= 32) return launch_siso_step_t<32, T>(sp, stream);
  if (sp.kp.D <= 64) return launch_siso_step_t<64, T>(sp, stream);
  if (sp.kp.D <= 128) return launch_siso_step_t<128, T>(sp, stream);
  return launch_siso_step_t<256, T>(sp, stream);
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
