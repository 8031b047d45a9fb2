// MIMO decode kernels.
//
// mimo_row_kernel (full-step fused).  One CTA owns 8 heads (one warp per
// head) and a chunk of consecutive batch rows; each thread issues all of a
// row's independent loads before using any of them, and four CTAs share an
// SM so that their rows hide each other's latency.  Per row:
//   A (all threads)  RMSNorm of the R B-rows and R C-rows (shared by every
//                    head of the CTA), the head scalars DT / exp(A DT) /
//                    trap (lane = head), and the accumulated RoPE angles
//                    (one sincosf per thread and angle, written back to
//                    angle_state), into a double-buffered shared block, so
//                    one barrier per row suffices;
//   B (warp / head)  x_r = mimo_x x (one transpose-reduction for all ranks);
//                    Bx = RoPE(sum_r x_r (Bn_r + bias_r)) -- RoPE is linear,
//                    so rotating the rank sum equals summing the rotated
//                    ranks (src/kernels/utils.py:133 with B_proj from
//                    src/models/mamba3.py:330-332); the trapezoidal update;
//                    y_r = <Cn_r + cbias_r, RoPE^-1(h)> (a rotation is
//                    orthogonal: <RoPE(c), h> = <c, RoPE^-1(h)>);
//                    y = sum_r (y_r + D x_r) mimo_o[r] * silu(z).
// Parameters are read through the read-only cache, where a CTA's 8 heads
// stay resident across its rows.
// mimo_decode_kernel (m3_kernels.cuh) serves everything else: the
// state-update-only entry points and shapes the row kernel does not take
// (head counts that are not a multiple of 8, headdim > 128, mixed dtypes).
#include "m3_async.cuh"
#include "m3_kernels.cuh"

namespace m3 {

namespace {

template <typename T> __device__ __forceinline__ float to_f(T v);
template <> __device__ __forceinline__ float to_f<float>(float v) { return v; }
template <> __device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }

// Sum each v[r] over the 32 lanes; every lane ends with all R totals.
// log2(R) halving exchanges (each lane keeps half of its live values and
// trades the other half with its partner), 5 - log2(R) plain butterfly
// steps, then R broadcasts: 5 + 2R - 1 - log2(R) shuffles instead of 5R.
template <int R>
__device__ __forceinline__ void warp_allreduce_ranks(float (&v)[R]) {
  constexpr int LR = R == 1 ? 0 : R == 2 ? 1 : R == 4 ? 2 : 3;
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int i = 0; i < LR; ++i) {
    const int off = 16 >> i;
    const int half = (R >> i) / 2;
    const bool upper = (lane & off) != 0;
#pragma unroll
    for (int q = 0; q < half; ++q) {
      const float send = upper ? v[q] : v[q + half];
      const float keep = upper ? v[q + half] : v[q];
      v[q] = keep + __shfl_xor_sync(kFullMask, send, off);
    }
  }
  float t = v[0];
#pragma unroll
  for (int off = 16 >> LR; off > 0; off >>= 1) t += __shfl_xor_sync(kFullMask, t, off);
  // lane l now holds the total of rank l >> (5 - LR)
#pragma unroll
  for (int r = 0; r < R; ++r) v[r] = __shfl_sync(kFullMask, t, r << (5 - LR));
}

// Loads through the non-coherent (read-only) path: parameters and the
// in_proj output are never written by the kernel.
template <typename T> __device__ __forceinline__ float ldg_f(const T *p);
template <> __device__ __forceinline__ float ldg_f<float>(const float *p) { return __ldg(p); }
template <> __device__ __forceinline__ float ldg_f<__nv_bfloat16>(const __nv_bfloat16 *p) {
  return __bfloat162float(__ldg(p));
}
template <int VW, typename T>
__device__ __forceinline__ void ldg_vec(const T *p, float (&v)[VW]) {
  if constexpr (sizeof(T) == 4) {
    if constexpr (VW == 4) {
      const float4 t = __ldg(reinterpret_cast<const float4 *>(p));
      v[0] = t.x; v[1] = t.y; v[2] = t.z; v[3] = t.w;
    } else {
      const float2 t = __ldg(reinterpret_cast<const float2 *>(p));
      v[0] = t.x; v[1] = t.y;
    }
  } else {
    if constexpr (VW == 4) {
      const uint2 t = __ldg(reinterpret_cast<const uint2 *>(p));
      const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&t.x));
      const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&t.y));
      v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y;
    } else {
      const unsigned t = __ldg(reinterpret_cast<const unsigned *>(p));
      const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&t));
      v[0] = a.x; v[1] = a.y;
    }
  }
}

__device__ __forceinline__ void st_vec_global(float *p, const float (&v)[4]) {
  asm volatile("st.global.v4.f32 [%0], {%1,%2,%3,%4};" ::"l"(p), "f"(v[0]), "f"(v[1]), "f"(v[2]), "f"(v[3])
               : "memory");
}
__device__ __forceinline__ void st_vec_global(float *p, const float (&v)[2]) {
  asm volatile("st.global.v2.f32 [%0], {%1,%2};" ::"l"(p), "f"(v[0]), "f"(v[1]) : "memory");
}

constexpr int kRowWarps = 8;  // heads per CTA of the row kernel

// Everything one thread needs from one batch row, loaded before first use.
template <int BD, int R, int KP>
struct RowRegs {
  static constexpr int VW = MimoShape<BD>::VW, F = MimoShape<BD>::F, KPL = MimoShape<BD>::KPL;
  static constexpr int NRW = (2 * R + kRowWarps - 1) / kRowWarps;  // norm rows per warp
  static constexpr int NA = BD / 64 > 0 ? BD / 64 : 1;             // angles per thread
  float h[F][VW], bx[F][VW];  // this warp's head state
  float x[KP];                // x of this warp's head, lanes over headdim
  float raw[NRW][KPL];        // B/C rows this warp normalizes
  float sc[3];                // warp 0, lane < heads: dd_dt, dd_A, trap_raw of head `lane`
  float ang[NA], araw[NA];    // angle state + increment of this thread's angles
};

// The row kernel: see the file comment.  One CTA = kRowWarps heads x a chunk
// of consecutive batch rows; every warp owns one head.
template <int BD, int R, typename T, int KP>
__global__ void __launch_bounds__(kRowWarps * 32, 4) mimo_row_kernel(const KParams p, const int rows_per_cta) {
  using Sh = MimoShape<BD>;
  using RR = RowRegs<BD, R, KP>;
  constexpr int VW = Sh::VW, F = Sh::F, KPL = Sh::KPL, NPAIR = VW / 2, NRW = RR::NRW, NA = RR::NA;
  using V = typename VecOf<VW>::T;

  // double-buffered per-row work block: normalized rows [2R][BD], head
  // scalars [8][4], cos/sin [8][A][2]
  extern __shared__ __align__(16) float smem[];
  const int A = p.A;
  const int wstride = 2 * R * BD + 4 * kRowWarps + 2 * kRowWarps * A;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int H = p.H, P = p.P, D = p.D;
  const int ngrp = H / kRowWarps;
  const int grp = blockIdx.x % ngrp;
  const int b0 = (blockIdx.x / ngrp) * rows_per_cta;
  const int b1 = min(p.B, b0 + rows_per_cta);
  const int h0 = grp * kRowWarps;
  const int hh = h0 + warp;
  const T *zx = static_cast<const T *>(p.zx);
  const int so = 2 * p.d_inner + 2 * p.d_bc;  // dd_dt[H] dd_A[H] trap[H] angle[A]

  // state and angle state: written by the previous step's kernel (two or
  // more launches back), safe to read before pdl_wait()
  auto load_state = [&](int b, RR &r) {
    const int64_t sbase = ((int64_t)b * H + hh) * D;
#pragma unroll
    for (int f = 0; f < F; ++f) {
      const int col = (lane + 32 * f) * VW;
      if (col < D) {
        ld_vec<VW>(p.h + sbase + col, r.h[f]);
        ld_vec<VW>(p.bx + sbase + col, r.bx[f]);
      }
    }
#pragma unroll
    for (int n = 0; n < NA; ++n) {
      const int i = tid + n * kRowWarps * 32;
      const int w = i / A, a = i - w * A;
      if (w < kRowWarps) r.ang[n] = p.ang[((int64_t)b * H + h0 + w) * A + a];
    }
  };
  // the in_proj row: produced by the preceding kernel, read after pdl_wait()
  auto load_zx = [&](int b, RR &r) {
    const T *row = zx + (int64_t)b * p.zx_sb;
#pragma unroll
    for (int k = 0; k < KP; ++k) {
      const int pp = lane + 32 * k;
      r.x[k] = pp < P ? ldg_f(row + p.d_inner + (int64_t)hh * P + pp) : 0.f;
    }
#pragma unroll
    for (int j = 0; j < NRW; ++j) {
      const int rr = warp + kRowWarps * j;
      const int col0 = 2 * p.d_inner + (rr < R ? 0 : p.d_bc) + (rr % R) * D;
#pragma unroll
      for (int q = 0; q < KPL; ++q) {
        const int d = lane + 32 * q;
        r.raw[j][q] = (rr < 2 * R && d < D) ? ldg_f(row + col0 + d) : 0.f;
      }
    }
    if (warp == 0 && lane < kRowWarps) {
      r.sc[0] = ldg_f(row + so + h0 + lane);
      r.sc[1] = ldg_f(row + so + H + h0 + lane);
      r.sc[2] = ldg_f(row + so + 2 * H + h0 + lane);
    }
#pragma unroll
    for (int n = 0; n < NA; ++n) {
      const int i = tid + n * kRowWarps * 32;
      const int w = i / A, a = i - w * A;
      if (w < kRowWarps) r.araw[n] = ldg_f(row + so + 3 * H + a);
    }
  };

  RR cur;
  if (b0 < b1) load_state(b0, cur);
  pdl_wait();
  pdl_trigger();
  for (int b = b0; b < b1; ++b) {
    if (b != b0) load_state(b, cur);
    load_zx(b, cur);
    const T *row = zx + (int64_t)b * p.zx_sb;
    float *wk = smem + ((b - b0) & 1) * wstride;
    float *nBC = wk, *wsc = wk + 2 * R * BD, *wrot = wsc + 4 * kRowWarps;

    // ---- phase A ----
    // RMSNorm of the 2R B/C rows (src/models/mamba3.py:202-203)
#pragma unroll
    for (int j = 0; j < NRW; ++j) {
      const int rr = warp + kRowWarps * j;
      if (rr < 2 * R) {
        const void *wn = rr < R ? p.wB : p.wC;
        float ss = 0.f;
#pragma unroll
        for (int q = 0; q < KPL; ++q) ss += cur.raw[j][q] * cur.raw[j][q];
        ss = group_sum<32>(ss);
        const float rms = sqrtf(ss / (float)D + kRmsEps);
#pragma unroll
        for (int q = 0; q < KPL; ++q) {
          const int d = lane + 32 * q;
          if (d < D) nBC[rr * BD + d] = cur.raw[j][q] / rms * ldg_f(static_cast<const T *>(wn) + d);
        }
      }
    }
    // head scalars, lane = head (src/models/mamba3.py:196-199)
    if (warp == 0 && lane < kRowWarps) {
      const float dd_A = cur.sc[1];
      float A_val;
      if (p.A_floor > 0.f) {
        // softplus(.) >= 0 > -A_floor for every non-NaN input, so the
        // clamp returns -A_floor; a NaN propagates as in torch.clamp
        A_val = dd_A != dd_A ? dd_A : p.A_floor;
      } else {
        const float sp = softplus_f(dd_A);
        A_val = -(sp > -p.A_floor ? -p.A_floor : sp);
      }
      const float DT = softplus_f(cur.sc[0] + ldg_f(static_cast<const T *>(p.dt_bias) + h0 + lane));
      const float tr = sigmoid_f(cur.sc[2]);
      float *sc = wsc + 4 * lane;
      sc[0] = expf(A_val * DT);
      sc[1] = DT;
      sc[2] = 1.f - tr;
      sc[3] = tr * 0.5f;
    }
    // accumulated angles -> cos/sin, written back (src/models/mamba3.py:326-327)
#pragma unroll
    for (int n = 0; n < NA; ++n) {
      const int i = tid + n * kRowWarps * 32;
      const int w = i / A, a = i - w * A;
      if (w < kRowWarps) {
        const float dd_dt = ldg_f(row + so + h0 + w);  // L1 hit: warp 0 loaded it
        const float DT = softplus_f(dd_dt + ldg_f(static_cast<const T *>(p.dt_bias) + h0 + w));
        const float ang = cur.ang[n] + cur.araw[n] * DT;
        p.ang[((int64_t)b * H + h0 + w) * A + a] = ang;
        float sn, cs;
        sincosf(ang, &sn, &cs);
        wrot[2 * i] = cs;
        wrot[2 * i + 1] = sn;
      }
    }
    __syncthreads();

    // ---- phase B: this warp's head ----
    {
      const float *sc = wsc + 4 * warp;
      const Coef c = {sc[0], sc[1], sc[2], sc[3]};
      const float dskip = ldg_f(static_cast<const T *>(p.Dp) + hh);
      const float *rot = wrot + 2 * warp * A;
      const T *mx = static_cast<const T *>(p.mx) + (int64_t)hh * R * P;
      const T *mo = static_cast<const T *>(p.mo) + (int64_t)hh * R * P;
      const T *bB = static_cast<const T *>(p.bB) + (int64_t)hh * R * D;
      const T *bC = static_cast<const T *>(p.bC) + (int64_t)hh * R * D;

      // x_r = sum_p x_p mimo_x[h, r, p]
      float xr[R];
#pragma unroll
      for (int r = 0; r < R; ++r) xr[r] = 0.f;
#pragma unroll
      for (int k = 0; k < KP; ++k) {
        const int pp = lane + 32 * k;
        if (pp < P) {
#pragma unroll
          for (int r = 0; r < R; ++r) xr[r] += cur.x[k] * ldg_f(mx + r * P + pp);
        }
      }
      warp_allreduce_ranks<R>(xr);

      // Bx, state update, inverse-rotated h for the readout
      float hr[F][VW];
      const int64_t sbase = ((int64_t)b * H + hh) * D;
#pragma unroll
      for (int f = 0; f < F; ++f) {
        const int col = (lane + 32 * f) * VW;
#pragma unroll
        for (int e = 0; e < VW; ++e) hr[f][e] = 0.f;
        if (col < D) {
          float cs[NPAIR], sn[NPAIR];
#pragma unroll
          for (int q = 0; q < NPAIR; ++q) {
            const int i = col / 2 + q;
            const bool on = i < A;
            cs[q] = on ? rot[2 * i] : 1.f;
            sn[q] = on ? rot[2 * i + 1] : 0.f;
          }
          float acc[VW];
#pragma unroll
          for (int e = 0; e < VW; ++e) acc[e] = 0.f;
#pragma unroll
          for (int r = 0; r < R; ++r) {
            const V nv = *reinterpret_cast<const V *>(nBC + r * BD + col);
            float bb[VW];
            ldg_vec<VW>(bB + r * D + col, bb);
            const float *n = reinterpret_cast<const float *>(&nv);
#pragma unroll
            for (int e = 0; e < VW; ++e) acc[e] += xr[r] * (n[e] + bb[e]);
          }
          float bxv[VW], hn[VW];
#pragma unroll
          for (int q = 0; q < NPAIR; ++q) {
            const float x1 = acc[2 * q], x2 = acc[2 * q + 1];
            bxv[2 * q] = x1 * cs[q] - x2 * sn[q];
            bxv[2 * q + 1] = x1 * sn[q] + x2 * cs[q];
          }
#pragma unroll
          for (int e = 0; e < VW; ++e) hn[e] = trap_update(c, bxv[e], cur.bx[f][e], cur.h[f][e]);
          st_vec_global(p.h + sbase + col, hn);
          st_vec_global(p.bx + sbase + col, bxv);
#pragma unroll
          for (int q = 0; q < NPAIR; ++q) {
            const float x1 = hn[2 * q], x2 = hn[2 * q + 1];
            hr[f][2 * q] = x1 * cs[q] + x2 * sn[q];
            hr[f][2 * q + 1] = x2 * cs[q] - x1 * sn[q];
          }
        }
      }

      // y_r = <Cn_r + cbias_r, RoPE^-1(h)> + D x_r
      float yr[R];
#pragma unroll
      for (int r = 0; r < R; ++r) {
        float part = 0.f;
#pragma unroll
        for (int f = 0; f < F; ++f) {
          const int col = (lane + 32 * f) * VW;
          if (col < D) {
            const V nv = *reinterpret_cast<const V *>(nBC + (R + r) * BD + col);
            float cc[VW];
            ldg_vec<VW>(bC + r * D + col, cc);
            const float *n = reinterpret_cast<const float *>(&nv);
#pragma unroll
            for (int e = 0; e < VW; ++e) part += (n[e] + cc[e]) * hr[f][e];
          }
        }
        yr[r] = part;
      }
      warp_allreduce_ranks<R>(yr);
#pragma unroll
      for (int r = 0; r < R; ++r) yr[r] += dskip * xr[r];

      // y_p = sum_r y_r mimo_o[h, r, p], gated by silu(z)
      const int64_t ybase = (int64_t)b * p.y_sb + (int64_t)hh * P;
#pragma unroll
      for (int k = 0; k < KP; ++k) {
        const int pp = lane + 32 * k;
        if (pp < P) {
          float yv = 0.f;
#pragma unroll
          for (int r = 0; r < R; ++r) yv += yr[r] * ldg_f(mo + r * P + pp);
          const float zv = ldg_f(row + (int64_t)hh * P + pp);
          st_any(p.y, ybase + pp, yv * silu_f(zv), p.y_dt);
        }
      }
    }
  }
}

int num_sms() {
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
  auto kern = mimo_row_kernel<BD, R, T, KP>;
  const size_t smem = 2 * (size_t)(2 * R * BD + 4 * kRowWarps + 2 * kRowWarps * kp.A) * sizeof(float);
  static bool attr = false;
  static size_t last_smem = (size_t)-1;
  static int last_per_sm = 1;
  if (!attr) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 96 * 1024);
    if (e != cudaSuccess) return e;
    attr = true;
  }
  if (smem != last_smem) {
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kRowWarps * 32, smem) != cudaSuccess ||
        per_sm < 1)
      per_sm = 1;
    last_smem = smem;
    last_per_sm = per_sm;
  }
  const int ngrp = kp.H / kRowWarps;
  const int slots = num_sms() * last_per_sm;
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
