// The MIMO row algorithm as a device function, shared by the standalone
// full-step kernel (m3_mimo.cu) and the single-launch decode step
// (m3_step.cu).  One CTA = kRowWarps heads x a run of batch rows; per row:
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
#pragma once

#include "m3_kernels.cuh"

namespace m3 {
namespace row {

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

// Floats of one row's shared work block (normalized B/C rows, head scalars,
// cos/sin of the angles); the row code double-buffers it.
__host__ __device__ constexpr int row_block_floats(int R, int BD, int A) {
  return 2 * R * BD + 4 * kRowWarps + 2 * kRowWarps * A;
}

// In_proj-output loads: read-only path, or L2-only when the same kernel
// wrote the data.
template <bool COHERENT, typename T> __device__ __forceinline__ float ldz(const T *p);
template <> __device__ __forceinline__ float ldz<false, float>(const float *p) { return __ldg(p); }
template <> __device__ __forceinline__ float ldz<false, __nv_bfloat16>(const __nv_bfloat16 *p) {
  return __bfloat162float(__ldg(p));
}
template <> __device__ __forceinline__ float ldz<true, float>(const float *p) { return __ldcg(p); }
template <> __device__ __forceinline__ float ldz<true, __nv_bfloat16>(const __nv_bfloat16 *p) {
  return __bfloat162float(__ldcg(p));
}

// Everything one thread needs from one batch row, loaded before first use
// (z only with ZL).
template <int BD, int R, int KP, bool ZL = false>
struct RowRegs {
  static constexpr int VW = MimoShape<BD>::VW, F = MimoShape<BD>::F, KPL = MimoShape<BD>::KPL;
  static constexpr int NRW = (2 * R + kRowWarps - 1) / kRowWarps;  // norm rows per warp
  static constexpr int NA = BD / 64 > 0 ? BD / 64 : 1;             // angles per thread
  float h[F][VW], bx[F][VW];  // this warp's head state
  float x[KP], z[ZL ? KP : 1];  // x and z of this warp's head, lanes over headdim
  float raw[NRW][KPL];        // B/C rows this warp normalizes
  float sc[3];                // warp 0, lane < heads: dd_dt, dd_A, trap_raw of head `lane`
  float ang[NA], araw[NA];    // angle state + increment of this thread's angles
};

// The per-head parameters a thread uses for every row.  With LOAD (callers
// with registers to spare) they are loaded once before the first row: the
// scalars and norm weights always, the phase-B vectors (mimo_x, mimo_o, B/C
// biases) when they fit (PRE).  Everything not held here is read through
// the read-only cache where it is used.
template <int BD, int R, int KP, bool LOAD>
struct HeadRegs {
  static constexpr int VW = MimoShape<BD>::VW, F = MimoShape<BD>::F, KPL = MimoShape<BD>::KPL;
  static constexpr int NRW = RowRegs<BD, R, KP>::NRW, NA = RowRegs<BD, R, KP>::NA;
  static constexpr bool PRE = LOAD && 2 * R * KP + 2 * R * F * VW <= 64;
  static constexpr int RP = PRE ? R : 1, KPP = PRE ? KP : 1, FP = PRE ? F : 1, VWP = PRE ? VW : 1;
  float mx[RP][KPP], mo[RP][KPP];        // mimo_x / mimo_o of this warp's head, lanes over headdim
  float bb[RP][FP][VWP], bc[RP][FP][VWP];  // B / C bias of this warp's head, lanes over d_state
  float dskip;                           // D of this warp's head
  float wn[NRW][KPL];                    // norm weights of the B/C rows this warp normalizes
  float dtb_head;                        // warp 0, lane < heads: dt_bias of head h0 + lane
  float dtb_ang[NA];                     // dt_bias of the head of each of this thread's angles
};

// One CTA's share of the row algorithm: the kRowWarps heads of head group
// `grp` for batch rows [b0, b1); every warp owns one head.  `smem` holds
// 2 * row_block_floats(R, BD, A) floats.  `pre()` runs once, after the first
// row's carried state has been requested and before anything produced by
// the preceding step of the pipeline is read.  ZX_COHERENT selects L2-only
// loads for an in_proj output written earlier by the same kernel (the
// read-only path may only serve data that is constant for the whole launch).
// PRELOAD holds the per-head parameters in registers (HeadRegs).
template <int BD, int R, typename T, int KP, bool ZX_COHERENT, bool PRELOAD, typename Pre>
__device__ __forceinline__ void mimo_row_block(const KParams &p, const int grp, const int b0, const int b1,
                                               float *smem, Pre &&pre) {
  using Sh = MimoShape<BD>;
  using RR = RowRegs<BD, R, KP, PRELOAD>;
  constexpr int VW = Sh::VW, F = Sh::F, KPL = Sh::KPL, NPAIR = VW / 2, NRW = RR::NRW, NA = RR::NA;
  using V = typename VecOf<VW>::T;

  // double-buffered per-row work block: normalized rows [2R][BD], head
  // scalars [8][4], cos/sin [8][A][2]
  const int A = p.A;
  const int wstride = row_block_floats(R, BD, A);

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int H = p.H, P = p.P, D = p.D;
  const int h0 = grp * kRowWarps;
  const int hh = h0 + warp;
  const T *zx = static_cast<const T *>(p.zx);
  const int so = 2 * p.d_inner + 2 * p.d_bc;  // dd_dt[H] dd_A[H] trap[H] angle[A]

  // state and angle state: written by the previous step's kernel (two or
  // more launches back), safe to read before pre()
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
  // the in_proj row: produced by the preceding step, read after pre()
  auto load_zx = [&](int b, RR &r) {
    const T *row = zx + (int64_t)b * p.zx_sb;
#pragma unroll
    for (int k = 0; k < KP; ++k) {
      const int pp = lane + 32 * k;
      r.x[k] = pp < P ? ldz<ZX_COHERENT>(row + p.d_inner + (int64_t)hh * P + pp) : 0.f;
      if constexpr (PRELOAD) r.z[k] = pp < P ? ldz<ZX_COHERENT>(row + (int64_t)hh * P + pp) : 0.f;
    }
#pragma unroll
    for (int j = 0; j < NRW; ++j) {
      const int rr = warp + kRowWarps * j;
      const int col0 = 2 * p.d_inner + (rr < R ? 0 : p.d_bc) + (rr % R) * D;
#pragma unroll
      for (int q = 0; q < KPL; ++q) {
        const int d = lane + 32 * q;
        r.raw[j][q] = (rr < 2 * R && d < D) ? ldz<ZX_COHERENT>(row + col0 + d) : 0.f;
      }
    }
    if (warp == 0 && lane < kRowWarps) {
      r.sc[0] = ldz<ZX_COHERENT>(row + so + h0 + lane);
      r.sc[1] = ldz<ZX_COHERENT>(row + so + H + h0 + lane);
      r.sc[2] = ldz<ZX_COHERENT>(row + so + 2 * H + h0 + lane);
    }
#pragma unroll
    for (int n = 0; n < NA; ++n) {
      const int i = tid + n * kRowWarps * 32;
      const int w = i / A, a = i - w * A;
      if (w < kRowWarps) r.araw[n] = ldz<ZX_COHERENT>(row + so + 3 * H + a);
    }
  };

  // the per-head parameters: constant for the whole launch
  using HR = HeadRegs<BD, R, KP, PRELOAD>;
  HR hp;
  if constexpr (PRELOAD) {
    const T *mxp = static_cast<const T *>(p.mx) + (int64_t)hh * R * P;
    const T *mop = static_cast<const T *>(p.mo) + (int64_t)hh * R * P;
    const T *bBp = static_cast<const T *>(p.bB) + (int64_t)hh * R * D;
    const T *bCp = static_cast<const T *>(p.bC) + (int64_t)hh * R * D;
    if constexpr (HR::PRE) {
#pragma unroll
      for (int r = 0; r < R; ++r) {
#pragma unroll
        for (int k = 0; k < KP; ++k) {
          const int pp = lane + 32 * k;
          hp.mx[r][k] = pp < P ? ldg_f(mxp + r * P + pp) : 0.f;
          hp.mo[r][k] = pp < P ? ldg_f(mop + r * P + pp) : 0.f;
        }
#pragma unroll
        for (int f = 0; f < F; ++f) {
          const int col = (lane + 32 * f) * VW;
          if (col < D) {
            ldg_vec<VW>(bBp + r * D + col, hp.bb[r][f]);
            ldg_vec<VW>(bCp + r * D + col, hp.bc[r][f]);
          } else {
#pragma unroll
            for (int e = 0; e < VW; ++e) hp.bb[r][f][e] = hp.bc[r][f][e] = 0.f;
          }
        }
      }
    }
    hp.dskip = ldg_f(static_cast<const T *>(p.Dp) + hh);
#pragma unroll
    for (int j = 0; j < NRW; ++j) {
      const int rr = warp + kRowWarps * j;
      const T *wn = static_cast<const T *>(rr < R ? p.wB : p.wC);
#pragma unroll
      for (int q = 0; q < KPL; ++q) {
        const int d = lane + 32 * q;
        hp.wn[j][q] = (rr < 2 * R && d < D) ? ldg_f(wn + d) : 0.f;
      }
    }
    hp.dtb_head = (warp == 0 && lane < kRowWarps) ? ldg_f(static_cast<const T *>(p.dt_bias) + h0 + lane) : 0.f;
#pragma unroll
    for (int n = 0; n < NA; ++n) {
      const int w = (tid + n * kRowWarps * 32) / A;
      hp.dtb_ang[n] = w < kRowWarps ? ldg_f(static_cast<const T *>(p.dt_bias) + h0 + w) : 0.f;
    }
  }

  RR cur;
  if (b0 < b1) load_state(b0, cur);
  pre();
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
        float ss = 0.f;
#pragma unroll
        for (int q = 0; q < KPL; ++q) ss += cur.raw[j][q] * cur.raw[j][q];
        ss = group_sum<32>(ss);
        const float rms = sqrtf(ss / (float)D + kRmsEps);
#pragma unroll
        for (int q = 0; q < KPL; ++q) {
          const int d = lane + 32 * q;
          if (d < D) {
            float w;
            if constexpr (PRELOAD) w = hp.wn[j][q];
            else w = ldg_f(static_cast<const T *>(rr < R ? p.wB : p.wC) + d);
            nBC[rr * BD + d] = cur.raw[j][q] / rms * w;
          }
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
      float dtb;
      if constexpr (PRELOAD) dtb = hp.dtb_head;
      else dtb = ldg_f(static_cast<const T *>(p.dt_bias) + h0 + lane);
      const float DT = softplus_f(cur.sc[0] + dtb);
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
        const float dd_dt = ldz<ZX_COHERENT>(row + so + h0 + w);  // cache hit: warp 0 loaded it
        float dtb;
        if constexpr (PRELOAD) dtb = hp.dtb_ang[n];
        else dtb = ldg_f(static_cast<const T *>(p.dt_bias) + h0 + w);
        const float DT = softplus_f(dd_dt + dtb);
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
      float dskip;
      if constexpr (PRELOAD) dskip = hp.dskip;
      else dskip = ldg_f(static_cast<const T *>(p.Dp) + hh);
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
          for (int r = 0; r < R; ++r) {
            if constexpr (HR::PRE) xr[r] += cur.x[k] * hp.mx[r][k];
            else xr[r] += cur.x[k] * ldg_f(mx + r * P + pp);
          }
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
            if constexpr (HR::PRE) {
#pragma unroll
              for (int e = 0; e < VW; ++e) bb[e] = hp.bb[r][f][e];
            } else {
              ldg_vec<VW>(bB + r * D + col, bb);
            }
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
            if constexpr (HR::PRE) {
#pragma unroll
              for (int e = 0; e < VW; ++e) cc[e] = hp.bc[r][f][e];
            } else {
              ldg_vec<VW>(bC + r * D + col, cc);
            }
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
          for (int r = 0; r < R; ++r) {
            if constexpr (HR::PRE) yv += yr[r] * hp.mo[r][k];
            else yv += yr[r] * ldg_f(mo + r * P + pp);
          }
          float zv;
          if constexpr (PRELOAD) zv = cur.z[k];
          else zv = ldz<ZX_COHERENT>(row + (int64_t)hh * P + pp);
          st_any(p.y, ybase + pp, yv * silu_f(zv), p.y_dt);
        }
      }
    }
  }
}

}  // namespace row
}  // namespace m3
