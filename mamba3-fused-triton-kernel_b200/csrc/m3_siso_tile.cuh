// Per-tile parameters of the SISO decode step, shared by the streamed SISO
// kernel (m3_siso.cu) and the single-launch step (m3_step_impl.cuh): the
// RMS-normalised, biased and rotated B / C rows of one (batch row, head)
// tile, its head scalars, x and silu(z), computed into a shared-memory
// parameter block (src/models/mamba3.py:196-215, 326-333;
// src/kernels/utils.py:31-44).
#pragma once

#include "m3_kernels.cuh"

namespace m3 {

namespace {

// Scalars of the current tile, kept in shared memory.
enum { kDecay = 0, kDT, kOmt, kHtr, kDskip, kGate, kNScalar = 8 };

// Shared-memory parameter block: tile parameters, then (full step) the
// norm weights, dt_bias and D of every head, loaded once per CTA.
struct ParBlock {
  float *sB, *sC, *sX, *sG, *sS, *wB, *wC, *dtb, *dsk;
};

template <int BD>
__device__ ParBlock par_block(unsigned char *base, const KParams &p) {
  ParBlock q;
  q.sB = reinterpret_cast<float *>(base);
  q.sC = q.sB + BD;
  q.sX = q.sC + BD;
  q.sG = q.sX + p.P;
  q.sS = q.sG + p.P;
  q.wB = q.sS + kNScalar;
  q.wC = q.wB + BD;
  q.dtb = q.wC + BD;
  q.dsk = q.dtb + p.H;
  return q;
}

template <typename T> __device__ __forceinline__ float to_f(T v);
template <> __device__ __forceinline__ float to_f<float>(float v) { return v; }
template <> __device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }

// RMSNorm + weight + bias + RoPE of the rank-0 B and C rows of one tile,
// into q.sB / q.sC, by one warp.  raw(d) / bias(d) fetch the inputs;
// ang_old(i) / ang_raw(i) the angle state and increment of pair i; the
// accumulated angle is written back to angle_state (src/models/mamba3.py:
// 202-215, 326-333; src/kernels/utils.py:31-44).
template <int BD, typename RawB, typename RawC, typename BiasB, typename BiasC, typename AngOld, typename AngRaw>
__device__ __forceinline__ void bc_rows(const KParams &p, const ParBlock &q, int t, float DT, RawB rawB, RawC rawC,
                                        BiasB biasB, BiasC biasC, AngOld ang_old, AngRaw ang_raw) {
  constexpr int KPL = SisoShape<BD>::KPL;
  const int lane = threadIdx.x & 31, D = p.D;
  float vb[KPL], vc[KPL];
  float ssb = 0.f, ssc = 0.f;
#pragma unroll
  for (int k = 0; k < KPL; ++k) {
    const int d = lane + 32 * k;
    vb[k] = d < D ? rawB(d) : 0.f;
    vc[k] = d < D ? rawC(d) : 0.f;
    ssb += vb[k] * vb[k];
    ssc += vc[k] * vc[k];
  }
  ssb = group_sum<32>(ssb);
  ssc = group_sum<32>(ssc);
  const float rmsb = sqrtf(ssb / (float)D + kRmsEps);
  const float rmsc = sqrtf(ssc / (float)D + kRmsEps);
#pragma unroll
  for (int k = 0; k < KPL; ++k) {
    const int d = lane + 32 * k;
    if (d < D) {
      vb[k] = vb[k] / rmsb * q.wB[d] + biasB(d);
      vc[k] = vc[k] / rmsc * q.wC[d] + biasC(d);
    }
    const bool rot = d < 2 * p.A;
    float sn = 0.f, cs = 1.f, ang = 0.f;
    if (rot) {
      ang = ang_old(d >> 1) + ang_raw(d >> 1) * DT;
      sincosf(ang, &sn, &cs);
    }
    const float ob = __shfl_xor_sync(kFullMask, vb[k], 1);
    const float oc = __shfl_xor_sync(kFullMask, vc[k], 1);
    if (rot) {
      if (d & 1) {
        vb[k] = ob * sn + vb[k] * cs;
        vc[k] = oc * sn + vc[k] * cs;
      } else {
        vb[k] = vb[k] * cs - ob * sn;
        vc[k] = vc[k] * cs - oc * sn;
        p.ang[(int64_t)t * p.A + (d >> 1)] = ang;
      }
    }
    if (d < D) {
      q.sB[d] = vb[k];
      q.sC[d] = vc[k];
    }
  }
}

// Scalars of head hh from dd_dt / dd_A / trap_raw (src/models/mamba3.py:196-199).
__device__ __forceinline__ void scalars_to_smem(const KParams &p, const ParBlock &q, int hh, float dd_dt,
                                                float dd_A, float tr_raw) {
  const float sp = softplus_f(dd_A);
  const float A = -(sp > -p.A_floor ? -p.A_floor : sp);  // clamp keeps NaN like torch
  const float DT = softplus_f(dd_dt + q.dtb[hh]);
  const float tr = sigmoid_f(tr_raw);
  q.sS[kDecay] = expf(A * DT);
  q.sS[kDT] = DT;
  q.sS[kOmt] = 1.f - tr;
  q.sS[kHtr] = tr * 0.5f;
  q.sS[kDskip] = q.dsk[hh];
  q.sS[kGate] = 1.f;
}

// Tile parameters read straight from global memory (full step on shapes
// the staged path cannot copy, and the state-update-only entry points).
template <int BD, bool FULL>
__device__ void tile_params_global(const KParams &p, const ParBlock &q, int b, int hh, int t) {
  const int tid = threadIdx.x, warp = tid >> 5, nthr = blockDim.x;
  const int P = p.P, D = p.D;
  if constexpr (FULL) {
    const int64_t zr = (int64_t)b * p.zx_sb;
    const int so = 2 * p.d_inner + 2 * p.d_bc;
    if (warp == 0) {
      const float dd_dt = ld_any(p.zx, zr + so + hh, p.zx_dt);
      const float DT = softplus_f(dd_dt + q.dtb[hh]);
      if ((tid & 31) == 0)
        scalars_to_smem(p, q, hh, dd_dt, ld_any(p.zx, zr + so + p.H + hh, p.zx_dt),
                        ld_any(p.zx, zr + so + 2 * p.H + hh, p.zx_dt));
      const int64_t colB = zr + 2 * p.d_inner, colC = zr + 2 * p.d_inner + p.d_bc;
      const int64_t acol = zr + so + 3 * p.H;
      bc_rows<BD>(
          p, q, t, DT, [&](int d) { return ld_any(p.zx, colB + d, p.zx_dt); },
          [&](int d) { return ld_any(p.zx, colC + d, p.zx_dt); },
          [&](int d) { return ld_any(p.bB, (int64_t)hh * D + d, p.par_dt); },
          [&](int d) { return ld_any(p.bC, (int64_t)hh * D + d, p.par_dt); },
          [&](int i) { return p.ang[(int64_t)t * p.A + i]; },
          [&](int i) { return ld_any(p.zx, acol + i, p.zx_dt); });
    }
    for (int i = tid; i < P; i += nthr) {
      q.sX[i] = ld_any(p.zx, zr + p.d_inner + (int64_t)hh * P + i, p.zx_dt);
      q.sG[i] = silu_f(ld_any(p.zx, zr + (int64_t)hh * P + i, p.zx_dt));
    }
  } else {
    if (tid == 0) {
      Coef c;
      float dskip;
      head_scalars_given(p, b, hh, c, dskip);
      q.sS[kDecay] = c.decay; q.sS[kDT] = c.DT; q.sS[kOmt] = c.omt; q.sS[kHtr] = c.htr;
      q.sS[kDskip] = dskip; q.sS[kGate] = p.z != nullptr ? 1.f : 0.f;
    }
    for (int i = tid; i < D; i += nthr) {
      q.sB[i] = p.Bp[(int64_t)b * p.B_sb + (int64_t)hh * p.B_sh + (int64_t)i * p.B_sd];
      q.sC[i] = p.Cp[(int64_t)b * p.C_sb + (int64_t)hh * p.C_sh + (int64_t)i * p.C_sd];
    }
    for (int i = tid; i < P; i += nthr) {
      q.sX[i] = ld_any(p.x, (int64_t)b * p.x_sb + (int64_t)hh * p.x_sh + (int64_t)i * p.x_sp, p.x_dt);
      if (p.z != nullptr)
        q.sG[i] = silu_f(ld_any(p.z, (int64_t)b * p.z_sb + (int64_t)hh * p.z_sh + (int64_t)i * p.z_sp, p.z_dt));
    }
  }
}

}  // namespace

}  // namespace m3
