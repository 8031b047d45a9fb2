// Mamba-3 single-token decode kernels for B200 (sm_100a).
//
// Two kernel families, each instantiated for the full-step fused variant
// (reads the raw in_proj output) and the state-update-only variant (reads
// precomputed B/C/dt/trap, as the reference's SSM kernels do):
//
//   siso_stream_kernel  (m3_siso.cu) persistent CTAs stream the contiguous
//                       (P, D) state tiles of ssm_state and bx_prev through
//                       a ring of shared-memory stages filled by 1-D bulk
//                       copies; a group of S lanes owns one state row
//                       (S = D/4 float4 columns, capped at 32) and reduces
//                       C.h with shuffles.
//   mimo_decode_kernel  one CTA per (batch, group of heads), one warp per
//                       head.  The (D,) state of a head is spread over the
//                       warp's lanes (2 or 4 floats per lane, so every RoPE
//                       pair is lane-local); RMSNorm of the rank-R B/C rows
//                       is done once per CTA into shared memory; the rank-R
//                       contractions are warp shuffles.
//
// Arithmetic follows the reference PyTorch decode (src/models/mamba3.py:
// 160-217, 306-353; src/kernels/utils.py:31-148) operation by operation in
// fp32, including the A = -(softplus(dd_A).clamp(max=-A_floor)) expression
// (which evaluates to +A_floor) and the torch softplus threshold of 20.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include <utility>

#include "m3_devcache.cuh"
#include "mamba3_b200.h"

namespace m3 {

constexpr float kRmsEps = 1e-5f;  // RMSNorm eps (src/models/mamba3.py:29)
constexpr unsigned kFullMask = 0xffffffffu;

// Everything a launch needs; filled on the host by the C-ABI layer.
struct KParams {
  int B, H, P, D, R, A;
  float A_floor;
  int d_inner, d_bc;  // d_bc = D * ngroups * R
  int heads_per_cta;  // MIMO only
  // full-step fused sources
  const void *zx; int64_t zx_sb; int zx_dt; int par_dt;
  const void *dt_bias, *Dp, *wB, *wC, *bB, *bC, *mx, *mo;
  // state-update-only sources
  const void *x; int64_t x_sb, x_sh, x_sp; int x_dt;
  const void *z; int64_t z_sb, z_sh, z_sp; int z_dt;
  const float *Bp; int64_t B_sb, B_sr, B_sh, B_sd;
  const float *Cp; int64_t C_sb, C_sr, C_sh, C_sd;
  const float *adt; int64_t adt_sb, adt_sh;
  const float *dt; int64_t dt_sb, dt_sh;
  const float *trap; int64_t tr_sb, tr_sh;
  const float *Dsk; int64_t D_sh;
  const float *smx; int64_t mx_sh, mx_sr, mx_sp;
  const float *smo; int64_t mo_sh, mo_sr, mo_sp;
  // carried state (in place) and output
  float *h, *bx, *ang;
  int L;  // tokens per sequence of a prefill launch (decode: unused)
  void *y; int64_t y_sb, y_sh, y_sp; int y_dt;
};

// ---------------------------------------------------------------------------
// programmatic dependent launch
// ---------------------------------------------------------------------------
// Every kernel of the library is launched with programmatic stream
// serialisation: it may start while the preceding kernel on the stream is
// still running.  Before reading anything that kernel produces (the in_proj
// output, the projection input) it executes pdl_wait(), which returns once
// the preceding grid has completed and its writes are visible; it calls
// pdl_wait() before pdl_trigger(), so a kernel's completion implies the
// completion of everything before it, and data written two or more kernels
// back (the carried state) may be read before the wait.  Without a
// preceding dependent launch both instructions are no-ops.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Launch `kernel` with programmatic stream serialisation.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                       Args &&...args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// scalar helpers
// ---------------------------------------------------------------------------

__device__ __forceinline__ float ld_any(const void *p, int64_t i, int dt) {
  return dt == M3_BF16 ? __bfloat162float(static_cast<const __nv_bfloat16 *>(p)[i])
                       : static_cast<const float *>(p)[i];
}

__device__ __forceinline__ void st_any(void *p, int64_t i, float v, int dt) {
  if (dt == M3_BF16)
    static_cast<__nv_bfloat16 *>(p)[i] = __float2bfloat16_rn(v);
  else
    static_cast<float *>(p)[i] = v;
}

// torch.nn.functional.softplus(beta=1, threshold=20)
__device__ __forceinline__ float softplus_f(float x) { return x > 20.f ? x : log1pf(expf(x)); }
__device__ __forceinline__ float sigmoid_f(float x) { return 1.f / (1.f + expf(-x)); }
__device__ __forceinline__ float silu_f(float x) { return x * sigmoid_f(x); }

// Sum over aligned groups of W lanes (W a power of two <= 32); every lane
// of the warp must call it.
template <int W>
__device__ __forceinline__ float group_sum(float v) {
#pragma unroll
  for (int o = W / 2; o > 0; o >>= 1) v += __shfl_xor_sync(kFullMask, v, o);
  return v;
}

// sin and cos of an accumulated RoPE angle, which grows without bound over
// a sequence: Cody-Waite reduction (Cody & Waite, "Software Manual for the
// Elementary Functions", 1980) by 2*pi with the constant split into a float
// head and a float tail -- each step one fma, whose product is exact -- then
// the hardware approximations on [-pi, pi], where their absolute error is
// about 4e-7.  Angles beyond 2^17 (and NaN) take the library's full-range
// sincosf, N angles at a time with one warp vote for that fallback.  Every
// lane of the warp must call it.
template <int N>
__device__ __forceinline__ void rope_sincos_n(const float (&x)[N], float (&s)[N], float (&c)[N]) {
  constexpr float kInvTwoPi = 0x1.45f306p-3f;   // 1 / (2 pi)
  constexpr float kTwoPiHi = 0x1.921fb6p+2f;    // 2 pi rounded to float
  constexpr float kTwoPiLo = -0x1.777a5cp-23f;  // 2 pi - kTwoPiHi, rounded to float
  bool big = false;
#pragma unroll
  for (int i = 0; i < N; ++i) {
    const float k = rintf(x[i] * kInvTwoPi);
    float r = fmaf(-k, kTwoPiHi, x[i]);
    r = fmaf(-k, kTwoPiLo, r);
    s[i] = __sinf(r);
    c[i] = __cosf(r);
    big = big || !(fabsf(x[i]) <= 131072.f);
  }
  if (__any_sync(kFullMask, big)) {
#pragma unroll
    for (int i = 0; i < N; ++i)
      if (!(fabsf(x[i]) <= 131072.f)) sincosf(x[i], &s[i], &c[i]);
  }
}

// 128-bit state accesses.  The state is touched exactly once per launch, so
// loads skip L1 allocation; L2 keeps its default policy so that a state that
// fits in L2 stays resident from one decode step to the next.
__device__ __forceinline__ float4 ld_state4(const float *p) {
  float4 v;
  asm volatile("ld.global.L1::no_allocate.v4.f32 {%0,%1,%2,%3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "l"(p));
  return v;
}
__device__ __forceinline__ float2 ld_state2(const float *p) {
  float2 v;
  asm volatile("ld.global.L1::no_allocate.v2.f32 {%0,%1}, [%2];" : "=f"(v.x), "=f"(v.y) : "l"(p));
  return v;
}
__device__ __forceinline__ void st_state4(float *p, float4 v) {
  *reinterpret_cast<float4 *>(p) = v;
}
__device__ __forceinline__ void st_state2(float *p, float2 v) {
  *reinterpret_cast<float2 *>(p) = v;
}

// One element of the exponential-trapezoidal update
// (src/kernels/utils.py:95-99):  bx = x*B;  blend = (1-trap)*bx +
// (trap*0.5)*(bx + bx_prev);  h = exp(ADT)*h + DT*blend.
struct Coef {
  float decay, DT, omt, htr;  // exp(ADT), DT, 1 - trap, trap * 0.5
};

__device__ __forceinline__ float trap_update(const Coef &c, float bx, float bx_prev, float h) {
  const float blend = c.omt * bx + c.htr * (bx + bx_prev);
  return c.decay * h + c.DT * blend;
}

// Per-(batch, head) scalars from the raw in_proj row
// (src/models/mamba3.py:196-199; the scalar section starts at
// 2*d_inner + 2*d_bc: dd_dt[H], dd_A[H], trap[H]).
__device__ __forceinline__ void head_scalars_from_zx(const KParams &p, int64_t zr, int hh, Coef &c,
                                                     float &dskip) {
  const int so = 2 * p.d_inner + 2 * p.d_bc;
  const float dd_dt = ld_any(p.zx, zr + so + hh, p.zx_dt);
  const float dd_A = ld_any(p.zx, zr + so + p.H + hh, p.zx_dt);
  const float tr_raw = ld_any(p.zx, zr + so + 2 * p.H + hh, p.zx_dt);
  const float sp = softplus_f(dd_A);
  // clamp(max=-A_floor) keeps a NaN, as torch.clamp does
  const float A = -(sp > -p.A_floor ? -p.A_floor : sp);
  c.DT = softplus_f(dd_dt + ld_any(p.dt_bias, hh, p.par_dt));
  c.decay = expf(A * c.DT);
  const float tr = sigmoid_f(tr_raw);
  c.omt = 1.f - tr;
  c.htr = tr * 0.5f;
  dskip = ld_any(p.Dp, hh, p.par_dt);
}

__device__ __forceinline__ void head_scalars_given(const KParams &p, int b, int hh, Coef &c,
                                                   float &dskip) {
  c.DT = p.dt[(int64_t)b * p.dt_sb + (int64_t)hh * p.dt_sh];
  c.decay = expf(p.adt[(int64_t)b * p.adt_sb + (int64_t)hh * p.adt_sh]);
  const float tr = p.trap[(int64_t)b * p.tr_sb + (int64_t)hh * p.tr_sh];
  c.omt = 1.f - tr;
  c.htr = tr * 0.5f;
  dskip = p.Dsk[(int64_t)hh * p.D_sh];
}

// ---------------------------------------------------------------------------
// SISO: state (B, H, P, D); one CTA per (b, h)
// ---------------------------------------------------------------------------

template <int BD>
struct SisoShape {
  static constexpr int BG = BD / 4;               // float4 columns per row (padded)
  static constexpr int S = BG < 32 ? BG : 32;     // lanes per row
  static constexpr int FPL = BG / S;              // float4 per lane per row
  static constexpr int RPW = 32 / S;              // rows per warp per pass
  static constexpr int KPL = BD >= 32 ? BD / 32 : 1;  // prologue elements per lane
};

// ---------------------------------------------------------------------------
// MIMO: state (B, H, D); one CTA per (b, group of heads), one warp per head
// ---------------------------------------------------------------------------

template <int VW> struct VecOf;
template <> struct VecOf<4> { using T = float4; };
template <> struct VecOf<2> { using T = float2; };

template <int BD>
struct MimoShape {
  static constexpr int VW = BD >= 128 ? 4 : 2;     // floats per lane vector
  static constexpr int NV = BD / VW;               // vectors per head row (padded)
  static constexpr int F = NV > 32 ? NV / 32 : 1;  // vectors per lane
  static constexpr int KPL = BD >= 32 ? BD / 32 : 1;
};

template <int VW>
__device__ __forceinline__ void ld_vec(const float *p, float (&v)[VW]) {
  if constexpr (VW == 4) {
    const float4 t = ld_state4(p);
    v[0] = t.x; v[1] = t.y; v[2] = t.z; v[3] = t.w;
  } else {
    const float2 t = ld_state2(p);
    v[0] = t.x; v[1] = t.y;
  }
}
template <int VW>
__device__ __forceinline__ void st_vec(float *p, const float (&v)[VW]) {
  if constexpr (VW == 4)
    st_state4(p, make_float4(v[0], v[1], v[2], v[3]));
  else
    st_state2(p, make_float2(v[0], v[1]));
}

template <int BD, int R, bool FULL>
__global__ void __launch_bounds__(256) mimo_decode_kernel(const KParams p) {
  using Sh = MimoShape<BD>;
  constexpr int VW = Sh::VW, F = Sh::F, KPL = Sh::KPL, NPAIR = VW / 2;

  extern __shared__ __align__(16) float smem[];  // FULL: [2R][BD] normalized B_r, C_r

  const int hpc = p.heads_per_cta;
  const int ngrp = (p.H + hpc - 1) / hpc;
  const int b = blockIdx.x / ngrp;
  const int hg = blockIdx.x - b * ngrp;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
  const int hh = hg * hpc + warp;
  const bool head_ok = warp < hpc && hh < p.H;
  const int D = p.D, P = p.P;
  const int64_t sbase = ((int64_t)b * p.H + hh) * D;
  const int64_t zr = (int64_t)b * p.zx_sb;

  // state of this warp's head, in flight during the prologue
  float hv[F][VW], bv[F][VW];
#pragma unroll
  for (int f = 0; f < F; ++f) {
    const int col = (lane + 32 * f) * VW;
    if (head_ok && col < D) {
      ld_vec<VW>(p.h + sbase + col, hv[f]);
      ld_vec<VW>(p.bx + sbase + col, bv[f]);
    } else {
#pragma unroll
      for (int e = 0; e < VW; ++e) hv[f][e] = bv[f][e] = 0.f;
    }
  }

  pdl_wait();
  pdl_trigger();

  if constexpr (FULL) {
    // RMSNorm of the R B-rows and R C-rows of this batch row, shared by
    // every head of the CTA (src/models/mamba3.py:202-203; "(r g n)" layout).
    for (int row = warp; row < 2 * R; row += nwarps) {
      const int r = row % R;
      const int col0 = 2 * p.d_inner + (row < R ? 0 : p.d_bc) + r * D;
      const void *wn = row < R ? p.wB : p.wC;
      float v[KPL];
      float ss = 0.f;
#pragma unroll
      for (int k = 0; k < KPL; ++k) {
        const int d = lane + 32 * k;
        v[k] = d < D ? ld_any(p.zx, zr + col0 + d, p.zx_dt) : 0.f;
        ss += v[k] * v[k];
      }
      ss = group_sum<32>(ss);
      const float rms = sqrtf(ss / (float)D + kRmsEps);
#pragma unroll
      for (int k = 0; k < KPL; ++k) {
        const int d = lane + 32 * k;
        if (d < D) smem[row * BD + d] = v[k] / rms * ld_any(wn, d, p.par_dt);
      }
    }
    __syncthreads();
  }
  if (!head_ok) return;

  Coef c;
  float dskip;
  if constexpr (FULL)
    head_scalars_from_zx(p, zr, hh, c, dskip);
  else
    head_scalars_given(p, b, hh, c, dskip);

  // RoPE coefficients of this lane's pairs; pair i covers entries (2i, 2i+1)
  // and is rotated iff i < A.  Each pair belongs to exactly one lane, which
  // also writes the accumulated angle back.
  float cs[F][NPAIR], sn[F][NPAIR];
  if constexpr (FULL) {
    const int acol = 2 * p.d_inner + 2 * p.d_bc + 3 * p.H;
    const int64_t abase = ((int64_t)b * p.H + hh) * p.A;
#pragma unroll
    for (int f = 0; f < F; ++f) {
#pragma unroll
      for (int q = 0; q < NPAIR; ++q) {
        const int i = (lane + 32 * f) * NPAIR + q;
        cs[f][q] = 1.f;
        sn[f][q] = 0.f;
        if (i < p.A) {
          const float ang = p.ang[abase + i] + ld_any(p.zx, zr + acol + i, p.zx_dt) * c.DT;
          p.ang[abase + i] = ang;
          sincosf(ang, &sn[f][q], &cs[f][q]);
        }
      }
    }
  }

  // x_r = sum_p x_p * mimo_x[h, r, p]   (src/kernels/utils.py:130)
  float xr[R];
#pragma unroll
  for (int r = 0; r < R; ++r) xr[r] = 0.f;
  for (int p0 = 0; p0 < P; p0 += 32) {
    const int pp = p0 + lane;
    if (pp < P) {
      float xp;
      if constexpr (FULL)
        xp = ld_any(p.zx, zr + p.d_inner + (int64_t)hh * P + pp, p.zx_dt);
      else
        xp = ld_any(p.x, (int64_t)b * p.x_sb + (int64_t)hh * p.x_sh + (int64_t)pp * p.x_sp, p.x_dt);
#pragma unroll
      for (int r = 0; r < R; ++r) {
        float m;
        if constexpr (FULL)
          m = ld_any(p.mx, ((int64_t)hh * R + r) * P + pp, p.par_dt);
        else
          m = p.smx[(int64_t)hh * p.mx_sh + (int64_t)r * p.mx_sr + (int64_t)pp * p.mx_sp];
        xr[r] += xp * m;
      }
    }
  }
#pragma unroll
  for (int r = 0; r < R; ++r) xr[r] = group_sum<32>(xr[r]);

  // B_r / C_r vector of this lane: FULL = RoPE(norm + bias[h, r]); else the
  // precomputed projection.
  auto bc_vec = [&](bool isC, int r, int f, float (&v)[VW]) {
    const int col = (lane + 32 * f) * VW;
    if constexpr (FULL) {
      const float *nrow = smem + (isC ? R + r : r) * BD + col;
      const void *bias = isC ? p.bC : p.bB;
      const int64_t bi = ((int64_t)hh * R + r) * D + col;
#pragma unroll
      for (int e = 0; e < VW; ++e) v[e] = nrow[e] + ld_any(bias, bi + e, p.par_dt);
#pragma unroll
      for (int q = 0; q < NPAIR; ++q) {
        const float x1 = v[2 * q], x2 = v[2 * q + 1];
        if ((lane + 32 * f) * NPAIR + q < p.A) {
          v[2 * q] = x1 * cs[f][q] - x2 * sn[f][q];
          v[2 * q + 1] = x1 * sn[f][q] + x2 * cs[f][q];
        }
      }
    } else {
      const float *src = isC ? p.Cp : p.Bp;
      const int64_t sb = isC ? p.C_sb : p.B_sb, sr = isC ? p.C_sr : p.B_sr;
      const int64_t sh = isC ? p.C_sh : p.B_sh, sd = isC ? p.C_sd : p.B_sd;
      const int64_t o = (int64_t)b * sb + (int64_t)r * sr + (int64_t)hh * sh;
#pragma unroll
      for (int e = 0; e < VW; ++e) v[e] = src[o + (int64_t)(col + e) * sd];
    }
  };

  // Bx = sum_r x_r * B_r   (utils.py:133), then the trapezoidal update
  float bxc[F][VW], hn[F][VW];
#pragma unroll
  for (int f = 0; f < F; ++f)
#pragma unroll
    for (int e = 0; e < VW; ++e) bxc[f][e] = 0.f;
#pragma unroll
  for (int r = 0; r < R; ++r) {
#pragma unroll
    for (int f = 0; f < F; ++f) {
      if ((lane + 32 * f) * VW < D) {
        float v[VW];
        bc_vec(false, r, f, v);
#pragma unroll
        for (int e = 0; e < VW; ++e) bxc[f][e] += xr[r] * v[e];
      }
    }
  }
#pragma unroll
  for (int f = 0; f < F; ++f)
#pragma unroll
    for (int e = 0; e < VW; ++e) hn[f][e] = trap_update(c, bxc[f][e], bv[f][e], hv[f][e]);

  // y_r = sum_d C_r[d] h[d] + D * x_r   (utils.py:143-145)
  float yr[R];
#pragma unroll
  for (int r = 0; r < R; ++r) {
    float part = 0.f;
#pragma unroll
    for (int f = 0; f < F; ++f) {
      if ((lane + 32 * f) * VW < D) {
        float v[VW];
        bc_vec(true, r, f, v);
#pragma unroll
        for (int e = 0; e < VW; ++e) part += v[e] * hn[f][e];
      }
    }
    yr[r] = group_sum<32>(part) + dskip * xr[r];
  }

#pragma unroll
  for (int f = 0; f < F; ++f) {
    const int col = (lane + 32 * f) * VW;
    if (col < D) {
      st_vec<VW>(p.h + sbase + col, hn[f]);
      st_vec<VW>(p.bx + sbase + col, bxc[f]);
    }
  }

  // y_p = sum_r y_r * mimo_o[h, r, p]  (utils.py:146), then * silu(z)
  const bool gate = FULL || p.z != nullptr;
  const int64_t ybase = (int64_t)b * p.y_sb + (int64_t)hh * p.y_sh;
  for (int p0 = 0; p0 < P; p0 += 32) {
    const int pp = p0 + lane;
    if (pp < P) {
      float yv = 0.f;
#pragma unroll
      for (int r = 0; r < R; ++r) {
        float m;
        if constexpr (FULL)
          m = ld_any(p.mo, ((int64_t)hh * R + r) * P + pp, p.par_dt);
        else
          m = p.smo[(int64_t)hh * p.mo_sh + (int64_t)r * p.mo_sr + (int64_t)pp * p.mo_sp];
        yv += yr[r] * m;
      }
      if (gate) {
        float zv;
        if constexpr (FULL)
          zv = ld_any(p.zx, zr + (int64_t)hh * P + pp, p.zx_dt);
        else
          zv = ld_any(p.z, (int64_t)b * p.z_sb + (int64_t)hh * p.z_sh + (int64_t)pp * p.z_sp, p.z_dt);
        yv = yv * silu_f(zv);
      }
      st_any(p.y, ybase + (int64_t)pp * p.y_sp, yv, p.y_dt);
    }
  }
}

// Launchers (defined in m3_siso.cu / m3_mimo.cu); return the launch status.
cudaError_t launch_siso(const KParams &kp, bool full, cudaStream_t stream);
cudaError_t launch_mimo(const KParams &kp, bool full, cudaStream_t stream);
// The streamed MIMO full-step kernel (m3_mimo_stream.cu); *taken is false
// when the call's shapes or alignment are outside its range.
cudaError_t launch_mimo_stream(const KParams &kp, cudaStream_t stream, bool *taken);
// The streamed kernel in prefill form: kp.B sequences of kp.L tokens each,
// in_proj / y rows b * L + t, state rows b (m3_mimo_stream.cu).
cudaError_t launch_mimo_prefill(const KParams &kp, cudaStream_t stream, bool *taken);
// SISO prefill (m3_siso_prefill.cu): kp.B sequences of kp.L tokens, one CTA per
// (sequence, head) with the state tile in registers; *taken false (nothing
// enqueued) for shapes outside its range.
cudaError_t launch_siso_prefill(const KParams &kp, cudaStream_t stream, bool *taken);
// The tcgen05 bf16 projection GEMM (m3_gemm.cu): y = x . w^T.
bool gemm_bf16_supported(const void *x, int64_t ldx, const void *w, int64_t ldw, const void *y, int64_t ldy, int M,
                         int N, int K);
int64_t gemm_bf16_workspace_bytes(int M, int N, int K);
cudaError_t launch_gemm_bf16(const void *x, int64_t ldx, const void *w, int64_t ldw, void *y, int64_t ldy, int M,
                             int N, int K, bool y_bf16, float *workspace, cudaStream_t stream);
// The split-precision fp32 GEMM on the same kernel (kind::tf32, three
// products per k step): y = (x + xl) . (w + wl)^T with x / w TF32 heads and
// xl / wl their remainders; and the head / remainder split of a matrix.
bool gemm_tf32x3_supported(const void *x, const void *xl, int64_t ldx, const void *w, const void *wl, int64_t ldw,
                           const void *y, int64_t ldy, int M, int N, int K);
cudaError_t launch_gemm_tf32x3(const float *x, const float *xl, int64_t ldx, const float *w, const float *wl,
                               int64_t ldw, float *y, int64_t ldy, int M, int N, int K, cudaStream_t stream);
cudaError_t launch_tf32_split(const float *x, int64_t ldx, float *hi, float *lo, int64_t ld, int rows, int cols,
                              cudaStream_t stream);
// The skinny bf16 GEMM for decode batches of up to kSkinnyMaxRows rows
// (m3_skinny.cu): y = x . w^T, weight streamed once through mma.sync.
constexpr int kSkinnyMaxRows = 64;
bool gemm_skinny_supported(const void *x, int64_t ldx, const void *w, int64_t ldw, const void *y, int64_t ldy, int M,
                           int N, int K);
cudaError_t launch_gemm_skinny(const void *x, int64_t ldx, const void *w, int64_t ldw, void *y, int64_t ldy, int M,
                               int N, int K, bool y_bf16, cudaStream_t stream);
cudaError_t launch_wait_timeout_probe(cudaStream_t stream);
cudaError_t launch_residual_rmsnorm(int dtype, const void *x, const void *o, const float *w, void *x_out, void *xn,
                                    int M, int N, int64_t ldx, int64_t ldo, int64_t ldxo, int64_t ldn, float eps,
                                    cudaStream_t stream);
int residual_rmsnorm_max_width();
cudaError_t launch_linear_small_m(const float *A, int64_t lda, const float *W, int64_t ldw, float *C, int64_t ldc,
                                  int M, int N, int K, cudaStream_t stream);

// Device error words of the kernel translation units (read, optionally clear).
int siso_device_error(bool reset);
int mimo_device_error(bool reset);
int mimo_stream_device_error(bool reset);
int siso_prefill_device_error(bool reset);
int gemm_device_error(bool reset);

// Heads handled by one CTA of the MIMO kernels.
int mimo_heads_per_cta(int H);

}  // namespace m3
