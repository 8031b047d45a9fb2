// MIMO decode kernels.
//
// mimo_stream_kernel (full-step fused, aligned shapes): one CTA owns a group
// of heads (one warp per head) and a chunk of consecutive batch rows.  The
// per-head parameters (B/C biases, the rank projections mimo_x / mimo_o,
// dt_bias, D, norm weights) are staged in shared memory once per CTA and
// reused for every row of the chunk.  For each batch row a ring stage is
// filled by 1-D bulk (TMA) copies of the row's B/C/x/z/scalar/angle sections
// of the in_proj output and of the heads' ssm_state / bx_prev / angle_state;
// the next rows land while the current one is computed.  Per row:
//   * RMSNorm of the R B-rows and R C-rows, shared by the CTA's heads;
//   * per head: x_r = mimo_x x (one warp transpose-reduction for all ranks),
//     Bx = RoPE(sum_r x_r (Bn_r + bias_r)) -- RoPE is linear, so rotating
//     the rank sum equals summing the rotated ranks (src/kernels/utils.py:
//     133 with B_proj from src/models/mamba3.py:330-332);
//     the trapezoidal update; y_r = <Cn_r + cbias_r, RoPE^-1(h)> (a
//     rotation is orthogonal, so <RoPE(c), h> = <c, RoPE^-1(h)>);
//     y = sum_r (y_r + D x_r) mimo_o[r] * silu(z).
// mimo_decode_kernel (m3_kernels.cuh) serves everything else: the
// state-update-only entry points and shapes the aligned path does not take.
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

struct MimoPlan {
  int rows_per_cta;  // consecutive batch rows per CTA
  int nstage;
  // byte offsets
  int par_off, nbc_off, ring_off, stage_bytes;
  // byte offsets inside a stage
  int o_raw, o_x, o_z, o_scal, o_h, o_bx, o_ang;
};

// Shared-memory parameter block (fp32) of a CTA with hpc heads.
template <int BD, int R>
struct ParLayout {
  int bB, bC, mx, mo, dtb, dsk, wB, wC, total;  // float offsets
  __host__ __device__ ParLayout(int hpc, int P) {
    bB = 0;
    bC = bB + hpc * R * BD;
    mx = bC + hpc * R * BD;
    mo = mx + hpc * R * P;
    dtb = mo + hpc * R * P;
    dsk = dtb + hpc;
    wB = dsk + hpc;
    wC = wB + BD;
    total = wC + BD;
  }
};

__device__ __forceinline__ void st_vec_global(float *p, const float (&v)[4]) {
  asm volatile("st.global.v4.f32 [%0], {%1,%2,%3,%4};" ::"l"(p), "f"(v[0]), "f"(v[1]), "f"(v[2]), "f"(v[3])
               : "memory");
}
__device__ __forceinline__ void st_vec_global(float *p, const float (&v)[2]) {
  asm volatile("st.global.v2.f32 [%0], {%1,%2};" ::"l"(p), "f"(v[0]), "f"(v[1]) : "memory");
}

template <int BD, int R, typename T>
__global__ void __launch_bounds__(256) mimo_stream_kernel(const KParams p, const MimoPlan mp) {
  using Sh = MimoShape<BD>;
  constexpr int VW = Sh::VW, F = Sh::F, KPL = Sh::KPL, NPAIR = VW / 2;
  using V = typename VecOf<VW>::T;

  extern __shared__ __align__(128) unsigned char smem_raw[];
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem_raw);
  float *par = reinterpret_cast<float *>(smem_raw + mp.par_off);
  float *nBC = reinterpret_cast<float *>(smem_raw + mp.nbc_off);  // [2R][BD]

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nwarps = blockDim.x >> 5;
  const int H = p.H, P = p.P, D = p.D, A = p.A;
  const int hpc = p.heads_per_cta;
  const int ngrp = (H + hpc - 1) / hpc;
  const int grp = blockIdx.x % ngrp;
  const int b0 = (blockIdx.x / ngrp) * mp.rows_per_cta;
  const int b1 = min(p.B, b0 + mp.rows_per_cta);
  const int h0 = grp * hpc;
  const int nh = min(hpc, H - h0);
  const ParLayout<BD, R> L(hpc, P);
  const T *zx = static_cast<const T *>(p.zx);
  const int so = 2 * p.d_inner + 2 * p.d_bc;  // scalar section: dd_dt[H] dd_A[H] trap[H] angle[A]

  if (tid == 0) {
    for (int s = 0; s < mp.nstage; ++s) mbar_init(smem_addr(&bars[s]), 1);
    mbar_init_fence();
  }
  __syncthreads();

  constexpr int es = sizeof(T);
  auto issue = [&](int k) {
    const int b = b0 + k;
    if (b >= b1) return;
    const int s = k % mp.nstage;
    unsigned char *st = smem_raw + mp.ring_off + (size_t)s * mp.stage_bytes;
    const uint32_t bar = smem_addr(&bars[s]);
    const T *row = zx + (int64_t)b * p.zx_sb;
    const uint32_t n_raw = 2u * R * D * es, n_xz = (uint32_t)nh * P * es, n_scal = (uint32_t)(3 * H + A) * es;
    const uint32_t n_hd = (uint32_t)nh * D * 4, n_ang = (uint32_t)nh * A * 4;
    mbar_arrive_expect_tx(bar, n_raw + 2 * n_xz + n_scal + 2 * n_hd + n_ang);
    const int64_t sb = ((int64_t)b * H + h0);
    bulk_g2s(smem_addr(st + mp.o_raw), row + 2 * p.d_inner, n_raw, bar);
    bulk_g2s(smem_addr(st + mp.o_x), row + p.d_inner + (int64_t)h0 * P, n_xz, bar);
    bulk_g2s(smem_addr(st + mp.o_z), row + (int64_t)h0 * P, n_xz, bar);
    bulk_g2s(smem_addr(st + mp.o_scal), row + so, n_scal, bar);
    bulk_g2s(smem_addr(st + mp.o_h), p.h + sb * D, n_hd, bar);
    bulk_g2s(smem_addr(st + mp.o_bx), p.bx + sb * D, n_hd, bar);
    bulk_g2s(smem_addr(st + mp.o_ang), p.ang + sb * A, n_ang, bar);
  };
  if (tid == 0)
    for (int k = 0; k < mp.nstage; ++k) issue(k);

  // ---- parameters of this CTA's heads -> shared memory (fp32) ----
  {
    const T *bB = static_cast<const T *>(p.bB), *bC = static_cast<const T *>(p.bC);
    const T *mx = static_cast<const T *>(p.mx), *mo = static_cast<const T *>(p.mo);
    const int nbias = nh * R * D;
    for (int i = tid; i < nbias; i += blockDim.x) {
      const int w = i / (R * D), rd = i - w * (R * D), r = rd / D, d = rd - r * D;
      const int64_t g = (int64_t)(h0 + w) * R * D + rd;
      par[L.bB + (w * R + r) * BD + d] = to_f(bB[g]);
      par[L.bC + (w * R + r) * BD + d] = to_f(bC[g]);
    }
    const int nm = nh * R * P;
    for (int i = tid; i < nm; i += blockDim.x) {
      const int64_t g = (int64_t)h0 * R * P + i;
      par[L.mx + i] = to_f(mx[g]);
      par[L.mo + i] = to_f(mo[g]);
    }
    for (int i = tid; i < nh; i += blockDim.x) {
      par[L.dtb + i] = to_f(static_cast<const T *>(p.dt_bias)[h0 + i]);
      par[L.dsk + i] = to_f(static_cast<const T *>(p.Dp)[h0 + i]);
    }
    for (int i = tid; i < D; i += blockDim.x) {
      par[L.wB + i] = to_f(static_cast<const T *>(p.wB)[i]);
      par[L.wC + i] = to_f(static_cast<const T *>(p.wC)[i]);
    }
  }
  __syncthreads();  // parameters staged (the first rows are already in flight)

  int k = 0;
  for (; b0 + k < b1; ++k) {
    const int b = b0 + k;
    const int s = k % mp.nstage;
    const bool ok = mbar_wait(smem_addr(&bars[s]), (uint32_t)((k / mp.nstage) & 1));
    if (__syncthreads_or(!ok)) break;
    const unsigned char *st = smem_raw + mp.ring_off + (size_t)s * mp.stage_bytes;
    const T *sRaw = reinterpret_cast<const T *>(st + mp.o_raw);
    const T *sX = reinterpret_cast<const T *>(st + mp.o_x);
    const T *sZ = reinterpret_cast<const T *>(st + mp.o_z);
    const T *sScal = reinterpret_cast<const T *>(st + mp.o_scal);
    const float *sH = reinterpret_cast<const float *>(st + mp.o_h);
    const float *sBx = reinterpret_cast<const float *>(st + mp.o_bx);
    const float *sAng = reinterpret_cast<const float *>(st + mp.o_ang);

    // RMSNorm of the 2R B/C rows of this batch row (src/models/mamba3.py:202-203)
    for (int row = warp; row < 2 * R; row += nwarps) {
      const float *w = par + (row < R ? L.wB : L.wC);
      float v[KPL];
      float ss = 0.f;
#pragma unroll
      for (int q = 0; q < KPL; ++q) {
        const int d = lane + 32 * q;
        v[q] = d < D ? to_f(sRaw[row * D + d]) : 0.f;
        ss += v[q] * v[q];
      }
      ss = group_sum<32>(ss);
      const float rms = sqrtf(ss / (float)D + kRmsEps);
#pragma unroll
      for (int q = 0; q < KPL; ++q) {
        const int d = lane + 32 * q;
        if (d < D) nBC[row * BD + d] = v[q] / rms * w[d];
      }
    }
    __syncthreads();

    if (warp < nh) {
      const int w = warp, hh = h0 + w;
      // scalars (src/models/mamba3.py:196-199)
      const float dd_dt = to_f(sScal[hh]), dd_A = to_f(sScal[H + hh]), tr_raw = to_f(sScal[2 * H + hh]);
      const float sp = softplus_f(dd_A);
      const float Aval = -(sp > -p.A_floor ? -p.A_floor : sp);
      Coef c;
      c.DT = softplus_f(dd_dt + par[L.dtb + w]);
      c.decay = expf(Aval * c.DT);
      const float tr = sigmoid_f(tr_raw);
      c.omt = 1.f - tr;
      c.htr = tr * 0.5f;
      const float dskip = par[L.dsk + w];

      // angles of this lane's RoPE pairs (angle_state += angle_raw * DT)
      float cs[F][NPAIR], sn[F][NPAIR];
      const int64_t abase = ((int64_t)b * H + hh) * A;
#pragma unroll
      for (int f = 0; f < F; ++f)
#pragma unroll
        for (int q = 0; q < NPAIR; ++q) {
          const int i = (lane + 32 * f) * NPAIR + q;
          cs[f][q] = 1.f;
          sn[f][q] = 0.f;
          if (i < A) {
            const float ang = sAng[w * A + i] + to_f(sScal[3 * H + i]) * c.DT;
            p.ang[abase + i] = ang;
            sincosf(ang, &sn[f][q], &cs[f][q]);
          }
        }

      // x_r = sum_p x_p mimo_x[h, r, p]
      float xr[R];
#pragma unroll
      for (int r = 0; r < R; ++r) xr[r] = 0.f;
      for (int p0 = 0; p0 < P; p0 += 32) {
        const int pp = p0 + lane;
        if (pp < P) {
          const float xp = to_f(sX[w * P + pp]);
#pragma unroll
          for (int r = 0; r < R; ++r) xr[r] += xp * par[L.mx + (w * R + r) * P + pp];
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
          float acc[VW];
#pragma unroll
          for (int e = 0; e < VW; ++e) acc[e] = 0.f;
#pragma unroll
          for (int r = 0; r < R; ++r) {
            const V nv = *reinterpret_cast<const V *>(nBC + r * BD + col);
            const V bv = *reinterpret_cast<const V *>(par + L.bB + (w * R + r) * BD + col);
            const float *n = reinterpret_cast<const float *>(&nv);
            const float *bb = reinterpret_cast<const float *>(&bv);
#pragma unroll
            for (int e = 0; e < VW; ++e) acc[e] += xr[r] * (n[e] + bb[e]);
          }
          float bxv[VW], hn[VW];
#pragma unroll
          for (int q = 0; q < NPAIR; ++q) {
            const float x1 = acc[2 * q], x2 = acc[2 * q + 1];
            bxv[2 * q] = x1 * cs[f][q] - x2 * sn[f][q];
            bxv[2 * q + 1] = x1 * sn[f][q] + x2 * cs[f][q];
          }
          const V ho = *reinterpret_cast<const V *>(sH + w * D + col);
          const V bo = *reinterpret_cast<const V *>(sBx + w * D + col);
          const float *hov = reinterpret_cast<const float *>(&ho);
          const float *bov = reinterpret_cast<const float *>(&bo);
#pragma unroll
          for (int e = 0; e < VW; ++e) hn[e] = trap_update(c, bxv[e], bov[e], hov[e]);
          st_vec_global(p.h + sbase + col, hn);
          st_vec_global(p.bx + sbase + col, bxv);
#pragma unroll
          for (int q = 0; q < NPAIR; ++q) {
            const float x1 = hn[2 * q], x2 = hn[2 * q + 1];
            hr[f][2 * q] = x1 * cs[f][q] + x2 * sn[f][q];
            hr[f][2 * q + 1] = x2 * cs[f][q] - x1 * sn[f][q];
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
            const V cv = *reinterpret_cast<const V *>(par + L.bC + (w * R + r) * BD + col);
            const float *n = reinterpret_cast<const float *>(&nv);
            const float *cc = reinterpret_cast<const float *>(&cv);
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
      for (int p0 = 0; p0 < P; p0 += 32) {
        const int pp = p0 + lane;
        if (pp < P) {
          float yv = 0.f;
#pragma unroll
          for (int r = 0; r < R; ++r) yv += yr[r] * par[L.mo + (w * R + r) * P + pp];
          yv = yv * silu_f(to_f(sZ[w * P + pp]));
          st_any(p.y, ybase + pp, yv, p.y_dt);
        }
      }
    }
    __syncthreads();  // stage s and nBC are free again
    if (tid == 0) issue(k + mp.nstage);
  }
  if (tid == 0) {  // only after a lost copy: bounded wait for what is still in flight
    for (int q = k; q < k + mp.nstage; ++q)
      if (b0 + q < b1) mbar_wait(smem_addr(&bars[q % mp.nstage]), (uint32_t)((q / mp.nstage) & 1), 1 << 16);
  }
}

int align128(int x) { return (x + 127) / 128 * 128; }

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

constexpr int kMaxSmem = 200 * 1024;

// Shared-memory plan of the aligned path; returns false if it does not fit.
template <int BD, int R>
bool mimo_plan(const KParams &kp, int es, int nstage, MimoPlan &mp, int *smem) {
  const int hpc = kp.heads_per_cta, P = kp.P, D = kp.D, A = kp.A, H = kp.H;
  const ParLayout<BD, R> L(hpc, P);
  mp.nstage = nstage;
  mp.par_off = 128;
  mp.nbc_off = mp.par_off + align128(L.total * 4);
  mp.ring_off = mp.nbc_off + align128(2 * R * BD * 4);
  int o = 0;
  mp.o_raw = o; o += align128(2 * R * D * es);
  mp.o_x = o; o += align128(hpc * P * es);
  mp.o_z = o; o += align128(hpc * P * es);
  mp.o_scal = o; o += align128((3 * H + A) * es);
  mp.o_h = o; o += align128(hpc * D * 4);
  mp.o_bx = o; o += align128(hpc * D * 4);
  mp.o_ang = o; o += align128(hpc * A * 4);
  mp.stage_bytes = o;
  *smem = mp.ring_off + nstage * mp.stage_bytes;
  return *smem <= kMaxSmem;
}

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Whether the aligned path can take this call: every bulk copy must start
// on a 16-byte boundary and move a multiple of 16 bytes.
bool stream_eligible(const KParams &kp, int es) {
  if (kp.zx_dt != kp.par_dt) return false;
  const int64_t zrow = kp.zx_sb * es;
  if (zrow % 16 || !aligned16(kp.zx) || !aligned16(kp.ang) || !aligned16(kp.h) || !aligned16(kp.bx)) return false;
  if ((kp.d_inner * es) % 16 || (kp.d_bc * es) % 16 || (kp.P * es) % 16) return false;
  if (((3 * kp.H + kp.A) * es) % 16 || (kp.A % 4) != 0) return false;
  return true;
}

template <int BD, int R, typename T>
cudaError_t launch_stream(KParams kp, cudaStream_t stream, bool *taken) {
  *taken = false;
  const int es = sizeof(T);
  if (!stream_eligible(kp, es)) return cudaSuccess;
  kp.heads_per_cta = kp.H < (R == 8 ? 4 : 8) ? kp.H : (R == 8 ? 4 : 8);
  MimoPlan mp;
  int smem = 0;
  if (!mimo_plan<BD, R>(kp, es, 3, mp, &smem) && !mimo_plan<BD, R>(kp, es, 2, mp, &smem)) return cudaSuccess;
  auto kern = mimo_stream_kernel<BD, R, T>;
  static bool attr = false;
  static int last_smem = -1, last_per_sm = 1, last_threads = 0;
  if (!attr) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxSmem);
    if (e != cudaSuccess) return e;
    attr = true;
  }
  const int threads = kp.heads_per_cta * 32;
  if (smem != last_smem || threads != last_threads) {
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, threads, smem) != cudaSuccess || per_sm < 1)
      per_sm = 1;
    last_smem = smem;
    last_threads = threads;
    last_per_sm = per_sm;
  }
  // batch rows per CTA: enough CTAs to fill every SM once, each reusing its
  // staged parameters over as many rows as that allows
  const int ngrp = (kp.H + kp.heads_per_cta - 1) / kp.heads_per_cta;
  const int slots = num_sms() * last_per_sm;
  const int64_t items = (int64_t)kp.B * ngrp;
  int rows = (int)((items + slots - 1) / slots);
  if (rows < 1) rows = 1;
  mp.rows_per_cta = rows;
  const int64_t grid = (int64_t)ngrp * ((kp.B + rows - 1) / rows);
  kern<<<(unsigned)grid, threads, smem, stream>>>(kp, mp);
  *taken = true;
  return cudaGetLastError();
}

template <int BD, int R>
cudaError_t launch_full_t(const KParams &kp, cudaStream_t stream) {
  bool taken = false;
  cudaError_t e = kp.zx_dt == M3_BF16 ? launch_stream<BD, R, __nv_bfloat16>(kp, stream, &taken)
                                      : launch_stream<BD, R, float>(kp, stream, &taken);
  if (e != cudaSuccess || taken) return e;
  // generic path
  const int ngrp = (kp.H + kp.heads_per_cta - 1) / kp.heads_per_cta;
  const unsigned grid = (unsigned)((int64_t)kp.B * ngrp);
  const size_t smem = (size_t)2 * R * BD * sizeof(float);
  mimo_decode_kernel<BD, R, true><<<grid, kp.heads_per_cta * 32, smem, stream>>>(kp);
  return cudaGetLastError();
}

template <int BD, int R>
cudaError_t launch_ssm_t(const KParams &kp, cudaStream_t stream) {
  const int ngrp = (kp.H + kp.heads_per_cta - 1) / kp.heads_per_cta;
  const unsigned grid = (unsigned)((int64_t)kp.B * ngrp);
  mimo_decode_kernel<BD, R, false><<<grid, kp.heads_per_cta * 32, 0, stream>>>(kp);
  return cudaGetLastError();
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
