// SISO decode: persistent streaming kernel over (batch, head) tiles.
//
// The SISO state of one (b, h) is a contiguous (P, D) fp32 tile in both
// ssm_state and bx_prev.  Each CTA walks its tiles in row-chunks of RT rows;
// a ring of NSTAGE shared-memory stages is kept full by 1-D bulk (TMA)
// copies, so up to NSTAGE chunks per CTA are in flight without holding
// registers.  Consumers read a chunk from shared memory, apply the
// exponential-trapezoidal update, write h and bx straight back to global
// memory with 128-bit stores and reduce C.h per row inside a lane group.
// Per-tile parameters (RMSNorm + bias + RoPE of B/C, scalars, x, silu(z))
// are computed while the following chunks are still landing.
//
// Reference arithmetic: src/kernels/fused_full_decode.py:37-225 (full step)
// and src/kernels/siso_decode.py:21-132 (state update only), in the
// operation order of src/kernels/utils.py:73-102.
#include "m3_async.cuh"
#include "m3_kernels.cuh"
#include "m3_siso_tile.cuh"

namespace m3 {

namespace {

constexpr int kSisoThreads = 256;
constexpr int kChunkFloats = 4096;  // state floats per tensor per stage (16 KB)
constexpr int kMaxSmem = 200 * 1024;

struct StreamPlan {
  int rt;           // rows per chunk
  int nchunk;       // chunks per (b, h) tile
  int nstage;       // ring depth
  int stage_bytes;  // bytes per stage
  int par_off;      // byte offset of the per-CTA parameter block
  int ring_off;     // byte offset of the ring
  // byte offsets inside a stage: state chunk, then (staged path) the tile header
  int o_h, o_bx, o_raw, o_x, o_z, o_scal, o_ang, o_bb, o_bc;
};

// Tile parameters of the full step from the header staged with chunk 0.
template <int BD, typename T>
__device__ void tile_params_staged(const KParams &p, const ParBlock &q, const StreamPlan &sp,
                                   const unsigned char *stage, int hh, int t) {
  const int tid = threadIdx.x, warp = tid >> 5, nthr = blockDim.x;
  const int H = p.H, D = p.D, P = p.P;
  const T *raw = reinterpret_cast<const T *>(stage + sp.o_raw);   // [B row | C row]
  const T *xs = reinterpret_cast<const T *>(stage + sp.o_x);
  const T *zs = reinterpret_cast<const T *>(stage + sp.o_z);
  const T *scal = reinterpret_cast<const T *>(stage + sp.o_scal);  // dd_dt[H] dd_A[H] trap[H] angle[A]
  const float *ang = reinterpret_cast<const float *>(stage + sp.o_ang);
  const unsigned char *bb = stage + sp.o_bb, *bc = stage + sp.o_bc;
  if (warp == 0) {
    const float dd_dt = to_f(scal[hh]);
    const float DT = softplus_f(dd_dt + q.dtb[hh]);
    if ((tid & 31) == 0) scalars_to_smem(p, q, hh, dd_dt, to_f(scal[H + hh]), to_f(scal[2 * H + hh]));
    bc_rows<BD>(
        p, q, t, DT, [&](int d) { return to_f(raw[d]); }, [&](int d) { return to_f(raw[D + d]); },
        [&](int d) { return ld_any(bb, d, p.par_dt); }, [&](int d) { return ld_any(bc, d, p.par_dt); },
        [&](int i) { return ang[i]; }, [&](int i) { return to_f(scal[3 * H + i]); });
  }
  for (int i = tid; i < P; i += nthr) {
    q.sX[i] = to_f(xs[i]);
    q.sG[i] = silu_f(to_f(zs[i]));
  }
}

__device__ __forceinline__ void st_global4(float *p, float4 v) {
  asm volatile("st.global.v4.f32 [%0], {%1,%2,%3,%4};" ::"l"(p), "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w)
               : "memory");
}

// FULL: full step (else state-update only).  STAGED: the tile header comes
// with chunk 0 through the ring (T = element type of the in_proj output).
template <int BD, bool FULL, bool STAGED, typename T>
__global__ void __launch_bounds__(kSisoThreads) siso_stream_kernel(const KParams p, const StreamPlan sp) {
  using Sh = SisoShape<BD>;
  constexpr int S = Sh::S, FPL = Sh::FPL, RPW = Sh::RPW;

  extern __shared__ __align__(128) unsigned char smem_raw[];
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem_raw);
  const ParBlock q = par_block<BD>(smem_raw + sp.par_off, p);
  unsigned char *ring = smem_raw + sp.ring_off;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int P = p.P, D = p.D, G = D >> 2;
  const int ntiles = p.B * p.H;
  const int nslots = (blockDim.x >> 5) * RPW;
  const int slot = warp * RPW + lane / S;
  const int j = lane % S;

  // k-th chunk of this CTA: tile blockIdx.x + (k / nchunk) * gridDim.x, chunk k % nchunk
  auto tile_of = [&](int k) { return (int)blockIdx.x + (k / sp.nchunk) * (int)gridDim.x; };

  if (tid == 0) {
    for (int s = 0; s < sp.nstage; ++s) mbar_init(smem_addr(&bars[s]), 1);
    mbar_init_fence();
  }
  __syncthreads();

  const int es_z = sizeof(T), pes_p = p.par_dt == M3_BF16 ? 2 : 4;
  auto header_bytes = [&]() -> uint32_t {
    return 2u * D * es_z + 2u * P * es_z + (uint32_t)(3 * p.H + p.A) * es_z + (uint32_t)p.A * 4 +
           2u * D * pes_p;
  };
  auto issue_header = [&](int k) {
    const int t = tile_of(k);
    const int b = t / p.H, hh = t - b * p.H;
    const uint32_t bar = smem_addr(&bars[k % sp.nstage]);
    unsigned char *st = ring + (size_t)(k % sp.nstage) * sp.stage_bytes;
    const T *row = static_cast<const T *>(p.zx) + (int64_t)b * p.zx_sb;
    const uint32_t n_raw = 2u * D * es_z, n_xz = (uint32_t)P * es_z, n_scal = (uint32_t)(3 * p.H + p.A) * es_z;
    const uint32_t n_ang = (uint32_t)p.A * 4, n_bias = (uint32_t)D * pes_p;
    bulk_g2s(smem_addr(st + sp.o_raw), row + 2 * p.d_inner, n_raw, bar);
    bulk_g2s(smem_addr(st + sp.o_x), row + p.d_inner + (int64_t)hh * P, n_xz, bar);
    bulk_g2s(smem_addr(st + sp.o_z), row + (int64_t)hh * P, n_xz, bar);
    bulk_g2s(smem_addr(st + sp.o_scal), row + 2 * p.d_inner + 2 * p.d_bc, n_scal, bar);
    bulk_g2s(smem_addr(st + sp.o_ang), p.ang + (int64_t)t * p.A, n_ang, bar);
    bulk_g2s(smem_addr(st + sp.o_bb), static_cast<const unsigned char *>(p.bB) + (size_t)hh * n_bias, n_bias, bar);
    bulk_g2s(smem_addr(st + sp.o_bc), static_cast<const unsigned char *>(p.bC) + (size_t)hh * n_bias, n_bias, bar);
  };
  // Chunk k of this CTA into stage k % nstage: the state chunk and, for the
  // first chunk of a tile on the staged path, the tile header.  The header
  // comes from the in_proj output (the preceding kernel's product), so the
  // first stages' headers are issued after pdl_wait() (with_header false
  // arms the barrier for them but leaves their copies to issue_header).
  auto issue = [&](int k, bool with_header) {
    const int t = tile_of(k);
    if (t >= ntiles) return;
    const int c = k % sp.nchunk;
    const int r0 = c * sp.rt;
    const int nr = min(sp.rt, P - r0);
    const int s = k % sp.nstage;
    const uint32_t bytes = (uint32_t)nr * (uint32_t)D * 4u;
    const uint32_t bar = smem_addr(&bars[s]);
    const size_t goff = ((size_t)t * P + r0) * D;
    unsigned char *st = ring + (size_t)s * sp.stage_bytes;
    uint32_t tx = 2 * bytes;
    if constexpr (STAGED) {
      if (c == 0) tx += header_bytes();
    }
    mbar_arrive_expect_tx(bar, tx);
    bulk_g2s(smem_addr(st + sp.o_h), p.h + goff, bytes, bar);
    bulk_g2s(smem_addr(st + sp.o_bx), p.bx + goff, bytes, bar);
    if constexpr (STAGED) {
      if (c == 0 && with_header) issue_header(k);
    }
  };
  if (tid == 0)
    for (int k = 0; k < sp.nstage; ++k) issue(k, false);

  if constexpr (FULL) {  // per-CTA constants: norm weights, dt_bias, D
    for (int i = tid; i < D; i += blockDim.x) {
      q.wB[i] = ld_any(p.wB, i, p.par_dt);
      q.wC[i] = ld_any(p.wC, i, p.par_dt);
    }
    for (int i = tid; i < p.H; i += blockDim.x) {
      q.dtb[i] = ld_any(p.dt_bias, i, p.par_dt);
      q.dsk[i] = ld_any(p.Dp, i, p.par_dt);
    }
  }
  pdl_wait();
  pdl_trigger();
  if constexpr (STAGED) {
    if (tid == 0)
      for (int k = 0; k < sp.nstage; ++k)
        if (tile_of(k) < ntiles && k % sp.nchunk == 0) issue_header(k);
  }
  __syncthreads();

  int k = 0;
  for (;; ++k) {
    const int t = tile_of(k);
    if (t >= ntiles) break;
    const int c = k % sp.nchunk;
    const int b = t / p.H, hh = t - b * p.H;
    const int s = k % sp.nstage;
    const unsigned char *st = ring + (size_t)s * sp.stage_bytes;
    if constexpr (STAGED) {
      const bool ok = mbar_wait(smem_addr(&bars[s]), (uint32_t)((k / sp.nstage) & 1));
      if (__syncthreads_or(!ok)) break;  // a lost copy: stop and drain
      if (c == 0) {
        tile_params_staged<BD, T>(p, q, sp, st, hh, t);
        __syncthreads();
      }
    } else {
      if (c == 0) {
        tile_params_global<BD, FULL>(p, q, b, hh, t);
        __syncthreads();
      }
      const bool ok = mbar_wait(smem_addr(&bars[s]), (uint32_t)((k / sp.nstage) & 1));
      if (__syncthreads_or(!ok)) break;
    }

    const float *sh = reinterpret_cast<const float *>(st + sp.o_h);
    const float *sbx = reinterpret_cast<const float *>(st + sp.o_bx);
    const int r0 = c * sp.rt;
    const int nr = min(sp.rt, P - r0);
    const Coef cf = {q.sS[kDecay], q.sS[kDT], q.sS[kOmt], q.sS[kHtr]};
    const float dskip = q.sS[kDskip];
    const bool gate = q.sS[kGate] != 0.f;
    float *hg = p.h + ((size_t)t * P + r0) * D;
    float *bg = p.bx + ((size_t)t * P + r0) * D;
    const int64_t ybase = (int64_t)b * p.y_sb + (int64_t)hh * p.y_sh;
    for (int rb = 0; rb < nr; rb += nslots) {
      const int row = rb + slot;
      const bool rok = row < nr;
      const float xp = rok ? q.sX[r0 + row] : 0.f;
      float part = 0.f;
#pragma unroll
      for (int f = 0; f < FPL; ++f) {
        const int col = j + S * f;
        if (rok && col < G) {
          const int o = row * G + col;
          const float4 ho = reinterpret_cast<const float4 *>(sh)[o];
          const float4 bo = reinterpret_cast<const float4 *>(sbx)[o];
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
          st_global4(hg + (size_t)o * 4, hn);
          st_global4(bg + (size_t)o * 4, bn);
        }
      }
      part = group_sum<S>(part);
      if (j == 0 && rok) {
        float yv = part + dskip * xp;
        if (gate) yv = yv * q.sG[r0 + row];
        st_any(p.y, ybase + (int64_t)(r0 + row) * p.y_sp, yv, p.y_dt);
      }
    }
    __syncthreads();  // stage s and the tile parameters are free again
    if (tid == 0) issue(k + sp.nstage, true);
  }
  // Normal exit: every issued chunk was consumed.  After a lost copy, wait
  // (bounded) for whatever this CTA still has in flight before leaving.
  if (tid == 0) {
    for (int q2 = k; q2 < k + sp.nstage; ++q2)
      if (tile_of(q2) < ntiles)
        mbar_wait(smem_addr(&bars[q2 % sp.nstage]), (uint32_t)((q2 / sp.nstage) & 1));  // full bound: a copy may still land
  }
}

int align128(int x) { return (x + 127) / 128 * 128; }

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Whether every header copy of the staged path starts on a 16-byte boundary
// and moves a multiple of 16 bytes.
bool staged_eligible(const KParams &kp) {
  const int es = kp.zx_dt == M3_BF16 ? 2 : 4, pes = kp.par_dt == M3_BF16 ? 2 : 4;
  if (!aligned16(kp.zx) || !aligned16(kp.ang) || !aligned16(kp.bB) || !aligned16(kp.bC)) return false;
  if ((kp.zx_sb * es) % 16 || (kp.d_inner * es) % 16 || (2 * kp.D * es) % 16) return false;
  if ((kp.P * es) % 16 || ((3 * kp.H + kp.A) * es) % 16 || (kp.A % 4) || (kp.D * pes) % 16) return false;
  return true;
}

StreamPlan make_plan(const KParams &kp, int BD, bool staged, int nstage, int *smem_bytes) {
  const int D = kp.D, P = kp.P;
  StreamPlan sp;
  sp.rt = kChunkFloats / D;
  if (sp.rt < 1) sp.rt = 1;
  if (sp.rt > P) sp.rt = P;
  sp.nchunk = (P + sp.rt - 1) / sp.rt;
  sp.nstage = nstage;
  int o = 0;
  sp.o_h = o; o += align128(sp.rt * D * 4);
  sp.o_bx = o; o += align128(sp.rt * D * 4);
  sp.o_raw = sp.o_x = sp.o_z = sp.o_scal = sp.o_ang = sp.o_bb = sp.o_bc = 0;
  if (staged) {
    const int es = kp.zx_dt == M3_BF16 ? 2 : 4, pes = kp.par_dt == M3_BF16 ? 2 : 4;
    sp.o_raw = o; o += align128(2 * D * es);
    sp.o_x = o; o += align128(P * es);
    sp.o_z = o; o += align128(P * es);
    sp.o_scal = o; o += align128((3 * kp.H + kp.A) * es);
    sp.o_ang = o; o += align128(kp.A * 4);
    sp.o_bb = o; o += align128(D * pes);
    sp.o_bc = o; o += align128(D * pes);
  }
  sp.stage_bytes = o;
  sp.par_off = 128;  // after the barriers
  const int par_floats = 2 * BD + 2 * P + kNScalar + 2 * BD + 2 * kp.H;
  sp.ring_off = sp.par_off + align128(par_floats * 4);
  *smem_bytes = sp.ring_off + sp.nstage * sp.stage_bytes;
  return sp;
}

int num_sms() { return sm_count_current(); }

template <int BD, bool FULL, bool STAGED, typename T>
cudaError_t launch_t(const KParams &kp, cudaStream_t stream) {
  int smem = 0;
  StreamPlan sp = make_plan(kp, BD, STAGED, 3, &smem);
  if (smem > kMaxSmem) sp = make_plan(kp, BD, STAGED, 2, &smem);
  if (smem > kMaxSmem) return cudaErrorInvalidValue;
  auto kern = siso_stream_kernel<BD, FULL, STAGED, T>;
  // Once per kernel and device: opt in to the largest ring any call may
  // need.  Then CTAs per SM for this ring size (per device, last size seen).
  static LaunchCache cache;
  if (cudaError_t e = ensure_smem_optin(cache, kern, kMaxSmem); e != cudaSuccess) return e;
  int per_sm = 0;
  if (occupancy_per_sm(cache, kern, kSisoThreads, (size_t)smem, &per_sm) != cudaSuccess || per_sm < 1) per_sm = 1;
  const int ntiles = kp.B * kp.H;
  int grid = num_sms() * per_sm;
  if (grid > ntiles) grid = ntiles;
  return launch_pdl(kern, dim3(grid), dim3(kSisoThreads), (size_t)smem, stream, kp, sp);
}

template <int BD>
cudaError_t launch_mode(const KParams &kp, bool full, cudaStream_t stream) {
  if (!full) return launch_t<BD, false, false, float>(kp, stream);
  if (staged_eligible(kp))
    return kp.zx_dt == M3_BF16 ? launch_t<BD, true, true, __nv_bfloat16>(kp, stream)
                               : launch_t<BD, true, true, float>(kp, stream);
  return launch_t<BD, true, false, float>(kp, stream);
}

// Waits on an mbarrier that nothing completes, with a short bound: the
// bounded-wait self test (the error word must read M3_DEVERR_TIMEOUT after).
__global__ void wait_timeout_probe_kernel() {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(smem_addr(&bar), 1);
    mbar_init_fence();
    mbar_wait(smem_addr(&bar), 0, 1000);
  }
}

}  // namespace

cudaError_t launch_siso(const KParams &kp, bool full, cudaStream_t stream) {
  if (kp.D <= 16) return launch_mode<16>(kp, full, stream);
  if (kp.D <= 32) return launch_mode<32>(kp, full, stream);
  if (kp.D <= 64) return launch_mode<64>(kp, full, stream);
  if (kp.D <= 128) return launch_mode<128>(kp, full, stream);
  return launch_mode<256>(kp, full, stream);
}

int siso_device_error(bool reset) { return device_error_of_this_unit(reset); }

cudaError_t launch_wait_timeout_probe(cudaStream_t stream) {
  wait_timeout_probe_kernel<<<1, 32, 0, stream>>>();
  return cudaGetLastError();
}

}  // namespace m3
