// MIMO full-step decode, streamed through shared memory.
//
// mimo_stream_kernel does what the row kernel (m3_mimo_row.cuh) does -- the
// whole MIMO decode update from the raw in_proj row (src/models/mamba3.py:
// 160-217, 306-353; src/kernels/utils.py:95-148) -- for the shapes where
// every piece of a batch row can be fetched by 1-D bulk (TMA) copies.  One
// CTA owns 8 heads (one warp each) and a run of consecutive batch rows:
//
//   * one thread keeps the next nstage-1 rows in flight: for each row it
//     copies the 8 heads' carried state (h, Bx_prev, angles) and the in_proj
//     pieces the CTA reads (x and z of its heads, the R B-rows and R C-rows,
//     the angle increments) into a ring stage, completing on that stage's
//     mbarrier, so the HBM latency of a row overlaps the arithmetic of the
//     rows before it;
//   * the per-(row, head) scalars (DT, exp(A DT), the trapezoid weights) are
//     computed once per 32 rows with one (row, head) pair per thread into a
//     double-buffered table, instead of once per warp and row;
//   * per row, each warp RMS-normalises one of the 2R B/C rows into shared
//     memory; the single CTA barrier of a row publishes them and frees the
//     previous row's stage for the next copy;
//   * each warp then updates its head: lane l owns state elements
//     [VW l, VW l + VW) (every RoPE pair lane-local) and head-dim elements
//     [PL l, PL l + PL), computes the rotation of its own pairs, and writes
//     h, Bx, the angles and y with vector stores.
//
// The per-head parameters (mimo_x, mimo_o, the B/C biases, the norm
// weights, D) stay in registers when they fit and are otherwise re-read
// through the read-only cache.  Every mbarrier wait is bounded; a lost copy
// stops the CTA, which then waits (bounded) for its other copies in flight.
#include "m3_async.cuh"
#include "m3_kernels.cuh"
#include "m3_mimo_row.cuh"

namespace m3 {

namespace {

constexpr int kWarps = 8;        // heads per CTA
constexpr int kTableRows = 32;   // rows per chunk of the head-scalar table
constexpr int kMaxStages = 8;  // mbarriers reserved; the ring uses 4 (one row a pass) or 6 (two)

// Byte layout of one launch's dynamic shared memory, computed on the host.
struct StreamLayout {
  int nstage, stage_bytes;
  int o_h, o_bx, o_ang, o_x, o_z, o_bc, o_araw;  // offsets inside a stage
  unsigned n_state, n_ang, n_xz, n_bc, n_araw;   // bytes of each copy
  unsigned tx_state, tx;                         // state bytes, all bytes of a stage
  int o_bars, o_table, o_nbc, o_ring, smem;      // offsets of the regions
  // per-head parameters of the CTA's 8 heads staged in shared memory by
  // bulk copies that complete with the first row (o_par < 0: read from
  // global memory instead); offsets inside the region and copy bytes
  int o_par, p_bB, p_bC, p_mx, p_mo, p_wB, p_wC, p_Dp, p_dtb;
  unsigned n_bBC, n_mxo, n_w, n_h8, n_par;
};

// Shared-memory loads of N consecutive elements (8- or 16-byte aligned for
// N > 1) into floats.
template <int N, typename T> __device__ __forceinline__ void lds_f(const T *p, float (&v)[N]);
template <> __device__ __forceinline__ void lds_f<1, float>(const float *p, float (&v)[1]) { v[0] = *p; }
template <> __device__ __forceinline__ void lds_f<2, float>(const float *p, float (&v)[2]) {
  const float2 t = *reinterpret_cast<const float2 *>(p);
  v[0] = t.x; v[1] = t.y;
}
template <> __device__ __forceinline__ void lds_f<4, float>(const float *p, float (&v)[4]) {
  const float4 t = *reinterpret_cast<const float4 *>(p);
  v[0] = t.x; v[1] = t.y; v[2] = t.z; v[3] = t.w;
}
template <> __device__ __forceinline__ void lds_f<1, __nv_bfloat16>(const __nv_bfloat16 *p, float (&v)[1]) {
  v[0] = __bfloat162float(*p);
}
template <> __device__ __forceinline__ void lds_f<2, __nv_bfloat16>(const __nv_bfloat16 *p, float (&v)[2]) {
  const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(p));
  v[0] = a.x; v[1] = a.y;
}
template <> __device__ __forceinline__ void lds_f<4, __nv_bfloat16>(const __nv_bfloat16 *p, float (&v)[4]) {
  const uint2 t = *reinterpret_cast<const uint2 *>(p);
  const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&t.x));
  const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&t.y));
  v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y;
}

// Global stores of N consecutive floats (aligned to N * 4 bytes).
template <int N> __device__ __forceinline__ void stg_f(float *p, const float (&v)[N]) {
  if constexpr (N == 4)
    asm volatile("st.global.v4.f32 [%0], {%1,%2,%3,%4};" ::"l"(p), "f"(v[0]), "f"(v[1]), "f"(v[2]), "f"(v[3])
                 : "memory");
  else if constexpr (N == 2)
    asm volatile("st.global.v2.f32 [%0], {%1,%2};" ::"l"(p), "f"(v[0]), "f"(v[1]) : "memory");
  else
    *p = v[0];
}

// y stores: N consecutive outputs as float or bf16 (aligned to their size).
template <int N> __device__ __forceinline__ void st_y(void *y, int64_t i, const float (&v)[N], int dt) {
  if (dt == M3_BF16) {
    __nv_bfloat16 *q = static_cast<__nv_bfloat16 *>(y) + i;
    if constexpr (N == 1) {
      *q = __float2bfloat16_rn(v[0]);
    } else {
#pragma unroll
      for (int j = 0; j < N; j += 2)
        *reinterpret_cast<__nv_bfloat162 *>(q + j) = __floats2bfloat162_rn(v[j], v[j + 1]);
    }
  } else {
    stg_f<N>(static_cast<float *>(y) + i, v);
  }
}

__device__ __forceinline__ float2 f2(float a, float b) { return make_float2(a, b); }

// Read-only global loads of N consecutive elements (aligned to their size).
template <int N, typename T> __device__ __forceinline__ void ldg_n(const T *p, float (&v)[N]) {
  if constexpr (N == 1)
    v[0] = row::ldg_f(p);
  else
    row::ldg_vec<N>(p, v);
}

// A parameter vector: from its staged copy (byte offset `off` in the
// shared-memory region at `base`) or from global memory.
template <int N, typename T>
__device__ __forceinline__ void ld_param(bool staged, const unsigned char *base, int off, const T *g, float (&v)[N]) {
  if (staged)
    lds_f<N, T>(reinterpret_cast<const T *>(base + off), v);
  else
    ldg_n<N>(g, v);
}

template <int BD, int R, typename T, int PL, int RP, bool SEQ>
__global__ void __launch_bounds__(kWarps * 32, 2) mimo_stream_kernel(const KParams p, const StreamLayout L,
                                                                      const int rows_per_cta) {
  using Sh = MimoShape<BD>;
  constexpr int VW = Sh::VW, F = Sh::F, NP = VW / 2;  // NP RoPE pairs per vector
  constexpr int NRW = (2 * R + kWarps - 1) / kWarps;   // B/C rows each warp normalises
  // per-head parameters held in registers when they fit beside RP rows' work
  constexpr bool KEEP_B = 2 * R * F * VW <= 32 / RP;   // B/C biases
  constexpr bool KEEP_M = 2 * R * PL <= 32 / RP;       // mimo_x / mimo_o
  constexpr int RB = KEEP_B ? R : 1, RM = KEEP_M ? R : 1;

  extern __shared__ __align__(128) unsigned char smem[];
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + L.o_bars);
  float4 *table = reinterpret_cast<float4 *>(smem + L.o_table);  // [2][kTableRows][8]
  float *nbc = reinterpret_cast<float *>(smem + L.o_nbc);        // [2][2R][BD]
  unsigned char *ring = smem + L.o_ring;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int H = p.H, P = p.P, D = p.D, A = p.A;
  const int ngrp = H / kWarps;
  const int grp = blockIdx.x % ngrp, h0 = grp * kWarps, hh = h0 + warp;
  // Decode: "rows" are batch rows b0 + k.  SEQ (prefill): they are the
  // p.L tokens of sequence bs -- in_proj / y rows bs * L + k -- and the
  // carried state of row bs stays in registers from the first token to the
  // last (read once, written once).
  static_assert(!SEQ || RP == 1, "a prefill CTA takes its tokens one at a time");
  const int bs = SEQ ? (int)(blockIdx.x / ngrp) : 0;
  const int b0 = SEQ ? 0 : (int)(blockIdx.x / ngrp) * rows_per_cta;
  const int nrows = SEQ ? p.L : min(p.B, b0 + rows_per_cta) - b0;
  auto zrow = [&](int k) -> int64_t { return SEQ ? (int64_t)bs * p.L + k : (int64_t)(b0 + k); };
  auto srow = [&](int k) -> int64_t { return SEQ ? (int64_t)bs : (int64_t)(b0 + k); };
  const int S = L.nstage;
  const T *zx = static_cast<const T *>(p.zx);
  const int so = 2 * p.d_inner + 2 * p.d_bc;  // dd_dt[H] dd_A[H] trap[H] angle[A]

  if (tid == 0) {
    for (int s = 0; s < S; ++s) mbar_init(smem_addr(&bars[s]), 1);
    mbar_init_fence();
  }
  __syncthreads();

  // Row k of this CTA into stage s (= k % S), issued by one thread.  The
  // carried state was written by the previous step's kernel (two or more
  // launches back) and may be requested before pdl_wait(); the in_proj
  // pieces only after it.  (Spreading the copies over warp 0's lanes, each
  // lane selecting its own source and size, was measured slower.)
  auto issue_state = [&](int k, int s) {
    unsigned char *st = ring + (size_t)s * L.stage_bytes;
    const uint32_t bar = smem_addr(&bars[s]);
    const int64_t rh = srow(k) * H + h0;
    if (SEQ && k > 0) {  // later tokens carry the state in registers
      mbar_arrive_expect_tx(bar, L.tx - L.tx_state);
      return;
    }
    mbar_arrive_expect_tx(bar, L.tx);
    bulk_g2s(smem_addr(st + L.o_h), p.h + rh * D, L.n_state, bar);
    bulk_g2s(smem_addr(st + L.o_bx), p.bx + rh * D, L.n_state, bar);
    bulk_g2s(smem_addr(st + L.o_ang), p.ang + rh * A, L.n_ang, bar);
  };
  auto issue_zx = [&](int k, int s) {
    unsigned char *st = ring + (size_t)s * L.stage_bytes;
    const uint32_t bar = smem_addr(&bars[s]);
    const T *row = zx + zrow(k) * p.zx_sb;
    bulk_g2s(smem_addr(st + L.o_x), row + p.d_inner + (int64_t)h0 * P, L.n_xz, bar);
    bulk_g2s(smem_addr(st + L.o_z), row + (int64_t)h0 * P, L.n_xz, bar);
    bulk_g2s(smem_addr(st + L.o_bc), row + 2 * p.d_inner, L.n_bc, bar);
    bulk_g2s(smem_addr(st + L.o_araw), row + so + 3 * H, L.n_araw, bar);
  };

  const int npre = min(S - RP, nrows);
  const bool par_smem = L.o_par >= 0;
  unsigned char *par = smem + (par_smem ? L.o_par : 0);
  if (tid == 0) {
    if (par_smem) {
      // the parameters join row 0's phase (their bytes are added before row
      // 0's arrival below): constant for the launch, so requested before
      // the preceding kernel completes
      const uint32_t bar = smem_addr(&bars[0]);
      const int es = (int)sizeof(T);
      mbar_expect_tx(bar, L.n_par);
      bulk_g2s(smem_addr(par + L.p_bB), static_cast<const T *>(p.bB) + (int64_t)h0 * R * D, L.n_bBC, bar);
      bulk_g2s(smem_addr(par + L.p_bC), static_cast<const T *>(p.bC) + (int64_t)h0 * R * D, L.n_bBC, bar);
      bulk_g2s(smem_addr(par + L.p_mx), static_cast<const T *>(p.mx) + (int64_t)h0 * R * P, L.n_mxo, bar);
      bulk_g2s(smem_addr(par + L.p_mo), static_cast<const T *>(p.mo) + (int64_t)h0 * R * P, L.n_mxo, bar);
      bulk_g2s(smem_addr(par + L.p_wB), p.wB, L.n_w, bar);
      bulk_g2s(smem_addr(par + L.p_wC), p.wC, L.n_w, bar);
      bulk_g2s(smem_addr(par + L.p_Dp), static_cast<const unsigned char *>(p.Dp) + (size_t)h0 * es, L.n_h8, bar);
      bulk_g2s(smem_addr(par + L.p_dtb), static_cast<const unsigned char *>(p.dt_bias) + (size_t)h0 * es, L.n_h8,
               bar);
    }
    for (int k = 0; k < npre; ++k) issue_state(k, k);
  }

  // ---- per-head parameters, constant for the launch: read from the staged
  // shared-memory copy once row 0 has landed, or from global memory ----
  const T *mxp = static_cast<const T *>(p.mx) + (int64_t)hh * R * P;
  const T *mop = static_cast<const T *>(p.mo) + (int64_t)hh * R * P;
  const T *bBp = static_cast<const T *>(p.bB) + (int64_t)hh * R * D;
  const T *bCp = static_cast<const T *>(p.bC) + (int64_t)hh * R * D;
  constexpr int es = (int)sizeof(T);
  float mx[RM][PL], mo[RM][PL];
  float bb[RB][F][VW], bc[RB][F][VW];
  float wn[NRW][F][VW];  // norm weights of the B/C rows this warp normalises
  float dskip, dtb_t;    // D of this warp's head; dt_bias of the table column's head
  auto load_params = [&]() {
    if constexpr (KEEP_M) {
#pragma unroll
      for (int r = 0; r < R; ++r) {
        const int e0 = (warp * R + r) * P + lane * PL;
        ld_param<PL>(par_smem, par, L.p_mx + e0 * es, mxp + r * P + lane * PL, mx[r]);
        ld_param<PL>(par_smem, par, L.p_mo + e0 * es, mop + r * P + lane * PL, mo[r]);
      }
    }
    if constexpr (KEEP_B) {
#pragma unroll
      for (int r = 0; r < R; ++r)
#pragma unroll
        for (int f = 0; f < F; ++f) {
          const int col = (lane + 32 * f) * VW;
          if (col < D) {
            const int e0 = (warp * R + r) * D + col;
            ld_param<VW>(par_smem, par, L.p_bB + e0 * es, bBp + r * D + col, bb[r][f]);
            ld_param<VW>(par_smem, par, L.p_bC + e0 * es, bCp + r * D + col, bc[r][f]);
          } else {
#pragma unroll
            for (int e = 0; e < VW; ++e) bb[r][f][e] = bc[r][f][e] = 0.f;
          }
        }
    }
#pragma unroll
    for (int j = 0; j < NRW; ++j) {
      const int rr = warp + kWarps * j;
      const T *w = static_cast<const T *>(rr < R ? p.wB : p.wC);
#pragma unroll
      for (int f = 0; f < F; ++f) {
        const int col = (lane + 32 * f) * VW;
        if (rr < 2 * R && col < D) {
          ld_param<VW>(par_smem, par, (rr < R ? L.p_wB : L.p_wC) + col * es, w + col, wn[j][f]);
        } else {
#pragma unroll
          for (int e = 0; e < VW; ++e) wn[j][f][e] = 0.f;
        }
      }
    }
    float t[1];
    ld_param<1>(par_smem, par, L.p_Dp + warp * es, static_cast<const T *>(p.Dp) + hh, t);
    dskip = t[0];
    ld_param<1>(par_smem, par, L.p_dtb + (tid & 7) * es, static_cast<const T *>(p.dt_bias) + h0 + (tid & 7), t);
    dtb_t = t[0];
  };
  if (!par_smem) load_params();
  const float inv_d = 1.f / (float)D;

  // ---- head-scalar table: thread (j = tid / 8, w = tid % 8) owns row j of
  // a 32-row chunk and head h0 + w (src/models/mamba3.py:196-199) ----
  float traw[3];
  auto table_load = [&](int c) {
    const int k = c * kTableRows + (tid >> 3);
    if (k < nrows) {
      const T *sr = zx + zrow(k) * p.zx_sb + so + h0 + (tid & 7);
      traw[0] = row::ldg_f(sr);
      traw[1] = row::ldg_f(sr + H);
      traw[2] = row::ldg_f(sr + 2 * H);
    }
  };
  auto table_store = [&](int c) {
    const int k = c * kTableRows + (tid >> 3);
    if (k < nrows) {
      const float dd_A = traw[1];
      float A_val;
      if (p.A_floor > 0.f) {
        // softplus(.) >= 0 > -A_floor for every non-NaN input, so the clamp
        // returns -A_floor; a NaN propagates as in torch.clamp
        A_val = dd_A != dd_A ? dd_A : p.A_floor;
      } else {
        const float sp = softplus_f(dd_A);
        A_val = -(sp > -p.A_floor ? -p.A_floor : sp);
      }
      const float DT = softplus_f(traw[0] + dtb_t);
      const float tr = sigmoid_f(traw[2]);
      // h = exp(A DT) h + DT ((1 - tr) Bx + tr/2 (Bx + Bx_prev))
      //   = exp(A DT) h + c1 Bx + c2 Bx_prev   (src/kernels/utils.py:95-99)
      table[(c & 1) * kTableRows * kWarps + tid] =
          make_float4(expf(A_val * DT), DT * (1.f - tr * 0.5f), DT * (tr * 0.5f), DT);
    }
  };

  pdl_wait();
  pdl_trigger();
  if (tid == 0)
    for (int k = 0; k < npre; ++k) issue_zx(k, k);
  table_load(0);  // stored after the first row's norms, so the loads overlap its wait

  // A pass takes RP consecutive rows: their waits, their norms, ONE CTA
  // barrier, then each warp updates its head for all RP rows in lockstep, so
  // the rows' dependency chains (loads, reductions, shuffles) overlap.  A row
  // past the end aliases the pass's first row (same stage and inputs) with
  // its stores suppressed.  Stage sk / parity pk of row k advance without
  // division.
  // prefill: the state carried from token to token (this lane's elements)
  float carry_h[F][VW], carry_bx[F][VW], carry_a1 = 0.f, carry_av[F][NP];
  int k = 0, sk = 0, pass = 0;
  uint32_t pk = 0;
  for (; k < nrows; k += RP, ++pass) {
    const bool from_stage = !SEQ || k == 0;      // state from the ring (else registers)
    const bool write_state = !SEQ || k == nrows - 1;
    int sj[RP];
    uint32_t pj[RP];
    bool live[RP];
    int kj[RP];
    {
      int s_ = sk;
      uint32_t p_ = pk;
#pragma unroll
      for (int j = 0; j < RP; ++j) {
        live[j] = k + j < nrows;
        kj[j] = live[j] ? k + j : k;
        sj[j] = live[j] ? s_ : sj[0];
        pj[j] = live[j] ? p_ : pj[0];
        if (++s_ == S) {
          s_ = 0;
          p_ ^= 1u;
        }
      }
      sk = s_;
      pk = p_;
    }
    bool ok = true;
#pragma unroll
    for (int j = 0; j < RP; ++j)
      if (j == 0 || live[j]) ok = mbar_wait(smem_addr(&bars[sj[j]]), pj[j]) && ok;
    if (pass == 0 && par_smem) load_params();  // staged with row 0

    // ---- phase A: RMSNorm of each row's 2R B/C rows (src/models/mamba3.py:34-36) ----
#pragma unroll
    for (int j = 0; j < RP; ++j) {
      if (j > 0 && !live[j]) continue;
      const unsigned char *st = ring + (size_t)sj[j] * L.stage_bytes;
      float *nb = nbc + ((pass & 1) * RP + j) * 2 * R * BD;
      const T *sbc = reinterpret_cast<const T *>(st + L.o_bc);
#pragma unroll
      for (int q = 0; q < NRW; ++q) {
        const int rr = warp + kWarps * q;
        if (rr < 2 * R) {
          float v[F][VW];
          float ss = 0.f;
#pragma unroll
          for (int f = 0; f < F; ++f) {
            const int col = (lane + 32 * f) * VW;
            if (col < D) {
              lds_f<VW, T>(sbc + rr * D + col, v[f]);
            } else {
#pragma unroll
              for (int e = 0; e < VW; ++e) v[f][e] = 0.f;
            }
#pragma unroll
            for (int e = 0; e < VW; ++e) ss = fmaf(v[f][e], v[f][e], ss);
          }
          ss = group_sum<32>(ss);
          const float rinv = rsqrtf(ss * inv_d + kRmsEps);
#pragma unroll
          for (int f = 0; f < F; ++f) {
            const int col = (lane + 32 * f) * VW;
            if (col < D) {
              float o[VW];
#pragma unroll
              for (int e = 0; e < VW; ++e) o[e] = __fmul_rn(__fmul_rn(v[f][e], rinv), wn[q][f][e]);
              if constexpr (VW == 4)
                *reinterpret_cast<float4 *>(nb + rr * BD + col) = make_float4(o[0], o[1], o[2], o[3]);
              else
                *reinterpret_cast<float2 *>(nb + rr * BD + col) = make_float2(o[0], o[1]);
            }
          }
        }
      }
    }
    if (k == 0) table_store(0);
    // next table chunk: raw scalars requested 8 rows before they are stored,
    // stored 16 rows before the chunk starts (its buffer was last read two or
    // more passes ago, which the barriers since then have retired)
    if (k % kTableRows == kTableRows / 4 && (k / kTableRows + 1) * kTableRows < nrows) table_load(k / kTableRows + 1);
    if (k % kTableRows == kTableRows / 2 && (k / kTableRows + 1) * kTableRows < nrows) table_store(k / kTableRows + 1);

    // the one barrier of a pass: normalised rows visible, the previous
    // pass's stages free
    if (__syncthreads_or(!ok)) break;
    if (tid == 0) {
#pragma unroll
      for (int j = 0; j < RP; ++j) {
        const int kn = k + S - RP + j;  // into the stage of row k - RP + j
        if (kn < nrows) {
          int sn = sj[0] - RP + j;
          if (sn < 0) sn += S;
          issue_state(kn, sn);
          issue_zx(kn, sn);
        }
      }
    }

    // ---- phase B: this warp's head, RP rows ----
    const unsigned char *st[RP];
    const float *nbj[RP];
    float4 hs[RP];
#pragma unroll
    for (int j = 0; j < RP; ++j) {
      st[j] = ring + (size_t)sj[j] * L.stage_bytes;
      nbj[j] = nbc + ((pass & 1) * RP + j) * 2 * R * BD;
      hs[j] = table[((kj[j] / kTableRows) & 1) * kTableRows * kWarps + (kj[j] % kTableRows) * kWarps + warp];
    }

    // accumulated angles of this lane's RoPE pairs, written back
    // (src/models/mamba3.py:326-327); angle_state + angle_raw * DT, rounded
    // after each operation as the reference's two tensor operations are
    float rc[RP][F][NP], rs[RP][F][NP];
    if (NP == 2 && A <= 32) {
      // lanes own pairs (2l, 2l+1): one angle per lane, then each lane
      // fetches the cos/sin of its two pairs
      float a[RP], sn[RP], cs[RP];
#pragma unroll
      for (int j = 0; j < RP; ++j) {
        a[j] = 0.f;
        if (lane < A) {
          const float *sang = reinterpret_cast<const float *>(st[j] + L.o_ang) + warp * A;
          const T *sraw = reinterpret_cast<const T *>(st[j] + L.o_araw);
          float raw[1];
          lds_f<1, T>(sraw + lane, raw);
          a[j] = __fadd_rn(from_stage ? sang[lane] : carry_a1, __fmul_rn(raw[0], hs[j].w));
          if constexpr (SEQ) carry_a1 = a[j];
          if (live[j] && write_state) p.ang[(srow(kj[j]) * H + hh) * A + lane] = a[j];
        }
      }
      rope_sincos_n<RP>(a, sn, cs);
      const int src = (2 * lane) & 31;
      const bool mine = 2 * lane < A;
#pragma unroll
      for (int j = 0; j < RP; ++j) {
        const float c0 = __shfl_sync(kFullMask, cs[j], src), s0 = __shfl_sync(kFullMask, sn[j], src);
        const float c1 = __shfl_sync(kFullMask, cs[j], src + 1), s1 = __shfl_sync(kFullMask, sn[j], src + 1);
        rc[j][0][0] = mine ? c0 : 1.f;
        rs[j][0][0] = mine ? s0 : 0.f;
        rc[j][0][NP - 1] = mine ? c1 : 1.f;
        rs[j][0][NP - 1] = mine ? s1 : 0.f;
#pragma unroll
        for (int f = 1; f < F; ++f)
#pragma unroll
          for (int q = 0; q < NP; ++q) {
            rc[j][f][q] = 1.f;
            rs[j][f][q] = 0.f;
          }
      }
    } else {
      // every lane computes its own pairs (A is a multiple of 4, so a
      // vector's NP pairs rotate together)
#pragma unroll
      for (int f = 0; f < F; ++f) {
        const int i0 = (lane + 32 * f) * NP;
        const bool on = i0 < A;
        const int ic = on ? i0 : 0;
        float a[RP * NP], sn[RP * NP], cs[RP * NP];
#pragma unroll
        for (int j = 0; j < RP; ++j) {
          const float *sang = reinterpret_cast<const float *>(st[j] + L.o_ang) + warp * A;
          const T *sraw = reinterpret_cast<const T *>(st[j] + L.o_araw);
          float av[NP], raw[NP];
          if (from_stage) {
            lds_f<NP, float>(sang + ic, av);
          } else {
#pragma unroll
            for (int q = 0; q < NP; ++q) av[q] = carry_av[f][q];
          }
          lds_f<NP, T>(sraw + ic, raw);
#pragma unroll
          for (int q = 0; q < NP; ++q) av[q] = __fadd_rn(av[q], __fmul_rn(raw[q], hs[j].w));
          if constexpr (SEQ) {
#pragma unroll
            for (int q = 0; q < NP; ++q) carry_av[f][q] = av[q];
          }
          if (on && live[j] && write_state) stg_f<NP>(p.ang + (srow(kj[j]) * H + hh) * A + i0, av);
#pragma unroll
          for (int q = 0; q < NP; ++q) a[j * NP + q] = av[q];
        }
        rope_sincos_n<RP * NP>(a, sn, cs);
#pragma unroll
        for (int j = 0; j < RP; ++j)
#pragma unroll
          for (int q = 0; q < NP; ++q) {
            rc[j][f][q] = on ? cs[j * NP + q] : 1.f;
            rs[j][f][q] = on ? sn[j * NP + q] : 0.f;
          }
      }
    }

    // x_r = sum_p x_p mimo_x[h, r, p]
    float xr[RP][R];
#pragma unroll
    for (int j = 0; j < RP; ++j) {
      const T *sx = reinterpret_cast<const T *>(st[j] + L.o_x) + warp * P;
      float xv[PL];
      lds_f<PL, T>(sx + lane * PL, xv);
#pragma unroll
      for (int r = 0; r < R; ++r) {
        float t = 0.f;
#pragma unroll
        for (int q = 0; q < PL; ++q) {
          float m;
          if constexpr (KEEP_M) {
            m = mx[r][q];
          } else {
            float t1[1];
            ld_param<1>(par_smem, par, L.p_mx + ((warp * R + r) * P + lane * PL + q) * es, mxp + r * P + lane * PL + q, t1);
            m = t1[0];
          }
          t = fmaf(xv[q], m, t);
        }
        xr[j][r] = t;
      }
    }
#pragma unroll
    for (int j = 0; j < RP; ++j) row::warp_allreduce_ranks<R>(xr[j]);

    // Bx = RoPE(sum_r x_r (Bn_r + bias_r)), the trapezoidal update, and the
    // readout y_r = <Cn_r + cbias_r, RoPE^-1(h)> (rotations are orthogonal)
    float2 part[RP][R];
#pragma unroll
    for (int j = 0; j < RP; ++j)
#pragma unroll
      for (int r = 0; r < R; ++r) part[j][r] = f2(0.f, 0.f);
#pragma unroll
    for (int f = 0; f < F; ++f) {
      const int col = (lane + 32 * f) * VW;
      if (col < D) {
        float hv[RP][VW], bp[RP][VW];
        float2 acc[RP][NP];
#pragma unroll
        for (int j = 0; j < RP; ++j) {
          if (from_stage) {
            lds_f<VW, float>(reinterpret_cast<const float *>(st[j] + L.o_h) + warp * D + col, hv[j]);
            lds_f<VW, float>(reinterpret_cast<const float *>(st[j] + L.o_bx) + warp * D + col, bp[j]);
          } else {
#pragma unroll
            for (int e = 0; e < VW; ++e) {
              hv[j][e] = carry_h[f][e];
              bp[j][e] = carry_bx[f][e];
            }
          }
#pragma unroll
          for (int q = 0; q < NP; ++q) acc[j][q] = f2(0.f, 0.f);
        }
#pragma unroll
        for (int r = 0; r < R; ++r) {
          float bias[VW];
          if constexpr (KEEP_B) {
#pragma unroll
            for (int e = 0; e < VW; ++e) bias[e] = bb[r][f][e];
          } else {
            ld_param<VW>(par_smem, par, L.p_bB + ((warp * R + r) * D + col) * es, bBp + r * D + col, bias);
          }
#pragma unroll
          for (int j = 0; j < RP; ++j) {
            float n[VW];
            lds_f<VW, float>(nbj[j] + r * BD + col, n);
            const float2 xx = f2(xr[j][r], xr[j][r]);
#pragma unroll
            for (int q = 0; q < NP; ++q)
              acc[j][q] =
                  __ffma2_rn(xx, __fadd2_rn(f2(n[2 * q], n[2 * q + 1]), f2(bias[2 * q], bias[2 * q + 1])), acc[j][q]);
          }
        }
        float hr[RP][VW];
#pragma unroll
        for (int j = 0; j < RP; ++j) {
          const float2 dec2 = f2(hs[j].x, hs[j].x), c12 = f2(hs[j].y, hs[j].y), c22 = f2(hs[j].z, hs[j].z);
          float bxv[VW], hn[VW];
#pragma unroll
          for (int q = 0; q < NP; ++q) {
            const float c = rc[j][f][q], sn = rs[j][f][q];
            // rotations with their roundings spelled out, so that every
            // instantiation (one or two rows a pass) rounds a row alike
            bxv[2 * q] = fmaf(acc[j][q].x, c, __fmul_rn(-acc[j][q].y, sn));
            bxv[2 * q + 1] = fmaf(acc[j][q].x, sn, __fmul_rn(acc[j][q].y, c));
            const float2 t = __ffma2_rn(c22, f2(bp[j][2 * q], bp[j][2 * q + 1]),
                                        __ffma2_rn(c12, f2(bxv[2 * q], bxv[2 * q + 1]),
                                                   __fmul2_rn(dec2, f2(hv[j][2 * q], hv[j][2 * q + 1]))));
            hn[2 * q] = t.x;
            hn[2 * q + 1] = t.y;
            hr[j][2 * q] = fmaf(t.x, c, __fmul_rn(t.y, sn));
            hr[j][2 * q + 1] = fmaf(t.y, c, __fmul_rn(-t.x, sn));
          }
          if constexpr (SEQ) {
#pragma unroll
            for (int e = 0; e < VW; ++e) {
              carry_h[f][e] = hn[e];
              carry_bx[f][e] = bxv[e];
            }
          }
          if (live[j] && write_state) {
            const int64_t gbase = (srow(kj[j]) * H + hh) * D;
            stg_f<VW>(p.h + gbase + col, hn);
            stg_f<VW>(p.bx + gbase + col, bxv);
          }
        }
#pragma unroll
        for (int r = 0; r < R; ++r) {
          float bias[VW];
          if constexpr (KEEP_B) {
#pragma unroll
            for (int e = 0; e < VW; ++e) bias[e] = bc[r][f][e];
          } else {
            ld_param<VW>(par_smem, par, L.p_bC + ((warp * R + r) * D + col) * es, bCp + r * D + col, bias);
          }
#pragma unroll
          for (int j = 0; j < RP; ++j) {
            float n[VW];
            lds_f<VW, float>(nbj[j] + (R + r) * BD + col, n);
#pragma unroll
            for (int q = 0; q < NP; ++q)
              part[j][r] = __ffma2_rn(__fadd2_rn(f2(n[2 * q], n[2 * q + 1]), f2(bias[2 * q], bias[2 * q + 1])),
                                      f2(hr[j][2 * q], hr[j][2 * q + 1]), part[j][r]);
          }
        }
      }
    }
    float yr[RP][R];
#pragma unroll
    for (int j = 0; j < RP; ++j)
#pragma unroll
      for (int r = 0; r < R; ++r) yr[j][r] = part[j][r].x + part[j][r].y;
#pragma unroll
    for (int j = 0; j < RP; ++j) row::warp_allreduce_ranks<R>(yr[j]);

    // y_p = sum_r (y_r + D x_r) mimo_o[h, r, p], gated by silu(z)
#pragma unroll
    for (int j = 0; j < RP; ++j) {
      const T *sz = reinterpret_cast<const T *>(st[j] + L.o_z) + warp * P;
      float zv[PL], yv[PL];
      lds_f<PL, T>(sz + lane * PL, zv);
#pragma unroll
      for (int q = 0; q < PL; ++q) {
        float t = 0.f;
#pragma unroll
        for (int r = 0; r < R; ++r) {
          float m;
          if constexpr (KEEP_M) {
            m = mo[r][q];
          } else {
            float t1[1];
            ld_param<1>(par_smem, par, L.p_mo + ((warp * R + r) * P + lane * PL + q) * es, mop + r * P + lane * PL + q, t1);
            m = t1[0];
          }
          t = fmaf(fmaf(dskip, xr[j][r], yr[j][r]), m, t);
        }
        yv[q] = t * __fdividef(zv[q], 1.f + __expf(-zv[q]));
      }
      if (live[j]) st_y<PL>(p.y, zrow(kj[j]) * p.y_sb + (int64_t)hh * P + lane * PL, yv, p.y_dt);
    }
  }
  // Normal exit: every issued row was consumed.  After a lost copy, wait
  // (bounded) for this CTA's copies still in flight before leaving.
  if (tid == 0 && k < nrows) {
    for (int q = k; q < min(nrows, k + S - RP); ++q)
      mbar_wait(smem_addr(&bars[q % S]), (uint32_t)((q / S) & 1));  // full bound: a copy may still land
  }
}

int align16(int x) { return (x + 15) & ~15; }

int num_sms_cached() { return sm_count_current(); }

bool aligned(const void *p, unsigned a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; }

// Whether every copy of the streamed kernel starts on a 16-byte boundary and
// moves a multiple of 16 bytes, and every vector access is aligned.
bool stream_eligible(const KParams &kp) {
  const int es = kp.zx_dt == M3_BF16 ? 2 : 4, esy = kp.y_dt == M3_BF16 ? 2 : 4;
  if (kp.zx_dt != kp.par_dt || kp.H % kWarps != 0 || kp.d_bc != kp.R * kp.D) return false;
  if (kp.P % 32 != 0 || kp.P > 128 || kp.D < 33 || kp.D > 256 || kp.D % 4 != 0 || kp.A % 4 != 0) return false;
  if (!aligned(kp.zx, 16) || !aligned(kp.h, 16) || !aligned(kp.bx, 16) || !aligned(kp.ang, 16) || !aligned(kp.y, 16) ||
      !aligned(kp.bB, 16) || !aligned(kp.bC, 16) || !aligned(kp.mx, 16) || !aligned(kp.mo, 16) ||
      !aligned(kp.wB, 16) || !aligned(kp.wC, 16))
    return false;
  if ((kp.zx_sb * es) % 16 || (kp.y_sb * esy) % 16 || (2 * kp.d_inner * es) % 16) return false;
  const int64_t so = 2 * (int64_t)kp.d_inner + 2 * (int64_t)kp.d_bc;
  if (((so + 3 * kp.H) * es) % 16 || (kp.A * es) % 16 || (2 * kp.R * kp.D * es) % 16) return false;
  return true;
}

StreamLayout make_layout(const KParams &kp, int BD, int nstage, int rp, bool stage_par) {
  const int es = kp.zx_dt == M3_BF16 ? 2 : 4;
  StreamLayout L = {};
  L.n_state = (unsigned)(kWarps * kp.D * 4);
  L.n_ang = (unsigned)(kWarps * kp.A * 4);
  L.n_xz = (unsigned)(kWarps * kp.P * es);
  L.n_bc = (unsigned)(2 * kp.R * kp.D * es);
  L.n_araw = (unsigned)(kp.A * es);
  L.tx_state = 2 * L.n_state + L.n_ang;
  L.tx = L.tx_state + 2 * L.n_xz + L.n_bc + L.n_araw;
  int o = 0;
  L.o_h = o; o += align16((int)L.n_state);
  L.o_bx = o; o += align16((int)L.n_state);
  L.o_ang = o; o += align16((int)L.n_ang);
  L.o_x = o; o += align16((int)L.n_xz);
  L.o_z = o; o += align16((int)L.n_xz);
  L.o_bc = o; o += align16((int)L.n_bc);
  L.o_araw = o; o += align16((int)L.n_araw);
  L.stage_bytes = align16(o);
  L.nstage = nstage;
  int g = 0;
  L.o_bars = g; g += align16(kMaxStages * 8);
  L.o_table = g; g += 2 * kTableRows * kWarps * 16;
  L.o_nbc = g; g += 2 * rp * 2 * kp.R * BD * 4;
  L.o_ring = g; g += nstage * L.stage_bytes;
  L.o_par = -1;
  L.n_bBC = (unsigned)(kWarps * kp.R * kp.D * es);
  L.n_mxo = (unsigned)(kWarps * kp.R * kp.P * es);
  L.n_w = (unsigned)(kp.D * es);
  L.n_h8 = (unsigned)(kWarps * es);
  const bool can = (L.n_w % 16) == 0 && aligned(kp.Dp, 16) && aligned(kp.dt_bias, 16);
  if (stage_par && can) {
    L.o_par = g;
    L.p_bB = 0;
    L.p_bC = L.p_bB + (int)L.n_bBC;
    L.p_mx = L.p_bC + (int)L.n_bBC;
    L.p_mo = L.p_mx + (int)L.n_mxo;
    L.p_wB = L.p_mo + (int)L.n_mxo;
    L.p_wC = L.p_wB + (int)L.n_w;
    L.p_Dp = L.p_wC + (int)L.n_w;
    L.p_dtb = L.p_Dp + (int)L.n_h8;
    L.n_par = (unsigned)(L.p_dtb + (int)L.n_h8);
    g += (int)L.n_par;
  }
  L.smem = g;
  return L;
}

template <int BD, int R, typename T, int PL, int RP, bool SEQ>
cudaError_t launch_stream_rp(const KParams &kp, const StreamLayout &L, cudaStream_t stream) {
  auto kern = mimo_stream_kernel<BD, R, T, PL, RP, SEQ>;
  static LaunchCache cache;
  if (cudaError_t e = ensure_smem_optin(cache, kern, 227 * 1024); e != cudaSuccess) return e;
  const int ngrp = kp.H / kWarps;
  if constexpr (SEQ) {  // one CTA per (sequence, head group), all tokens of it
    const int64_t grid = (int64_t)ngrp * kp.B;
    return launch_pdl(kern, dim3((unsigned)grid), dim3(kWarps * 32), (size_t)L.smem, stream, kp, L, 0);
  }
  int per_sm = 0;
  if (occupancy_per_sm(cache, kern, kWarps * 32, (size_t)L.smem, &per_sm) != cudaSuccess || per_sm < 1) per_sm = 1;
  const int sms = num_sms_cached();
  const int64_t slots = (int64_t)sms * per_sm;
  const int64_t items = (int64_t)kp.B * ngrp;
  int rows = (int)((items + slots - 1) / slots);
  if (rows < 1) rows = 1;
  const int64_t grid = (int64_t)ngrp * ((kp.B + rows - 1) / rows);
  return launch_pdl(kern, dim3((unsigned)grid), dim3(kWarps * 32), (size_t)L.smem, stream, kp, L, rows);
}

// Ring depth: up to 4 stages (no deeper than the CTA's rows -- batch rows,
// or tokens in a prefill -- need), with the per-head parameters staged in
// shared memory when that still lets two CTAs share an SM (else they are
// read from global memory in the prologue).  One row a pass: two-row passes
// (RP = 2) were measured slower per row (3.0 us a pass against 0.9 us a row
// at d2048 / batch 256).
template <int BD, int R, typename T, int PL, bool SEQ>
cudaError_t launch_stream_t(const KParams &kp, cudaStream_t stream) {
  const int ngrp = kp.H / kWarps;
  const int64_t slots = (int64_t)num_sms_cached() * 2;
  const int64_t rows = SEQ ? (int64_t)kp.L : ((int64_t)kp.B * ngrp + slots - 1) / slots;
  int want = (int)(rows + 1 < 4 ? rows + 1 : 4);
  if (want < 2) want = 2;
  StreamLayout L = make_layout(kp, BD, want, 1, true);
  if (L.smem > 110 * 1024) {
    L = make_layout(kp, BD, 2, 1, false);
    for (int s = want; s >= 2; --s) {
      L = make_layout(kp, BD, s, 1, false);
      if (L.smem <= 110 * 1024) break;
    }
  }
  if (L.smem > 227 * 1024) return cudaErrorInvalidValue;
  return launch_stream_rp<BD, R, T, PL, 1, SEQ>(kp, L, stream);
}

template <int BD, int R, typename T, bool SEQ>
cudaError_t launch_stream_p(const KParams &kp, cudaStream_t stream) {
  if (kp.P == 32) return launch_stream_t<BD, R, T, 1, SEQ>(kp, stream);
  if (kp.P == 64) return launch_stream_t<BD, R, T, 2, SEQ>(kp, stream);
  return launch_stream_t<BD, R, T, 4, SEQ>(kp, stream);  // P == 128 (others are not taken)
}

template <int BD, typename T, bool SEQ>
cudaError_t launch_stream_r(const KParams &kp, cudaStream_t stream) {
  switch (kp.R) {
    case 1: return launch_stream_p<BD, 1, T, SEQ>(kp, stream);
    case 2: return launch_stream_p<BD, 2, T, SEQ>(kp, stream);
    case 4: return launch_stream_p<BD, 4, T, SEQ>(kp, stream);
    default: return launch_stream_p<BD, 8, T, SEQ>(kp, stream);
  }
}

template <typename T, bool SEQ>
cudaError_t launch_stream_d(const KParams &kp, cudaStream_t stream) {
  if (kp.D <= 64) return launch_stream_r<64, T, SEQ>(kp, stream);
  if (kp.D <= 128) return launch_stream_r<128, T, SEQ>(kp, stream);
  return launch_stream_r<256, T, SEQ>(kp, stream);
}

bool stream_takes(const KParams &kp) {
  return stream_eligible(kp) && (kp.P == 32 || kp.P == 64 || kp.P == 128) &&
         (kp.R == 1 || kp.R == 2 || kp.R == 4 || kp.R == 8);
}

}  // namespace

cudaError_t launch_mimo_stream(const KParams &kp, cudaStream_t stream, bool *taken) {
  *taken = false;
  if (!stream_takes(kp)) return cudaSuccess;
  *taken = true;
  return kp.zx_dt == M3_BF16 ? launch_stream_d<__nv_bfloat16, false>(kp, stream)
                             : launch_stream_d<float, false>(kp, stream);
}

cudaError_t launch_mimo_prefill(const KParams &kp, cudaStream_t stream, bool *taken) {
  *taken = false;
  if (kp.L < 1 || !stream_takes(kp)) return cudaSuccess;
  *taken = true;
  return kp.zx_dt == M3_BF16 ? launch_stream_d<__nv_bfloat16, true>(kp, stream)
                             : launch_stream_d<float, true>(kp, stream);
}

int mimo_stream_device_error(bool reset) { return device_error_of_this_unit(reset); }

}  // namespace m3
