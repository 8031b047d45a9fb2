// SISO prefill: the full SISO step in sequence form.
//
// One CTA per (sequence b, head hh) walks the sequence's L tokens.  The
// head's (P, D) state tile stays in the registers of eight update warps
// from the first token to the last (read once, written once); the previous
// token's B x is rank one (x_prev[p] * B_prev[d]) and is rebuilt from the
// previous token's x and B in shared memory, so only the incoming bx_prev
// of token 0 is read from global memory and only the last token's B x is
// written back.
//
// Tokens move in chunks of TC.  A chunk's slices of the in_proj rows (the
// B|C rows, the head's x and z, the scalar section) arrive by bulk copies
// into one of two ring slots on one mbarrier.  Four producer warps prepare
// a whole chunk while the update warps advance the state through the
// previous one, each warp a quarter of the chunk's tokens: RMSNorm of the B and
// C rows, the norm weights and the head's biases, the rotation of both by
// the accumulated angles (one sin/cos per angle serves both rows), x and
// silu(z), and the head scalars (warp 8, every token).  The tokens a warp
// prepares are independent chains (only the angle accumulation runs token
// after token, per lane, and both warps run it over the whole chunk so
// that each carries the angles on), so their latencies overlap; with two
// producer warps the update warps still waited for them at the barrier.  One CTA
// barrier per chunk hands a chunk from the producers to
// the update warps, which run the chunk's tokens back to back; three chunk
// buffers hold the chunk being updated, the one before it (its last token's
// x and B) and the one being prepared.
//
// Per element and token the update is
//     h = exp(A DT) h + DT (1 - trap/2) x[p] B[d] + DT trap/2 x_prev[p] B_prev[d]
// (the exponential-trapezoidal step of src/kernels/utils.py:73-102 with its
// two B x terms grouped per row), y[p] = (sum_d C[d] h[p, d] + D x[p]) silu(z[p]).
// Reference: src/kernels/fused_full_decode.py:37-225 applied token after
// token, as src/models/mamba3.py:242-304 walks a sequence.
#include <type_traits>

#include "m3_async.cuh"
#include "m3_kernels.cuh"

namespace m3 {

namespace {

constexpr int kUpdWarps = 8;
constexpr int kPrepWarps = 4;
constexpr int kThreads = (kUpdWarps + kPrepWarps) * 32;
constexpr int kSlots = 2;        // ring slots (chunks in flight)
constexpr int kChunkBufs = 3;    // prepared-chunk buffers
constexpr int kMaxHFloats = 64;  // state floats per update thread

template <int BD>
struct PrefShape {
  static constexpr int BG = BD / 4;             // float4 columns per row (padded)
  static constexpr int S = BG < 8 ? BG : 8;     // lanes per row
  static constexpr int FPL = BG / S;            // float4 per lane per row
  static constexpr int RPW = 32 / S;            // rows per warp per pass
  static constexpr int ROWS = kUpdWarps * RPW;  // rows per pass of the CTA
  static constexpr int KPL = BD >= 32 ? BD / 32 : 1;  // producer elements per lane
  static constexpr int TC = BD >= 256 ? 4 : 12;  // tokens per chunk
};

// Byte offsets of the shared-memory regions.
struct PrefLayout {
  int o_w;          // wB[BD] wC[BD] bias_B[BD] bias_C[BD] (floats)
  int o_chunk;      // kChunkBufs x chunk buffer
  int tok_floats;   // per token: sB[BD] sC[BD] sX[P] sG[P] sc[4], padded to float4
  int chunk_bytes;
  int o_ring;       // kSlots x TC stages
  int stage_bytes;
  int s_raw, s_x, s_z, s_scal;  // offsets inside a stage
  int tx;           // bytes landing per token
  int smem;
};

int align128(int x) { return (x + 127) / 128 * 128; }

PrefLayout make_layout(const KParams &kp, int BD, int TC) {
  const int es = kp.zx_dt == M3_BF16 ? 2 : 4;
  PrefLayout L;
  L.o_w = 128;  // the ring's barriers first
  L.tok_floats = (2 * BD + 2 * kp.P + 4 + 3) / 4 * 4;
  L.chunk_bytes = align128(TC * L.tok_floats * 4);
  L.o_chunk = L.o_w + align128(4 * BD * 4);
  L.o_ring = L.o_chunk + kChunkBufs * L.chunk_bytes;
  int o = 0;
  L.s_raw = o; o += align128(2 * kp.D * es);
  L.s_x = o; o += align128(kp.P * es);
  L.s_z = o; o += align128(kp.P * es);
  L.s_scal = o; o += align128((3 * kp.H + kp.A) * es);
  L.stage_bytes = o;
  L.tx = 2 * kp.D * es + 2 * kp.P * es + (3 * kp.H + kp.A) * es;
  L.smem = L.o_ring + kSlots * TC * L.stage_bytes;
  return L;
}

template <typename T> __device__ __forceinline__ float to_f(T v);
template <> __device__ __forceinline__ float to_f<float>(float v) { return v; }
template <> __device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }

__device__ __forceinline__ float2 f2(float a) { return make_float2(a, a); }

template <int BD, int NP, typename T>
__global__ void __launch_bounds__(kThreads, 2) siso_prefill_kernel(const KParams p, const PrefLayout lay) {
  using Sh = PrefShape<BD>;
  constexpr int S = Sh::S, FPL = Sh::FPL, RPW = Sh::RPW, ROWS = Sh::ROWS, KPL = Sh::KPL, TC = Sh::TC;

  extern __shared__ __align__(128) unsigned char smem_raw[];
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem_raw);
  float *wB = reinterpret_cast<float *>(smem_raw + lay.o_w);
  float *wC = wB + BD, *bBh = wC + BD, *bCh = bBh + BD;
  unsigned char *ring = smem_raw + lay.o_ring;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int H = p.H, P = p.P, D = p.D, A = p.A, G = D >> 2, L = p.L;
  const int b = blockIdx.x / H, hh = blockIdx.x - b * H;
  const int tile = blockIdx.x;  // (b, hh) of the state tensors
  const int nchunk = (L + TC - 1) / TC;
  const bool producer = warp >= kUpdWarps;
  const bool issuer = tid == kUpdWarps * 32;  // lane 0 of warp 8

  auto ntok = [&](int c) { return min(TC, L - c * TC); };
  // prepared token t: sB = tok(t), sC = +BD, sX = +2BD, sG = +2BD+P, sc = +2BD+2P
  auto tok = [&](int t) {
    return reinterpret_cast<float *>(smem_raw + lay.o_chunk + ((t / TC) % kChunkBufs) * lay.chunk_bytes) +
           (t % TC) * lay.tok_floats;
  };
  auto stage = [&](int c, int i) { return ring + (size_t)((c % kSlots) * TC + i) * lay.stage_bytes; };
  // all copies of chunk c into its slot, on the slot's barrier (issuer only)
  auto issue_chunk = [&](int c) {
    const int n = ntok(c);
    const uint32_t bar = smem_addr(&bars[c % kSlots]);
    const int es = (int)sizeof(T);
    mbar_arrive_expect_tx(bar, (uint32_t)(n * lay.tx));
    for (int i = 0; i < n; ++i) {
      unsigned char *st = stage(c, i);
      const T *row = static_cast<const T *>(p.zx) + ((int64_t)b * L + c * TC + i) * p.zx_sb;
      bulk_g2s(smem_addr(st + lay.s_raw), row + 2 * p.d_inner, (uint32_t)(2 * D * es), bar);
      bulk_g2s(smem_addr(st + lay.s_x), row + p.d_inner + (int64_t)hh * P, (uint32_t)(P * es), bar);
      bulk_g2s(smem_addr(st + lay.s_z), row + (int64_t)hh * P, (uint32_t)(P * es), bar);
      bulk_g2s(smem_addr(st + lay.s_scal), row + 2 * p.d_inner + 2 * p.d_bc, (uint32_t)((3 * H + A) * es), bar);
    }
  };

  if (tid == 0) {
    for (int s = 0; s < kSlots; ++s) mbar_init(smem_addr(&bars[s]), 1);
    mbar_init_fence();
  }
  // per-CTA constants: norm weights, the head's biases, dt_bias and D
  for (int i = tid; i < BD; i += kThreads) {
    const bool in = i < D;
    wB[i] = in ? ld_any(p.wB, i, p.par_dt) : 0.f;
    wC[i] = in ? ld_any(p.wC, i, p.par_dt) : 0.f;
    bBh[i] = in ? ld_any(p.bB, (int64_t)hh * D + i, p.par_dt) : 0.f;
    bCh[i] = in ? ld_any(p.bC, (int64_t)hh * D + i, p.par_dt) : 0.f;
  }
  const float dtb = ld_any(p.dt_bias, hh, p.par_dt);
  const float dskip = ld_any(p.Dp, hh, p.par_dt);

  // Warp roles.  Both branches pass the same CTA barriers in the same
  // order: one after the constants, one after chunk 0's preparation, one per
  // chunk; a lost copy (a producer's wait that gave up) ends every loop at
  // the same barrier.
  const int rsub = lane / S, j = lane % S;
  if (producer) {
    const int pw = warp - kUpdWarps;  // tokens [pw * TH, (pw + 1) * TH) of each chunk
    const float invD = 1.f / (float)D;
    constexpr int TH = TC / kPrepWarps;
    float ang[KPL];  // carried angles (written two or more kernels back)
#pragma unroll
    for (int k = 0; k < KPL; ++k) {
      const int d = lane + 32 * k;
      ang[k] = d < 2 * A ? p.ang[(int64_t)tile * A + (d >> 1)] : 0.f;
    }
    pdl_wait();  // the in_proj rows are the preceding kernel's product
    pdl_trigger();
    __syncthreads();  // barriers initialised, constants in shared memory
    int issued = 0;
    if (issuer)
      for (; issued < kSlots && issued < nchunk; ++issued) issue_chunk(issued);

    // Chunk c's parameters into its buffer: RMSNorm + weight + head bias +
    // RoPE of the B and C rows of each token (src/models/mamba3.py:202-215,
    // 326-333; src/kernels/utils.py:31-44), the angles advanced by
    // angle_raw * DT token after token.
    auto prepare = [&](int c) -> bool {
      if (!mbar_wait(smem_addr(&bars[c % kSlots]), (uint32_t)((c / kSlots) & 1))) return false;
      const int n = ntok(c);
      // this chunk's ring slot and token buffers, addressed from two bases
      const unsigned char *slot = stage(c, 0);
      const int sbytes = lay.stage_bytes, tf = lay.tok_floats;
      float *cbuf = tok(c * TC);
      // DT of token i on lane i, then to every lane
      float dt_l = 0.f;
      if (lane < n) dt_l = softplus_f(to_f(reinterpret_cast<const T *>(slot + lane * sbytes + lay.s_scal)[hh]) + dtb);
      float DT[TC];
#pragma unroll
      for (int i = 0; i < TC; ++i) DT[i] = __shfl_sync(kFullMask, dt_l, i);
      if (pw == 0 && lane < n) {  // head scalars of token `lane`
        const T *scal = reinterpret_cast<const T *>(slot + lane * sbytes + lay.s_scal);
        const float sp = softplus_f(to_f(scal[H + hh]));
        const float Ah = -(sp > -p.A_floor ? -p.A_floor : sp);  // clamp keeps NaN like torch
        const float tr = sigmoid_f(to_f(scal[2 * H + hh]));
        const float htr = tr * 0.5f;
        float *sc = cbuf + lane * tf + 2 * BD + 2 * P;
        sc[0] = expf(Ah * dt_l);
        sc[1] = dt_l * ((1.f - tr) + htr);
        sc[2] = dt_l * htr;
      }
      // the angle accumulation over the whole chunk; this warp keeps the
      // angles of its own tokens
      float an[TH][KPL];
#pragma unroll
      for (int i = 0; i < TC; ++i) {
        const bool live = i < n;
        const T *araw = reinterpret_cast<const T *>(slot + (live ? i : 0) * sbytes + lay.s_scal) + 3 * H;
#pragma unroll
        for (int k = 0; k < KPL; ++k) {
          const int d = lane + 32 * k;
          if (live && d < 2 * A) ang[k] = ang[k] + to_f(araw[d >> 1]) * DT[i];
          if (i / TH == pw) an[i % TH][k] = ang[k];
        }
      }
      // raw B and C rows of this warp's tokens, their squared sums
      float vb[TH][KPL], vc[TH][KPL], sb[TH], scq[TH];
#pragma unroll
      for (int u = 0; u < TH; ++u) {
        const int i = pw * TH + u;
        const bool live = i < n;
        const T *raw = reinterpret_cast<const T *>(slot + (live ? i : 0) * sbytes + lay.s_raw);
        sb[u] = 0.f;
        scq[u] = 0.f;
#pragma unroll
        for (int k = 0; k < KPL; ++k) {
          const int d = lane + 32 * k;
          vb[u][k] = (live && d < D) ? to_f(raw[d]) : 0.f;
          vc[u][k] = (live && d < D) ? to_f(raw[D + d]) : 0.f;
          sb[u] += vb[u][k] * vb[u][k];
          scq[u] += vc[u][k] * vc[u][k];
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1)
#pragma unroll
        for (int u = 0; u < TH; ++u) {
          sb[u] += __shfl_xor_sync(kFullMask, sb[u], o);
          scq[u] += __shfl_xor_sync(kFullMask, scq[u], o);
        }
#pragma unroll
      for (int u = 0; u < TH; ++u) {
        const int i = pw * TH + u;
        const float ib = rsqrtf(sb[u] * invD + kRmsEps);
        const float ic = rsqrtf(scq[u] * invD + kRmsEps);
        float sn[KPL], cs[KPL];
        rope_sincos_n<KPL>(an[u], sn, cs);
        float *out = cbuf + (i < n ? i : 0) * tf;
#pragma unroll
        for (int k = 0; k < KPL; ++k) {
          const int d = lane + 32 * k;
          float xb = vb[u][k], xc = vc[u][k];
          if (d < D) {
            xb = xb * ib * wB[d] + bBh[d];
            xc = xc * ic * wC[d] + bCh[d];
          }
          const bool rot = d < 2 * A;
          const float ob = __shfl_xor_sync(kFullMask, xb, 1);
          const float oc = __shfl_xor_sync(kFullMask, xc, 1);
          if (rot) {
            xb = (d & 1) ? ob * sn[k] + xb * cs[k] : xb * cs[k] - ob * sn[k];
            xc = (d & 1) ? oc * sn[k] + xc * cs[k] : xc * cs[k] - oc * sn[k];
          }
          if (i < n && d < BD) {
            out[d] = d < D ? xb : 0.f;
            out[BD + d] = d < D ? xc : 0.f;
          }
        }
      }
      // x and silu(z) of this warp's tokens
#pragma unroll
      for (int u = 0; u < TH; ++u) {
        const int i = pw * TH + u;
        if (i >= n) break;
        const T *xs = reinterpret_cast<const T *>(slot + i * sbytes + lay.s_x);
        const T *zs = reinterpret_cast<const T *>(slot + i * sbytes + lay.s_z);
        float *dst = cbuf + i * tf + 2 * BD;
        for (int e = lane; e < P; e += 32) {
          const float z = to_f(zs[e]);
          dst[e] = to_f(xs[e]);
          dst[P + e] = __fdividef(z, 1.f + __expf(-z));
        }
      }
      return true;
    };

    bool failed = __syncthreads_or(!prepare(0));
    if (!failed && issuer && issued < nchunk) issue_chunk(issued++);
    for (int c = 0; !failed && c < nchunk; ++c) {
      const bool ok = c + 1 < nchunk ? prepare(c + 1) : true;
      failed = __syncthreads_or(!ok);
      // the slot of chunk c + 1 is consumed: refill it
      if (!failed && issuer && issued < nchunk) issue_chunk(issued++);
    }
    if (failed) {
      // A lost copy: the state is left as it was.  Wait (bounded) for the
      // chunks still in flight (the last kSlots issued) before leaving.
      if (issuer)
        for (int k = issued > kSlots ? issued - kSlots : 0; k < issued; ++k)
          mbar_wait(smem_addr(&bars[k % kSlots]), (uint32_t)((k / kSlots) & 1));  // full bound: a copy may still land
      return;
    }
    if (pw == 0) {
#pragma unroll
      for (int k = 0; k < KPL; ++k) {
        const int d = lane + 32 * k;
        if (d < 2 * A && !(d & 1)) p.ang[(int64_t)tile * A + (d >> 1)] = ang[k];
      }
    }
    return;
  }

  // update warps: the (P, D) tile in registers (written two or more kernels
  // back, so it may be read before pdl_wait())
  float4 hreg[NP][FPL];
  {
    const float *hg = p.h + (size_t)tile * P * D;
#pragma unroll
    for (int q = 0; q < NP; ++q) {
      const int r = q * ROWS + warp * RPW + rsub;
#pragma unroll
      for (int f = 0; f < FPL; ++f) {
        const int col = j + S * f;
        hreg[q][f] = (r < P && col < G) ? reinterpret_cast<const float4 *>(hg + (size_t)r * D)[col]
                                        : make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
  }
  pdl_wait();
  pdl_trigger();
  __syncthreads();

  // Token t (prepared parameters at cur, token t - 1's at prv): h advanced
  // in registers, y rows stored.  FIRST: the previous B x comes from the
  // bx_prev state, else from prv.
  const int64_t ybase = (int64_t)b * L * p.y_sb + (int64_t)hh * P;
  auto update = [&](int t, const float *cur, const float *prv, auto first_tag) {
    constexpr bool FIRST = decltype(first_tag)::value;
    const float *sc = cur + 2 * BD + 2 * P;
    const float2 dec2 = f2(sc[0]);
    const float a1 = sc[1], a2 = sc[2];
    // column groups outer, passes inner: each float4 of B, C and the
    // previous B is read from shared memory once and used for every row
    float xv[NP];
    float2 ax[NP], axp[NP], acc[NP];
#pragma unroll
    for (int q = 0; q < NP; ++q) {
      const int r = q * ROWS + warp * RPW + rsub;
      xv[q] = r < P ? cur[2 * BD + r] : 0.f;
      ax[q] = f2(a1 * xv[q]);
      axp[q] = f2(0.f);
      if constexpr (!FIRST) axp[q] = f2(a2 * (r < P ? prv[2 * BD + r] : 0.f));
      acc[q] = f2(0.f);
    }
#pragma unroll
    for (int f = 0; f < FPL; ++f) {
      const int col = j + S * f;
      const float4 Bq = reinterpret_cast<const float4 *>(cur)[col];
      const float4 Cq = reinterpret_cast<const float4 *>(cur + BD)[col];
      float4 Bp = make_float4(0.f, 0.f, 0.f, 0.f);
      if constexpr (!FIRST) Bp = reinterpret_cast<const float4 *>(prv)[col];
#pragma unroll
      for (int q = 0; q < NP; ++q) {
        float2 lo, hi;
        if constexpr (FIRST) {
          const int r = q * ROWS + warp * RPW + rsub;
          float4 bo = make_float4(0.f, 0.f, 0.f, 0.f);
          if (r < P && col < G) bo = reinterpret_cast<const float4 *>(p.bx + ((size_t)tile * P + r) * D)[col];
          lo = __fmul2_rn(f2(a2), make_float2(bo.x, bo.y));
          hi = __fmul2_rn(f2(a2), make_float2(bo.z, bo.w));
        } else {
          lo = __fmul2_rn(axp[q], make_float2(Bp.x, Bp.y));
          hi = __fmul2_rn(axp[q], make_float2(Bp.z, Bp.w));
        }
        lo = __ffma2_rn(ax[q], make_float2(Bq.x, Bq.y), lo);
        hi = __ffma2_rn(ax[q], make_float2(Bq.z, Bq.w), hi);
        float2 h0 = make_float2(hreg[q][f].x, hreg[q][f].y), h1 = make_float2(hreg[q][f].z, hreg[q][f].w);
        h0 = __ffma2_rn(dec2, h0, lo);
        h1 = __ffma2_rn(dec2, h1, hi);
        hreg[q][f] = make_float4(h0.x, h0.y, h1.x, h1.y);
        acc[q] = __ffma2_rn(make_float2(Cq.x, Cq.y), h0, acc[q]);
        acc[q] = __ffma2_rn(make_float2(Cq.z, Cq.w), h1, acc[q]);
      }
    }
#pragma unroll
    for (int q = 0; q < NP; ++q) {
      const int r = q * ROWS + warp * RPW + rsub;
      const float part = group_sum<S>(acc[q].x + acc[q].y);
      if (j == 0 && r < P) {
        const float yv = (part + dskip * xv[q]) * cur[2 * BD + P + r];
        st_any(p.y, ybase + (int64_t)t * p.y_sb + r, yv, p.y_dt);
      }
    }
  };

  bool failed = __syncthreads_or(false);
  for (int c = 0; !failed && c < nchunk; ++c) {
    const int n = ntok(c);
    int i = 0;
    const int tf = lay.tok_floats;
    const float *cb = tok(c * TC);
    if (c == 0) {
      update(0, cb, cb, std::true_type{});
      i = 1;
    }
    // token i of the chunk follows token i - 1 (the previous chunk's last for i = 0)
    for (const float *prv = i ? cb : tok(c * TC - 1); i < n; ++i) {
      update(c * TC + i, cb + i * tf, prv, std::false_type{});
      prv = cb + i * tf;
    }
    failed = __syncthreads_or(false);
  }
  if (failed) return;

  // write the carried state back once: h and the last token's B x (rank one)
  const float *last = tok(L - 1);
  float *hw = p.h + (size_t)tile * P * D;
  float *bw = p.bx + (size_t)tile * P * D;
#pragma unroll
  for (int q = 0; q < NP; ++q) {
    const int r = q * ROWS + warp * RPW + rsub;
    if (r >= P) continue;
    const float xv = last[2 * BD + r];
#pragma unroll
    for (int f = 0; f < FPL; ++f) {
      const int col = j + S * f;
      if (col < G) {
        const float4 Bl = reinterpret_cast<const float4 *>(last)[col];
        reinterpret_cast<float4 *>(hw + (size_t)r * D)[col] = hreg[q][f];
        reinterpret_cast<float4 *>(bw + (size_t)r * D)[col] = make_float4(xv * Bl.x, xv * Bl.y, xv * Bl.z, xv * Bl.w);
      }
    }
  }
}

bool aligned16(const void *q) { return (reinterpret_cast<uintptr_t>(q) & 15u) == 0; }

// Rows per update thread: the smallest NP in {1, 2, 4} with NP passes
// covering P and at most kMaxHFloats state floats per thread.
template <int BD>
int passes_for(int P) {
  using Sh = PrefShape<BD>;
  for (int np = 1; np <= 4; np *= 2)
    if (np * Sh::ROWS >= P && np * Sh::FPL * 4 <= kMaxHFloats) return np;
  return 0;
}

template <int BD, int NP, typename T>
cudaError_t launch_np(const KParams &kp, const PrefLayout &lay, cudaStream_t stream) {
  auto kern = siso_prefill_kernel<BD, NP, T>;
  static LaunchCache cache;
  if (lay.smem > 48 * 1024)
    if (cudaError_t e = ensure_smem_optin(cache, kern, lay.smem); e != cudaSuccess) return e;
  return launch_pdl(kern, dim3((unsigned)(kp.B * kp.H)), dim3(kThreads), (size_t)lay.smem, stream, kp, lay);
}

template <int BD, typename T>
cudaError_t launch_bd(const KParams &kp, const PrefLayout &lay, int np, cudaStream_t stream) {
  constexpr int FPL = PrefShape<BD>::FPL;
  if (np == 1) return launch_np<BD, 1, T>(kp, lay, stream);
  if constexpr (2 * FPL * 4 <= kMaxHFloats)
    if (np == 2) return launch_np<BD, 2, T>(kp, lay, stream);
  if constexpr (4 * FPL * 4 <= kMaxHFloats)
    if (np == 4) return launch_np<BD, 4, T>(kp, lay, stream);
  return cudaErrorInvalidValue;
}

template <int BD>
cudaError_t launch_dt(const KParams &kp, bool *taken, cudaStream_t stream) {
  const int np = passes_for<BD>(kp.P);
  if (np == 0) return cudaSuccess;
  const PrefLayout lay = make_layout(kp, BD, PrefShape<BD>::TC);
  if (lay.smem > 110 * 1024) return cudaSuccess;  // two CTAs per SM
  *taken = true;
  return kp.zx_dt == M3_BF16 ? launch_bd<BD, __nv_bfloat16>(kp, lay, np, stream)
                             : launch_bd<BD, float>(kp, lay, np, stream);
}

// Whether every copy of a token's header starts on a 16-byte boundary and
// moves a multiple of 16 bytes, and the state rows are float4-addressable.
bool prefill_eligible(const KParams &kp) {
  const int es = kp.zx_dt == M3_BF16 ? 2 : 4;
  if (kp.R != 1 || kp.D % 4 || kp.D > 256 || kp.L <= 0) return false;
  if (!aligned16(kp.zx) || !aligned16(kp.h) || !aligned16(kp.bx)) return false;
  if ((kp.zx_sb * es) % 16 || (kp.d_inner * es) % 16 || (2 * kp.D * es) % 16) return false;
  if ((kp.P * es) % 16 || ((3 * kp.H + kp.A) * es) % 16) return false;
  if ((int64_t)kp.B * kp.H > 0x7fffffff) return false;
  return true;
}

}  // namespace

cudaError_t launch_siso_prefill(const KParams &kp, cudaStream_t stream, bool *taken) {
  *taken = false;
  if (!prefill_eligible(kp)) return cudaSuccess;
  if (kp.D <= 16) return launch_dt<16>(kp, taken, stream);
  if (kp.D <= 32) return launch_dt<32>(kp, taken, stream);
  if (kp.D <= 64) return launch_dt<64>(kp, taken, stream);
  if (kp.D <= 128) return launch_dt<128>(kp, taken, stream);
  return launch_dt<256>(kp, taken, stream);
}

int siso_prefill_device_error(bool reset) { return device_error_of_this_unit(reset); }

}  // namespace m3
