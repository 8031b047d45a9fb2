// bf16 projection GEMM on the 5th-generation tensor cores (tcgen05).
//
// y[M, N] = x[M, K] . w[N, K]^T for the decode step's projections
// (nn.Linear without bias, src/models/mamba3.py:115,158), where M is the
// batch and N, K are layer widths.  The weight rows are the MMA's M
// dimension (128 per CTA) and the batch rows its N dimension (up to 256 per
// CTA), so a decode batch of <= 256 rows is one tile column:
//
//   * warp 0 / lane 0 streams k-tiles of 64 elements through an S-stage
//     shared-memory ring with TMA (cp.async.bulk.tensor.2d, 128-byte swizzle):
//     the weight tile (128 x 64) and the batch tile (NB x 64);
//   * warp 1 / lane 0 issues four tcgen05.mma (kind::f16: bf16 operands,
//     fp32 accumulation) per k-tile into one TMEM accumulator of 128 lanes x
//     NB columns, and hands each stage back with tcgen05.commit;
//   * the tile width (batch rows per CTA) and a K split are planned per call
//     so that the CTAs fill the SMs; a split runs its CTAs as one thread-block
//     cluster (up to 4): every CTA writes its fp32 partial tile to the
//     caller's workspace, and after a cluster barrier CTA j sums slice j of the
//     batch rows over the cluster's partials (from L2) and writes it.
//     Distributed shared memory was tried for that exchange and measured at
//     about 15 GB/s per CTA -- far slower than L2.
//
// All four warps drain TMEM (tcgen05.ld, warp w owns lanes 32w..32w+31).
// Every mbarrier wait is bounded and records M3_DEVERR_TIMEOUT when it gives
// up; the cluster barrier is reached on every path.  No load uses cluster
// multicast.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "m3_async.cuh"
#include "m3_kernels.cuh"

namespace m3 {

namespace {

constexpr int kTileN = 128;  // weight rows per CTA (MMA M)
constexpr int kTileK = 64;   // k per stage: one 128-byte swizzle row of bf16
constexpr int kThreads = 128;
constexpr int kMaxSplit = 4;
constexpr int kSmemBudget = 200 * 1024;
constexpr int kMaxStages = 8;

struct GemmArgs {
  int M, N;
  int nb;          // batch rows per tile (multiple of 16, <= 256)
  int ktiles;      // k-tiles per split
  int ktotal;      // k-tiles of K
  int nsplit;      // CTAs per cluster along K
  int nstage;      // ring depth
  int stage_a;     // bytes of a weight tile
  int stage_b;     // bytes of a batch tile
  int tmem_cols;   // allocated accumulator columns
  void *y;
  int64_t ldy;
  int y_bf16;
  float *ws;       // split-K partial tiles (nsplit > 1)
};

// UMMA shared-memory descriptor of a K-major operand in the 128-byte swizzle
// layout TMA writes: rows of 128 bytes, 8-row groups 1024 bytes apart
// (stride byte offset), descriptor version 1, layout type 2 (128B swizzle).
// Stepping K by 16 elements inside the swizzle row adds 32 bytes to the
// start address.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFF) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap *map, int x, int y, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}

__device__ __forceinline__ void mma_bf16(uint32_t tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem),
      "l"(a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}

__device__ __forceinline__ void mma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// 16 consecutive accumulator columns of this thread's TMEM lane (read them
// after tmem_wait).
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

__global__ void __launch_bounds__(kThreads, 1)
    gemm_bf16_kernel(const __grid_constant__ CUtensorMap tw, const __grid_constant__ CUtensorMap tx, const GemmArgs g) {
  extern __shared__ unsigned char smem_raw[];
  unsigned char *smem =
      reinterpret_cast<unsigned char *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  const int S = g.nstage;
  unsigned char *ringA = smem;
  unsigned char *ringB = smem + (size_t)S * g.stage_a;
  const int ring_bytes = S * (g.stage_a + g.stage_b);
  const int part_bytes = g.nb * kTileN * 4;
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + (ring_bytes > part_bytes ? ring_bytes : part_bytes));
  uint64_t *full = bars, *empty = bars + S, *accum = bars + 2 * S;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 2 * S + 1);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n0 = blockIdx.x * kTileN, m0 = blockIdx.y * g.nb;
  const int split = blockIdx.z;  // rank in the cluster (cluster dims 1 x 1 x nsplit)
  const int kt0 = split * g.ktiles;
  const int nkt = max(0, min(g.ktiles, g.ktotal - kt0));

  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(tmem_slot)),
                 "r"(g.tmem_cols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (tid == 32) {
    for (int s = 0; s < S; ++s) {
      mbar_init(smem_addr(&full[s]), 1);
      mbar_init(smem_addr(&empty[s]), 1);
    }
    mbar_init(smem_addr(accum), 1);
    mbar_init_fence();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  // the weights are constant: the first stages' weight tiles are requested
  // before waiting for the preceding kernel, whose product the batch rows are
  const int npre = min(S, nkt);
  if (tid == 0) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tw)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tx)) : "memory");
    for (int i = 0; i < npre; ++i) {
      const uint32_t bar = smem_addr(&full[i]);
      mbar_arrive_expect_tx(bar, (uint32_t)(g.stage_a + g.stage_b));
      tma_load_2d(smem_addr(ringA + (size_t)i * g.stage_a), &tw, (kt0 + i) * kTileK, n0, bar);
    }
  }
  pdl_wait();
  pdl_trigger();

  if (tid == 0) {
    // producer: k-tile i into stage i % S, after the MMAs of k-tile i - S
    // have released it
    for (int i = 0; i < npre; ++i)
      tma_load_2d(smem_addr(ringB + (size_t)i * g.stage_b), &tx, (kt0 + i) * kTileK, m0, smem_addr(&full[i]));
    int s = npre % S;
    uint32_t ph = npre == S ? 1u : 0u;
    int issued = npre;
    for (int i = npre; i < nkt; ++i) {
      if (!mbar_wait(smem_addr(&empty[s]), ph ^ 1u)) break;
      const uint32_t bar = smem_addr(&full[s]);
      mbar_arrive_expect_tx(bar, (uint32_t)(g.stage_a + g.stage_b));
      const int kx = (kt0 + i) * kTileK;
      tma_load_2d(smem_addr(ringA + (size_t)s * g.stage_a), &tw, kx, n0, bar);
      tma_load_2d(smem_addr(ringB + (size_t)s * g.stage_b), &tx, kx, m0, bar);
      issued = i + 1;
      if (++s == S) {
        s = 0;
        ph ^= 1u;
      }
    }
    // every copy this thread issued has landed before the CTA moves on
    // (immediate on the normal path, where the MMAs consumed them)
    for (int j = issued > S ? issued - S : 0; j < issued; ++j)
      mbar_wait(smem_addr(&full[j % S]), (uint32_t)((j / S) & 1));  // full bound: a copy may still land
  } else if (tid == 32) {
    // MMA issuer: D[128 x nb] (+)= W_tile[128 x 64] . X_tile[nb x 64]^T
    const uint32_t idesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(g.nb >> 3) << 17) |
                           ((uint32_t)(kTileN >> 4) << 24);
    int s = 0;
    uint32_t ph = 0;
    for (int i = 0; i < nkt; ++i) {
      if (!mbar_wait(smem_addr(&full[s]), ph)) break;
      tc_fence_after();
      const uint32_t a0 = smem_addr(ringA + (size_t)s * g.stage_a);
      const uint32_t b0 = smem_addr(ringB + (size_t)s * g.stage_b);
#pragma unroll
      for (int j = 0; j < kTileK / 16; ++j)
        mma_bf16(tmem, sw128_desc(a0 + 32 * j), sw128_desc(b0 + 32 * j), idesc, (i | j) != 0 ? 1u : 0u);
      mma_commit(smem_addr(&empty[s]));
      if (++s == S) {
        s = 0;
        ph ^= 1u;
      }
    }
    mma_commit(smem_addr(accum));  // arrives once every MMA issued above has completed
  }
  __syncwarp();

  mbar_wait(smem_addr(accum), 0);
  __syncwarp();
  tc_fence_after();
  const int nl = 32 * warp + lane;
  const uint32_t trow = tmem + ((uint32_t)(32 * warp) << 16);
  // Drain the accumulator 64 columns (batch rows) at a time: up to four
  // tcgen05.ld per wait; `put(m, value)` stores column m of this thread's row.
  auto drain = [&](auto &&put) {
    for (int c0 = 0; c0 < g.nb; c0 += 64) {  // nb is a multiple of 16
      uint32_t v[4][16];
#pragma unroll
      for (int q = 0; q < 4; ++q)
        if (c0 + 16 * q < g.nb) tmem_ld16(trow + (uint32_t)(c0 + 16 * q), v[q]);
      tmem_wait();
#pragma unroll
      for (int q = 0; q < 4; ++q)
        if (c0 + 16 * q < g.nb)
#pragma unroll
          for (int j = 0; j < 16; ++j) put(c0 + 16 * q + j, nkt > 0 ? __uint_as_float(v[q][j]) : 0.f);
    }
  };
  const int n = n0 + 4 * lane;
  auto store_row = [&](int m, const float4 a4) {
    const float o[4] = {a4.x, a4.y, a4.z, a4.w};
    if (g.y_bf16) {
      __nv_bfloat16 *yr = static_cast<__nv_bfloat16 *>(g.y) + (int64_t)m * g.ldy;
      if (n + 3 < g.N && ((g.ldy | n) & 3) == 0) {
        __nv_bfloat162 lo = __floats2bfloat162_rn(o[0], o[1]), hi = __floats2bfloat162_rn(o[2], o[3]);
        uint2 pk;
        pk.x = *reinterpret_cast<uint32_t *>(&lo);
        pk.y = *reinterpret_cast<uint32_t *>(&hi);
        *reinterpret_cast<uint2 *>(yr + n) = pk;
      } else {
#pragma unroll
        for (int e = 0; e < 4; ++e)
          if (n + e < g.N) yr[n + e] = __float2bfloat16_rn(o[e]);
      }
    } else {
      float *yr = static_cast<float *>(g.y) + (int64_t)m * g.ldy;
      if (n + 3 < g.N && ((g.ldy | n) & 3) == 0) {
        *reinterpret_cast<float4 *>(yr + n) = a4;
      } else {
#pragma unroll
        for (int e = 0; e < 4; ++e)
          if (n + e < g.N) yr[n + e] = o[e];
      }
    }
  };

  if (g.nsplit > 1) {
    // split-K: this CTA's fp32 partial tile -> workspace [m][n] (each warp
    // store one 128-byte row segment), a cluster barrier, then CTA `split`
    // sums batch rows [r0, r1) of the tile over the cluster's partials from L2
    const size_t tile = (size_t)blockIdx.y * gridDim.x + blockIdx.x;
    float *tws = g.ws + tile * g.nsplit * g.nb * kTileN;
    float *mine = tws + (size_t)split * g.nb * kTileN;
    drain([&](int m, float v) { __stcg(mine + (size_t)m * kTileN + nl, v); });
    tc_fence_before();
    cluster_sync();  // release / acquire at cluster scope: every partial is visible
    const int per = (g.nb + g.nsplit - 1) / g.nsplit;
    const int r0 = split * per, r1 = min(g.nb, r0 + per);
    constexpr int RU = 4;  // rows per warp and pass: RU x nsplit loads in flight
    for (int base = r0; base < r1; base += 4 * RU) {
      float4 acc[RU];
#pragma unroll
      for (int u = 0; u < RU; ++u) acc[u] = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int q = 0; q < kMaxSplit; ++q) {
        if (q < g.nsplit) {
#pragma unroll
          for (int u = 0; u < RU; ++u) {
            const int mm = base + 4 * u + warp;
            if (mm < r1) {
              const float4 t = __ldcg(reinterpret_cast<const float4 *>(tws + ((size_t)q * g.nb + mm) * kTileN + 4 * lane));
              acc[u].x += t.x; acc[u].y += t.y; acc[u].z += t.z; acc[u].w += t.w;
            }
          }
        }
      }
#pragma unroll
      for (int u = 0; u < RU; ++u) {
        const int mm = base + 4 * u + warp;
        if (mm < r1 && m0 + mm < g.M) store_row(m0 + mm, acc[u]);
      }
    }
  } else {
    // whole K here: accumulator -> shared memory part[m][n] (the ring it
    // overwrites was last written by TMA and read by the finished MMAs),
    // then coalesced row stores
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    float *part = reinterpret_cast<float *>(smem);
    drain([&](int m, float v) { part[m * kTileN + nl] = v; });
    tc_fence_before();
    __syncthreads();
    for (int mm = warp; mm < g.nb && m0 + mm < g.M; mm += 4)
      store_row(m0 + mm, *reinterpret_cast<const float4 *>(part + mm * kTileN + 4 * lane));
  }

  __syncthreads();
  tc_fence_after();
  if (warp == 0)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(g.tmem_cols) : "memory");
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// 2-D bf16 tensor map: `rows` rows of `cols` elements, `ld` elements apart;
// boxes of 64 columns x `box_rows` rows, 128-byte swizzle, zero fill.
bool make_map(CUtensorMap *map, const void *ptr, int64_t rows, int64_t cols, int64_t ld, int box_rows) {
  auto fn = encode_fn();
  if (fn == nullptr) return false;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(ld * 2)};
  cuuint32_t box[2] = {(cuuint32_t)kTileK, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(ptr), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int sm_count() { return sm_count_current(); }

// Tile width (batch rows per CTA) and K split of one call: the cheapest by
// a simple model -- each k-tile moves its weight and batch tiles at about
// 100 GB/s per SM (the operands mostly come from L2), CTAs beyond one per SM
// run in further waves, and a split adds the partial tiles' write and read.
struct GemmPlan {
  int nb, ntiles, mchunks, ktotal, ktiles, nsplit;
};

GemmPlan plan_gemm(int M, int N, int K) {
  const int sms = sm_count();
  const int ntiles = (N + kTileN - 1) / kTileN, ktotal = (K + kTileK - 1) / kTileK;
  const int mr = (M + 15) / 16 * 16;
  GemmPlan best = {};
  double best_cost = 1e30;
  for (int nb : {256, 128, 64, 32, 16}) {
    if (nb > mr && nb != 16 && (nb >> 1) >= mr) continue;  // skip widths twice the batch or more
    const int b = nb < mr ? nb : mr;
    const int mchunks = (M + b - 1) / b, tiles = ntiles * mchunks;
    int nsplit = tiles >= sms ? 1 : sms / tiles;
    nsplit = nsplit < 1 ? 1 : nsplit > kMaxSplit ? kMaxSplit : nsplit;
    if (nsplit > ktotal) nsplit = ktotal;
    const int ktiles = (ktotal + nsplit - 1) / nsplit;
    nsplit = (ktotal + ktiles - 1) / ktiles;  // every split gets at least one k-tile
    const int waves = (tiles * nsplit + sms - 1) / sms;
    const double us_per_ktile = (kTileN * kTileK * 2.0 + b * kTileK * 2.0) / 1.0e5;
    double cost = waves * ktiles * us_per_ktile + b * kTileN * 4.0 / 1.0e5;
    if (nsplit > 1) cost += 2.0 * b * kTileN * 4.0 / 1.0e5 + 0.7;
    if (cost < best_cost) {
      best_cost = cost;
      best = {b, ntiles, mchunks, ktotal, ktiles, nsplit};
    }
  }
  return best;
}

}  // namespace

bool gemm_bf16_supported(const void *x, int64_t ldx, const void *w, int64_t ldw, const void *y, int64_t ldy, int M,
                         int N, int K) {
  auto al = [](const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  return M > 0 && N > 0 && K >= kTileK && K % 8 == 0 && ldx % 8 == 0 && ldw % 8 == 0 && ldx >= K && ldw >= K &&
         ldy >= N && al(x) && al(w) && al(y) && encode_fn() != nullptr;
}

int64_t gemm_bf16_workspace_bytes(int M, int N, int K) {
  if (M <= 0 || N <= 0 || K < kTileK) return 0;
  const GemmPlan pl = plan_gemm(M, N, K);
  if (pl.nsplit <= 1) return 0;
  return (int64_t)pl.ntiles * pl.mchunks * pl.nsplit * pl.nb * kTileN * 4;
}

cudaError_t launch_gemm_bf16(const void *x, int64_t ldx, const void *w, int64_t ldw, void *y, int64_t ldy, int M,
                             int N, int K, bool y_bf16, float *workspace, cudaStream_t stream) {
  const GemmPlan pl = plan_gemm(M, N, K);
  GemmArgs g = {};
  g.M = M;
  g.N = N;
  g.nb = pl.nb;
  g.ktotal = pl.ktotal;
  g.ktiles = pl.ktiles;
  g.nsplit = pl.nsplit;
  if (g.nsplit > 1 && workspace == nullptr) return cudaErrorInvalidValue;
  g.ws = workspace;
  g.stage_a = kTileN * kTileK * 2;
  g.stage_b = g.nb * kTileK * 2;
  int S = kSmemBudget / (g.stage_a + g.stage_b);
  S = S > kMaxStages ? kMaxStages : S;
  if (S > g.ktiles) S = g.ktiles < 2 ? 2 : g.ktiles;
  g.nstage = S;
  g.tmem_cols = 32;
  while (g.tmem_cols < g.nb) g.tmem_cols <<= 1;
  g.y = y;
  g.ldy = ldy;
  g.y_bf16 = y_bf16 ? 1 : 0;
  const int ring = S * (g.stage_a + g.stage_b), part = g.nb * kTileN * 4;
  const int smem = 1024 + (ring > part ? ring : part) + (2 * S + 2) * 8;

  CUtensorMap tw, tx;
  if (!make_map(&tw, w, N, K, ldw, kTileN) || !make_map(&tx, x, M, K, ldx, g.nb)) return cudaErrorInvalidValue;

  static LaunchCache cache;
  if (cudaError_t e = ensure_smem_optin(cache, gemm_bf16_kernel, 227 * 1024); e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)pl.ntiles, (unsigned)pl.mchunks, (unsigned)g.nsplit);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = (size_t)smem;
  cfg.stream = stream;
  cudaLaunchAttribute attrs[2];
  int na = 0;
  attrs[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attrs[na].val.programmaticStreamSerializationAllowed = 1;
  ++na;
  if (g.nsplit > 1) {
    attrs[na].id = cudaLaunchAttributeClusterDimension;
    attrs[na].val.clusterDim.x = 1;
    attrs[na].val.clusterDim.y = 1;
    attrs[na].val.clusterDim.z = (unsigned)g.nsplit;
    ++na;
  }
  cfg.attrs = attrs;
  cfg.numAttrs = na;
  cudaError_t e = cudaLaunchKernelEx(&cfg, gemm_bf16_kernel, tw, tx, g);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

int gemm_device_error(bool reset) { return device_error_of_this_unit(reset); }

}  // namespace m3
