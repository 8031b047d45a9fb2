// Skinny bf16 projection GEMM for decode batches of up to 64 rows.
//
// C[M, N] = X[M, K] . W[N, K]^T (nn.Linear without bias, the decode step's
// in_proj / out_proj, src/models/mamba3.py:115,158) when M, the number of
// sequences a GPU decodes, is small: the weight is then read once from HBM
// and the batch rows are tiny, so the GEMM is a stream of the weight through
// the tensor cores, and what sets its speed is how many weight bytes are in
// flight per SM.
//
//   * mma.sync.m16n8k16 (bf16 in, fp32 accumulate).  A 16x16 A fragment
//     holds, on lane (g = lane / 4, q = lane % 4), elements (g | g + 8,
//     2q + {0, 1} | 2q + 8 + {0, 1}); the B fragment (g, 2q + {0, 1} |
//     2q + 8 + {0, 1}).  The sum over k does not depend on the order of k,
//     so the kernel gives its k index a permutation under which those are
//     exactly the eight consecutive elements [8q, 8q + 8) of a 32-wide K
//     block: lane q's one 16-byte load of a weight row (and of each of its
//     two batch rows) feeds two MMAs, physical k 8q + {0..3} in the first and
//     8q + {4..7} in the second; the four lanes of a group cover the block.
//   * A warp owns NT * 8 weight rows and a run of K blocks, and keeps MT x NT
//     accumulator tiles (all the batch rows).  Its lanes stream their
//     16-byte pieces of the weight rows (from HBM) and of the batch rows (L2
//     hits: the batch operand is read by every CTA) into a private S-stage
//     ring in shared memory with cp.async, S - 1 K blocks ahead of the MMAs;
//     each lane reads back only what it wrote, so the ring needs no barrier.
//   * The 8 warps of a CTA split the CTA's K range, and the CS CTAs of a
//     thread-block cluster split K between them: the warps' partial tiles
//     are added in shared memory in warp order, then each CTA of the cluster
//     adds its share of the tile over the cluster's CTAs in rank order
//     through distributed shared memory and writes it -- a fixed order
//     throughout, so results are deterministic.
#include "m3_kernels.cuh"

namespace m3 {

namespace {

constexpr int kSkinnySmemBudget = 200 * 1024;

__device__ __forceinline__ uint32_t skinny_smem_addr(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// 16 bytes global -> shared, bypassing L1: the first `bytes` (16 or 0)
// read from `src`, the rest of the 16 zero-filled.
__device__ __forceinline__ void cp_async16(uint32_t dst, const void *src, uint32_t bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(bytes) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

__device__ __forceinline__ void skinny_cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ uint32_t skinny_cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ float ld_peer_f32(uint32_t addr, uint32_t rank) {
  uint32_t a;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(a) : "r"(addr), "r"(rank));
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(a) : "memory");
  return v;
}

// d (+)= a . b for one m16n8k16 tile (not volatile: the compiler may
// interleave independent tiles).
__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  asm(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

template <int MT, int NT, int S, int WARPS>
constexpr size_t skinny_smem_bytes() {
  return (size_t)WARPS * S * (NT + 2 * MT) * 32 * 16;
}

// MT: 16-row tiles of the batch (M <= 16 MT); NT: 8-row tiles of the weight
// per warp (a CTA's N tile is NT * 8 rows); S: ring stages; WARPS: warps
// of a CTA; MINB: CTAs per SM the registers are budgeted for.  The grid is (N tiles x CS) CTAs in clusters of CS along K; a
// CTA takes kbc K blocks of 32 and each of its warps kpw of those.
template <int MT, int NT, int S, int WARPS, int MINB>
__global__ void __launch_bounds__(WARPS * 32, MINB)
    skinny_kernel(const __nv_bfloat16 *__restrict__ X, int64_t ldx, const __nv_bfloat16 *__restrict__ W, int64_t ldw,
                  void *C, int64_t ldc, int M, int N, int K, int c_bf16, int cs, int kbc, int kpw) {
  constexpr int SLOTS = NT + 2 * MT;  // 16-byte pieces per lane per K block
  constexpr int PER = MT * NT * 4;    // accumulator floats per lane
  static_assert(WARPS * 32 * PER * sizeof(float) <= skinny_smem_bytes<MT, NT, S, WARPS>(),
                "the reduction reuses the ring");
  extern __shared__ __align__(16) uint4 ring[];  // [warps][S][SLOTS][32 lanes]
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = lane >> 2, q = lane & 3;
  const uint32_t rank = skinny_cluster_rank();
  const int n0 = (blockIdx.x / cs) * NT * 8;
  const int nkb = (K + 31) / 32;
  const int cb0 = (int)rank * kbc, cb1 = min(nkb, cb0 + kbc);
  const int kb0 = cb0 + warp * kpw, kb1 = min(cb1, kb0 + kpw);

  // this lane's weight rows and batch rows, and the bytes each of its
  // pieces reads (0 past the last row: the piece is zero-filled and reads
  // nothing; the address is then clamped to the operand's first row)
  const __nv_bfloat16 *wrow[NT];
  uint32_t wsz[NT];
#pragma unroll
  for (int t = 0; t < NT; ++t) {
    const int n = n0 + t * 8 + g;
    wsz[t] = n < N ? 16u : 0u;
    wrow[t] = W + (int64_t)(n < N ? n : 0) * ldw + 8 * q;
  }
  const __nv_bfloat16 *xrow[MT][2];
  uint32_t xsz[MT][2];
#pragma unroll
  for (int t = 0; t < MT; ++t)
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int m = t * 16 + g + 8 * h;
      xsz[t][h] = m < M ? 16u : 0u;
      xrow[t][h] = X + (int64_t)(m < M ? m : 0) * ldx + 8 * q;
    }

  uint4 *mine = ring + (size_t)warp * S * SLOTS * 32 + lane;
  const uint32_t mine_s = skinny_smem_addr(mine);
  // stage K block kb into ring slot `slot` (an empty group past the warp's range)
  auto issue = [&](int kb, int slot) {
    if (kb < kb1) {
      // K is a multiple of 8, so a piece is wholly inside or past the end
      // of its row; past the end it reads nothing at the row's start
      const bool kok = kb * 32 + 8 * q < K;
      const int k = kok ? kb * 32 : 0;
      const uint32_t base = mine_s + (uint32_t)(slot * SLOTS * 32 * 16);
#pragma unroll
      for (int t = 0; t < NT; ++t) cp_async16(base + t * 512, wrow[t] + k, kok ? wsz[t] : 0u);
#pragma unroll
      for (int t = 0; t < MT; ++t)
#pragma unroll
        for (int h = 0; h < 2; ++h)
          cp_async16(base + (NT + 2 * t + h) * 512, xrow[t][h] + k, kok ? xsz[t][h] : 0u);
    }
    cp_async_commit();
  };

  float acc[MT][NT][4];
#pragma unroll
  for (int a = 0; a < MT; ++a)
#pragma unroll
    for (int b = 0; b < NT; ++b)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[a][b][e] = 0.f;

  pdl_wait();  // the batch rows are the preceding kernel's output
  pdl_trigger();
#pragma unroll
  for (int s = 0; s < S - 1; ++s) issue(kb0 + s, s);
  int slot = 0, fill = S - 1;
  for (int kb = kb0; kb < kb1; ++kb) {
    issue(kb + S - 1, fill);
    cp_async_wait<S - 1>();
    const uint4 *p = mine + slot * SLOTS * 32;
    uint4 wv[NT], xv[MT][2];
#pragma unroll
    for (int t = 0; t < NT; ++t) wv[t] = p[t * 32];
#pragma unroll
    for (int t = 0; t < MT; ++t)
#pragma unroll
      for (int h = 0; h < 2; ++h) xv[t][h] = p[(NT + 2 * t + h) * 32];
    // physical k 8q + 0..3 for every tile (A rows g / g + 8, B column g),
    // then 8q + 4..7: a tile's two products are MT x NT issues apart
#pragma unroll
    for (int a = 0; a < MT; ++a)
#pragma unroll
      for (int b = 0; b < NT; ++b)
        mma16816(acc[a][b], xv[a][0].x, xv[a][1].x, xv[a][0].y, xv[a][1].y, wv[b].x, wv[b].y);
#pragma unroll
    for (int a = 0; a < MT; ++a)
#pragma unroll
      for (int b = 0; b < NT; ++b)
        mma16816(acc[a][b], xv[a][0].z, xv[a][1].z, xv[a][0].w, xv[a][1].w, wv[b].z, wv[b].w);
    slot = slot + 1 == S ? 0 : slot + 1;
    fill = fill + 1 == S ? 0 : fill + 1;
  }
  cp_async_wait_all();
  __syncthreads();  // every warp is done with its ring: the reduction reuses it

  // partial tiles of the CTA's warps, added in warp order into warp 0's slots
  float *red = reinterpret_cast<float *>(ring);  // [warps][32 lanes][PER]
  {
    float *dst = red + ((size_t)warp * 32 + lane) * PER;
#pragma unroll
    for (int a = 0; a < MT; ++a)
#pragma unroll
      for (int b = 0; b < NT; ++b)
#pragma unroll
        for (int e = 0; e < 4; ++e) dst[(a * NT + b) * 4 + e] = acc[a][b][e];
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < 32 * PER; idx += blockDim.x) {
    float s = red[idx];
    for (int w = 1; w < WARPS; ++w) s += red[(size_t)w * 32 * PER + idx];
    red[idx] = s;
  }
  // the cluster's partial tiles, added in rank order; CTA `rank` writes
  // fragment positions [rank * share, (rank + 1) * share)
  skinny_cluster_sync();
  const int share = (32 * PER + cs - 1) / cs;
  const int i0 = (int)rank * share, i1 = min(32 * PER, i0 + share);
  const uint32_t red_s = skinny_smem_addr(red);
  for (int idx = i0 + threadIdx.x; idx < i1; idx += blockDim.x) {
    float s = 0.f;
    for (int c = 0; c < cs; ++c) s += ld_peer_f32(red_s + idx * 4, (uint32_t)c);
    // fragment position -> (batch row, weight row)
    const int ln = idx / PER, r = idx - ln * PER;
    const int e = r & 3, ab = r >> 2, b = ab % NT, a = ab / NT;
    const int m = a * 16 + (ln >> 2) + ((e & 2) ? 8 : 0);
    const int n = n0 + b * 8 + 2 * (ln & 3) + (e & 1);
    if (m < M && n < N) {
      if (c_bf16)
        static_cast<__nv_bfloat16 *>(C)[(int64_t)m * ldc + n] = __float2bfloat16_rn(s);
      else
        static_cast<float *>(C)[(int64_t)m * ldc + n] = s;
    }
  }
  skinny_cluster_sync();  // no CTA leaves while another reads its shared memory
}

// The K split over a cluster of CS CTAs: the CS that minimises waves / CS
// over `slots` resident CTAs (each CTA's share of the stream shrinks with
// CS), smallest on ties, such that every warp keeps at least one K block.
inline int skinny_cluster_split(int tiles, int nkb, int warps, int slots) {
  int cs = 1;
  double best = 1e30;
  for (int c = 1; c <= 8; c *= 2) {
    if (c > 1 && (nkb + c - 1) / c < warps) break;
    const double cost = (double)((tiles * c + slots - 1) / slots) / c;
    if (cost < best * 0.999) best = cost, cs = c;
  }
  return cs;
}

template <int MT, int NT, int S, int WARPS, int MINB = 1>
cudaError_t launch_skinny_t(const void *x, int64_t ldx, const void *w, int64_t ldw, void *y, int64_t ldy, int M,
                            int N, int K, bool y_bf16, int cs, cudaStream_t stream) {
  auto kern = skinny_kernel<MT, NT, S, WARPS, MINB>;
  constexpr size_t smem = skinny_smem_bytes<MT, NT, S, WARPS>();
  static_assert(smem <= kSkinnySmemBudget, "ring too large");
  static LaunchCache cache;
  if (cudaError_t e = ensure_smem_optin(cache, kern, (int)smem); e != cudaSuccess) return e;
  const int tiles = (N + NT * 8 - 1) / (NT * 8);
  const int nkb = (K + 31) / 32;
  if (cs <= 0) {
    int per_sm = 1;
    if (cudaError_t e = occupancy_per_sm(cache, kern, WARPS * 32, smem, &per_sm); e != cudaSuccess) return e;
    cs = skinny_cluster_split(tiles, nkb, WARPS, sm_count_current() * (per_sm > 0 ? per_sm : 1));
  }
  const int kbc = (nkb + cs - 1) / cs;
  const int kpw = (kbc + WARPS - 1) / WARPS;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(tiles * cs));
  cfg.blockDim = dim3(WARPS * 32);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = (unsigned)cs;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, static_cast<const __nv_bfloat16 *>(x), ldx,
                                     static_cast<const __nv_bfloat16 *>(w), ldw, y, ldy, M, N, K, y_bf16 ? 1 : 0, cs,
                                     kbc, kpw);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

}  // namespace

bool gemm_skinny_supported(const void *x, int64_t ldx, const void *w, int64_t ldw, const void *y, int64_t ldy, int M,
                           int N, int K) {
  auto al = [](const void *p, unsigned a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; };
  return M >= 0 && M <= kSkinnyMaxRows && N > 0 && K > 0 && K % 8 == 0 && ldx % 8 == 0 && ldw % 8 == 0 &&
         ldx >= K && ldw >= K && ldy >= N && al(x, 16) && al(w, 16) && al(y, 4);
}

cudaError_t launch_gemm_skinny(const void *x, int64_t ldx, const void *w, int64_t ldw, void *y, int64_t ldy, int M,
                               int N, int K, bool y_bf16, cudaStream_t stream) {
  // Tile shapes measured fastest on B200 for the d_model 2048 stack's
  // in_proj (9440 x 2048) and out_proj (2048 x 4096): at 16 rows, 32-row
  // weight tiles and 3 stages with two CTAs per SM (16 warps); at 32 and
  // 64 rows one CTA per SM (the accumulators' registers).
  if (M <= 16) return launch_skinny_t<1, 4, 3, 8, 2>(x, ldx, w, ldw, y, ldy, M, N, K, y_bf16, 0, stream);
  if (M <= 32) return launch_skinny_t<2, 4, 3, 8, 1>(x, ldx, w, ldw, y, ldy, M, N, K, y_bf16, 0, stream);
  return launch_skinny_t<4, 4, 4, 8, 1>(x, ldx, w, ldw, y, ldy, M, N, K, y_bf16, 0, stream);
}

}  // namespace m3
