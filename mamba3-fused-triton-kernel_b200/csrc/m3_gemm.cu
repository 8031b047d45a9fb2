// bf16 projection GEMM on the 5th-generation tensor cores (tcgen05), for
// the decode step's projections (nn.Linear without bias,
// src/models/mamba3.py:115,158): y[M, N] = x[M, K] . w[N, K]^T, M the batch.
// One kernel, gemm_pair_kernel: pairs of SMs (tcgen05.mma.cta_group::2),
// TMA-fed shared-memory rings, fp32 accumulation in TMEM, an optional K
// split over independent pairs.  Design notes above the kernel.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "m3_async.cuh"
#include "m3_kernels.cuh"

namespace m3 {

namespace {

constexpr int kTileK = 64;  // k per stage: one 128-byte swizzle row of bf16

// Operand kinds of the paired-SM GEMM.
//   kKindBF16    bf16 operands, one tcgen05.mma (kind::f16) per 16 k
//   kKindTF32x3  fp32 operands given as TF32 heads and remainders
//                (x = hi + lo, hi exactly representable in TF32), three
//                tcgen05.mma (kind::tf32) per 8 k: hi.hi + hi.lo + lo.hi, the
//                split-precision product of ~fp32 accuracy (the dropped
//                lo.lo term is ~2^-22 relative)
constexpr int kKindBF16 = 0;
constexpr int kKindTF32x3 = 1;
template <int KIND> struct PairKind;
template <> struct PairKind<kKindBF16> {
  static constexpr int kTileK = 64;  // elements of a 128-byte row
  static constexpr int kPlanes = 1;  // operand planes per matrix
  static constexpr uint32_t kFormat = 1;  // BF16
};
template <> struct PairKind<kKindTF32x3> {
  static constexpr int kTileK = 32;
  static constexpr int kPlanes = 2;  // hi, lo
  static constexpr uint32_t kFormat = 2;  // TF32
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

// 2-D tensor map of bf16 (f32 = false) or fp32 elements: `rows` rows of
// `cols` elements, `ld` elements apart; boxes of one 128-byte row (64 bf16 or
// 32 fp32 columns) x `box_rows` rows, 128-byte swizzle, zero fill.
bool make_map(CUtensorMap *map, const void *ptr, int64_t rows, int64_t cols, int64_t ld, int box_rows,
              bool f32 = false) {
  auto fn = encode_fn();
  if (fn == nullptr) return false;
  const int es = f32 ? 4 : 2;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(ld * es)};
  cuuint32_t box[2] = {(cuuint32_t)(128 / es), (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  return fn(map, f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(ptr),
            dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int sm_count() { return sm_count_current(); }

// ---------------------------------------------------------------------------
// Paired-SM projection GEMM (tcgen05 .cta_group::2).
//
// y[M, N] = x[M, K] . w[N, K]^T for the decode step's projections, with the
// batch rows as the MMA's M and the weight rows as its N: a pair of SMs (a
// two-CTA cluster) owns 256 batch rows (128 per CTA, on its TMEM lanes) and
// nt weight rows (nt / 2 loaded by each CTA), and the even CTA issues one
// tcgen05.mma.cta_group::2 per 16 k that reads both CTAs' shared memory.
// Each SM therefore streams half of the pair's weight tile; the batch rows
// (at decode sizes a few hundred KB, resident in L2) are re-read per tile.
// A thread owns one batch row of the accumulator, so the epilogue writes
// contiguous 32-byte row segments straight from TMEM.  Batch rows past M are
// zero-filled by TMA and cost no memory traffic.
//
// K may be split over `nsplit` pairs for shapes with few weight tiles: every
// pair but the last to finish writes its fp32 partial tile to the caller's
// workspace and takes a ticket; the last sums all partials in split order
// (its own from TMEM), so the result does not depend on arrival order, and
// resets the ticket.  Nobody waits on anybody; no co-scheduling is assumed.
//
//   warp 0 / lane 0   TMA producer (both CTAs): its 128 batch rows and its
//                     nt / 2 weight rows per 64-k tile into an S-stage ring;
//                     both CTAs' copies complete on the even CTA's barrier
//   warp 1            TMEM allocation for the pair (both CTAs); lane 0 of
//                     the even CTA issues the MMAs and releases each stage
//                     in BOTH CTAs with one multicast tcgen05.commit
//   warps 2-5         epilogue: warp w reads TMEM lanes 32 (w % 4) .. + 31
//
// No copy uses cluster multicast.  Every mbarrier wait is bounded; on a
// timeout the thread records M3_DEVERR_TIMEOUT and carries on, so both CTAs
// reach every cluster barrier.
// ---------------------------------------------------------------------------

constexpr int kPairBatch = 128;   // batch rows per CTA (MMA M = 256 per pair)
constexpr int kPairThreads = 192;
constexpr int kPairMaxSplit = 16;
constexpr int kPairSmem = 200 * 1024;
// Split-K tickets live at the start of the workspace, before any partial
// tile, at the same place for every shape (a workspace serves many shapes).
constexpr int kPairMaxTickets = 8192;
constexpr int64_t kPairTicketBytes = kPairMaxTickets * 4;
constexpr int kPairMaxStages = 8;

struct PairArgs {
  int M, N;
  int nt;          // weight rows per pair tile (multiple of 32, <= 256)
  int ntn;         // pair tiles along N
  int ktiles;      // k-tiles per split
  int ktotal;      // k-tiles of K
  int nsplit;      // pairs along K
  int nstage;      // ring depth
  int stage_b;     // bytes of this CTA's half of a weight tile (nt / 2 rows)
  int nacc;        // accumulators the k-tiles alternate between (1 or 2)
  int tmem_cols;   // accumulator columns allocated per CTA (>= nacc * nt)
  void *y;
  int64_t ldy;
  int y_bf16;
  float *part;        // split K: fp32 partials, [tile][half][split][128][nt]
  unsigned *tickets;  // split K: arrivals per [tile][half], zero between calls
};

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// The shared::cluster address of `addr` (a shared::cta address of this CTA's
// layout) in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t peer_addr(uint32_t addr, uint32_t rank) {
  uint32_t d;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(d) : "r"(addr), "r"(rank));
  return d;
}

// 2-D TMA load into this CTA's shared memory whose completion is counted on
// the pair's even CTA's barrier `bar` (a shared::cluster address).
__device__ __forceinline__ void tma_load_2d_pair(uint32_t dst, const CUtensorMap *map, int x, int y, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
      "[%4];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}

__device__ __forceinline__ void mma_bf16_pair(uint32_t tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem),
      "l"(a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}
__device__ __forceinline__ void mma_tf32_pair(uint32_t tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem),
      "l"(a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}

// Arrive once on barrier `bar` (same shared::cta offset) of every CTA in
// `cta_mask` when all MMAs this thread issued have completed.
__device__ __forceinline__ void mma_commit_to_pair(uint32_t bar, uint16_t cta_mask) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster"
      ".multicast::cluster.b64 [%0], %1;" ::"r"(bar),
      "h"(cta_mask)
      : "memory");
}

// Named barrier of the four epilogue warps.
__device__ __forceinline__ void epi_sync() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

// 16 consecutive outputs v of row m from column n: 32-byte bf16 / 4 x
// 16-byte fp32 stores where the row allows, else element by element.
__device__ __forceinline__ void store16(const PairArgs &g, int m, int n, const float (&v)[16]) {
  if (m >= g.M || n >= g.N) return;
  const bool vec = n + 15 < g.N && ((g.ldy | n) & 7) == 0;
  if (g.y_bf16) {
    __nv_bfloat16 *yr = static_cast<__nv_bfloat16 *>(g.y) + (int64_t)m * g.ldy + n;
    if (vec) {
      uint32_t pk[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        __nv_bfloat162 b = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
        pk[i] = *reinterpret_cast<uint32_t *>(&b);
      }
      reinterpret_cast<uint4 *>(yr)[0] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
      reinterpret_cast<uint4 *>(yr)[1] = make_uint4(pk[4], pk[5], pk[6], pk[7]);
    } else {
#pragma unroll
      for (int i = 0; i < 16; ++i)
        if (n + i < g.N) yr[i] = __float2bfloat16_rn(v[i]);
    }
  } else {
    float *yr = static_cast<float *>(g.y) + (int64_t)m * g.ldy + n;
    if (vec) {
#pragma unroll
      for (int i = 0; i < 4; ++i)
        reinterpret_cast<float4 *>(yr)[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
    } else {
#pragma unroll
      for (int i = 0; i < 16; ++i)
        if (n + i < g.N) yr[i] = v[i];
    }
  }
}

// tw / tx: the weight and batch operands (bf16; TF32 heads for kKindTF32x3),
// twl / txl: their TF32 remainders (kKindTF32x3 only; unused otherwise).
// A stage holds, per plane, this CTA's 128 batch rows and nt / 2 weight rows
// of one 128-byte k-tile.
template <int KIND>
__global__ void __launch_bounds__(kPairThreads, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap tw, const __grid_constant__ CUtensorMap tx,
                     const __grid_constant__ CUtensorMap twl, const __grid_constant__ CUtensorMap txl,
                     const PairArgs g) {
  using K_ = PairKind<KIND>;
  constexpr int kTileK = K_::kTileK, NPL = K_::kPlanes;
  extern __shared__ unsigned char smem_raw[];  // no static shared memory: the opt-in is the whole 227 KB
  unsigned char *smem =
      reinterpret_cast<unsigned char *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  constexpr int kStageA = kPairBatch * 128;  // this CTA's batch rows x one 128-byte k-tile, per plane
  const int S = g.nstage;
  unsigned char *ringA = smem;                                  // [S][NPL][kStageA]
  unsigned char *ringB = smem + (size_t)S * NPL * kStageA;      // [S][NPL][stage_b]
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + (size_t)S * NPL * (kStageA + g.stage_b));
  uint64_t *full = bars, *empty = bars + S, *accum = bars + 2 * S, *redbar = bars + 2 * S + 2;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 2 * S + 1);
  int *s_last = reinterpret_cast<int *>(tmem_slot + 1);  // shares the slot's 8 bytes

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t rank = cluster_rank();  // the cluster is the pair: rank 0 (even CTA) or 1
  const int half = (int)(rank & 1u);
  const bool leader = half == 0;
  const int pair = (int)blockIdx.x >> 1;
  const int kq = pair % g.nsplit, tile = pair / g.nsplit;
  const int tn = tile % g.ntn, tm = tile / g.ntn;
  const int n0 = tn * g.nt;                             // the pair's weight rows (output columns)
  const int nw = n0 + half * (g.nt >> 1);               // this CTA's half of them
  const int mb = tm * 2 * kPairBatch + half * kPairBatch;  // this CTA's batch rows
  const int kt0 = kq * g.ktiles;
  const int nkt = max(0, min(g.ktiles, g.ktotal - kt0));
  // Every pair reads the same batch rows; walking K in the same order, all
  // pairs would ask L2 for the same lines at once.  Each pair tile starts
  // its walk at its own k-tile (both CTAs of the pair alike), which spreads
  // the requests over the batch tile.
  const int krot = nkt > 0 ? (int)(((unsigned)tile * 7u) % (unsigned)nkt) : 0;
  auto kx_of = [&](int i) { int k = i + krot; return (kt0 + (k >= nkt ? k - nkt : k)) * kTileK; };
  const uint16_t pair_mask = 3;
  const uint32_t stage_tx = 2u * (uint32_t)(NPL * (kStageA + g.stage_b));  // both CTAs' copies of a stage

  if (tid == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(smem_addr(&full[s]), 1);
      mbar_init(smem_addr(&empty[s]), 1);
    }
    mbar_init(smem_addr(accum), 1);
    mbar_init(smem_addr(redbar), 1);
    mbar_init_fence();
  }
  if (warp == 1) {  // the pair's accumulator: the same columns in both CTAs
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(tmem_slot)),
                 "r"(g.tmem_cols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  cluster_sync();  // both CTAs' barriers are initialised and their TMEM allocated
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t full_lead = peer_addr(smem_addr(&full[0]), 0);  // the even CTA's `full` barriers

  // the weights are constant: the first stages' weight tiles are requested
  // before waiting for the preceding kernel, whose product the batch rows are
  const int npre = min(S, nkt);
  if (warp == 0 && lane == 0) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tw)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tx)) : "memory");
    if constexpr (NPL == 2) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&twl)) : "memory");
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&txl)) : "memory");
    }
    for (int i = 0; i < npre; ++i) {
      if (leader) mbar_arrive_expect_tx(smem_addr(&full[i]), stage_tx);
      unsigned char *b = ringB + (size_t)i * NPL * g.stage_b;
      tma_load_2d_pair(smem_addr(b), &tw, kx_of(i), nw, full_lead + 8u * i);
      if constexpr (NPL == 2) tma_load_2d_pair(smem_addr(b + g.stage_b), &twl, kx_of(i), nw, full_lead + 8u * i);
    }
  }
  pdl_wait();
  pdl_trigger();

  if (warp == 0) {
    if (lane == 0) {
      // producer: k-tile i into stage i % S once the MMAs of k-tile i - S
      // (in both CTAs) have released it
      for (int i = 0; i < npre; ++i) {
        unsigned char *a = ringA + (size_t)i * NPL * kStageA;
        tma_load_2d_pair(smem_addr(a), &tx, kx_of(i), mb, full_lead + 8u * i);
        if constexpr (NPL == 2) tma_load_2d_pair(smem_addr(a + kStageA), &txl, kx_of(i), mb, full_lead + 8u * i);
      }
      int s = npre % S;
      uint32_t ph = npre == S ? 1u : 0u;
      int issued = npre;
      for (int i = npre; i < nkt; ++i) {
        if (!mbar_wait(smem_addr(&empty[s]), ph ^ 1u)) break;
        if (leader) mbar_arrive_expect_tx(smem_addr(&full[s]), stage_tx);
        const int kx = kx_of(i);
        unsigned char *b = ringB + (size_t)s * NPL * g.stage_b;
        unsigned char *a = ringA + (size_t)s * NPL * kStageA;
        tma_load_2d_pair(smem_addr(b), &tw, kx, nw, full_lead + 8u * s);
        if constexpr (NPL == 2) tma_load_2d_pair(smem_addr(b + g.stage_b), &twl, kx, nw, full_lead + 8u * s);
        tma_load_2d_pair(smem_addr(a), &tx, kx, mb, full_lead + 8u * s);
        if constexpr (NPL == 2) tma_load_2d_pair(smem_addr(a + kStageA), &txl, kx, mb, full_lead + 8u * s);
        issued = i + 1;
        if (++s == S) {
          s = 0;
          ph ^= 1u;
        }
      }
      // the even CTA waits until the last stages' copies (both CTAs') have
      // landed before the pair moves on (immediate on the normal path, where
      // the MMAs consumed them)
      if (leader)
        for (int j = issued > S ? issued - S : 0; j < issued; ++j)
          mbar_wait(smem_addr(&full[j % S]), (uint32_t)((j / S) & 1));
    }
    __syncwarp();
  } else if (warp == 1) {
    if (leader && lane == 0) {
      // D[256 x nt] (+)= X_pair[256 x k] . W_pair[nt x k]^T per k-tile;
      // instruction descriptor: fp32 accumulator, A and B in the kind's
      // format, both K-major, N / 8 and M / 16
      const uint32_t idesc = (1u << 4) | (K_::kFormat << 7) | (K_::kFormat << 10) |
                             ((uint32_t)(g.nt >> 3) << 17) | ((uint32_t)((2 * kPairBatch) >> 4) << 24);
      int s = 0;
      uint32_t ph = 0;
      for (int i = 0; i < nkt; ++i) {
        if (!mbar_wait(smem_addr(&full[s]), ph)) break;
        tc_fence_after();
        const uint32_t a0 = smem_addr(ringA + (size_t)s * NPL * kStageA);
        const uint32_t b0 = smem_addr(ringB + (size_t)s * NPL * g.stage_b);
        // with two accumulators, k-tile i adds into accumulator i % 2: two
        // independent chains of MMAs
        const int ai = g.nacc == 2 ? (i & 1) : 0;
        const uint32_t d = tmem + (uint32_t)(ai * g.nt);
        // four 32-byte k steps per 128-byte row (16 bf16 or 8 TF32 each)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const uint32_t acc = (i >> (g.nacc - 1) | j) != 0 ? 1u : 0u;
          if constexpr (KIND == kKindBF16) {
            mma_bf16_pair(d, sw128_desc(a0 + 32 * j), sw128_desc(b0 + 32 * j), idesc, acc);
          } else {
            const uint64_t ah = sw128_desc(a0 + 32 * j), al = sw128_desc(a0 + kStageA + 32 * j);
            const uint64_t bh = sw128_desc(b0 + 32 * j), bl = sw128_desc(b0 + g.stage_b + 32 * j);
            mma_tf32_pair(d, ah, bh, idesc, acc);
            mma_tf32_pair(d, ah, bl, idesc, 1u);
            mma_tf32_pair(d, al, bh, idesc, 1u);
          }
        }
        mma_commit_to_pair(smem_addr(&empty[s]), pair_mask);
        if (++s == S) {
          s = 0;
          ph ^= 1u;
        }
      }
      mma_commit_to_pair(smem_addr(accum), pair_mask);  // once every MMA above has completed
    }
    __syncwarp();
  } else {
    // epilogue: TMEM lane q is batch row mb + q; its nt columns are the
    // output columns n0 .. n0 + nt - 1 of that row
    mbar_wait(smem_addr(accum), 0);
    __syncwarp();
    tc_fence_after();
    const int q = 32 * (warp & 3) + lane, m = mb + q;
    const uint32_t trow = tmem + ((uint32_t)(32 * (warp & 3)) << 16);
    // 32 accumulator columns from c0 (both accumulators added), zero when
    // this split had no k-tile (a second accumulator gets one only when nkt >= 2)
    auto load32 = [&](int c0, float (&f)[32]) {
      uint32_t v[2][16], w[2][16];
      tmem_ld16(trow + (uint32_t)c0, v[0]);
      tmem_ld16(trow + (uint32_t)(c0 + 16), v[1]);
      if (g.nacc == 2) {
        tmem_ld16(trow + (uint32_t)(g.nt + c0), w[0]);
        tmem_ld16(trow + (uint32_t)(g.nt + c0 + 16), w[1]);
      }
      tmem_wait();
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        float a = nkt > 0 ? __uint_as_float(v[j >> 4][j & 15]) : 0.f;
        if (g.nacc == 2 && nkt > 1) a += __uint_as_float(w[j >> 4][j & 15]);
        f[j] = a;
      }
    };
    if (g.nsplit == 1) {
      for (int c0 = 0; c0 < g.nt; c0 += 32) {
        float f[32];
        load32(c0, f);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          float o[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) o[j] = f[16 * h + j];
          store16(g, m, n0 + c0 + 16 * h, o);
        }
      }
    } else {
      // split K: this pair's partial tile -> its slot, stored column-major
      // ([nt][128]: a warp writes 128 contiguous bytes per column); the
      // last of the nsplit pairs to take a ticket sums the slots in split
      // order (its own from TMEM) and writes the rows
      const size_t slot_elems = (size_t)kPairBatch * g.nt;
      float *slot0 = g.part + ((size_t)tile * 2 + half) * g.nsplit * slot_elems;
      float *mine = slot0 + (size_t)kq * slot_elems;
      for (int c0 = 0; c0 < g.nt; c0 += 32) {
        float f[32];
        load32(c0, f);
#pragma unroll
        for (int j = 0; j < 32; ++j) __stcg(mine + (size_t)(c0 + j) * kPairBatch + q, f[j]);
      }
      __threadfence();
      epi_sync();
      if (warp == 2 && lane == 0) *s_last = atomicAdd(&g.tickets[tile * 2 + half], 1u) == (unsigned)(g.nsplit - 1);
      epi_sync();
      if (*s_last) {
        __threadfence();
        // the other pairs' slots, into the idle ring when they fit (one
        // bulk copy each), else read from L2 column by column
        const uint32_t slot_bytes = (uint32_t)(slot_elems * 4);
        const bool staged = (int64_t)(g.nsplit - 1) * slot_bytes <= (int64_t)S * NPL * (kStageA + g.stage_b);
        float *ring = reinterpret_cast<float *>(smem);
        auto other = [&](int p) -> int { return p < kq ? p : p - 1; };  // staging index of slot p
        if (staged) {
          if (warp == 2 && lane == 0) {
            asm volatile("fence.proxy.async.global;" ::: "memory");  // the slots were written by generic stores
            const uint32_t rb = smem_addr(redbar);
            mbar_arrive_expect_tx(rb, (uint32_t)(g.nsplit - 1) * slot_bytes);
            for (int p = 0; p < g.nsplit; ++p) {
              if (p == kq) continue;
              const char *src = reinterpret_cast<const char *>(slot0 + (size_t)p * slot_elems);
              const uint32_t dst = smem_addr(ring + (size_t)other(p) * slot_elems);
              for (uint32_t off = 0; off < slot_bytes; off += 32768u) {
                const uint32_t len = slot_bytes - off < 32768u ? slot_bytes - off : 32768u;
                bulk_g2s(dst + off, src + off, len, rb);
              }
            }
          }
          mbar_wait(smem_addr(redbar), 0);
        }
        for (int c0 = 0; c0 < g.nt; c0 += 32) {
          float own[32], f[32];
          load32(c0, own);
#pragma unroll
          for (int j = 0; j < 32; ++j) f[j] = 0.f;
          for (int p = 0; p < g.nsplit; ++p) {
            if (p == kq) {
#pragma unroll
              for (int j = 0; j < 32; ++j) f[j] += own[j];
            } else if (staged) {
              const float *src = ring + (size_t)other(p) * slot_elems + (size_t)c0 * kPairBatch + q;
#pragma unroll
              for (int j = 0; j < 32; ++j) f[j] += src[(size_t)j * kPairBatch];
            } else {
              const float *src = slot0 + (size_t)p * slot_elems + (size_t)c0 * kPairBatch + q;
              float t[32];
#pragma unroll
              for (int j = 0; j < 32; ++j) t[j] = __ldcg(src + (size_t)j * kPairBatch);
#pragma unroll
              for (int j = 0; j < 32; ++j) f[j] += t[j];
            }
          }
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            float o[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) o[j] = f[16 * h + j];
            store16(g, m, n0 + c0 + 16 * h, o);
          }
        }
        if (warp == 2 && lane == 0) g.tickets[tile * 2 + half] = 0u;
      }
    }
  }
  tc_fence_before();
  cluster_sync();  // both CTAs are done with their accumulators
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(g.tmem_cols) : "memory");
  }
}

// Pair tiles and K split of one call, the cheapest by a model measured on
// B200: a pair spends about 0.33 us per 64-k tile whatever the tile width
// (at nt = 256 that is the tensor cores' full rate), pairs beyond one per SM
// pair run in further waves, and a split adds about a microsecond plus the
// last pair's copy of the other partial tiles (~200 GB/s).
struct PairPlan {
  int nt, ntn, ntm, ktotal, ktiles, nsplit, nacc;
};

PairPlan plan_pair(int M, int N, int K) {
  const int sms = sm_count();
  const int ntm = (M + 2 * kPairBatch - 1) / (2 * kPairBatch);
  const int ktotal = (K + kTileK - 1) / kTileK;
  PairPlan best = {};
  double best_cost = 1e30;
  for (int nt : {256, 128, 64, 32}) {
    const int ntn = (N + nt - 1) / nt;
    int nsmax = sms / (2 * ntn * ntm);
    nsmax = nsmax < 1 ? 1 : nsmax > kPairMaxSplit ? kPairMaxSplit : nsmax;
    for (int ns0 = 1; ns0 <= nsmax && ns0 <= ktotal; ns0 *= 2) {
      const int ktiles = (ktotal + ns0 - 1) / ns0;
      const int ns = (ktotal + ktiles - 1) / ktiles;
      const int waves = (2 * ntn * ntm * ns + sms - 1) / sms;
      double cost = waves * ktiles * 0.33;  // us
      if (ns > 1) cost += waves * (1.0 + (ns - 1) * (double)kPairBatch * nt * 4.0 / 2.0e5);
      if (cost < best_cost - 1e-9) {
        best_cost = cost;
        best = {nt, ntn, ntm, ktotal, ktiles, ns, 1};
      }
    }
  }
  return best;
}

// Split-K workspace: the tickets (fixed region), then the partial tiles.
int64_t pair_workspace_bytes(const PairPlan &p) {
  return p.nsplit > 1 ? kPairTicketBytes + (int64_t)p.ntn * p.ntm * 2 * p.nsplit * kPairBatch * p.nt * 4 : 0;
}

// TF32x3 tile plan: no K split (the fp32 path is taken for batches of
// several hundred rows and more, which give enough pair tiles); the tile
// width with the least waves x k-tiles x per-k-tile time, measured on B200
// at 1.5x the 128-wide tile's for the 256-wide one (4096 x 5248 x 1024:
// 213 us at nt 256 in 5 waves, 254 us at nt 128 in 9).
PairPlan plan_pair_tf32(int M, int N, int K) {
  const int sms = sm_count();
  const int ntm = (M + 2 * kPairBatch - 1) / (2 * kPairBatch);
  const int ktotal = (K + PairKind<kKindTF32x3>::kTileK - 1) / PairKind<kKindTF32x3>::kTileK;
  PairPlan best = {};
  double best_cost = 1e30;
  for (int nt : {256, 128}) {
    const int ntn = (N + nt - 1) / nt;
    const int waves = (2 * ntn * ntm + sms - 1) / sms;
    const double cost = waves * ktotal * (nt == 256 ? 1.0 : 0.66);
    if (cost < best_cost - 1e-9) {
      best_cost = cost;
      best = {nt, ntn, ntm, ktotal, ktotal, 1, 1};
    }
  }
  return best;
}

// x / w: the batch and weight operands (TF32 heads for kKindTF32x3), xl / wl
// their TF32 remainders (kKindTF32x3 only).
template <int KIND>
cudaError_t launch_gemm_pair(const void *x, const void *xl, int64_t ldx, const void *w, const void *wl, int64_t ldw,
                             void *y, int64_t ldy, int M, int N, int K, bool y_bf16, void *workspace,
                             const PairPlan &pl, cudaStream_t stream) {
  using K_ = PairKind<KIND>;
  constexpr bool kF32 = KIND == kKindTF32x3;
  PairArgs g = {};
  g.M = M;
  g.N = N;
  g.nt = pl.nt;
  g.ntn = pl.ntn;
  g.ktotal = pl.ktotal;
  g.ktiles = pl.ktiles;
  g.nsplit = pl.nsplit;
  if (g.nt % 32 != 0 || g.nt > 256 || g.nsplit < 1 || g.nsplit > kPairMaxSplit) return cudaErrorInvalidValue;
  if (g.nsplit > 1) {
    if (workspace == nullptr || pl.ntn * pl.ntm * 2 > kPairMaxTickets) return cudaErrorInvalidValue;
    g.tickets = static_cast<unsigned *>(workspace);
    g.part = reinterpret_cast<float *>(static_cast<char *>(workspace) + kPairTicketBytes);
  }
  g.nacc = pl.nacc == 2 && 2 * pl.nt <= 512 ? 2 : 1;
  g.stage_b = (g.nt / 2) * 128;
  const int stage = K_::kPlanes * (kPairBatch * 128 + g.stage_b);
  int S = kPairSmem / stage;
  S = S > kPairMaxStages ? kPairMaxStages : S;
  if (S > g.ktiles) S = g.ktiles < 2 ? 2 : g.ktiles;
  g.nstage = S;
  g.tmem_cols = 32;
  while (g.tmem_cols < g.nacc * g.nt) g.tmem_cols <<= 1;
  g.y = y;
  g.ldy = ldy;
  g.y_bf16 = y_bf16 ? 1 : 0;
  const int smem = 1024 + S * stage + (2 * S + 3) * 8;
  if (smem > 227 * 1024) return cudaErrorInvalidValue;

  CUtensorMap tw, tx, twl, txl;
  if (!make_map(&tw, w, N, K, ldw, g.nt / 2, kF32) || !make_map(&tx, x, M, K, ldx, kPairBatch, kF32))
    return cudaErrorInvalidValue;
  if (kF32) {
    if (!make_map(&twl, wl, N, K, ldw, g.nt / 2, true) || !make_map(&txl, xl, M, K, ldx, kPairBatch, true))
      return cudaErrorInvalidValue;
  } else {
    twl = tw;
    txl = tx;
  }

  auto kern = gemm_pair_kernel<KIND>;
  static LaunchCache cache;
  if (cudaError_t e = ensure_smem_optin(cache, kern, 227 * 1024); e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(2 * g.nsplit * pl.ntn * pl.ntm));
  cfg.blockDim = dim3(kPairThreads);
  cfg.dynamicSmemBytes = (size_t)smem;
  cfg.stream = stream;
  cudaLaunchAttribute attrs[2];
  attrs[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attrs[0].val.programmaticStreamSerializationAllowed = 1;
  attrs[1].id = cudaLaunchAttributeClusterDimension;
  attrs[1].val.clusterDim.x = 2;
  attrs[1].val.clusterDim.y = 1;
  attrs[1].val.clusterDim.z = 1;
  cfg.attrs = attrs;
  cfg.numAttrs = 2;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, tw, tx, twl, txl, g);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

// The TF32 head / remainder split of an fp32 matrix (rows x cols, rows ld
// elements apart): hi = x with its 13 low mantissa bits cleared (exactly a
// TF32 value), lo = x - hi (exact in fp32).  One thread per 4 elements.
__global__ void __launch_bounds__(256) tf32_split_kernel(const float *__restrict__ x, int64_t ldx,
                                                         float *__restrict__ hi, float *__restrict__ lo, int64_t ld,
                                                         int rows, int cols4) {
  pdl_wait();
  pdl_trigger();
  const int64_t n = (int64_t)rows * cols4;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / cols4, c = (i - r * cols4) * 4;
    const float4 v = *reinterpret_cast<const float4 *>(x + r * ldx + c);
    float4 h, l;
    h.x = __uint_as_float(__float_as_uint(v.x) & 0xFFFFE000u);
    h.y = __uint_as_float(__float_as_uint(v.y) & 0xFFFFE000u);
    h.z = __uint_as_float(__float_as_uint(v.z) & 0xFFFFE000u);
    h.w = __uint_as_float(__float_as_uint(v.w) & 0xFFFFE000u);
    l.x = v.x - h.x;
    l.y = v.y - h.y;
    l.z = v.z - h.z;
    l.w = v.w - h.w;
    *reinterpret_cast<float4 *>(hi + r * ld + c) = h;
    *reinterpret_cast<float4 *>(lo + r * ld + c) = l;
  }
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
  return pair_workspace_bytes(plan_pair(M, N, K));
}

cudaError_t launch_gemm_bf16(const void *x, int64_t ldx, const void *w, int64_t ldw, void *y, int64_t ldy, int M,
                             int N, int K, bool y_bf16, float *workspace, cudaStream_t stream) {
  return launch_gemm_pair<kKindBF16>(x, nullptr, ldx, w, nullptr, ldw, y, ldy, M, N, K, y_bf16, workspace,
                                     plan_pair(M, N, K), stream);
}

bool gemm_tf32x3_supported(const void *x, const void *xl, int64_t ldx, const void *w, const void *wl, int64_t ldw,
                           const void *y, int64_t ldy, int M, int N, int K) {
  auto al = [](const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  return M > 0 && N > 0 && K >= 32 && K % 4 == 0 && ldx % 4 == 0 && ldw % 4 == 0 && ldx >= K && ldw >= K &&
         ldy >= N && al(x) && al(xl) && al(w) && al(wl) && al(y) && encode_fn() != nullptr;
}

cudaError_t launch_gemm_tf32x3(const float *x, const float *xl, int64_t ldx, const float *w, const float *wl,
                               int64_t ldw, float *y, int64_t ldy, int M, int N, int K, cudaStream_t stream) {
  return launch_gemm_pair<kKindTF32x3>(x, xl, ldx, w, wl, ldw, y, ldy, M, N, K, false, nullptr,
                                       plan_pair_tf32(M, N, K), stream);
}

cudaError_t launch_tf32_split(const float *x, int64_t ldx, float *hi, float *lo, int64_t ld, int rows, int cols,
                              cudaStream_t stream) {
  const int cols4 = cols / 4;
  const int64_t n = (int64_t)rows * cols4;
  int64_t blocks = (n + 255) / 256;
  const int64_t cap = (int64_t)sm_count() * 8;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  return launch_pdl(tf32_split_kernel, dim3((unsigned)blocks), dim3(256), 0, stream, x, ldx, hi, lo, ld, rows, cols4);
}

int gemm_device_error(bool reset) { return device_error_of_this_unit(reset); }

}  // namespace m3
