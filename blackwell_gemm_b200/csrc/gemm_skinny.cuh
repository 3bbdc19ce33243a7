// Skinny-M GEMM for sm_100a (M <= 256, the HBM-bound decode shapes):
// C = A * B^T computed as C^T = B * A^T, so the big operand B supplies the
// MMA's 128-row M dimension and the few rows of A its N dimension
// (Mp = M rounded up to a supported MMA N of 16..256).  The tensor core then
// does almost no wasted work and each SM only streams its share of B
// through a deep shared-memory ring; the reference can run none of these
// shapes except v1 at M = 128 (its kernels need M % 256 == 0).
//
// One CTA per SM, persistent over work units (128-row block of B, K slice);
// cta_group::1 tcgen05.mma M=128 N=Mp K=16 into a double-buffered TMEM
// accumulator (128 lanes x Mp fp32 columns per buffer).  Warp roles:
//   warp 0     TMA producer (B box 64 x 128, A box 64 x Mp)
//   warp 1     TMEM owner and MMA issuer
//   warps 2-5  epilogue: TMEM lane quarter -> smem [m][n] fp32 -> TMA
//              reduce-add into the zeroed fp32 workspace W (M x N); a
//              separate pass rounds W to bf16 C.  (Finishing a tile inside
//              the kernel, by the warp whose reduce-adds complete last, was
//              measured slower: waiting for each unit's reduce-adds stalls
//              the epilogue, which stalls the MMA.)
// All waits are the bounded waits of gemm_kernel.cuh.
#pragma once
#include "gemm_kernel.cuh"

namespace b200 {

// Every CTA reads the same rows of A.  Units that walk their K blocks in
// the same order ask L2 for the same A slab at the same moment; starting
// tile t's walk at an offset spreads those reads over t-dependent slabs.
// K block number i (0 <= i < len) of a unit of tile t out of T:
__device__ __forceinline__ int skinny_kb(int kb0, int len, int i, int t, int T) {
  const int rot = (int)(((long long)t * len) / T) % len;
  int j = i + rot;
  if (j >= len) j -= len;
  return kb0 + j;
}

// kTiles: 128-row blocks of B per work unit.  Every CTA streams its own rows
// of B but re-reads A's slab for each unit, and each SM's inflow is the
// limit in this HBM-bound regime, so a unit of kTiles blocks sharing one A
// slab per K step cuts A's share of the inflow kTiles-fold.
// kPair: 2-CTA pairs (stream-K kernel only): the pair MMA is M = 256 rows of
// B (128 per CTA) by N = Mp rows of A, and each CTA holds Mp / 2 of A's rows.
template <int kMp, int kSlabs, int kTiles = 1, bool kPair = false>
struct SkinnyCfg {
  static_assert(kMp % 16 == 0 && kMp >= 16 && kMp <= 256, "MMA N must be 16..256, step 16");
  static_assert(kTiles * kMp <= 512, "an accumulator of kTiles x Mp columns exceeds TMEM");
  static_assert(!kPair || (kTiles == 1 && kMp >= 32), "pairs: one block per CTA, Mp >= 32");
  // Two accumulators (the epilogue of one unit overlaps the next unit's
  // MMAs) when they fit in TMEM's 512 columns, else one.
  static constexpr int kAccBufs = 2 * kTiles * kMp <= 512 ? 2 : 1;
  static constexpr int kRowsB = 128;                       // MMA M: rows of B per block
  static constexpr int kBK = kSlabs * kSlabK;              // K per stage
  static constexpr int kSlabB = kRowsB * kSlabK * 2;       // 16 KiB
  static constexpr int kRowsA = kPair ? kMp / 2 : kMp;     // rows of A per CTA
  static constexpr int kSlabA = kRowsA * kSlabK * 2;
  static constexpr int kBytesB = kTiles * kSlabs * kSlabB;
  static constexpr int kBytesA = kSlabs * kSlabA;
  static constexpr int kStageBytes = kBytesB + kBytesA;
  static constexpr int kChunk = kMp < 32 ? kMp : 32;       // epilogue columns per pass
  static constexpr int kStoreBuf = 32 * kChunk * 4;        // [kChunk m][32 n] fp32
  static constexpr int kStoreBytes = 4 * 2 * kStoreBuf;    // 4 warps x 2 buffers
  static constexpr int kStagesFit = (kSmemBudget - kStoreBytes - kSmemReserve) / kStageBytes;
  static constexpr int kStages = kStagesFit > 16 ? 16 : kStagesFit;
  static constexpr int kSmemBytes = kStages * kStageBytes + kStoreBytes + 1024;
  static constexpr int kTmemCols = kAccBufs * kTiles * kMp;
  static constexpr int kTmemAlloc = kTmemCols <= 32    ? 32
                                    : kTmemCols <= 64  ? 64
                                    : kTmemCols <= 128 ? 128
                                    : kTmemCols <= 256 ? 256
                                                       : 512;  // power of two >= 32
  static constexpr int kThreads = 192;
  static_assert(kStages >= 2, "ring too shallow");
};

// Largest K-slab count <= `want` whose stages still leave a ring of three.
constexpr int skinny_fit_slabs(int mp, int want, int tiles = 1) {
  for (int s = want; s > 1; --s) {
    const int chunk = mp < 32 ? mp : 32;
    const int store = 4 * 2 * 32 * chunk * 4;
    const int stage = s * (tiles * 128 * kSlabK * 2 + mp * kSlabK * 2);
    if ((kSmemBudget - store - kSmemReserve) / stage >= 3) return s;
  }
  return 1;
}

struct SkinnyArgs {
  int M, N, K;
  int l2_hint;       // 1: B loads evict-first, A loads evict-last in L2
  int tiles;         // ceil(N / 128)
  int groups;        // ceil(tiles / kTiles): the units' blocks of B
  int k_blocks;      // ceil(K / kBK)
  int splits;        // K slices per group
  int kb_per_split;
  int* status;
  unsigned long long timeout_ns;
};

template <int kMp, int kSlabs, int kTiles>
__global__ void __launch_bounds__(192, 1)
gemm_skinny_kernel(const __grid_constant__ CUtensorMap tmap_b,   // N x K, box 64 x 128
                   const __grid_constant__ CUtensorMap tmap_a,   // M x K, box 64 x Mp
                   const __grid_constant__ CUtensorMap tmap_w,   // W fp32 M x N, box 32 x kChunk
                   const SkinnyArgs args) {
  using P = SkinnyCfg<kMp, kSlabs, kTiles>;
  constexpr int kStages = P::kStages;
  extern __shared__ uint8_t smem_raw[];
  __shared__ alignas(8) uint64_t bar_full[kStages];
  __shared__ alignas(8) uint64_t bar_empty[kStages];
  __shared__ alignas(8) uint64_t bar_acc_full[2];
  __shared__ alignas(8) uint64_t bar_acc_empty[2];
  __shared__ alignas(8) uint64_t bar_drain;
  __shared__ uint32_t tmem_slot;
  __shared__ uint32_t abort_word;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int units = args.groups * args.splits;
  const uint32_t smem_base = (smem_u32(smem_raw) + 1023u) & ~1023u;
  const uint32_t store_base = smem_base + kStages * P::kStageBytes;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(smem_u32(&bar_full[s]), 1);
      mbar_init(smem_u32(&bar_empty[s]), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(smem_u32(&bar_acc_full[b]), 1);
      mbar_init(smem_u32(&bar_acc_empty[b]), 4);
    }
    mbar_init(smem_u32(&bar_drain), 1);
    abort_word = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    prefetch_tmap(&tmap_b);
    prefetch_tmap(&tmap_a);
    prefetch_tmap(&tmap_w);
  }
  if (warp == 1) {
    tmem_alloc_1(smem_u32(&tmem_slot), P::kTmemAlloc);
    tmem_relinquish_1();
  }
  tc_fence_before_sync();
  __syncthreads();
  tc_fence_after_sync();
  const uint32_t tmem_base = tmem_slot;

  WaitCtx wctx;
  wctx.status = args.status;
  wctx.timeout_ns = args.timeout_ns;
  wctx.abort_local = smem_u32(&abort_word);
  wctx.abort_peer = smem_u32(&abort_word);  // no peer CTA: both words are this CTA's

  auto unit_range = [&](int u, int* tile, int* kb0, int* kb1) {
    *tile = u / args.splits;
    const int s = u - *tile * args.splits;
    *kb0 = s * args.kb_per_split;
    const int end = *kb0 + args.kb_per_split;
    *kb1 = end < args.k_blocks ? end : args.k_blocks;
  };

  if (warp == 0) {
    if (lane == 0) {
      const uint64_t pol_b = args.l2_hint ? l2_policy_evict_first() : l2_policy_evict_normal();
      const uint64_t pol_a = args.l2_hint ? l2_policy_evict_last() : l2_policy_evict_normal();
      uint32_t stage = 0, phase = 0;
      bool ok = true;
      for (int u = blockIdx.x; ok && u < units; u += gridDim.x) {
        int tile, kb0, kb1;
        unit_range(u, &tile, &kb0, &kb1);
        for (int i = 0; i < kb1 - kb0; ++i) {
          const int kb = skinny_kb(kb0, kb1 - kb0, i, tile, args.groups);
          if (!wait_bounded(smem_u32(&bar_empty[stage]), phase ^ 1u, wctx, kErrWaitEmpty)) {
            ok = false;
            break;
          }
          const uint32_t sb = smem_base + stage * P::kStageBytes;
          const uint32_t fb = smem_u32(&bar_full[stage]);
          mbar_arrive_expect_tx(fb, P::kStageBytes);
          // B's slabs first, back to back, so each row's consecutive 128 B
          // segments are requested together.
#pragma unroll
          for (int sl = 0; sl < kSlabs; ++sl)
#pragma unroll
            for (int b = 0; b < kTiles; ++b)
              tma_load_2d_hint(sb + (b * kSlabs + sl) * P::kSlabB, &tmap_b,
                               kb * P::kBK + sl * kSlabK, (tile * kTiles + b) * P::kRowsB, fb,
                               pol_b);
#pragma unroll
          for (int sl = 0; sl < kSlabs; ++sl)
            tma_load_2d_hint(sb + P::kBytesB + sl * P::kSlabA, &tmap_a, kb * P::kBK + sl * kSlabK,
                             0, fb, pol_a);
          if (++stage == kStages) { stage = 0; phase ^= 1u; }
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = make_idesc_bf16_f32(P::kRowsB, kMp);
      uint32_t stage = 0, phase = 0;
      int it = 0;
      bool ok = true;
      for (int u = blockIdx.x; ok && u < units; u += gridDim.x, ++it) {
        int tile, kb0, kb1;
        unit_range(u, &tile, &kb0, &kb1);
        const uint32_t buf = it % P::kAccBufs, acc_phase = (it / P::kAccBufs) & 1;
        if (!wait_bounded(smem_u32(&bar_acc_empty[buf]), acc_phase ^ 1u, wctx, kErrWaitAccEmpty))
          break;
        tc_fence_after_sync();
        const uint32_t d_tmem = tmem_base + buf * kTiles * kMp;
        for (int kb = kb0; kb < kb1; ++kb) {  // slabs arrive in the producer's order
          if (!wait_bounded(smem_u32(&bar_full[stage]), phase, wctx, kErrWaitFull)) {
            ok = false;
            break;
          }
          tc_fence_after_sync();
          const uint32_t sb = smem_base + stage * P::kStageBytes;
#pragma unroll
          for (int sl = 0; sl < kSlabs; ++sl) {
            const uint64_t adesc_small = make_sdesc_k128(sb + P::kBytesB + sl * P::kSlabA);
#pragma unroll
            for (int b = 0; b < kTiles; ++b) {
              const uint64_t bdesc_big = make_sdesc_k128(sb + (b * kSlabs + sl) * P::kSlabB);
#pragma unroll
              for (int k = 0; k < kSlabK / kMmaK; ++k)
                umma_bf16_1(d_tmem + b * kMp, bdesc_big + 2ull * k, adesc_small + 2ull * k, idesc,
                            (kb != kb0 || sl != 0 || k != 0) ? 1u : 0u);
            }
          }
          umma_commit_1(smem_u32(&bar_empty[stage]));
          if (++stage == kStages) { stage = 0; phase ^= 1u; }
        }
        if (!ok) break;
        umma_commit_1(smem_u32(&bar_acc_full[buf]));
      }
      umma_commit_1(smem_u32(&bar_drain));
      if (!mbar_try_wait(smem_u32(&bar_drain), 0))
        wait_slow(smem_u32(&bar_drain), 0, wctx, kErrWaitDrain, false);
    }
    __syncwarp();
  } else {
    // Epilogue: warp w reads TMEM lanes 32 (w % 4) .. + 31 = rows n of B.
    const int quarter = warp & 3;
    const uint32_t my_store = store_base + (warp - 2) * 2 * P::kStoreBuf;
    uint32_t nstore = 0;
    int it = 0;
    for (int u = blockIdx.x; u < units; u += gridDim.x, ++it) {
      int tile, kb0, kb1;
      unit_range(u, &tile, &kb0, &kb1);
      const uint32_t buf = it % P::kAccBufs, acc_phase = (it / P::kAccBufs) & 1;
      int ok = 0;
      if (lane == 0) ok = wait_bounded(smem_u32(&bar_acc_full[buf]), acc_phase, wctx, kErrWaitAccFull);
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) break;
      tc_fence_after_sync();
      // Block b of the unit: TMEM columns b Mp .. b Mp + Mp - 1 of buffer buf.
      constexpr int kChunks = kTiles * (kMp / P::kChunk);
#pragma unroll 1
      for (int cb = 0; cb < kChunks; ++cb) {
        const int b = cb / (kMp / P::kChunk);
        const int c = cb - b * (kMp / P::kChunk);
        const uint32_t tbase =
            tmem_base + (buf * kTiles + b) * kMp + ((uint32_t)(quarter * 32) << 16);
        const int n0 = (tile * kTiles + b) * P::kRowsB + quarter * 32;
        uint32_t v[P::kChunk];
        if constexpr (P::kChunk == 16) {
          tmem_ld_32x32b_x16(tbase + c * 16, *reinterpret_cast<uint32_t(*)[16]>(v));
        } else {
          tmem_ld_32x32b_x32(tbase + c * 32, *reinterpret_cast<uint32_t(*)[32]>(v));
        }
        tmem_wait_ld();
        if (cb == kChunks - 1) {
          tc_fence_before_sync();
          __syncwarp();
          if (lane == 0) mbar_arrive_local(smem_u32(&bar_acc_empty[buf]));
        }
        if (n0 >= args.N) continue;  // a block of the last unit past N (B read as zeros)
        const uint32_t sb = my_store + (nstore & 1u) * P::kStoreBuf;
        if (lane == 0) bulk_wait_group_read<1>();
        __syncwarp();
        // Row j of the box is m = c*kChunk + j; column `lane` is n = n0 + lane.
#pragma unroll
        for (int j = 0; j < P::kChunk; ++j) st_shared_u32(sb + j * 128u + lane * 4u, v[j]);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          tma_reduce_add_2d(&tmap_w, sb, n0, c * P::kChunk);
          bulk_commit_group();
        }
        ++nstore;
      }
    }
    if (lane == 0) bulk_wait_group<0>();
    __syncwarp();
  }

  tc_fence_before_sync();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after_sync();
    tmem_dealloc_1(tmem_base, P::kTmemAlloc);
  }
}

}  // namespace b200

namespace b200 {

// ---------------------------------------------------------------------------
// Cluster split-K variant: no workspace, one launch.  A cluster owns one
// block of B and splits K over S slices; slice p accumulates K blocks
// [p * kb_per, (p+1) * kb_per) into its own TMEM.  The grid is not
// persistent: blocks x cluster-size CTAs, one work unit each.
//   * one-CTA slices (kPair = false): the cluster is S CTAs (S = 1, 2, 4 or
//     8, a launch attribute), the block is 128 rows of B, CTA r is slice r;
//     tcgen05.mma.cta_group::1 M = 128, N = Mp.
//   * pair slices (kPair): the cluster is S 2-CTA pairs (2S = 2, 4 or 8 CTAs;
//     ranks 2p and 2p + 1 form pair p, the even rank leads), the block is 256
//     rows of B, CTA half h = rank & 1 loads its 128 of them and rows
//     [h Mp/2, (h+1) Mp/2) of A, and the pair leader issues
//     tcgen05.mma.cta_group::2 M = 256, N = Mp.  Each SM then streams its
//     rows of B but only half of A's slab: every SM's inflow (its TMA loads
//     are capped at ~76 GB/s each, from L2 or DRAM) carries B + A/2 per K
//     step instead of B + A, which is what bounds these kernels from M = 64 up.
// The S partial sums of each row of C are added through distributed shared
// memory (see the reduction below).
template <int kMp, int kStagesWanted, bool kPair = false>
struct SkinnyClusterCfg {
  static_assert(!kPair || kMp >= 32, "pairs: each CTA holds Mp / 2 >= 16 rows of A");
  static constexpr int kRowsB = 128;                      // rows of B per CTA
  static constexpr int kRowsA = kPair ? kMp / 2 : kMp;    // rows of A per CTA
  static constexpr int kBlockRows = kPair ? 2 * kRowsB : kRowsB;
  static constexpr int kSlabB = kRowsB * kSlabK * 2;      // 16 KiB
  static constexpr int kSlabA = kRowsA * kSlabK * 2;
  static constexpr int kStageBytes = kSlabB + kSlabA;
  static constexpr int kChunk = kMp < 32 ? kMp : 32;      // accumulator columns per TMEM load
  static constexpr int kStages = kStagesWanted;
  static constexpr int kSmemBytes = kStages * kStageBytes + 1024;
  // the ring doubles as the reduction area: every slice's partial of every
  // row of this CTA's 128 columns, 128 x Mp fp32
  static_assert(kStages * kStageBytes >= kRowsB * kMp * 4, "ring too small to reduce in");
  static constexpr int kTmemAlloc = kMp <= 32 ? 32 : kMp;
  static constexpr int kThreads = 192;
  static_assert(kSmemBytes <= kSmemBudget - 1024, "does not fit in shared memory");
};

struct SkinnyClusterArgs {
  int M, N, K;
  int l2_hint;
  int k_blocks;       // ceil(K / 64)
  int kb_per;         // K blocks per slice
  int ldc;            // C row stride (elements)
  __nv_bfloat16* C;
  int* status;
  unsigned long long timeout_ns;
};

// The cluster kernel's cross-slice reduction, for S slices (a compile-time
// count, so every register index below is static).  Rows of C (columns of
// the accumulator) are dealt to the slices in contiguous blocks: slice o owns
// rows [o R, (o+1) R), R = Mp / S.  Each slice's partials land in the owner's
// shared memory laid out [source slice][lane quarter q][lane][row i of R]
// fp32, so the rows one thread owes one owner are contiguous: it pushes them
// with 16-byte DSMEM stores (8-byte for two rows) and the owner reads them
// back with vector loads.  The 16-byte groups of a thread's rows are
// permuted by lane (skc_group) so that the eight lanes of a quarter warp,
// whose rows lie R x 4 bytes apart, hit eight different groups of banks.
template <int kR>
__device__ __forceinline__ uint32_t skc_group(int g, int lane) {
  constexpr int kG = kR / 4;  // 16-byte groups per thread row
  if constexpr (kG <= 1) {
    return (uint32_t)g;
  } else {
    constexpr int kShift = kG >= 8 ? 0 : kG == 4 ? 1 : 2;
    constexpr int kMask = (kG >= 8 ? 8 : kG) - 1;
    return (uint32_t)(g ^ ((lane >> kShift) & kMask));
  }
}

// Pushes columns [c0, c0 + kChunk) of this thread's accumulator row (v).
template <int S, int kMp, int kChunk>
__device__ __forceinline__ void skc_push(const uint32_t (&v)[kChunk], int c0, uint32_t area,
                                         uint32_t slice, uint32_t half, bool pair, int q,
                                         int lane) {
  constexpr int kR = kMp / S;                      // rows per owner
  constexpr int kRun = kR < kChunk ? kR : kChunk;  // contiguous rows per owner in this chunk
  static_assert(kRun >= 2 && (kRun == 2 || kRun % 4 == 0), "rows per store run");
  const uint32_t row_base =
      area + (((slice * 4u + (uint32_t)q) * 32u + (uint32_t)lane) * kR) * 4u;
#pragma unroll
  for (int j0 = 0; j0 < kChunk; j0 += kRun) {
    const int row = c0 + j0;  // first row of C of this run
    const int o = row / kR, i0 = row % kR;
    const uint32_t base =
        cluster_map(row_base, pair ? 2u * (uint32_t)o + half : (uint32_t)o);
    if constexpr (kRun == 2) {
      st_shared_cluster_v2(base + 4u * (uint32_t)i0, v[j0], v[j0 + 1]);
    } else {
#pragma unroll
      for (int i = 0; i < kRun; i += 4)
        st_shared_cluster_v4(base + 16u * skc_group<kR>((i0 + i) / 4, lane), v[j0 + i],
                             v[j0 + i + 1], v[j0 + i + 2], v[j0 + i + 3]);
    }
  }
}

// The owner's part: rows [slice R, (slice+1) R) of C at column n, each the
// sum of the S slices' partials in slice order, stored as bf16.
template <int S, int kMp>
__device__ __forceinline__ void skc_finish(uint32_t area, uint32_t slice, int q, int lane, int n,
                                           const SkinnyClusterArgs& args) {
  constexpr int kR = kMp / S;
  constexpr int kStep = kR == 2 ? 2 : 4;
#pragma unroll 1
  for (int i0 = 0; i0 < kR; i0 += kStep) {
    float acc[kStep];
#pragma unroll
    for (int i = 0; i < kStep; ++i) acc[i] = 0.f;
#pragma unroll
    for (int r = 0; r < S; ++r) {
      const uint32_t src =
          area + ((((uint32_t)r * 4u + (uint32_t)q) * 32u + (uint32_t)lane) * kR) * 4u +
          (kStep == 2 ? 4u * (uint32_t)i0 : 16u * skc_group<kR>(i0 / 4, lane));
      if constexpr (kStep == 2) {
        float a, b;
        ld_shared_v2_f32(src, a, b);
        acc[0] += a;
        acc[1] += b;
      } else {
        float a, b, c, d;
        ld_shared_v4_f32(src, a, b, c, d);
        acc[0] += a;
        acc[1] += b;
        acc[2] += c;
        acc[3] += d;
      }
    }
#pragma unroll
    for (int i = 0; i < kStep; ++i) {
      const int m = (int)slice * kR + i0 + i;
      if (m < args.M) args.C[(long long)m * args.ldc + n] = __float2bfloat16_rn(acc[i]);
    }
  }
}

template <int kMp, int kStages, bool kPair = false>
__global__ void __launch_bounds__(192)
gemm_skinny_cluster_kernel(const __grid_constant__ CUtensorMap tmap_b,   // N x K, box 64 x 128
                           const __grid_constant__ CUtensorMap tmap_a,   // M x K, box 64 x Mp (pairs: Mp / 2)
                           const SkinnyClusterArgs args) {
  using P = SkinnyClusterCfg<kMp, kStages, kPair>;
  extern __shared__ uint8_t smem_raw[];
  __shared__ alignas(8) uint64_t bar_full[kStages];
  __shared__ alignas(8) uint64_t bar_empty[kStages];
  __shared__ alignas(8) uint64_t bar_acc_full;
  __shared__ uint32_t tmem_slot;
  __shared__ uint32_t abort_word;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const uint32_t csize = cluster_nctarank();
  const uint32_t half = kPair ? (rank & 1u) : 0u;      // this CTA's half of a pair block
  const uint32_t leader = kPair ? (rank & ~1u) : rank;  // the pair's MMA issuer
  const uint32_t slice = kPair ? (rank >> 1) : rank;   // K slice
  const uint32_t slices = kPair ? (csize >> 1) : csize;
  const int tile = blockIdx.x / (int)csize;
  const int kb0 = (int)slice * args.kb_per;
  const int kb1 = kb0 + args.kb_per < args.k_blocks ? kb0 + args.kb_per : args.k_blocks;
  const int row0 = tile * P::kBlockRows + (int)half * P::kRowsB;  // this CTA's first row of B
  const uint32_t smem_base = (smem_u32(smem_raw) + 1023u) & ~1023u;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(smem_u32(&bar_full[s]), kPair ? 2 : 1);  // pairs: both CTAs' bytes, in the leader
      mbar_init(smem_u32(&bar_empty[s]), 1);
    }
    mbar_init(smem_u32(&bar_acc_full), 1);
    abort_word = 0;
    fence_mbar_init_cluster();
    prefetch_tmap(&tmap_b);
    prefetch_tmap(&tmap_a);
  }
  if (warp == 1) {
    if constexpr (kPair) {
      tmem_alloc_pair(smem_u32(&tmem_slot), P::kTmemAlloc);
      tmem_relinquish_pair();
    } else {
      tmem_alloc_1(smem_u32(&tmem_slot), P::kTmemAlloc);
      tmem_relinquish_1();
    }
  }
  tc_fence_before_sync();
  // Every CTA of the cluster has started and initialised its barriers before
  // any peer signals them or writes its shared memory.
  cluster_sync_all();
  tc_fence_after_sync();
  const uint32_t tmem_base = tmem_slot;

  WaitCtx wctx;
  wctx.status = args.status;
  wctx.timeout_ns = args.timeout_ns;
  wctx.abort_local = smem_u32(&abort_word);
  wctx.abort_peer = kPair ? cluster_map(smem_u32(&abort_word), rank ^ 1u) : smem_u32(&abort_word);

  bool acc_ok = true;
  if (warp == 0) {
    if (lane == 0) {
      uint32_t stage = 0, phase = 0;
      const uint64_t pol_b = args.l2_hint ? l2_policy_evict_first() : l2_policy_evict_normal();
      const uint64_t pol_a = args.l2_hint ? l2_policy_evict_last() : l2_policy_evict_normal();
      // K blocks in order (starting each block of B at a rotated K block, as
      // the split-K kernel does, measured ~1 us slower here at M = 16 and 64
      // after a written flush, and the same with L2 clean).
      for (int i = 0; i < kb1 - kb0; ++i) {
        const int kb = kb0 + i;
        if (!wait_bounded(smem_u32(&bar_empty[stage]), phase ^ 1u, wctx, kErrWaitEmpty)) break;
        const uint32_t sb = smem_base + stage * P::kStageBytes;
        if constexpr (kPair) {
          // The pair MMA commits a freed slot to the leader's empty barrier
          // only; the leader's producer passes it on to its peer's.  (One
          // commit arriving in both CTAs at once measured the same.)
          if (half == 0 && i >= kStages)
            mbar_arrive_cluster(cluster_map(smem_u32(&bar_empty[stage]), rank + 1u));
          const uint32_t fb = cluster_map(smem_u32(&bar_full[stage]), leader);
          mbar_arrive_expect_tx_cluster(fb, P::kStageBytes);
          tma_load_2d_pair_hint(sb, &tmap_b, kb * kSlabK, row0, fb, pol_b);
          tma_load_2d_pair_hint(sb + P::kSlabB, &tmap_a, kb * kSlabK, (int)half * P::kRowsA, fb,
                                pol_a);
        } else {
          const uint32_t fb = smem_u32(&bar_full[stage]);
          mbar_arrive_expect_tx(fb, P::kStageBytes);
          tma_load_2d_hint(sb, &tmap_b, kb * kSlabK, row0, fb, pol_b);
          tma_load_2d_hint(sb + P::kSlabB, &tmap_a, kb * kSlabK, 0, fb, pol_a);
        }
        if (++stage == kStages) { stage = 0; phase ^= 1u; }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0 && half == 0) {
      const uint32_t idesc = make_idesc_bf16_f32(P::kBlockRows, kMp);
      uint32_t stage = 0, phase = 0;
      for (int kb = kb0; kb < kb1; ++kb) {
        if (!wait_bounded(smem_u32(&bar_full[stage]), phase, wctx, kErrWaitFull)) break;
        tc_fence_after_sync();
        const uint32_t sb = smem_base + stage * P::kStageBytes;
        const uint64_t bdesc_big = make_sdesc_k128(sb);
        const uint64_t adesc_small = make_sdesc_k128(sb + P::kSlabB);
#pragma unroll
        for (int k = 0; k < kSlabK / kMmaK; ++k) {
          const uint32_t acc = (kb != kb0 || k != 0) ? 1u : 0u;
          if constexpr (kPair)
            umma_bf16_pair(tmem_base, bdesc_big + 2ull * k, adesc_small + 2ull * k, idesc, acc);
          else
            umma_bf16_1(tmem_base, bdesc_big + 2ull * k, adesc_small + 2ull * k, idesc, acc);
        }
        if constexpr (kPair)
          umma_commit_pair(cluster_map(smem_u32(&bar_empty[stage]), rank));
        else
          umma_commit_1(smem_u32(&bar_empty[stage]));
        if (++stage == kStages) { stage = 0; phase ^= 1u; }
      }
      // Each completes once every MMA above has (also when there were none);
      // the epilogues of both halves wait for it before TMEM is read or freed.
      if constexpr (kPair) {
        umma_commit_pair(cluster_map(smem_u32(&bar_acc_full), rank));
        umma_commit_pair(cluster_map(smem_u32(&bar_acc_full), rank + 1u));
      } else {
        umma_commit_1(smem_u32(&bar_acc_full));
      }
    }
    __syncwarp();
  } else {
    int ok = 0;
    if (lane == 0) ok = wait_bounded(smem_u32(&bar_acc_full), 0, wctx, kErrWaitAccFull);
    acc_ok = __shfl_sync(0xffffffffu, ok, 0) != 0;
    tc_fence_after_sync();
  }

  // Cross-slice reduction (skc_push / skc_finish).  Once every CTA of the
  // cluster has seen its MMAs complete (first barrier), no operand load or
  // MMA touches any ring any more, so the rings become the reduction area:
  // every slice pushes all its partial rows into their owners' rings with
  // fire-and-forget DSMEM stores, one barrier makes them visible, and each
  // owner adds its rows' partials in slice order and stores them as bf16.
  // (Earlier forms, on an 8192-row B: a remote load per row and slice, 5 us
  // at Mp = 16 and 15 us at Mp = 64; 4-byte pushes in 32-row chunks with a
  // barrier each, 6 and 12 us at Mp = 64 and 128.)  All 6 warps take part in
  // the barriers; the 4 epilogue warps move the data.
  const bool empty_slice = kb1 <= kb0;  // this slice saw no K blocks: its TMEM holds nothing
  const int quarter = warp & 3;
  const int n_local = quarter * 32 + lane;  // row of B within this CTA's 128 = column of C
  const int n = row0 + n_local;
  cluster_sync_all();
  if (warp >= 2) {
#pragma unroll 1
    for (int c = 0; c < kMp / P::kChunk; ++c) {
      uint32_t v[P::kChunk];
      if (acc_ok && !empty_slice) {
        if constexpr (P::kChunk == 16)
          tmem_ld_32x32b_x16(tmem_base + ((uint32_t)(quarter * 32) << 16) + c * 16,
                             *reinterpret_cast<uint32_t(*)[16]>(v));
        else
          tmem_ld_32x32b_x32(tmem_base + ((uint32_t)(quarter * 32) << 16) + c * 32,
                             *reinterpret_cast<uint32_t(*)[32]>(v));
        tmem_wait_ld();
      } else {
#pragma unroll
        for (int j = 0; j < P::kChunk; ++j) v[j] = 0u;
      }
      const int c0 = c * P::kChunk;
      switch (slices) {
        case 1: skc_push<1, kMp, P::kChunk>(v, c0, smem_base, slice, half, kPair, quarter, lane); break;
        case 2: skc_push<2, kMp, P::kChunk>(v, c0, smem_base, slice, half, kPair, quarter, lane); break;
        case 4: skc_push<4, kMp, P::kChunk>(v, c0, smem_base, slice, half, kPair, quarter, lane); break;
        default: skc_push<8, kMp, P::kChunk>(v, c0, smem_base, slice, half, kPair, quarter, lane); break;
      }
    }
  }
  cluster_sync_all();
  if (warp >= 2 && n < args.N) {
    switch (slices) {
      case 1: skc_finish<1, kMp>(smem_base, slice, quarter, lane, n, args); break;
      case 2: skc_finish<2, kMp>(smem_base, slice, quarter, lane, n, args); break;
      case 4: skc_finish<4, kMp>(smem_base, slice, quarter, lane, n, args); break;
      default: skc_finish<8, kMp>(smem_base, slice, quarter, lane, n, args); break;
    }
  }

  tc_fence_before_sync();
  if constexpr (kPair) {
    // both CTAs of the pair are done with its TMEM before either frees it,
    // and neither exits before the pair's deallocation has completed
    cluster_sync_all();
    if (warp == 1) {
      tc_fence_after_sync();
      tmem_dealloc_pair(tmem_base, P::kTmemAlloc);
    }
    cluster_sync_all();
  } else {
    __syncthreads();
    if (warp == 1) {
      tc_fence_after_sync();
      tmem_dealloc_1(tmem_base, P::kTmemAlloc);
    }
  }
}

}  // namespace b200

namespace b200 {

// ---------------------------------------------------------------------------
// Stream-K variant: every SM streams the same number of B bytes, in one
// launch, with no workspace clear of the output and no rounding pass.  The
// problem's work items, (128-row block of B = tile) x (K block), are laid
// out tile by tile and cut into G contiguous ranges of equal length, one per
// CTA (G = SMs).  A range is the tail of one tile, whole tiles, then the
// head of another:
//   * a whole tile: the epilogue rounds TMEM to bf16 and TMA-stores C^T;
//   * part of a tile: the epilogue writes the fp32 partial into slot j of
//     the tile (j = this CTA's position among the tile's n contributors, in
//     K order) and raises flag (tile, j, lane quarter).
// After its range every contributor finishes a share of each partial tile
// it touched: the tile's output is cut into pieces (lane quarter, 32
// columns), contributor j takes pieces j, j + n, ... (for n = 2 the second
// contributor takes all: it then waits only for the CTA below it, while a
// share would make both wait for each other); for each it waits,
// bounded, for the n flags of the piece's quarter, loads the n slot
// granules of the piece, adds them in K order, rounds and stores C.
// Spreading the fix-up this way keeps
// every SM's share of slot reads at about one slot per partial tile; a
// single finishing CTA per tile read all n slots and was the critical path.
// A slot is laid out [lane quarter][Mp m][32 n] fp32, so a piece of a slot
// (kChunk x 32 floats) is contiguous.
// Contributors wait for CTAs of higher index too, so the launch is
// cooperative: all G CTAs are resident together.  Slots live in a per-call
// workspace; flags are raised to the call's epoch (the launcher's per-stream
// flag arrays, or cleared per-call flags).
struct SkinnyStreamArgs {
  int M, N, K;
  int l2_hint;
  int tiles;         // ceil(N / (kTiles x 128))
  int k_blocks;      // K blocks per tile, ceil(K / kBK)
  long long total;   // tiles x k_blocks
  int max_seg;       // slots per tile
  float* slots;      // [tiles][max_seg][4 quarters][kTiles x kMp][32] fp32
  unsigned int* flags;  // [tiles][max_seg][4], below `epoch` at launch
  unsigned int epoch;   // value a raised flag takes in this call
  int* status;
  unsigned long long timeout_ns;
};

// First CTA (of G) whose range [c total / G, (c+1) total / G) holds item x.
__device__ __forceinline__ int stream_owner(long long x, long long total, int G) {
  return (int)(((x + 1) * G + total - 1) / total) - 1;
}

// kPair (launched in 2-CTA clusters): a tile is 256 rows of B, CTA r of the
// pair loads its own 128 of them and rows [r Mp/2, (r+1) Mp/2) of A, and the
// pair leader issues tcgen05.mma.cta_group::2 (M = 256, N = Mp), which reads
// both CTAs' shared memory: each SM streams its rows of B but only half of
// A's slab, where a single CTA re-reads A's whole slab per 128 rows of B.
// Each CTA's TMEM holds its own 128 rows x Mp columns, so the epilogue, the
// slots and the fix-up are the single-CTA kernel's, per CTA half h = 2 t + r
// of tile t; the ranges of (tile, K block) items are per pair.
template <int kMp, int kSlabs, int kTiles = 1, bool kPair = false>
__global__ void __launch_bounds__(192, 1)
gemm_skinny_stream_kernel(const __grid_constant__ CUtensorMap tmap_b,   // N x K, box 64 x 128
                          const __grid_constant__ CUtensorMap tmap_a,   // M x K, box 64 x Mp (pairs: Mp / 2)
                          const __grid_constant__ CUtensorMap tmap_c,   // C bf16 M x N, box 32 x kChunk
                          const SkinnyStreamArgs args) {
  using P = SkinnyCfg<kMp, kSlabs, kTiles, kPair>;
  static_assert(P::kAccBufs == 2, "the stream-K kernel double-buffers its accumulator");
  constexpr int kStages = P::kStages;
  constexpr int kChunk = P::kChunk;
  // A tile is kTiles 128-row blocks of B sharing each A slab; its
  // accumulator is kMpT = kTiles x Mp TMEM columns (block i at i x Mp), read
  // by the epilogue in kMpT / kChunk chunks, kCpb of them per block.
  constexpr int kMpT = kTiles * kMp;
  constexpr int kTileRows = (kPair ? 2 : kTiles) * P::kRowsB;
  // rows of B one slot / flag unit covers: a tile, or a pair tile's CTA half
  constexpr int kUnitRows = kPair ? P::kRowsB : kTileRows;
  constexpr int kCpb = kMp / kChunk;
  extern __shared__ uint8_t smem_raw[];
  __shared__ alignas(8) uint64_t bar_full[kStages];
  __shared__ alignas(8) uint64_t bar_empty[kStages];
  __shared__ alignas(8) uint64_t bar_acc_full[2];
  __shared__ alignas(8) uint64_t bar_acc_empty[2];
  __shared__ alignas(8) uint64_t bar_drain;
  __shared__ uint32_t tmem_slot;
  __shared__ uint32_t abort_word;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = kPair ? cluster_ctarank() : 0u;
  const int worker = kPair ? (int)(blockIdx.x >> 1) : (int)blockIdx.x;  // pair or CTA
  const int G = kPair ? (int)(gridDim.x >> 1) : (int)gridDim.x;
  const long long lo = (long long)worker * args.total / G;
  const long long hi = (long long)(worker + 1) * args.total / G;
  const int KB = args.k_blocks;
  const uint32_t smem_base = (smem_u32(smem_raw) + 1023u) & ~1023u;
  const uint32_t store_base = smem_base + kStages * P::kStageBytes;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(smem_u32(&bar_full[s]), kPair ? 2 : 1);  // pairs: both CTAs' bytes, in the leader
      mbar_init(smem_u32(&bar_empty[s]), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(smem_u32(&bar_acc_full[b]), 1);
      mbar_init(smem_u32(&bar_acc_empty[b]), kPair ? 8 : 4);  // every epilogue warp (of the pair)
    }
    mbar_init(smem_u32(&bar_drain), 1);
    abort_word = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    prefetch_tmap(&tmap_b);
    prefetch_tmap(&tmap_a);
    prefetch_tmap(&tmap_c);
  }
  if (warp == 1) {
    if constexpr (kPair) {
      tmem_alloc_pair(smem_u32(&tmem_slot), P::kTmemAlloc);
      tmem_relinquish_pair();
    } else {
      tmem_alloc_1(smem_u32(&tmem_slot), P::kTmemAlloc);
      tmem_relinquish_1();
    }
  }
  tc_fence_before_sync();
  if constexpr (kPair) cluster_sync_all(); else __syncthreads();
  tc_fence_after_sync();
  const uint32_t tmem_base = tmem_slot;

  WaitCtx wctx;
  wctx.status = args.status;
  wctx.timeout_ns = args.timeout_ns;
  wctx.abort_local = smem_u32(&abort_word);
  wctx.abort_peer = kPair ? cluster_map(smem_u32(&abort_word), rank ^ 1u) : smem_u32(&abort_word);

  // Segments of [lo, hi): tile t, K blocks [kb0, kb1).
#define B200_FOR_SEGMENTS(...)                                                \
  for (long long pos = lo; pos < hi;) {                                       \
    const int t = (int)(pos / KB);                                            \
    const int kb0 = (int)(pos - (long long)t * KB);                           \
    const long long rest = hi - (long long)t * KB;                            \
    const int kb1 = rest < KB ? (int)rest : KB;                               \
    __VA_ARGS__                                                               \
    pos = (long long)t * KB + kb1;                                            \
  }

  if (warp == 0) {
    if (lane == 0) {
      const uint64_t pol_b = args.l2_hint ? l2_policy_evict_first() : l2_policy_evict_normal();
      const uint64_t pol_a = args.l2_hint ? l2_policy_evict_last() : l2_policy_evict_normal();
      uint32_t stage = 0, phase = 0;
      uint32_t filled = 0;  // ring slots this producer has filled (pairs: the leader forwards frees)
      bool ok = true;
      B200_FOR_SEGMENTS({
        for (int kb = kb0; ok && kb < kb1; ++kb) {
          if (!wait_bounded(smem_u32(&bar_empty[stage]), phase ^ 1u, wctx, kErrWaitEmpty)) {
            ok = false;
            break;
          }
          const uint32_t sb = smem_base + stage * P::kStageBytes;
          if constexpr (kPair) {
            // The pair MMA commits a freed slot to the leader's empty barrier
            // only; the leader's producer passes it on to the peer's.
            if (rank == 0 && filled >= (uint32_t)kStages)
              mbar_arrive_cluster(cluster_map(smem_u32(&bar_empty[stage]), 1));
            ++filled;
            const uint32_t fb = cluster_map(smem_u32(&bar_full[stage]), 0);
            mbar_arrive_expect_tx_cluster(fb, P::kStageBytes);
#pragma unroll
            for (int sl = 0; sl < kSlabs; ++sl)
              tma_load_2d_pair_hint(sb + sl * P::kSlabB, &tmap_b, kb * P::kBK + sl * kSlabK,
                                    t * kTileRows + (int)rank * P::kRowsB, fb, pol_b);
#pragma unroll
            for (int sl = 0; sl < kSlabs; ++sl)
              tma_load_2d_pair_hint(sb + P::kBytesB + sl * P::kSlabA, &tmap_a,
                                    kb * P::kBK + sl * kSlabK, (int)rank * P::kRowsA, fb, pol_a);
          } else {
            const uint32_t fb = smem_u32(&bar_full[stage]);
            mbar_arrive_expect_tx(fb, P::kStageBytes);
#pragma unroll
            for (int i = 0; i < kTiles; ++i)
#pragma unroll
              for (int sl = 0; sl < kSlabs; ++sl)
                tma_load_2d_hint(sb + (i * kSlabs + sl) * P::kSlabB, &tmap_b,
                                 kb * P::kBK + sl * kSlabK, t * kTileRows + i * P::kRowsB, fb,
                                 pol_b);
#pragma unroll
            for (int sl = 0; sl < kSlabs; ++sl)
              tma_load_2d_hint(sb + P::kBytesB + sl * P::kSlabA, &tmap_a,
                               kb * P::kBK + sl * kSlabK, 0, fb, pol_a);
          }
          if (++stage == kStages) { stage = 0; phase ^= 1u; }
        }
        if (!ok) break;
      })
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0 && rank == 0) {
      const uint32_t idesc = make_idesc_bf16_f32(kPair ? 2 * P::kRowsB : P::kRowsB, kMp);
      uint32_t stage = 0, phase = 0;
      int it = 0;
      bool ok = true;
      B200_FOR_SEGMENTS({
        const uint32_t buf = it & 1, acc_phase = (it >> 1) & 1;
        if (!wait_bounded(smem_u32(&bar_acc_empty[buf]), acc_phase ^ 1u, wctx, kErrWaitAccEmpty))
          break;
        tc_fence_after_sync();
        const uint32_t d_tmem = tmem_base + buf * kMpT;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!wait_bounded(smem_u32(&bar_full[stage]), phase, wctx, kErrWaitFull)) {
            ok = false;
            break;
          }
          tc_fence_after_sync();
          const uint32_t sb = smem_base + stage * P::kStageBytes;
#pragma unroll
          for (int sl = 0; sl < kSlabs; ++sl) {
            const uint64_t adesc = make_sdesc_k128(sb + P::kBytesB + sl * P::kSlabA);
#pragma unroll
            for (int k = 0; k < kSlabK / kMmaK; ++k)
#pragma unroll
              for (int i = 0; i < kTiles; ++i) {
                const uint64_t bdesc = make_sdesc_k128(sb + (i * kSlabs + sl) * P::kSlabB);
                const uint32_t acc = (kb != kb0 || sl != 0 || k != 0) ? 1u : 0u;
                if constexpr (kPair)
                  umma_bf16_pair(d_tmem + i * kMp, bdesc + 2ull * k, adesc + 2ull * k, idesc, acc);
                else
                  umma_bf16_1(d_tmem + i * kMp, bdesc + 2ull * k, adesc + 2ull * k, idesc, acc);
              }
          }
          if constexpr (kPair)
            umma_commit_pair(cluster_map(smem_u32(&bar_empty[stage]), 0));
          else
            umma_commit_1(smem_u32(&bar_empty[stage]));
          if (++stage == kStages) { stage = 0; phase ^= 1u; }
        }
        if (!ok) break;
        if constexpr (kPair) {
          umma_commit_pair(cluster_map(smem_u32(&bar_acc_full[buf]), 0));
          umma_commit_pair(cluster_map(smem_u32(&bar_acc_full[buf]), 1));
        } else {
          umma_commit_1(smem_u32(&bar_acc_full[buf]));
        }
        ++it;
      })
      // Every MMA this thread issued must finish before TMEM is freed.
      if constexpr (kPair)
        umma_commit_pair(cluster_map(smem_u32(&bar_drain), 0));
      else
        umma_commit_1(smem_u32(&bar_drain));
      if (!mbar_try_wait(smem_u32(&bar_drain), 0))
        wait_slow(smem_u32(&bar_drain), 0, wctx, kErrWaitDrain, false);
    }
    __syncwarp();
  } else {
    // Epilogue: warp w holds TMEM lanes 32 (w % 4) .. + 31 = rows n of B
    // (columns of C); register j of a chunk is row m = c kChunk + j of C.
    const int quarter = warp & 3;
    const uint32_t my_store = store_base + (warp - 2) * 2 * P::kStoreBuf;
    uint32_t nstore = 0;
    int it = 0;
    // Partial tiles of this range (at most two: the first and the last
    // segment), finished after the range: tile, this CTA's slot, slots.
    int fix_t[2] = {0, 0}, fix_j[2] = {0, 0}, fix_n[2] = {0, 0};
    int nfix = 0;
    bool alive = true;
    // Rounds 32 (or Mp) rows of C held as fp32 bits in v and TMA-stores them
    // through this warp's staging buffers ([kChunk m][32 n] bf16) at lane
    // quarter q of tile t.
    auto store_bf16 = [&](const uint32_t* v, int t, int q, int c) {
      // chunk c: block c / kCpb of the tile, rows (c % kCpb) kChunk .. of C
      const uint32_t sb = my_store + (nstore & 1u) * P::kStoreBuf;
      if (lane == 0) bulk_wait_group_read<1>();
      __syncwarp();
#pragma unroll
      for (int j = 0; j < kChunk; ++j) {
        const __nv_bfloat16 h = __float2bfloat16_rn(__uint_as_float(v[j]));
        st_shared_u16(sb + (j * 32 + lane) * 2u, *reinterpret_cast<const uint16_t*>(&h));
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        tma_store_2d(&tmap_c, sb, t * kUnitRows + (c / kCpb) * P::kRowsB + q * 32,
                     (c % kCpb) * kChunk);
        bulk_commit_group();
      }
      ++nstore;
    };
    B200_FOR_SEGMENTS({
      if (!alive) break;
      const uint32_t buf = it & 1, acc_phase = (it >> 1) & 1;
      int ok = 0;
      if (lane == 0) ok = wait_bounded(smem_u32(&bar_acc_full[buf]), acc_phase, wctx, kErrWaitAccFull);
      if (!__shfl_sync(0xffffffffu, ok, 0)) {
        alive = false;
        break;
      }
      tc_fence_after_sync();
      const uint32_t tbase = tmem_base + buf * kMpT + ((uint32_t)(quarter * 32) << 16);
      const bool whole = kb0 == 0 && kb1 == KB;
      const int first = stream_owner((long long)t * KB, args.total, G);
      const int j = worker - first;
      // slot / flag unit: the tile, or this CTA's half of a pair tile
      const int h = kPair ? 2 * t + (int)rank : t;
      float* slot = args.slots + ((long long)h * args.max_seg + j) * kMpT * P::kRowsB +
                    quarter * kMpT * 32 + lane;
#pragma unroll 1
      for (int c = 0; c < kMpT / kChunk; ++c) {
        uint32_t v[kChunk];
        if constexpr (kChunk == 16)
          tmem_ld_32x32b_x16(tbase + c * 16, *reinterpret_cast<uint32_t(*)[16]>(v));
        else
          tmem_ld_32x32b_x32(tbase + c * 32, *reinterpret_cast<uint32_t(*)[32]>(v));
        tmem_wait_ld();
        if (c == kMpT / kChunk - 1) {
          tc_fence_before_sync();
          __syncwarp();
          if (lane == 0) {
            if constexpr (kPair)
              mbar_arrive_cluster(cluster_map(smem_u32(&bar_acc_empty[buf]), 0));
            else
              mbar_arrive_local(smem_u32(&bar_acc_empty[buf]));
          }
        }
        if (whole) {
          store_bf16(v, h, quarter, c);
        } else {
          // slot[quarter][m][lane]: each warp-wide store covers 128 contiguous bytes
#pragma unroll
          for (int jj = 0; jj < kChunk; ++jj) slot[(c * kChunk + jj) * 32] = __uint_as_float(v[jj]);
        }
      }
      if (!whole) {
        const int n = stream_owner((long long)t * KB + KB - 1, args.total, G) - first + 1;
        // (With two contributors the second finishes the tile from its own
        // quarters of its own slot: no other warp reads them.)
        if (n != 2 || j != 1) {
          asm volatile("fence.acq_rel.gpu;" ::: "memory");
          __syncwarp();
          if (lane == 0)
            st_release_gpu_u32(args.flags + ((long long)h * args.max_seg + j) * 4 + quarter,
                               args.epoch);
        }
        if (nfix < 2) {
          fix_t[nfix] = h;
          fix_j[nfix] = j;
          fix_n[nfix] = n;
          ++nfix;
        }
      }
      ++it;
    })
    // Finish the partial tiles.  A tile's output is cut into pieces (lane
    // quarter q, chunk c); contributor j of the tile's n finishes pieces
    // j, j + n, j + 2n, ..., dealt in turn over its four epilogue warps
    // (n = 2: contributor 1 finishes all of them, each warp its quarter).  A
    // warp waits, bounded, for all flags of its tiles (one warp-wide poll
    // covers a tile's 4n flags), then loads the pieces' slot granules with
    // 16-byte loads, adds each piece's n granules in K order, rounds and
    // stores it.  (Bulk copies of the granules
    // need a generic-to-async proxy fence first, which waits for this
    // warp's C stores still in flight and cost more than the loads.)
    constexpr int kChunks = kMpT / kChunk;
    constexpr int kPieces = 4 * kChunks;
    // At most a whole tile (n = 2) plus a third of another (n >= 3).
    constexpr int kMaxMine = (kPieces + kPieces / 3) / 4 + 2;
    int mine[kMaxMine];  // (f << 8) | piece
    int nmine = 0;
    int has = 0;  // bit f: this warp finishes pieces of tile f
    {
      int dealt = 0;
#pragma unroll 1
      for (int f = 0; f < nfix; ++f) {
        if (fix_n[f] == 2) {
          // Two contributors: the second (whose range starts with the tile,
          // so its partial is ready first) finishes the whole tile, each
          // warp its own lane quarter, and waits only for the CTA below it.
          if (fix_j[f] == 1)
#pragma unroll 1
            for (int pc = quarter; pc < kPieces && nmine < kMaxMine; pc += 4) {
              mine[nmine++] = (f << 8) | pc;
              has |= 1 << f;
            }
          continue;
        }
#pragma unroll 1
        for (int pc = fix_j[f]; pc < kPieces; pc += fix_n[f], ++dealt)
          if ((dealt & 3) == warp - 2 && nmine < kMaxMine) {
            mine[nmine++] = (f << 8) | pc;
            has |= 1 << f;
          }
      }
    }
#pragma unroll 1
    for (int f = 0; alive && f < nfix; ++f) {
      if (!((has >> f) & 1)) continue;
      const unsigned int* tflags = args.flags + (long long)fix_t[f] * args.max_seg * 4;
      // flags of slots other than this CTA's own when it finishes alone
      const int nflags = fix_n[f] == 2 ? 4 : 4 * fix_n[f];
#pragma unroll 1
      for (int base = 0; alive && base < nflags; base += 32) {
        const int idx = base + lane;
        const unsigned long long t0 = globaltimer_ns();
        for (;;) {
          const bool up = idx >= nflags || (int)(ld_acquire_gpu_u32(tflags + idx) - args.epoch) >= 0;
          if (__all_sync(0xffffffffu, up)) break;
          int give_up = 0;
          if (lane == 0 && globaltimer_ns() - t0 > args.timeout_ns) {
            atomicCAS(args.status, 0, kErrWaitPartial);
            give_up = 1;
          }
          if (__shfl_sync(0xffffffffu, give_up, 0)) {
            alive = false;
            break;
          }
          __nanosleep(64);
        }
      }
    }
    __syncwarp();  // orders every lane after the flags the other lanes acquired
    // A granule (kChunk m x 32 n fp32) is kVec float4 per lane: float4 i of
    // lane l holds m = l / 8 + 4 i, n = 4 (l % 8) .. + 3.  The granules of
    // this warp's pieces are loaded in sequence (piece by piece, slots in K
    // order), kRound at a time whatever piece they belong to; a piece is
    // rounded and stored when its last granule has been added.
    constexpr int kVec = kChunk / 4;
    constexpr int kRound = 4;
    const long long slot_floats = (long long)kMpT * P::kRowsB;
    auto granule = [&](int x, int sl) {
      const int f = mine[x] >> 8, pc = mine[x] & 255;
      return args.slots + ((long long)fix_t[f] * args.max_seg + sl) * slot_floats +
             ((pc & 3) * kMpT + (pc >> 2) * kChunk) * 32 + 4 * lane;
    };
    auto store_piece = [&](const float4* acc, int x) {
      const int f = mine[x] >> 8, pc = mine[x] & 255;
      const uint32_t sb = my_store + (nstore & 1u) * P::kStoreBuf;
      if (lane == 0) bulk_wait_group_read<1>();
      __syncwarp();
#pragma unroll
      for (int i = 0; i < kVec; ++i) {
        const __nv_bfloat162 lo = __floats2bfloat162_rn(acc[i].x, acc[i].y);
        const __nv_bfloat162 hi = __floats2bfloat162_rn(acc[i].z, acc[i].w);
        st_shared_v2(sb + (((lane >> 3) + 4 * i) * 32 + 4 * (lane & 7)) * 2u,
                     *reinterpret_cast<const uint32_t*>(&lo), *reinterpret_cast<const uint32_t*>(&hi));
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        tma_store_2d(&tmap_c, sb,
                     fix_t[f] * kUnitRows + ((pc >> 2) / kCpb) * P::kRowsB + (pc & 3) * 32,
                     ((pc >> 2) % kCpb) * kChunk);
        bulk_commit_group();
      }
      ++nstore;
    };
    float4 acc[kVec];
#pragma unroll
    for (int i = 0; i < kVec; ++i) acc[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    int lx = 0, ls = 0;  // next granule to load: piece lx, slot ls
#pragma unroll 1
    while (alive && lx < nmine) {
      float4 xv[kRound][kVec];
      int gx[kRound];
      int cnt = 0;
#pragma unroll
      for (int u = 0; u < kRound; ++u) {
        if (lx < nmine) {
          const float* g = granule(lx, ls);
#pragma unroll
          for (int i = 0; i < kVec; ++i) xv[u][i] = ld_global_cg_v4(g + 128 * i);
          gx[u] = lx;
          if (++ls == fix_n[mine[lx] >> 8]) {
            ls = 0;
            ++lx;
          }
          cnt = u + 1;
        }
      }
#pragma unroll
      for (int u = 0; u < kRound; ++u) {
        if (u < cnt) {
#pragma unroll
          for (int i = 0; i < kVec; ++i) {
            acc[i].x += xv[u][i].x;
            acc[i].y += xv[u][i].y;
            acc[i].z += xv[u][i].z;
            acc[i].w += xv[u][i].w;
          }
          const bool last = u + 1 < cnt ? gx[u + 1] != gx[u] : lx > gx[u];
          if (last) {
            store_piece(acc, gx[u]);
#pragma unroll
            for (int i = 0; i < kVec; ++i) acc[i] = make_float4(0.f, 0.f, 0.f, 0.f);
          }
        }
      }
    }
    // (the staging buffers' reads only: the stores' global writes complete with the grid)
    if (lane == 0) bulk_wait_group_read<0>();
    __syncwarp();
  }
#undef B200_FOR_SEGMENTS

  tc_fence_before_sync();
  if constexpr (kPair) cluster_sync_all(); else __syncthreads();
  if (warp == 1) {
    tc_fence_after_sync();
    if constexpr (kPair)
      tmem_dealloc_pair(tmem_base, P::kTmemAlloc);
    else
      tmem_dealloc_1(tmem_base, P::kTmemAlloc);
  }
  if constexpr (kPair) cluster_sync_all();
}

}  // namespace b200
