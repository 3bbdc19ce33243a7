// Host/device shared layout rules of the sm_100a BF16 GEMM: the tile
// geometry, the tcgen05 instruction and shared-memory descriptors, and the
// persistent tile rasteriser.  Everything here is plain integer arithmetic so
// the CPU tests can check it through the C-ABI without a GPU.
//
// Geometry (one 2-CTA cluster = one "pair"):
//   pair tile        256 (M) x 256 or 512 (N), K stepped in blocks of 64/128
//   per CTA          128 rows of A and, per 256-wide N sub-tile, 128 rows of
//                    B (its half of the sub-tile)
//   MMA              tcgen05.mma.cta_group::2.kind::f16, M=256 N=256 K=16
//   accumulator      fp32 in TMEM, 128 lanes x 256 columns per CTA per
//                    sub-tile; 512 columns in all
// The reference computes the same 256x256 cluster tile with BK=64
// (kernel_v8.cu:775-833, launch_matmul_v8<128, 256, 64>).
#pragma once
#include <stdint.h>

#if defined(__CUDACC__)
#define B200_HD __host__ __device__ __forceinline__
#else
#define B200_HD static inline
#endif

namespace b200 {

constexpr int kPairM = 256;        // rows of C per pair tile
constexpr int kSubN = 256;         // columns of one N sub-tile (= MMA N)
constexpr int kCtaM = 128;         // rows of A (and of C) owned by one CTA
constexpr int kCtaN = 128;         // rows of B per sub-tile loaded by one CTA
constexpr int kSlabK = 64;         // K elements per 128 B swizzle slab (one TMA box)
constexpr int kSlabBytes = 128 * kSlabK * 2;   // 16 KiB: one 128-row operand slab
constexpr int kMmaK = 16;          // K per tcgen05.mma kind::f16
constexpr int kTmemCols = 512;     // the whole TMEM of an SM
constexpr int kStoreCols = 64;     // epilogue chunk width (one 128 B swizzle row of bf16)
constexpr int kStoreBufBytes = 32 * kStoreCols * 2;        // 4 KiB: 32 rows x 64 columns
constexpr int kSmemBudget = 227 * 1024;                    // opt-in shared memory per CTA
constexpr int kSmemReserve = 1024 + 1024;                  // 1 KiB alignment + static/barriers

// Output modes of the epilogue.
enum OutMode : int {
  kOutBf16 = 0,    // C bf16 = round(acc)                    (the GEMM)
  kOutF32 = 1,     // C fp32 = acc                           (K-split partials)
  kOutF32Add = 2,  // C fp32 += acc, by TMA reduce-add       (split-K workspace)
  kOutBf16Epi = 3, // C bf16 = round(alpha acc + bias[n] + beta R[m][n])
  kOutKsplit = 4,  // K-split over ranks: peers' tiles sent, own rows summed + rounded
};

// Kernel configuration.
//   kSlabs  K slabs of 64 per pipeline stage (stage K = 64 * kSlabs)
//   kSubW   width of one N sub-tile (= MMA N): 256, or 128 / 64 for grids too
//           small to occupy every SM with 256-wide tiles (kNSub = 1 only);
//           each CTA loads kSubW / 2 rows of B per sub-tile
//   kNSub   N sub-tiles per pair tile: 1 -> 256 x kSubW pair tiles with
//           two TMEM accumulators (epilogue of tile i overlaps the MMAs of
//           tile i+1); 2 -> 256 x 512 pair tiles with one 512-column
//           accumulator, where each A slab feeds two MMAs, so 25% fewer
//           operand bytes cross L2 per FLOP, at the cost of the MMA waiting
//           for the epilogue to drain TMEM once per tile.
// A stage holds kSlabs slabs of A, then kNSub x kSlabs slabs of B (16 KiB
// each, 1 KiB aligned); the ring depth is whatever fits beside the epilogue
// staging buffers.
template <int kSlabs, int kNSub, int kSubW = kSubN>
struct Cfg {
  static_assert(kSubW == 256 || (kNSub == 1 && (kSubW == 128 || kSubW == 64)),
                "sub-tiles are 256 wide, or 128 / 64 wide in single-sub-tile configurations");
  static constexpr int kRowsB = kSubW / 2;              // rows of B per CTA per sub-tile
  static constexpr int kSlabB = kRowsB * kSlabK * 2;    // bytes of one B slab (1 KiB multiple)
  static constexpr int kTileN = kNSub * kSubW;
  static constexpr int kAccBufs = kNSub == 1 ? 2 : 1;
  static constexpr int kEpiWarps = 4 * kNSub;          // one per (lane quarter, sub-tile)
  static constexpr int kWarps = 2 + kEpiWarps;         // producer, MMA, epilogue
  static constexpr int kThreads = 32 * kWarps;
  static constexpr int kBK = kSlabs * kSlabK;
  static constexpr int kBytesA = kSlabs * kSlabBytes;
  static constexpr int kBytesB = kNSub * kSlabs * kSlabB;
  static constexpr int kStageBytes = kBytesA + kBytesB;
  // 256-wide tiles: two staging buffers per epilogue warp, so storing chunk
  // c overlaps converting chunk c+1.  512-wide tiles: the epilogue first
  // moves its whole TMEM slice into registers (as packed bf16) to free the
  // single accumulator early, then stores from registers through one buffer.
  static constexpr int kStoreBufs = kNSub == 1 ? 2 : 1;
  static constexpr int kStoreBytes = kEpiWarps * kStoreBufs * kStoreBufBytes;
  static constexpr int kStages = (kSmemBudget - kStoreBytes - kSmemReserve) / kStageBytes;
  static constexpr int kSmemBytes = kStages * kStageBytes + kStoreBytes + 1024;
  static_assert(kStages >= 2, "pipeline needs at least two stages");
  static_assert(kAccBufs * kTileN <= kTmemCols, "accumulators exceed TMEM");
};

// ---------------------------------------------------------------------------
// tcgen05 instruction descriptor for kind::f16 (PTX ISA "Instruction
// descriptor" table): bits 4-5 D format (1 = f32), 7-9 A format (1 = bf16),
// 10-12 B format (1 = bf16), 15/16 A/B major (0 = K-major), 17-22 N>>3,
// 24-28 M>>4.  The reference packs the same fields (kernel_v8.cu:450-455).
B200_HD uint32_t make_idesc_bf16_f32(int mma_m, int mma_n) {
  return (1u << 4) | (1u << 7) | (1u << 10) |
         ((uint32_t)(mma_n >> 3) << 17) | ((uint32_t)(mma_m >> 4) << 24);
}

// Shared-memory matrix descriptor for a K-major operand tile written by TMA
// with 128 B swizzling: rows of 128 B, 8-row swizzle atoms of 1024 B.
//   bits  0-13 start address >> 4
//   bits 16-29 leading byte offset >> 4 (unused for swizzled K-major: 0)
//   bits 32-45 stride byte offset >> 4 (1024 B between 8-row groups)
//   bits 46-47 descriptor version (1 on sm_100)
//   bits 49-51 base offset (0: atoms are 1024 B aligned)
//   bits 61-63 layout (2 = 128 B swizzle)
// Same encoding as the reference's make_smem_desc (kernel_v1.cu:159-164).
B200_HD uint64_t make_sdesc_k128(uint32_t smem_addr) {
  return (uint64_t)((smem_addr & 0x3FFFFu) >> 4) |
         ((uint64_t)(1024u >> 4) << 32) |
         (1ull << 46) |
         (2ull << 61);
}

// ---------------------------------------------------------------------------
// Persistent tile rasteriser.  Pair tiles are numbered 0..tiles-1 and pair p
// of P processes tiles p, p+P, p+2P, ...; consecutive numbers are therefore
// in flight at the same time.  Numbers walk across a band of |group| tiles
// of one dimension before stepping along the other, so the ~74 tiles in
// flight touch about |group| + 74/|group| distinct 256-row blocks of A and B
// instead of 2*74: that keeps the working set of one wave inside the 126 MB
// L2.  group > 0 makes bands of tile-rows (sweeping N), group < 0 bands of
// tile-columns (sweeping M).  Odd bands sweep backwards (serpentine), so the
// last operand blocks of one band are the first of the next.  The reference
// instead deals a Hilbert curve over the tile grid
// (kernel_v8.cu:338-358,796-820); both are permutations of the grid.
B200_HD void tile_coord(int t, int tiles_m, int tiles_n, int group, int* tm, int* tn) {
  const bool cols = group < 0;
  const int g = cols ? -group : group;
  const int banded = cols ? tiles_n : tiles_m;   // dimension cut into bands
  const int swept = cols ? tiles_m : tiles_n;    // dimension each band sweeps
  const int band_tiles = g * swept;
  const int band = t / band_tiles;
  const int first = band * g;
  int width = banded - first;
  if (width > g) width = g;
  const int r = t - band * band_tiles;
  const int a = first + r % width;
  int b = r / width;
  if (band & 1) b = swept - 1 - b;
  *tm = cols ? b : a;
  *tn = cols ? a : b;
}

// ---------------------------------------------------------------------------
// Stream-K split of the tail tiles (shared by the kernel and the CPU tests).
// The tail's (tile, K block) items, item = tile * k_blocks + kb, are cut into
// G contiguous ranges, pair p taking [p items / G, (p+1) items / G), where G
// = min(pairs, items) so that no range is empty.

B200_HD int sk_range_pairs(long long items, int pairs) {
  return items < pairs ? (int)items : pairs;
}

B200_HD void sk_range(int pair, long long items, int G, long long* lo, long long* hi) {
  *lo = (long long)pair * items / G;
  *hi = (long long)(pair + 1) * items / G;
}

// First pair (of G) whose range holds item x.
B200_HD int sk_owner(long long x, long long items, int G) {
  return (int)(((x + 1) * G + items - 1) / items) - 1;
}

// Next segment of a pair's range [lo, *pos), walked from its end: the tile
// holding item *pos - 1 and its K blocks [kb0, kb1) inside the range; moves
// *pos to the segment's first item.  A pair thus meets first the head of the
// tile it shares with the next pair and last the tail of the tile it
// finishes.  Requires *pos > lo.
B200_HD void sk_next_segment(long long lo, long long* pos, int k_blocks, int* t, int* kb0,
                             int* kb1) {
  const int tile = (int)((*pos - 1) / k_blocks);
  const long long base = (long long)tile * k_blocks;
  *kb1 = (int)(*pos - base);
  *kb0 = lo > base ? (int)(lo - base) : 0;
  *t = tile;
  *pos = base + *kb0;
}

}  // namespace b200
