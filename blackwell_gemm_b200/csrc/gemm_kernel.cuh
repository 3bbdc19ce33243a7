// Persistent, warp-specialised BF16 GEMM for sm_100a:  C = A * B^T
//   A  M x K bf16, row stride lda (K-major)
//   B  N x K bf16, row stride ldb (K-major; the reference's "(K,N) view of an
//      N x K buffer", matmul.cpp:25-39)
//   C  M x N bf16, row stride ldc, fp32 accumulation, round-to-nearest-even
//
// One 2-CTA cluster ("pair") owns a 256 x (256 * kNSub) tile of C at a time
// (configurations in gemm_layout.h, Cfg).  Warp roles per CTA:
//   warp 0     TMA producer: fills the shared-memory ring of {A 128 x BK,
//              kNSub x B 128 x BK}
//   warp 1     TMEM owner; in the pair leader also the MMA issuer
//              (tcgen05.mma.cta_group::2, kNSub MMAs per K16 step)
//   warps 2..  epilogue, 4 per N sub-tile: tcgen05.ld -> bf16 -> swizzled
//              smem -> TMA store, one warp per (TMEM lane quarter, sub-tile),
//              each with its own two 4 KiB staging buffers so no epilogue
//              warp waits for another
// Pipelines:
//   full[s]/empty[s]        ring stage s (full lives in the leader: both
//                           producers arrive on it; empty lives in each CTA)
//   acc_full[b]/acc_empty[b] TMEM accumulator b (two 256-column buffers for
//                           256-wide tiles, so the epilogue of tile i
//                           overlaps the MMAs of tile i+1; one 512-column
//                           buffer for 512-wide tiles)
// Reference behaviour followed: kernel_v8.cu:360-773 (same math, same tile,
// same TMA/UMMA/epilogue data path); the scheduling here is a static
// persistent walk over a grouped raster (gemm_layout.h) instead of cluster
// launch control, and every wait is bounded (a stuck pipeline records an
// error code in `status` and the kernel returns instead of spinning).
#pragma once
#include <cuda.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "gemm_layout.h"
#include "ksplit_fused.cuh"
#include "sm100_ptx.cuh"

// TMEM loads (32 columns each) in flight per wait when a 512-wide tile's
// epilogue drains its single accumulator into registers (plain bf16 output).
#ifndef B200_DRAIN_BATCH
#define B200_DRAIN_BATCH 4
#endif

namespace b200 {

struct EpiArgs {
  float alpha, beta;
  const __nv_bfloat16* bias;   // N values (or null)
  const __nv_bfloat16* resid;  // M x N, row stride ldr (or null)
  int ldr;
};

struct GemmArgs {
  int M, N, K;
  int tiles_m, tiles_n, k_blocks, group;
  int splits;        // K slices per tile (split-K); 1 = whole K per tile
  int kb_per_split;  // K blocks per slice (the last slice may be shorter)
  int* status;                    // device error word (0 = ok)
  unsigned long long timeout_ns;  // bound on any single pipeline wait
  long long* prof;                // intra-kernel profiler rows (nullptr: off)
  int prof_entries;
  // Fused epilogue (kOutBf16Epi): C = round(alpha acc + bias[n] + beta R[m][n]);
  // bias and resid may be null, resid may alias C.
  EpiArgs epi;
  // K-split exchange (kOutKsplit only): see ksplit_fused.cuh.
  KsArgs ks;
  // L2 eviction policy of the A and B loads: 0 normal, 1 evict-first,
  // 2 evict-last.
  int l2_a, l2_b;
  // Work split.  Tiles [0, dp_tiles) (x splits) are dealt whole, pair p
  // taking units p, p + P, ...; a stream-K tail of sk_tiles further tiles is
  // cut into sk_items = sk_tiles x k_blocks (tile, K block) items, pair p
  // taking the contiguous range [p items / G, (p+1) items / G) (G = min(P,
  // items)) and walking it from its end.  A tile cut between pairs is finished by the pair
  // holding its last K blocks -- the first segment of that pair's range,
  // which it reaches last -- by adding the fp32 pieces the earlier pairs
  // left in sk_slots to its accumulator (bf16 output only).
  int dp_tiles, sk_tiles;
  long long sk_items;
  float* sk_slots;          // [pair][pieces][kPieceFloats]: the pair's piece of a tile it does not finish
  unsigned int* sk_flags;   // [pair][pieces], below sk_epoch at launch
  unsigned int sk_epoch;    // value a raised flag takes in this call
  // Dynamic dealing of the data-parallel units (null: static, pair p takes
  // units p, p + P, ...): sched[0] counts tickets taken after the first
  // wave, sched[1] pairs that are done; both 0 at launch, and the last pair
  // to finish sets them back to 0 (see WorkIter).
  unsigned int* sched;
};

__device__ __forceinline__ uint64_t l2_policy(int code) {
  return code == 1 ? l2_policy_evict_first()
                   : code == 2 ? l2_policy_evict_last() : l2_policy_evict_normal();
}

// Error codes written to GemmArgs::status by a wait that ran out.
enum : int {
  kErrWaitEmpty = 0x1001,     // producer waited on a ring slot
  kErrWaitFull = 0x1002,      // MMA waited on TMA data
  kErrWaitAccEmpty = 0x1003,  // MMA waited on the epilogue to free TMEM
  kErrWaitAccFull = 0x1004,   // epilogue waited on the MMA
  kErrWaitDrain = 0x1005,     // final wait for outstanding MMAs
  kErrWaitProbe = 0x1006,     // self-test kernel (wait that nothing releases)
  kErrWaitPeer = 0x1007,      // K-split: a peer's piece of an own tile never arrived
  kErrWaitPartial = 0x1008,   // stream-K: an earlier CTA's partial tile never arrived
  kErrWaitSched = 0x1009,     // dynamic dealing: a slot of the pair's unit ring
};

// Intra-kernel profiler tags; numbering and row format follow the
// reference's profiler.h:4-13,22-50 (row = [count, (smid, tag, start_ns,
// duration_ns) x entries]).  Recording stops when a row is full.
enum ProfTag : int {
  kTagSetup = 0, kTagIssueTMA, kTagIssueMMA, kTagWaitTMA, kTagWaitMMA,
  kTagWaitMainloop, kTagWaitEpilogue, kTagEpilogue,
};

template <bool kOn>
struct Prof {
  long long* row = nullptr;
  int cap = 0, cnt = 0, sm = 0;
  long long t0 = 0;
  int tag = 0;
  __device__ __forceinline__ void init(long long* base, int entries, int row_idx) {
    if constexpr (kOn) {
      row = base + (long long)row_idx * (1 + 4 * entries);
      cap = entries;
      sm = (int)smid();
    }
  }
  __device__ __forceinline__ void start(int t) {
    if constexpr (kOn) { tag = t; t0 = (long long)globaltimer_ns(); }
  }
  __device__ __forceinline__ void stop() {
    if constexpr (kOn) {
      if (cnt < cap) {
        long long* e = row + 1 + 4 * cnt;
        e[0] = sm; e[1] = tag; e[2] = t0; e[3] = (long long)globaltimer_ns() - t0;
        ++cnt;
      }
    }
  }
  __device__ __forceinline__ void flush() {
    if constexpr (kOn) row[0] = cnt;
  }
};

struct WaitCtx {
  int* status;
  unsigned long long timeout_ns;
  uint32_t abort_local;  // shared::cta address of this CTA's abort word
  uint32_t abort_peer;   // shared::cluster address of the peer's abort word
};

__device__ __forceinline__ uint32_t ld_volatile_shared(uint32_t addr) {
  uint32_t v;
  asm volatile("ld.volatile.shared.u32 %0, [%1];" : "=r"(v) : "r"(addr) : "memory");
  return v;
}

// Wait for `parity` on a local mbarrier.  Each poll may sleep up to
// kPollSuspendNs (it returns as soon as the phase completes).  Gives up when
// the abort word is set (another warp of the pair already gave up) or once
// timeout_ns has passed; in the latter case it records `code`, raises both
// CTAs' abort words and returns false so the caller can leave its loop and
// reach the teardown.  The bound is timeout_ns plus at most one burst of
// polls.
template <bool kAcqCluster = false>
__device__ __noinline__ bool wait_slow(uint32_t bar, uint32_t parity, const WaitCtx& w, int code,
                                       bool honour_abort) {
  const unsigned long long t0 = globaltimer_ns();
  for (;;) {
    // Poll in bursts; the abort word and the clock are read once per burst.
#pragma unroll 1
    for (int i = 0; i < 32; ++i)
      if (kAcqCluster ? mbar_try_wait_acq_cluster(bar, parity) : mbar_try_wait(bar, parity))
        return true;
    if (honour_abort && ld_volatile_shared(w.abort_local) != 0) return false;
    if (globaltimer_ns() - t0 > w.timeout_ns) {
      atomicCAS(w.status, 0, code);
      asm volatile("st.volatile.shared.u32 [%0], %1;" :: "r"(w.abort_local), "r"(1u) : "memory");
      st_cluster_u32(w.abort_peer, 1u);
      return false;
    }
  }
}

__device__ __forceinline__ bool wait_bounded(uint32_t bar, uint32_t parity, const WaitCtx& w,
                                             int code) {
  if (mbar_try_wait(bar, parity)) return true;
  return wait_slow(bar, parity, w, code, true);
}

// wait_bounded with acquire semantics at cluster scope (data written into
// this CTA's shared memory by the other CTA of the pair).
__device__ __forceinline__ bool wait_bounded_acq_cluster(uint32_t bar, uint32_t parity,
                                                         const WaitCtx& w, int code) {
  if (mbar_try_wait_acq_cluster(bar, parity)) return true;
  return wait_slow<true>(bar, parity, w, code, true);
}

// In place on 32 consecutive accumulator columns of one row (fp32 bits):
// v = alpha v + bias[col..] + beta resid[row][col..].  Rows >= M and columns
// >= N are left as they are (the store clips them).  Bias and residual rows
// are read with 16-byte loads (both are 16-byte aligned by contract).
__device__ __forceinline__ void epi_apply(uint32_t (&v)[32], const EpiArgs& e, int M, int N,
                                          int row, int col) {
  float f[32];
#pragma unroll
  for (int j = 0; j < 32; ++j) f[j] = e.alpha * __uint_as_float(v[j]);
  const bool full = col + 32 <= N;
  auto add8 = [&](const __nv_bfloat16* p, int j0, float scale) {
    const uint4 u = *reinterpret_cast<const uint4*>(p);
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      f[j0 + 2 * q] += scale * __uint_as_float(w[q] << 16);
      f[j0 + 2 * q + 1] += scale * __uint_as_float(w[q] & 0xFFFF0000u);
    }
  };
  if (e.bias != nullptr) {
    if (full) {
#pragma unroll
      for (int q = 0; q < 4; ++q) add8(e.bias + col + 8 * q, 8 * q, 1.0f);
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (col + j < N) f[j] += __bfloat162float(e.bias[col + j]);
    }
  }
  if (e.resid != nullptr && row < M) {
    const __nv_bfloat16* r = e.resid + (long long)row * e.ldr + col;
    if (full) {
#pragma unroll
      for (int q = 0; q < 4; ++q) add8(r + 8 * q, 8 * q, e.beta);
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (col + j < N) f[j] += e.beta * __bfloat162float(r[j]);
    }
  }
#pragma unroll
  for (int j = 0; j < 32; ++j) v[j] = __float_as_uint(f[j]);
}

// K-split exchange: the whole (converged) warp waits until *flag, a word in
// this GPU's memory that a peer raises, reaches `epoch`.  Every lane reads it
// with acquire semantics at system scope, so each lane's later loads see the
// peer's piece.  Gives up when the pair's abort word is set or after
// timeout_ns (records kErrWaitPeer and raises both abort words); the verdict
// is warp-uniform.
template <bool kSys = true>
__device__ __noinline__ bool wait_peer_flag(const unsigned int* flag, unsigned int epoch,
                                            const WaitCtx& w, unsigned long long timeout_ns,
                                            int code = kErrWaitPeer) {
  const int lane = threadIdx.x & 31;
  unsigned long long t0 = 0;
  for (int round = 0;; ++round) {
    const unsigned int v = kSys ? ld_acquire_sys_u32(flag) : ld_acquire_gpu_u32(flag);
    const bool ok = (int)(v - epoch) >= 0;
    if (__all_sync(0xffffffffu, ok)) return true;
    int give_up = 0;
    if (lane == 0) {
      const unsigned long long now = globaltimer_ns();
      if (round == 0) t0 = now;
      if (ld_volatile_shared(w.abort_local) != 0) {
        give_up = 1;
      } else if (now - t0 > timeout_ns) {
        atomicCAS(w.status, 0, code);
        asm volatile("st.volatile.shared.u32 [%0], %1;" ::"r"(w.abort_local), "r"(1u) : "memory");
        st_cluster_u32(w.abort_peer, 1u);
        give_up = 1;
      }
    }
    if (__shfl_sync(0xffffffffu, give_up, 0)) return false;
    __nanosleep(256);
  }
}

// K-split exchange, own tile: v (fp32 bits of this rank's partial, columns
// 32h..32h+31 of this lane's row) <- P_0 + P_1 + ... + P_{P-1}, summed left to
// right in rank order.  `recv` points at this lane's float4 of source 0's
// piece in this rank's receive slots; source q's piece is q * stride floats
// further.
__device__ __forceinline__ void ks_accumulate(uint32_t (&v)[32], const float* recv,
                                              long long stride, int h, int rank, int nranks) {
  float s[32];
  auto add_src = [&](int q, bool first) {
    const float* p = recv + q * stride + h * 8 * 128;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float4 x = ld_global_cg_v4(p + j * 128);
      if (first) {
        s[4 * j] = x.x; s[4 * j + 1] = x.y; s[4 * j + 2] = x.z; s[4 * j + 3] = x.w;
      } else {
        s[4 * j] += x.x; s[4 * j + 1] += x.y; s[4 * j + 2] += x.z; s[4 * j + 3] += x.w;
      }
    }
  };
  if (rank == 0) {
#pragma unroll
    for (int j = 0; j < 32; ++j) s[j] = __uint_as_float(v[j]);
  } else {
    add_src(0, true);
  }
#pragma unroll 1
  for (int q = 1; q < nranks; ++q) {
    if (q == rank) {
#pragma unroll
      for (int j = 0; j < 32; ++j) s[j] += __uint_as_float(v[j]);
    } else {
      add_src(q, false);
    }
  }
#pragma unroll
  for (int j = 0; j < 32; ++j) v[j] = __float_as_uint(s[j]);
}

// K-split exchange: owner of 256-row tile tm and the index of the piece
// (32 rows x 256 columns) that epilogue warp `quarter` of CTA `cta` holds for
// 256-column block cb.
__device__ __forceinline__ long long ks_piece(const KsArgs& ks, int tm, int cb, int cblocks,
                                              int cta, int quarter, int* owner) {
  *owner = tm / ks.tiles_m_own;
  return ((long long)((tm - *owner * ks.tiles_m_own) * cblocks + cb) * 2 + cta) * 4 + quarter;
}

// K-split exchange, another owner's tile (and stream-K partial tiles): write
// this warp's piece (TMEM columns tbase .. tbase + 255, fp32) into `dst`
// (piece layout), hand the accumulator back after its last column, then --
// unless `flag` is null -- raise `flag` to `epoch` once every lane's stores
// are visible system-wide.
template <bool kSys = true>
__device__ __forceinline__ void ks_send_piece(uint32_t tbase, float* dst, unsigned int* flag,
                                              unsigned int epoch, uint32_t acc_empty) {
  const int lane = threadIdx.x & 31;
  dst += 4 * lane;
#pragma unroll 1
  for (int c = 0; c < kSubN / 32; ++c) {
    uint32_t v[32];
    tmem_ld_32x32b_x32(tbase + c * 32, v);
    tmem_wait_ld();
    if (c == kSubN / 32 - 1) {
      tc_fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(acc_empty);
    }
#pragma unroll
    for (int j = 0; j < 8; ++j)
      st_global_v4(dst + (c * 8 + j) * 128, v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
  }
  if (flag == nullptr) return;
  if constexpr (kSys) {
    fence_acq_rel_sys();
    __syncwarp();
    if (lane == 0) st_release_sys_u32(flag, epoch);
  } else {
    asm volatile("fence.acq_rel.gpu;" ::: "memory");
    __syncwarp();
    if (lane == 0) st_release_gpu_u32(flag, epoch);
  }
}

// Stream-K tail tile: v (this pair's fp32 partial, columns 32h .. 32h+31 of
// this lane's row) <- P_c0 + P_c0+1 + ... + P_last + v, the earlier pairs'
// pieces in K order then this pair's own.  `piece` points at this lane's
// float4 of pair c0's piece; pair c's is (c - c0) * stride floats further.
__device__ __forceinline__ void sk_accumulate(uint32_t (&v)[32], const float* piece,
                                              long long stride, int heads, int h) {
  float s[32];
#pragma unroll 1
  for (int c = 0; c < heads; ++c) {
    const float* p = piece + c * stride + h * 8 * 128;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float4 x = ld_global_cg_v4(p + j * 128);
      if (c == 0) {
        s[4 * j] = x.x; s[4 * j + 1] = x.y; s[4 * j + 2] = x.z; s[4 * j + 3] = x.w;
      } else {
        s[4 * j] += x.x; s[4 * j + 1] += x.y; s[4 * j + 2] += x.z; s[4 * j + 3] += x.w;
      }
    }
  }
#pragma unroll
  for (int j = 0; j < 32; ++j) v[j] = __float_as_uint(s[j] + __uint_as_float(v[j]));
}

// Work unit u -> tile (tm, tn) and its K-block range [kb0, kb1).  In the
// K-split exchange the tiles come in P phases, phase f over the rows of
// owner (rank + 1 + f) mod P, each phase rastered like a whole grid.
template <int kOut>
__device__ __forceinline__ void unit_coord(int u, const GemmArgs& a, int* tm, int* tn, int* kb0,
                                           int* kb1) {
  const int t = u / a.splits;
  const int s = u - t * a.splits;
  if constexpr (kOut == kOutKsplit) {
    const int own = a.ks.tiles_m_own * a.tiles_n;
    const int phase = t / own;
    int owner = a.ks.rank + 1 + phase;
    if (owner >= a.ks.nranks) owner -= a.ks.nranks;
    tile_coord(t - phase * own, a.ks.tiles_m_own, a.tiles_n, a.group, tm, tn);
    *tm += owner * a.ks.tiles_m_own;
  } else {
    tile_coord(t, a.tiles_m, a.tiles_n, a.group, tm, tn);
  }
  *kb0 = s * a.kb_per_split;
  const int end = *kb0 + a.kb_per_split;
  *kb1 = end < a.k_blocks ? end : a.k_blocks;
}

// Pairs taking stream-K work: all P, or one per item when there are fewer
// items, so that no range is empty (sk_range_pairs, gemm_layout.h).
__device__ __forceinline__ int sk_pairs(const GemmArgs& a, int P) {
  return sk_range_pairs(a.sk_items, P);
}

// Dynamic dealing of data-parallel units.  The first wave is static (pair p
// takes unit p); after that the pair leader's producer thread (the fetcher)
// takes tickets from the global counter GemmArgs::sched[0] -- unit = P +
// ticket -- and publishes each unit it will process in a ring of
// kSchedDepth slots held in both CTAs' shared memory (a unit, or -1 for "no
// more work"), with a full barrier per slot in each CTA and an empty
// barrier per slot in the leader.  Every other role of the pair (the peer's
// producer, the MMA thread, every epilogue warp of both CTAs) takes the units
// from the ring in the same order and frees its slot.  Units are therefore
// handed out in increasing order as pairs become free, so the tiles in flight
// stay a compact window of the raster however the pairs' speeds drift, and
// no pair idles while another still has several tiles queued.  The ring
// never deadlocks: the fetcher waits for slot reuse only on units at least
// kSchedDepth behind, whose data it has already loaded.
constexpr int kSchedDepth = 8;

struct SchedRing {
  uint32_t full;          // shared::cta address of this CTA's full[0]
  uint32_t full_self;     // shared::cluster address of this CTA's full[0] (fetcher)
  uint32_t unit;          // shared::cta address of this CTA's unit[0]
  uint32_t empty_leader;  // shared::cluster address of the leader's empty[0]
  uint32_t empty_local;   // shared::cta address of the leader's empty[0] (fetcher)
  uint32_t full_peer;     // shared::cluster address of the peer's full[0] (fetcher)
  uint32_t unit_peer;     // shared::cluster address of the peer's unit[0] (fetcher)
};

enum SchedRole : int {
  kSchedStatic = 0,  // GemmArgs::sched is null: pair p takes units p, p + P, ...
  kSchedFetch = 1,   // the leader's producer thread: takes tickets, publishes units
  kSchedTake = 2,    // one thread takes published units
  kSchedTakeWarp = 3 // a whole warp: lane 0 takes, the unit is broadcast
};

// One pair's work, in order: its stream-K segments (a tile and a K-block
// range within it), last tile first, then its data-parallel units.  Walking
// the stream-K range backwards makes a pair compute the head of the tile it
// shares with the next pair first and the tail of the tile it finishes last;
// doing the stream-K work before the whole tiles lets that tail's epilogue
// (which adds the heads) overlap the next tile's MMAs.
struct WorkIter {
  int u, dp_units, npairs;
  long long lo, pos;  // stream-K range still to walk: [lo, pos)
  int role, n, ticket;
  unsigned int* counter;
  SchedRing ring;
  const WaitCtx* w;
  __device__ __forceinline__ void init(const GemmArgs& a, int pair, int P, int sched_role = kSchedStatic,
                                       const SchedRing* r = nullptr, const WaitCtx* wc = nullptr) {
    npairs = P;
    u = pair;
    dp_units = a.dp_tiles * a.splits;
    lo = pos = 0;
    const int G = sk_pairs(a, P);
    if (a.sk_tiles > 0 && pair < G) sk_range(pair, a.sk_items, G, &lo, &pos);
    role = a.sched != nullptr ? sched_role : kSchedStatic;
    counter = a.sched;
    n = 0;
    ticket = pair;  // the first wave is dealt statically
    if (r != nullptr) ring = *r;
    w = wc;
  }
  // Fetcher: publish the next unit (or -1) in the ring, then take the next
  // ticket (its latency hides behind the loads of the unit just published).
  // -2 when a wait ran out.
  __device__ __forceinline__ int publish() {
    const uint32_t slot = n % kSchedDepth, lap = n / kSchedDepth;
    ++n;
    // (acquire at cluster scope: the peer's takers read their slot before
    // arriving, and this thread then overwrites it remotely)
    if (!wait_bounded_acq_cluster(ring.empty_local + slot * 8u, (lap & 1u) ^ 1u, *w, kErrWaitSched))
      return -2;
    const int unit = ticket < dp_units ? ticket : -1;
    st_shared_u32(ring.unit + slot * 4u, (uint32_t)unit);
    st_cluster_u32(ring.unit_peer + slot * 4u, (uint32_t)unit);
    mbar_arrive_release_cluster(ring.full_self + slot * 8u);
    mbar_arrive_release_cluster(ring.full_peer + slot * 8u);
    if (unit >= 0) ticket = npairs + (int)atomicAdd(counter, 1u);
    return unit;
  }
  // Taker (one thread): the next published unit, -2 when a wait ran out.
  __device__ __forceinline__ int take() {
    const uint32_t slot = n % kSchedDepth, lap = n / kSchedDepth;
    ++n;
    if (!wait_bounded_acq_cluster(ring.full + slot * 8u, lap & 1u, *w, kErrWaitSched)) return -2;
    const int unit = ld_shared_s32(ring.unit + slot * 4u);
    mbar_arrive_release_cluster(ring.empty_leader + slot * 8u);
    return unit;
  }
  // Next work: tile (tm, tn), K blocks [kb0, kb1), stream-K tile index sk_t
  // (-1 for a data-parallel unit).  False when the pair's work is done.
  template <int kOut, bool kSK>
  __device__ __forceinline__ bool next(const GemmArgs& a, int* tm, int* tn, int* kb0, int* kb1,
                                       int* sk_t) {
    if constexpr (kSK) {
      if (pos > lo) {
        int t;
        sk_next_segment(lo, &pos, a.k_blocks, &t, kb0, kb1);
        tile_coord(a.dp_tiles + t, a.tiles_m, a.tiles_n, a.group, tm, tn);
        *sk_t = t;
        return true;
      }
    }
    int unit;
    if (role == kSchedStatic) {
      if (u >= dp_units) return false;
      unit = u;
      u += npairs;
    } else if (role == kSchedFetch) {
      unit = publish();
    } else if (role == kSchedTake) {
      unit = take();
    } else {
      int v = 0;
      if ((threadIdx.x & 31) == 0) v = take(); else ++n;
      unit = __shfl_sync(0xffffffffu, v, 0);
    }
    if (unit < 0) return false;
    unit_coord<kOut>(unit, a, tm, tn, kb0, kb1);
    *sk_t = -1;
    return true;
  }
  // Fetcher, once after its loop however it ended: count this pair done; the
  // last pair resets the counters for the next launch on the stream.  The
  // fence orders this pair's last ticket before its "done", so no ticket is
  // taken after the reset.
  __device__ __forceinline__ void finish() {
    if (role != kSchedFetch) return;
    __threadfence();
    if (atomicAdd(counter + 1, 1u) == (unsigned int)npairs - 1u) {
      atomicExch(counter, 0u);
      atomicExch(counter + 1, 0u);
    }
  }
};

__device__ __forceinline__ uint32_t pack_bf16x2(uint32_t lo, uint32_t hi) {
  __nv_bfloat162 h = __floats2bfloat162_rn(__uint_as_float(lo), __uint_as_float(hi));
  return *reinterpret_cast<uint32_t*>(&h);
}

template <bool kProfile, int kSlabs, int kNSub, int kOut, int kSubW = kSubN, bool kSK = false>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(Cfg<kSlabs, kNSub, kSubW>::kThreads, 1)
gemm_bf16_pair_kernel(const __grid_constant__ CUtensorMap tmap_a,
                      const __grid_constant__ CUtensorMap tmap_b,
                      const __grid_constant__ CUtensorMap tmap_c,
                      const GemmArgs args) {
  using P = Cfg<kSlabs, kNSub, kSubW>;
  static_assert(kOut == kOutBf16 || kOut == kOutKsplit || kNSub == 1,
                "fp32 outputs and fused epilogues use 256-wide pair tiles");
  static_assert(kSubW == kSubN || kOut == kOutBf16, "narrow sub-tiles: plain bf16 output only");
  static_assert(!kSK || (kOut == kOutBf16 && kSubW == kSubN && kNSub == 1 && !kProfile),
                "stream-K tails: 256 x 256 pair tiles (double-buffered TMEM), bf16 output, "
                "no profiler");
  constexpr int kStages = P::kStages;
  constexpr int kAccBufs = P::kAccBufs;
  extern __shared__ uint8_t smem_raw[];
  __shared__ alignas(8) uint64_t bar_full[kStages];
  __shared__ alignas(8) uint64_t bar_empty[kStages];
  __shared__ alignas(8) uint64_t bar_acc_full[kAccBufs];
  __shared__ alignas(8) uint64_t bar_acc_empty[kAccBufs];
  __shared__ alignas(8) uint64_t bar_drain;
  __shared__ alignas(8) uint64_t bar_sched_full[kSchedDepth];
  __shared__ alignas(8) uint64_t bar_sched_empty[kSchedDepth];
  __shared__ int sched_unit[kSchedDepth];
  __shared__ uint32_t tmem_slot;
  __shared__ uint32_t abort_word;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const int pair = blockIdx.x >> 1;
  const int npairs = gridDim.x >> 1;
  // Work units: (tile, K slice) pairs, unit u = tile * splits + slice.

  // 1 KiB aligned start: the 128 B swizzle atoms (8 rows x 128 B) must be.
  const uint32_t smem_base = (smem_u32(smem_raw) + 1023u) & ~1023u;
  const uint32_t store_base = smem_base + kStages * P::kStageBytes;

  Prof<kProfile> prof;
  if constexpr (kProfile) {
    if (lane == 0) {
      prof.init(args.prof, args.prof_entries, blockIdx.x * P::kWarps + warp);
      prof.start(kTagSetup);
    }
  }

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(smem_u32(&bar_full[s]), 2);   // one expect_tx arrive per CTA
      mbar_init(smem_u32(&bar_empty[s]), 1);  // one tcgen05.commit (or its forward)
    }
    for (int b = 0; b < kAccBufs; ++b) {
      mbar_init(smem_u32(&bar_acc_full[b]), 1);
      mbar_init(smem_u32(&bar_acc_empty[b]), 2 * P::kEpiWarps);  // every epilogue warp of the pair
    }
    mbar_init(smem_u32(&bar_drain), 1);
    for (int s = 0; s < kSchedDepth; ++s) {
      mbar_init(smem_u32(&bar_sched_full[s]), 1);  // the fetcher's publication
      // (leader) the peer's producer, the MMA thread, every epilogue warp of the pair
      mbar_init(smem_u32(&bar_sched_empty[s]), 2 + 2 * P::kEpiWarps);
    }
    abort_word = 0;
    fence_mbar_init_cluster();
    prefetch_tmap(&tmap_a);
    prefetch_tmap(&tmap_b);
    prefetch_tmap(&tmap_c);
  }
  if (warp == 1) {
    tmem_alloc_pair(smem_u32(&tmem_slot), kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before_sync();
  cluster_sync_all();
  tc_fence_after_sync();
  const uint32_t tmem_base = tmem_slot;

  WaitCtx wctx;
  wctx.status = args.status;
  wctx.timeout_ns = args.timeout_ns;
  wctx.abort_local = smem_u32(&abort_word);
  wctx.abort_peer = cluster_map(smem_u32(&abort_word), rank ^ 1u);

  SchedRing ring;
  ring.full = smem_u32(&bar_sched_full[0]);
  ring.full_self = cluster_map(ring.full, rank);
  ring.unit = smem_u32(&sched_unit[0]);
  ring.empty_leader = cluster_map(smem_u32(&bar_sched_empty[0]), 0);
  ring.empty_local = smem_u32(&bar_sched_empty[0]);
  ring.full_peer = cluster_map(ring.full, rank ^ 1u);
  ring.unit_peer = cluster_map(ring.unit, rank ^ 1u);

  if constexpr (kProfile) {
    if (lane == 0) prof.stop();
  }

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      const uint32_t full_leader = cluster_map(smem_u32(&bar_full[0]), 0);
      const uint32_t empty_peer = cluster_map(smem_u32(&bar_empty[0]), 1);
      const uint64_t pol_a = l2_policy(args.l2_a), pol_b = l2_policy(args.l2_b);
      uint32_t stage = 0, phase = 0;
      uint32_t filled = 0;  // ring slots this producer has filled so far
      bool ok = true;
      WorkIter wi;
      wi.init(args, pair, npairs, rank == 0 ? kSchedFetch : kSchedTake, &ring, &wctx);
      int tm, tn, kb0, kb1, skt;
      while (ok && wi.template next<kOut, kSK>(args, &tm, &tn, &kb0, &kb1, &skt)) {
        const int a_row = tm * kPairM + (int)rank * kCtaM;
        const int b_row = tn * P::kTileN + (int)rank * P::kRowsB;
        for (int kb = kb0; kb < kb1; ++kb) {
          if constexpr (kProfile) prof.start(kTagWaitMMA);
          if (!wait_bounded(smem_u32(&bar_empty[stage]), phase ^ 1u, wctx, kErrWaitEmpty)) {
            ok = false;
            break;
          }
          // The MMA commits a freed slot only to the leader's empty barrier
          // (one tcgen05.commit per stage); the leader's producer passes each
          // completion on to the peer's empty barrier.
          if (rank == 0 && filled >= (uint32_t)kStages) mbar_arrive_cluster(empty_peer + stage * 8u);
          ++filled;
          if constexpr (kProfile) { prof.stop(); prof.start(kTagIssueTMA); }
          const uint32_t fb = full_leader + stage * 8u;
          const uint32_t sa = smem_base + stage * P::kStageBytes;
          mbar_arrive_expect_tx_cluster(fb, P::kStageBytes);
#pragma unroll
          for (int sl = 0; sl < kSlabs; ++sl) {
            const int x = kb * P::kBK + sl * kSlabK;
            tma_load_2d_pair_hint(sa + sl * kSlabBytes, &tmap_a, x, a_row, fb, pol_a);
#pragma unroll
            for (int sub = 0; sub < kNSub; ++sub)
              tma_load_2d_pair_hint(sa + P::kBytesA + (sub * kSlabs + sl) * P::kSlabB, &tmap_b,
                                    x, b_row + sub * kSubW, fb, pol_b);
          }
          if constexpr (kProfile) prof.stop();
          if (++stage == kStages) { stage = 0; phase ^= 1u; }
        }
      }
      wi.finish();
      if constexpr (kProfile) prof.flush();
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA
    if (rank == 0 && lane == 0) {
      const uint32_t idesc = make_idesc_bf16_f32(kPairM, kSubW);
      const uint32_t empty_self = cluster_map(smem_u32(&bar_empty[0]), 0);
      const uint32_t accf_self = cluster_map(smem_u32(&bar_acc_full[0]), 0);
      const uint32_t accf_peer = cluster_map(smem_u32(&bar_acc_full[0]), 1);
      uint32_t stage = 0, phase = 0;
      int it = 0;
      bool ok = true;
      WorkIter wi;
      wi.init(args, pair, npairs, kSchedTake, &ring, &wctx);
      int tm, tn, kb0, kb1, skt;
      while (ok && wi.template next<kOut, kSK>(args, &tm, &tn, &kb0, &kb1, &skt)) {
        const int my_it = it++;
        const uint32_t buf = my_it % kAccBufs, acc_phase = (my_it / kAccBufs) & 1;
        if constexpr (kProfile) prof.start(kTagWaitEpilogue);
        if (!wait_bounded(smem_u32(&bar_acc_empty[buf]), acc_phase ^ 1u, wctx, kErrWaitAccEmpty))
          break;
        if constexpr (kProfile) prof.stop();
        tc_fence_after_sync();
        const uint32_t d_tmem = tmem_base + buf * P::kTileN;
        for (int kb = kb0; kb < kb1; ++kb) {
          if constexpr (kProfile) prof.start(kTagWaitTMA);
          if (!wait_bounded(smem_u32(&bar_full[stage]), phase, wctx, kErrWaitFull)) {
            ok = false;
            break;
          }
          tc_fence_after_sync();
          if constexpr (kProfile) { prof.stop(); prof.start(kTagIssueMMA); }
          const uint32_t sa = smem_base + stage * P::kStageBytes;
#pragma unroll
          for (int sl = 0; sl < kSlabs; ++sl) {
            const uint64_t adesc = make_sdesc_k128(sa + sl * kSlabBytes);
#pragma unroll
            for (int k = 0; k < kSlabK / kMmaK; ++k) {
#pragma unroll
              for (int sub = 0; sub < kNSub; ++sub) {
                const uint64_t bdesc =
                    make_sdesc_k128(sa + P::kBytesA + (sub * kSlabs + sl) * P::kSlabB);
                // +32 B per K16 step inside the 128 B swizzled row (>>4 => +2)
                umma_bf16_pair(d_tmem + sub * kSubW, adesc + 2ull * k, bdesc + 2ull * k, idesc,
                               (kb != kb0 || sl != 0 || k != 0) ? 1u : 0u);
              }
            }
          }
          umma_commit_pair(empty_self + stage * 8u);
          if constexpr (kProfile) prof.stop();
          if (++stage == kStages) { stage = 0; phase ^= 1u; }
        }
        if (!ok) break;
        umma_commit_pair(accf_self + buf * 8u);
        umma_commit_pair(accf_peer + buf * 8u);
      }
      // Every MMA this thread issued must finish before TMEM is freed.
      umma_commit_pair(cluster_map(smem_u32(&bar_drain), 0));
      if (!mbar_try_wait(smem_u32(&bar_drain), 0))
        wait_slow(smem_u32(&bar_drain), 0, wctx, kErrWaitDrain, false);
    }
    if constexpr (kProfile) {
      if (lane == 0) prof.flush();
    }
    __syncwarp();
  } else {
    // ----------------------------------------------------------- epilogue
    // Warp w reads TMEM lane quarter w % 4 (hardware rule) of sub-tile
    // (w - 2) / 4: 32 rows x 256 columns per tile.
    const int quarter = warp & 3;
    const int ew = warp - 2;
    const int sub = ew >> 2;
    const uint32_t my_store = store_base + ew * P::kStoreBufs * kStoreBufBytes;
    const uint32_t acc_empty_leader = cluster_map(smem_u32(&bar_acc_empty[0]), 0);
    uint32_t nstore = 0;
    int it = 0;
    WorkIter wi;
    wi.init(args, pair, npairs, kSchedTakeWarp, &ring, &wctx);
    int tm, tn, kb0, kb1, skt;
    while (wi.template next<kOut, kSK>(args, &tm, &tn, &kb0, &kb1, &skt)) {
      const int my_it = it++;
      const uint32_t buf = my_it % kAccBufs, acc_phase = (my_it / kAccBufs) & 1;
      if constexpr (kProfile) {
        if (lane == 0) prof.start(kTagWaitMainloop);
      }
      // Lane 0 waits and the verdict is broadcast, so the warp stays converged
      // for the warp-collective tcgen05.ld below.
      int ok = 0;
      if (lane == 0) ok = wait_bounded(smem_u32(&bar_acc_full[buf]), acc_phase, wctx, kErrWaitAccFull);
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) break;
      tc_fence_after_sync();
      if constexpr (kProfile) {
        if (lane == 0) { prof.stop(); prof.start(kTagEpilogue); }
      }
      const uint32_t tbase =
          tmem_base + buf * P::kTileN + sub * kSubW + ((uint32_t)(quarter * 32) << 16);
      const int row0 = tm * kPairM + (int)rank * kCtaM + quarter * 32;
      const int col0 = tn * P::kTileN + sub * kSubW;
      // Stream-K tile cut between pairs: a piece that is not the tile's last
      // K blocks goes to this pair's slot for the pair that finishes the
      // tile; the last K blocks wait for the earlier pieces (heads) and add
      // them while draining (sk_heads > 0).
      int sk_heads = 0;
      const float* sk_piece = nullptr;
      constexpr long long kSkStride = 2LL * P::kEpiWarps * kPieceFloats;  // one pair's pieces
      if constexpr (kSK) {
        if (skt >= 0 && !(kb0 == 0 && kb1 == args.k_blocks)) {
          const int piece = (int)rank * P::kEpiWarps + ew;
          if (kb1 < args.k_blocks) {
            const long long slot = (long long)pair * 2 * P::kEpiWarps + piece;
            ks_send_piece<false>(tbase, args.sk_slots + slot * kPieceFloats,
                                 args.sk_flags + slot, args.sk_epoch,
                                 acc_empty_leader + buf * 8u);
            if constexpr (kProfile) {
              if (lane == 0) prof.stop();
            }
            continue;
          }
          const int c0 = sk_owner((long long)skt * args.k_blocks, args.sk_items,
                                  sk_pairs(args, npairs));
          bool ready = true;
#pragma unroll 1
          for (int c = c0; ready && c < pair; ++c)
            ready = wait_peer_flag<false>(args.sk_flags + (long long)c * 2 * P::kEpiWarps + piece,
                                          args.sk_epoch, wctx, args.timeout_ns, kErrWaitPartial);
          if (!ready) break;
          sk_heads = pair - c0;
          sk_piece = args.sk_slots + ((long long)c0 * 2 * P::kEpiWarps + piece) * kPieceFloats +
                     4 * lane;
        }
      }
      // Row `lane` of a 32x64 box is 8 chunks of 16 B; chunk j is stored at
      // position j ^ (row % 8) -- the TMA 128 B swizzle pattern.
      const uint32_t row_off = lane * 128u;
      if constexpr (kOut == kOutF32 || kOut == kOutF32Add) {
        // fp32: 8 chunks of 32 columns (128 B rows); chunk j of 16 B at
        // position j ^ (row % 8), as above.
#pragma unroll 1
        for (int c = 0; c < kSubN / 32; ++c) {
          uint32_t v[32];
          tmem_ld_32x32b_x32(tbase + c * 32, v);
          tmem_wait_ld();
          if (c == kSubN / 32 - 1) {
            tc_fence_before_sync();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(acc_empty_leader + buf * 8u);
          }
          const uint32_t sb = my_store + (nstore & 1u) * kStoreBufBytes;
          if (lane == 0) bulk_wait_group_read<1>();
          __syncwarp();
#pragma unroll
          for (int j = 0; j < 8; ++j)
            st_shared_v4(sb + row_off + ((uint32_t)(j ^ (lane & 7)) << 4), v[4 * j],
                         v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            if constexpr (kOut == kOutF32Add)
              tma_reduce_add_2d(&tmap_c, sb, col0 + c * 32, row0);
            else
              tma_store_2d(&tmap_c, sb, col0 + c * 32, row0);
            bulk_commit_group();
          }
          ++nstore;
        }
      } else if constexpr (kNSub == 1) {
        int out_row = row0;             // first row of this warp's 32 in C
        const float* recv = nullptr;    // K-split: own tile's received pieces
        long long recv_stride = 0;
        if constexpr (kOut == kOutKsplit) {
          const KsArgs& ks = args.ks;
          int owner;
          const long long piece = ks_piece(ks, tm, tn, args.tiles_n, (int)rank, quarter, &owner);
          if (owner != ks.rank) {
            // Another owner's tile: send this warp's piece into its receive
            // slot, then raise the piece's flag there.
            ks_send_piece(tbase, ks.recv[owner] + ks_slot_offset(ks, ks.rank, piece),
                          ks.flags[owner] + (long long)ks.rank * ks.pieces + piece, ks.epoch,
                          acc_empty_leader + buf * 8u);
            if constexpr (kProfile) {
              if (lane == 0) prof.stop();
            }
            continue;
          }
          // Own tile: every peer's piece must have arrived.
          bool arrived = true;
#pragma unroll 1
          for (int q = 0; arrived && q < ks.nranks; ++q)
            if (q != ks.rank)
              arrived = wait_peer_flag(ks.flags[ks.rank] + (long long)q * ks.pieces + piece,
                                       ks.epoch, wctx, ks.peer_timeout_ns);
          if (!arrived) break;
          recv = ks.recv[ks.rank] + ks_slot_offset(ks, 0, piece) + 4 * lane;
          recv_stride = (long long)ks.pieces * kPieceFloats;
          out_row = row0 - ks.rank * ks.tiles_m_own * kPairM;
        }
#pragma unroll 1
        for (int c = 0; c < kSubW / kStoreCols; ++c) {
          uint32_t v0[32], v1[32];
          tmem_ld_32x32b_x32(tbase + c * kStoreCols, v0);
          tmem_ld_32x32b_x32(tbase + c * kStoreCols + 32, v1);
          tmem_wait_ld();
          if constexpr (kOut == kOutBf16Epi) {
            epi_apply(v0, args.epi, args.M, args.N, row0 + lane, col0 + c * kStoreCols);
            epi_apply(v1, args.epi, args.M, args.N, row0 + lane, col0 + c * kStoreCols + 32);
          }
          if constexpr (kOut == kOutKsplit) {
            ks_accumulate(v0, recv, recv_stride, 2 * c, args.ks.rank, args.ks.nranks);
            ks_accumulate(v1, recv, recv_stride, 2 * c + 1, args.ks.rank, args.ks.nranks);
          }
          if constexpr (kSK) {
            if (sk_heads > 0) {
              sk_accumulate(v0, sk_piece, kSkStride, sk_heads, 2 * c);
              sk_accumulate(v1, sk_piece, kSkStride, sk_heads, 2 * c + 1);
            }
          }
          if (c == kSubW / kStoreCols - 1) {
            // All of this warp's part of the buffer is in registers: hand
            // TMEM back to the MMA.
            tc_fence_before_sync();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(acc_empty_leader + buf * 8u);
          }
          const uint32_t sb = my_store + (nstore & 1u) * kStoreBufBytes;
          if (lane == 0) bulk_wait_group_read<1>();  // the store that last used sb has read it
          __syncwarp();
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const uint32_t* v = j < 4 ? v0 + 8 * j : v1 + 8 * (j - 4);
            st_shared_v4(sb + row_off + ((uint32_t)(j ^ (lane & 7)) << 4),
                         pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]),
                         pack_bf16x2(v[4], v[5]), pack_bf16x2(v[6], v[7]));
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_2d(&tmap_c, sb, col0 + c * kStoreCols, out_row);
            bulk_commit_group();
          }
          ++nstore;
        }
      } else {
        int out_row = row0;
        const float* recv = nullptr;
        long long recv_stride = 0;
        if constexpr (kOut == kOutKsplit) {
          // As for 256-wide tiles, per 256-column sub-tile.
          const KsArgs& ks = args.ks;
          int owner;
          const long long piece =
              ks_piece(ks, tm, tn * kNSub + sub, args.tiles_n * kNSub, (int)rank, quarter, &owner);
          if (owner != ks.rank) {
            ks_send_piece(tbase, ks.recv[owner] + ks_slot_offset(ks, ks.rank, piece),
                          ks.flags[owner] + (long long)ks.rank * ks.pieces + piece, ks.epoch,
                          acc_empty_leader + buf * 8u);
            if constexpr (kProfile) {
              if (lane == 0) prof.stop();
            }
            continue;
          }
          bool arrived = true;
#pragma unroll 1
          for (int q = 0; arrived && q < ks.nranks; ++q)
            if (q != ks.rank)
              arrived = wait_peer_flag(ks.flags[ks.rank] + (long long)q * ks.pieces + piece,
                                       ks.epoch, wctx, ks.peer_timeout_ns);
          if (!arrived) break;
          recv = ks.recv[ks.rank] + ks_slot_offset(ks, 0, piece) + 4 * lane;
          recv_stride = (long long)ks.pieces * kPieceFloats;
          out_row = row0 - ks.rank * ks.tiles_m_own * kPairM;
        }
        // Drain this warp's 32 x 256 slice into registers as packed bf16
        // (128 registers per thread), release the accumulator, then store.
        // The MMA of the next tile waits for this drain (single accumulator),
        // so the loads go out kDrainBatch at a time with one wait each: the
        // drain takes kSubN / 32 / kDrainBatch load latencies, not kSubN / 32.
        // (One at a time where the K-split sums or the profiler need the
        // registers: batching there spills.)
        constexpr int kDrainBatch = (kOut == kOutBf16 && !kProfile) ? B200_DRAIN_BATCH : 1;
        static_assert((kSubN / 32) % kDrainBatch == 0, "drain batch must divide the chunks");
        uint32_t packed[kSubN / 2];
#pragma unroll
        for (int c = 0; c < kSubN / 32; c += kDrainBatch) {
          uint32_t v[kDrainBatch][32];
#pragma unroll
          for (int b = 0; b < kDrainBatch; ++b) tmem_ld_32x32b_x32(tbase + (c + b) * 32, v[b]);
          tmem_wait_ld();
#pragma unroll
          for (int b = 0; b < kDrainBatch; ++b) {
            if constexpr (kOut == kOutKsplit)
              ks_accumulate(v[b], recv, recv_stride, c + b, args.ks.rank, args.ks.nranks);
#pragma unroll
            for (int i = 0; i < 16; ++i)
              packed[(c + b) * 16 + i] = pack_bf16x2(v[b][2 * i], v[b][2 * i + 1]);
          }
        }
        tc_fence_before_sync();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(acc_empty_leader + buf * 8u);
#pragma unroll
        for (int c = 0; c < kSubN / kStoreCols; ++c) {
          if (lane == 0) bulk_wait_group_read<0>();  // the single buffer is free again
          __syncwarp();
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const uint32_t* p = packed + c * 32 + 4 * j;
            st_shared_v4(my_store + row_off + ((uint32_t)(j ^ (lane & 7)) << 4), p[0], p[1],
                         p[2], p[3]);
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_2d(&tmap_c, my_store, col0 + c * kStoreCols, out_row);
            bulk_commit_group();
          }
        }
      }
      if constexpr (kProfile) {
        if (lane == 0) prof.stop();
      }
    }
    // Only the staging buffers' reads must finish before the CTA's shared
    // memory goes away; the stores' global writes complete with the grid.
    if (lane == 0) bulk_wait_group_read<0>();
    if constexpr (kProfile) {
      if (lane == 0) prof.flush();
    }
    __syncwarp();
  }

  // ------------------------------------------------------------- teardown
  tc_fence_before_sync();
  cluster_sync_all();
  if (warp == 1) {
    tc_fence_after_sync();
    tmem_dealloc_pair(tmem_base, kTmemCols);
  }
  cluster_sync_all();
}

// Self-test of the bounded wait: one CTA pair waits on a barrier that nothing
// ever arrives on.  The wait must give up after timeout_ns, record
// kErrWaitProbe in *status and return; nothing faults or hangs.
__global__ void __cluster_dims__(2, 1, 1) wait_probe_kernel(int* status,
                                                            unsigned long long timeout_ns) {
  __shared__ alignas(8) uint64_t bar;
  __shared__ uint32_t abort_word;
  if (threadIdx.x == 0) {
    mbar_init(smem_u32(&bar), 1);
    abort_word = 0;
    fence_mbar_init_cluster();
  }
  cluster_sync_all();
  if (threadIdx.x == 0 && cluster_ctarank() == 0) {
    WaitCtx w;
    w.status = status;
    w.timeout_ns = timeout_ns;
    w.abort_local = smem_u32(&abort_word);
    w.abort_peer = cluster_map(smem_u32(&abort_word), 1);
    wait_bounded(smem_u32(&bar), 0, w, kErrWaitProbe);
  }
  cluster_sync_all();
}

// fp32 workspace (row stride ldw) -> bf16 C (row stride ldc), round to
// nearest even.  Eight columns per thread; vector loads and stores when the
// row has eight columns left and both rows are 16-byte aligned there.
__global__ void __launch_bounds__(256) cast_f32_to_bf16_kernel(const float* __restrict__ W,
                                                               int ldw, __nv_bfloat16* C,
                                                               int ldc, int M, int N,
                                                               EpiArgs epi, bool fused) {
  const int groups = (N + 7) / 8;
  const long long total = (long long)M * groups;
  for (long long g = blockIdx.x * (long long)blockDim.x + threadIdx.x; g < total;
       g += (long long)gridDim.x * blockDim.x) {
    const int row = (int)(g / groups);
    const int col = (int)(g - (long long)row * groups) * 8;
    const float* w = W + (long long)row * ldw + col;
    __nv_bfloat16* c = C + (long long)row * ldc + col;
    const int n_here = N - col < 8 ? N - col : 8;
    float f[8];
    if (n_here == 8) {
      const float4 a = *reinterpret_cast<const float4*>(w);
      const float4 b = *reinterpret_cast<const float4*>(w + 4);
      f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w;
      f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
    } else {
      for (int i = 0; i < 8; ++i) f[i] = i < n_here ? w[i] : 0.f;
    }
    if (fused) {
      // the same arithmetic as epi_apply: alpha acc + bias + beta resid
      for (int i = 0; i < n_here; ++i) {
        f[i] *= epi.alpha;
        if (epi.bias) f[i] += __bfloat162float(epi.bias[col + i]);
        if (epi.resid) f[i] += epi.beta * __bfloat162float(epi.resid[(long long)row * epi.ldr + col + i]);
      }
    }
    if (n_here == 8) {
      uint4 o;
      o.x = pack_bf16x2(__float_as_uint(f[0]), __float_as_uint(f[1]));
      o.y = pack_bf16x2(__float_as_uint(f[2]), __float_as_uint(f[3]));
      o.z = pack_bf16x2(__float_as_uint(f[4]), __float_as_uint(f[5]));
      o.w = pack_bf16x2(__float_as_uint(f[6]), __float_as_uint(f[7]));
      *reinterpret_cast<uint4*>(c) = o;
    } else {
      for (int i = 0; i < n_here; ++i) c[i] = __float2bfloat16_rn(f[i]);
    }
  }
}

}  // namespace b200
