// Fused K-split exchange over NVLink: the reduce-scatter of fp32 partials and
// the bf16 rounding happen inside the GEMM's epilogue, with plain stores and
// loads through CUDA IPC mappings of the peers' memory (no collective
// library, no bulk or tensor copies from peer memory).
//
// P ranks each hold the K-slice A[:, K_r], B[:, K_r] of one M x N x K GEMM.
// Rank r owns C rows [r M/P, (r+1) M/P) (whole 256-row pair tiles).  Every
// rank runs the persistent pair kernel over all M x N tiles of its partial,
// in P phases: phase f covers the tiles of owner (r + 1 + f) mod P, so a rank
// computes the other owners' tiles first and its own last.
//   * A tile of another owner o: each epilogue warp sends its 32 x 256 fp32
//     piece of the accumulator straight into o's receive slot for this
//     source (plain 16-byte stores into o's memory), then raises the piece's
//     flag in o's memory to the call's epoch (release at system scope).
//   * An own tile: each epilogue warp waits until every peer's flag for its
//     piece reaches the epoch (acquire at system scope, bounded), adds the
//     peers' pieces to the accumulator in rank order (P_0 + P_1 + ...), rounds
//     once to bf16 and stores its rows of this rank's C.
// Because every peer computes an owner's tiles one or more phases before the
// owner reaches them, the waits normally find the flags already raised, and
// the NVLink traffic overlaps the tensor-core work of the following phases.
//
// Piece layout (the exchange format, identical on both sides): a piece is the
// 32 rows x 256 columns one epilogue warp holds, 32 KiB of fp32.  The float4
// with columns 4f..4f+3 of lane l (row l of the warp's 32) sits at float
// offset 4 (32 f + l), so each warp-wide 16-byte access covers 512
// contiguous bytes.  Piece index p = ((t * 2 + cta) * 4 + quarter) for the
// owner-local tile t = (tm - o T) * tiles_n + tn (T = 256-row tiles per
// owner).
//
// Receive area of each rank (one IPC-exported allocation):
//   flags  uint32 [P sources][pieces]          epoch of the last piece received
//   slots  fp32   [2 parities][P sources][pieces][8192]
// A call with epoch e uses parity e & 1.  Reuse is safe without further
// handshakes: a source starts call e + 2 only after its call e + 1 finished,
// which needed the owner's call e + 1 pieces, which the owner sends only
// after its call e kernel -- the last reader of that parity -- completed.
// Flags only ever grow, so a flag left by an earlier call (or by a call with
// another shape) never satisfies a later epoch.
#pragma once
#include <stdint.h>

namespace b200 {

constexpr int kMaxRanks = 8;
constexpr int kPieceFloats = 32 * 256;

struct KsArgs {
  int rank, nranks;
  int tiles_m_own;            // 256-row pair tiles per owner (M / P / 256)
  int pieces;                 // pieces per owner in this call's layout
  unsigned int epoch;         // this call's epoch (>= 1)
  int parity;                 // epoch & 1
  unsigned long long peer_timeout_ns;
  float* recv[kMaxRanks];           // every rank's slots as mapped here
  unsigned int* flags[kMaxRanks];   // every rank's flags as mapped here
};

// Order this thread's earlier global stores (peer memory included) before
// its later ones at system scope.
__device__ __forceinline__ void fence_acq_rel_sys() {
  asm volatile("fence.acq_rel.sys;" ::: "memory");
}

__device__ __forceinline__ unsigned int ld_acquire_sys_u32(const unsigned int* p) {
  unsigned int v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_sys_u32(unsigned int* p, unsigned int v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ unsigned int ld_acquire_gpu_u32(const unsigned int* p) {
  unsigned int v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_gpu_u32(unsigned int* p, unsigned int v) {
  asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ void st_global_v4(float* p, uint32_t a, uint32_t b, uint32_t c,
                                             uint32_t d) {
  asm volatile("st.global.v4.b32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(a), "r"(b), "r"(c),
               "r"(d)
               : "memory");
}

__device__ __forceinline__ float4 ld_global_cg_v4(const float* p) {
  float4 v;
  asm volatile("ld.global.cg.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "l"(p)
               : "memory");
  return v;
}

// Owner-side location of piece p from `src` in a rank's receive area.
__device__ __forceinline__ long long ks_slot_offset(const KsArgs& ks, int src, long long p) {
  return (((long long)ks.parity * ks.nranks + src) * ks.pieces + p) * kPieceFloats;
}

}  // namespace b200
