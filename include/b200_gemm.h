/* C ABI of the sm_100a BF16 GEMM (libb200gemm.so).
 *
 * The reference exposes its GEMM as
 *     void matmul_vN(const nv_bfloat16 *A, const nv_bfloat16 *B,
 *                    nv_bfloat16 *C, int M, int N, int K);
 * (src/matmul.cpp:4-23, bodies e.g. src/kernels/kernel_v8.cu:830-833) and
 *     void profile_matmul_vN(..., int64_t *profiler_ptr, int num_entries);
 * (src/matmul.cpp:16-23, src/kernels/kernel_v8.cu:835-839).  The entry points
 * below replace those: same operand meaning (C = A * B^T, A is M x K
 * row-major, B is N x K row-major -- the reference's "(K,N) view of an N x K
 * buffer" -- and C is M x N row-major, bf16 in/out, fp32 accumulation), plus
 * explicit leading dimensions, an explicit CUDA stream (0 = legacy default
 * stream, where the reference launches) and a status code instead of silent
 * garbage on unsupported input.
 *
 * All pointers are device pointers.  Calls are asynchronous on `stream`.
 * Plain C types only; no torch types cross this boundary.
 */
#ifndef B200_GEMM_H_
#define B200_GEMM_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes returned by every entry point. */
#define B200_OK 0
#define B200_ERR_INVALID_ARGUMENT 1 /* null pointer, negative size, ld < width */
#define B200_ERR_ALIGNMENT 2        /* pointer or leading dimension not 16 B aligned */
#define B200_ERR_UNSUPPORTED_DEVICE 3 /* current device is not sm_100 */
#define B200_ERR_TENSOR_MAP 4       /* cuTensorMapEncodeTiled rejected the operand */
#define B200_ERR_LAUNCH 5           /* CUDA error at or before the launch */
#define B200_ERR_DEVICE_TIMEOUT 6   /* reserved: timeouts are read with b200_gemm_device_status */
#define B200_ERR_TOO_LARGE 7        /* a size exceeds what the entry point supports */

/* C = A * B^T, bf16 in and out, fp32 accumulation.
 * A: M x K, row stride lda elements.  B: N x K, row stride ldb.  C: M x N,
 * row stride ldc.  Requirements: lda >= K, ldb >= K, ldc >= N; lda, ldb, ldc
 * multiples of 8 and A, B, C 16-byte aligned (TMA); M, N, K >= 0.  M == 0 or
 * N == 0 is a no-op; K == 0 writes zeros.  Any other M, N, K is supported
 * (ragged edges are handled by the TMA bounds).
 * Replaces matmul_v1_2d ... matmul_v8 (src/matmul.cpp:4-13). */
int b200_gemm_bf16(const void* A, const void* B, void* C, int M, int N, int K, int lda, int ldb,
                   int ldc, void* stream);

/* fp32 C = A * B^T without rounding (the per-rank partial of a K-split GEMM:
 * partials are summed, then rounded once).  C row stride ldc is in floats
 * (a multiple of 4); other requirements as b200_gemm_bf16.  No reference
 * counterpart: the reference writes bf16 only. */
int b200_gemm_bf16_f32out(const void* A, const void* B, float* C, int M, int N, int K, int lda,
                          int ldb, int ldc, void* stream);

/* C = round(alpha * (A * B^T) + bias[n] + beta * R[m][n]) in one pass: the
 * fused epilogue of a transformer projection (scale, bias, residual add),
 * rounded to bf16 once.  bias: N bf16 values or NULL; residual R: M x N bf16
 * with row stride ldr (a multiple of 8) or NULL, and may be C itself; both
 * 16-byte aligned.  Other requirements as b200_gemm_bf16.  No reference
 * counterpart: the reference's epilogue only converts. */
int b200_gemm_bf16_epilogue(const void* A, const void* B, void* C, int M, int N, int K, int lda,
                            int ldb, int ldc, float alpha, const void* bias, float beta,
                            const void* residual, int ldr, void* stream);

/* The same GEMM on operands in HOST memory (A, B and C host pointers; page-
 * locked memory lets the transfers run asynchronously and overlap).  A and B
 * are uploaded in blocks of block_rows rows (0 = chosen: a quarter of the
 * larger of M and N, rounded up to 256), alternately; the GEMM of each block
 * of C starts as soon as its two blocks are up and the block comes back as
 * soon as it is done, on three internal streams, so uploads, GEMMs and
 * downloads overlap and the link moves data in both directions at once.
 * Device buffers (A, B and four C blocks) come from the library's per-device
 * pool.  Ordered after the work
 * already on `stream`, and `stream` waits for the result: the host buffers
 * must stay valid until then.  Strides as for b200_gemm_bf16 (no alignment
 * rule on the host side).  No reference counterpart (the reference takes
 * device tensors; its harness copies them serially). */
int b200_gemm_bf16_host(const void* A, const void* B, void* C, int M, int N, int K, int lda,
                        int ldb, int ldc, int block_rows, void* stream);

/* bf16 C = round-to-nearest-even(W) for an fp32 M x N matrix W (row stride
 * ldw floats, a multiple of 4; C row stride ldc, a multiple of 8).  The last
 * step of a K-split GEMM after the partials are summed.  No reference
 * counterpart. */
int b200_cast_f32_bf16(const float* W, int ldw, void* C, int ldc, int M, int N, void* stream);

/* Split-K for grids too small to occupy every SM (skinny M or N): 0 = chosen
 * per shape (default, B200_GEMM_SPLITS overrides), 1 = never, n = n slices.
 * Split-K calls accumulate into an fp32 workspace taken from a per-device
 * stream-ordered pool on the call's stream, then round once to bf16.
 * b200_gemm_get_splits reports the slice count a call would use. */
int b200_gemm_set_splits(int splits);
int b200_gemm_get_splits(int M, int N, int K, int* splits);

/* Skinny-M path (M <= 256, N >= 1024, K >= 512: C^T = B A^T so the large
 * operand B feeds the MMA's 128 rows): 0 = off (pair kernels only), 1 =
 * chosen per shape (default; B200_GEMM_SKINNY overrides), 2 = the
 * single-launch cluster kernel for every M, 3 = the stream-K kernel for
 * every M, 4 = the stream-K kernel on 2-CTA pairs (each CTA loads 128 rows
 * of B and half of A's rows; tcgen05.mma.cta_group::2 reads both) for every
 * M, 5 = the cluster kernel on 2-CTA pairs (K split over the pairs of a
 * cluster of 2, 4 or 8 CTAs, partials added in distributed shared memory)
 * for every M.  Calls with a fused epilogue take the workspace kernel
 * whatever the mode.  No reference counterpart. */
int b200_gemm_set_skinny_mode(int mode);

/* 128-row blocks of B per tile of the skinny stream-K kernel: 1, 2 (a
 * tile's two blocks share each slab of A, halving A's share of every SM's
 * L2 inflow; M <= 128 only; measured slower: twice the in-kernel fix-up) or
 * 0 = chosen, one (default; B200_GEMM_SKINNY_TILES overrides).  No
 * reference counterpart. */
int b200_gemm_set_skinny_tiles(int tiles);

/* Stream-K tail of the 256 x 256 pair-tile kernels: when the tiles are more than
 * one wave of the persistent grid but not a whole number of waves, the whole
 * waves run as usual and the remaining tiles' (tile, K block) items are split
 * evenly over all pairs; a tile cut between pairs is summed in the kernel by
 * the pair holding its last K blocks (fp32 pieces through a pool workspace,
 * one rounding).  0 = off, 1 = when the last wave would idle at least 3 % of
 * the pair-slots and K >= 4096 (default; B200_GEMM_STREAMK overrides), 2 =
 * whenever the last wave is partial, at any K.  The first stream-K call (pair tail or skinny
 * stream-K kernel) on each (device, stream) allocates that stream's flag
 * array with cudaMalloc, which may synchronise the device; it is cleared on
 * the stream itself.  No reference counterpart (the reference deals whole
 * tiles with cluster launch control). */
int b200_gemm_set_stream_k(int mode);

/* Dealing of whole tiles to the persistent pairs: 0 = static (default;
 * B200_GEMM_DYNAMIC overrides): pair p takes tiles p, p + P, ...; 1 =
 * dynamic: after a static first wave, each pair takes its next tile from a
 * device counter the moment it needs one, so the tiles in flight stay a
 * compact window of the raster and no pair idles while another has tiles
 * queued (measured no faster on the configuration shapes, slower on some:
 * the static deal stays the default).  The counters are two words per (device,
 * stream), made on the stream's first call (cudaMalloc) and left at zero by
 * every launch.  No reference counterpart (the reference steals work with
 * cluster launch control, src/kernels/kernel_v8.cu:608-653). */
int b200_gemm_set_dynamic(int mode);

/* Same GEMM with the intra-kernel profiler on (never split).  `profiler` is a device int64
 * buffer of rows x (1 + 4 * num_entries) entries, rows from
 * b200_gemm_profile_rows; row r = block * warps_per_cta + warp (warps per
 * CTA = threads from b200_gemm_launch_shape / 32) holds
 * [count, (smid, tag, start_ns, duration_ns) x count].  Writes past a row's
 * capacity are dropped.
 * Replaces profile_matmul_v5 ... profile_matmul_v8 (src/matmul.cpp:16-23). */
int b200_gemm_bf16_profile(const void* A, const void* B, void* C, int M, int N, int K, int lda,
                           int ldb, int ldc, int64_t* profiler, int num_entries, void* stream);

/* Rows the profiler buffer needs for an M x N x K launch on the current
 * device (grid size x warps per CTA).  No reference counterpart: the
 * reference sizes this buffer by hand and under-sizes it for v8
 * (src/bench_core.py:459-464 vs src/kernels/kernel_v8.cu:416). */
int b200_gemm_profile_rows(int M, int N, int K, int* rows);

/* Reads (and if `clear`, resets) the device error word of the current device
 * that the kernels write when a pipeline wait runs out.  Synchronises the
 * device.  *status_out = 0 when no wait has run out.  No reference
 * counterpart (the reference's waits never give up, kernel_v8.cu:60-76). */
int b200_gemm_device_status(int clear, int* status_out);

/* Process-wide tuning.
 *   tile_n        pair-tile width: 256 (two TMEM accumulators, epilogue
 *                 overlapped), 512 (one A slab feeds two MMAs: 25% fewer
 *                 operand bytes per FLOP), 128 or 64 (more, shorter tiles
 *                 for grids that leave SMs idle) or -1 to choose per shape;
 *                 0 keeps
 *   stage_slabs   K slabs of 64 per stage for 256-wide tiles (1: 6 stages of
 *                 K=64, 2: 3 stages of K=128); 0 keeps
 *   raster_group  band width, in tiles, of the persistent raster (positive:
 *                 bands of tile-rows, negative: bands of tile-columns); 0 keeps
 * Defaults come from B200_GEMM_TILE_N / B200_GEMM_SLABS / B200_GEMM_GROUP.
 * Plays the role of the reference's GEMM_L2_A/GEMM_L2_B environment knobs
 * (src/kernels/kernel_v8.cu:11-31). */
int b200_gemm_set_tuning(int tile_n, int stage_slabs, int raster_group);
int b200_gemm_get_tuning(int* tile_n, int* stage_slabs, int* raster_group);

/* Upper bound, in nanoseconds, on any single pipeline wait inside the GEMM
 * kernels of this process (default 2 s).  No reference counterpart. */
int b200_gemm_set_wait_timeout_ns(unsigned long long timeout_ns);

/* Launches a self-test kernel whose only wait is on a barrier nothing
 * releases, bounded by timeout_ns; the kernel records the timeout in the
 * device error word and returns.  Used by the failure-detection tests.  No
 * reference counterpart. */
int b200_gemm_wait_probe(unsigned long long timeout_ns, void* stream);

/* Short text for a status code. */
const char* b200_gemm_status_string(int status);

/* The same GEMM as b200_gemm_bf16, for callers that cannot let a library
 * allocate device memory: processes that reserve the GPU's memory up front
 * through their own allocator or arena (a later cudaMalloc would fail or
 * break their accounting) and latency-critical loops in which
 * cudaMalloc/cudaFree would synchronize the device.  b200_gemm_bf16 allocates
 * on a device's first call (an error word and a split-K memory pool) and its
 * split-K, skinny and stream-K calls draw workspaces from that pool; this
 * entry point allocates nothing.  Its scratch is one fixed 16 MiB device
 * array in the library, held by every GPU that loads the library until exit:
 * a 4-byte error word, 64 KiB - 256 B of epoch flags and 16 MiB - 64 KiB of
 * workspace (split-K fp32 accumulators, skinny stream-K slots).  Skinny M
 * (<= 256) runs the same skinny kernels as b200_gemm_bf16, with their
 * workspace in the array, or, where it would not fit, the cluster kernel
 * (no workspace).  Slice counts chosen per shape always fit; only a forced
 * one (b200_gemm_set_splits) can need more than the workspace, and such a
 * call returns B200_ERR_TOO_LARGE.  Grids that b200_gemm_bf16 would give a
 * stream-K tail run whole tiles here (the tail's slots exceed the array).
 * Every call shares the array; the parts that must start at zero are
 * cleared on the call's stream, and the flags take a new epoch per call.
 * Calls whose executions overlap on the GPU (other streams, other threads)
 * race on it, so callers serialise them.  A pipeline wait that runs out is
 * recorded in the array's error word, which stays set until
 * b200_gemm_noalloc_status reads and clears it.  The first call on a device
 * (or of b200_gemm_noalloc_status) also sets that device up (kernel
 * attributes, occupancy, the array's device address); make it before any
 * stream capture.  No counterpart in the reference, which has no scratch. */
int b200_gemm_bf16_noalloc(const void* A, const void* B, void* C, int M, int N, int K, int lda,
                           int ldb, int ldc, void* stream);

/* Reads (and if `clear`, resets) the error word of b200_gemm_bf16_noalloc's
 * array on the current device: 0, or the code of the first pipeline wait
 * that ran out in its kernels since the last clear (codes as for
 * b200_gemm_device_status).  Synchronises the device; allocates nothing.
 * No reference counterpart. */
int b200_gemm_noalloc_status(int clear, int* status_out);

/* The wait self-test of b200_gemm_wait_probe, recording into the
 * allocation-free entry point's error word instead (read it with
 * b200_gemm_noalloc_status).  Allocates nothing.  No reference counterpart. */
int b200_gemm_noalloc_wait_probe(unsigned long long timeout_ns, void* stream);

/* ---- Fused K-split over NVLink -------------------------------------------
 * One GEMM C = A B^T (M x N x K) split along K over P ranks, one process per
 * GPU: rank r holds A[:, K_r] (M x K_r) and B[:, K_r] (N x K_r) and receives
 * the bf16 rows [r M/P, (r+1) M/P) of C.  It replaces the multi-GPU K-split
 * sequence "fp32 partial (b200_gemm_bf16_f32out) -> collective
 * reduce-scatter (sum) -> b200_cast_f32_bf16" with one kernel per rank: each
 * rank computes the other owners' tiles first and writes their fp32
 * accumulators straight into the owner's memory over NVLink (CUDA IPC
 * mappings, plain stores), then computes its own tiles and adds the peers'
 * contributions in its epilogue (sum in rank order, one rounding).  No
 * reference counterpart (the reference is single-GPU); it is the fused form
 * of the reduce-scatter + cast step of the K-split configuration.
 *
 * Set-up, once per group (a collective: every rank, same arguments but its
 * own rank):
 *   b200_ksplit_create(rank, P, max_m, max_n, &comm, handle)  on rank's GPU;
 *       allocates 2 * max_m * round_up(max_n, 256) * 4 bytes plus flags and
 *       writes B200_KSPLIT_HANDLE_BYTES of exchange data to `handle`;
 *   all-gather the P handles (any transport, rank order);
 *   b200_ksplit_connect(comm, handles)  maps every peer's area.
 *   Every rank must return from connect before any rank calls the GEMM.
 * Calls (a collective: every rank, same order, same M and N, K_r >= 1):
 *   b200_ksplit_gemm_bf16(comm, A, B, C, M, N, K_r, lda, ldb, ldc, stream)
 *       M a multiple of 256 P, M x N within the created capacity; C is this
 *       rank's M/P x N block.  Asynchronous on `stream`; waits for peers are
 *       on the device and bounded (5 x the pipeline wait bound, 10 s by default):
 *       a missing peer sets the device error word (b200_gemm_device_status)
 *       and the kernel returns.
 * Tear-down: synchronize every rank's streams, barrier, then
 *   b200_ksplit_destroy(comm). */
#define B200_KSPLIT_HANDLE_BYTES 128
typedef struct b200_ksplit_comm b200_ksplit_comm;
int b200_ksplit_create(int rank, int nranks, int max_m, int max_n, b200_ksplit_comm** comm,
                       void* handle);
int b200_ksplit_connect(b200_ksplit_comm* comm, const void* handles);
int b200_ksplit_gemm_bf16(b200_ksplit_comm* comm, const void* A, const void* B, void* C, int M,
                          int N, int K, int lda, int ldb, int ldc, void* stream);
/* Calls this communicator has queued so far (the epoch of the last one). */
int b200_ksplit_epoch(const b200_ksplit_comm* comm, unsigned int* epoch);
int b200_ksplit_destroy(b200_ksplit_comm* comm);

/* Host-side layout rules, exported so they can be checked without a GPU. */
void b200_gemm_tile_coord(int t, int tiles_m, int tiles_n, int group, int* tm, int* tn);
uint32_t b200_gemm_idesc(int mma_m, int mma_n);
/* Stream-K split of a tail of `items` (tile, K block) items over `pairs`
 * pairs, as the kernel computes it: pairs taking work (min(pairs, items)),
 * pair p's item range [*lo, *hi), the first pair whose range holds item x,
 * and the next segment (tile, K blocks [kb0, kb1)) of a range walked from
 * its end (*pos moves to the segment's first item).  No reference
 * counterpart (the reference deals whole tiles). */
int b200_gemm_sk_range_pairs(long long items, int pairs);
void b200_gemm_sk_range(int pair, long long items, int range_pairs, long long* lo, long long* hi);
int b200_gemm_sk_owner(long long x, long long items, int range_pairs);
void b200_gemm_sk_next_segment(long long lo, long long* pos, int k_blocks, int* t, int* kb0,
                               int* kb1);
uint64_t b200_gemm_smem_desc(uint32_t smem_addr);
/* Launch geometry the GEMM would use: pair tiles, grid CTAs (0 if no
 * device), dynamic shared memory bytes and threads per CTA. */
int b200_gemm_launch_shape(int M, int N, int K, int* tiles, int* grid, int* smem_bytes,
                           int* threads);

#ifdef __cplusplus
}
#endif

#endif /* B200_GEMM_H_ */
