/* CPU oracle for the BF16 GEMM  C = A * B^T  (fp32 accumulation, bf16 out).
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker: only tests/,
 * __graft_entry__.smoke() and bench.py's CPU-baseline leg load it.  The
 * product path (blackwell_gemm_b200) never calls it and has no CPU fallback.
 *
 * What it restates (the reference has no CPU implementation; its arithmetic
 * is the tcgen05 kernel):
 *   - operands: A is M x K bf16 row-major, B is N x K bf16 row-major (the
 *     "(K,N) view of an N x K buffer" the reference binding passes,
 *     src/matmul.cpp:25-39, src/bench_core.py:110-111);
 *   - products of bf16 values accumulated in fp32
 *     (tcgen05.mma kind::f16 with an f32 D, src/kernels/kernel_v8.cu:450-455,
 *     554-589);
 *   - fp32 -> bf16 round-to-nearest-even of the accumulator
 *     (__float22bfloat162_rn, src/kernels/kernel_v8.cu:716).
 * The summation order is fixed (8 interleaved partial sums, combined
 * pairwise) and independent of the thread count, so results are
 * reproducible; it differs from the tensor core's order, which is why
 * non-exact inputs are compared with a tolerance.
 */
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

static inline float bf16_bits_to_f32(uint16_t h) {
  uint32_t u = (uint32_t)h << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

/* IEEE-754 round-to-nearest, ties-to-even, from fp32 to bf16: add half an
 * ulp of the target (0x7FFF) plus the parity of the kept part, truncate.
 * NaNs stay NaN (quiet bit forced). */
uint16_t oracle_f32_to_bf16(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  if ((u & 0x7FFFFFFFu) > 0x7F800000u) return (uint16_t)((u >> 16) | 0x0040u);
  u += 0x7FFFu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}

void oracle_round_bf16(const float* x, uint16_t* y, int64_t n) {
  for (int64_t i = 0; i < n; ++i) y[i] = oracle_f32_to_bf16(x[i]);
}

void oracle_bf16_to_f32(const uint16_t* x, float* y, int64_t n) {
  for (int64_t i = 0; i < n; ++i) y[i] = bf16_bits_to_f32(x[i]);
}

typedef struct {
  const float* Af;   /* M x K fp32 copy of A (row stride K) */
  const float* Bf;   /* N x K fp32 copy of B (row stride K) */
  float* C;
  int M, N, K, ldc;
  int r0, r1;        /* rows [r0, r1) of C */
} job_t;

enum { RB = 4, JB = 32, LANES = 8 };

static inline float lanes_sum(const float* acc) {
  /* pairwise: ((0+1)+(2+3)) + ((4+5)+(6+7)) */
  return ((acc[0] + acc[1]) + (acc[2] + acc[3])) + ((acc[4] + acc[5]) + (acc[6] + acc[7]));
}

/* Dot product of one A row with one B row in the oracle's fixed order:
 * lane l accumulates k = l, l+8, l+16, ... in order, tail elements go to
 * lanes 0.., then the 8 lanes are combined pairwise. */
static float dot_fixed(const float* a, const float* b, int K) {
  float acc[LANES] = {0};
  int k = 0;
  for (; k + LANES <= K; k += LANES)
    for (int l = 0; l < LANES; ++l) acc[l] += a[k + l] * b[k + l];
  for (int l = 0; k < K; ++k, ++l) acc[l] += a[k] * b[k];
  return lanes_sum(acc);
}

static void* run_job(void* arg) {
  const job_t* j = (const job_t*)arg;
  const int K = j->K;
  for (int n0 = 0; n0 < j->N; n0 += JB) {
    const int n1 = n0 + JB < j->N ? n0 + JB : j->N;
    int i = j->r0;
    /* RB rows at a time share each B row load; same per-element order as
     * dot_fixed, so the blocking never changes a result. */
    for (; i + RB <= j->r1; i += RB) {
      const float* a0 = j->Af + (int64_t)i * K;
      for (int n = n0; n < n1; ++n) {
        const float* b = j->Bf + (int64_t)n * K;
        float acc[RB][LANES];
        memset(acc, 0, sizeof(acc));
        int k = 0;
        for (; k + LANES <= K; k += LANES)
          for (int r = 0; r < RB; ++r)
            for (int l = 0; l < LANES; ++l) acc[r][l] += a0[(int64_t)r * K + k + l] * b[k + l];
        for (int r = 0; r < RB; ++r) {
          int kk = k;
          for (int l = 0; kk < K; ++kk, ++l) acc[r][l] += a0[(int64_t)r * K + kk] * b[kk];
          j->C[(int64_t)(i + r) * j->ldc + n] = lanes_sum(acc[r]);
        }
      }
    }
    for (; i < j->r1; ++i)
      for (int n = n0; n < n1; ++n)
        j->C[(int64_t)i * j->ldc + n] = dot_fixed(j->Af + (int64_t)i * K, j->Bf + (int64_t)n * K, K);
  }
  return NULL;
}

/* C (fp32, M x N, row stride ldc) = A * B^T.  A, B are bf16 bit patterns with
 * row strides lda, ldb.  nthreads <= 0 means 1.  Returns 0 on success. */
int oracle_gemm_f32(const uint16_t* A, const uint16_t* B, float* C, int M, int N, int K,
                    int lda, int ldb, int ldc, int nthreads) {
  if (M < 0 || N < 0 || K < 0 || lda < K || ldb < K || ldc < N) return 1;
  if (M == 0 || N == 0) return 0;
  float* Af = (float*)malloc(sizeof(float) * (size_t)M * (K > 0 ? K : 1));
  float* Bf = (float*)malloc(sizeof(float) * (size_t)N * (K > 0 ? K : 1));
  if (!Af || !Bf) {
    free(Af);
    free(Bf);
    return 2;
  }
  for (int i = 0; i < M; ++i) oracle_bf16_to_f32(A + (int64_t)i * lda, Af + (int64_t)i * K, K);
  for (int n = 0; n < N; ++n) oracle_bf16_to_f32(B + (int64_t)n * ldb, Bf + (int64_t)n * K, K);
  if (nthreads < 1) nthreads = 1;
  if (nthreads > M) nthreads = M;
  if (nthreads > 256) nthreads = 256;
  pthread_t th[256];
  int started[256];
  job_t jobs[256];
  const int per = (M + nthreads - 1) / nthreads;
  for (int t = 0; t < nthreads; ++t) {
    jobs[t].Af = Af;
    jobs[t].Bf = Bf;
    jobs[t].C = C;
    jobs[t].M = M;
    jobs[t].N = N;
    jobs[t].K = K;
    jobs[t].ldc = ldc;
    jobs[t].r0 = t * per < M ? t * per : M;
    jobs[t].r1 = (t + 1) * per < M ? (t + 1) * per : M;
  }
  for (int t = 1; t < nthreads; ++t)
    started[t] = pthread_create(&th[t], NULL, run_job, &jobs[t]) == 0;
  run_job(&jobs[0]);
  for (int t = 1; t < nthreads; ++t) {
    if (started[t])
      pthread_join(th[t], NULL);
    else
      run_job(&jobs[t]); /* thread creation failed: do the rows here */
  }
  free(Af);
  free(Bf);
  return 0;
}

/* bf16 output: the fp32 oracle rounded to nearest even. */
int oracle_gemm_bf16(const uint16_t* A, const uint16_t* B, uint16_t* C, int M, int N, int K,
                     int lda, int ldb, int ldc, int nthreads) {
  if (M <= 0 || N <= 0) return (M < 0 || N < 0) ? 1 : 0;
  float* Cf = (float*)malloc(sizeof(float) * (size_t)M * N);
  if (!Cf) return 2;
  int st = oracle_gemm_f32(A, B, Cf, M, N, K, lda, ldb, N, nthreads);
  if (st == 0)
    for (int i = 0; i < M; ++i)
      for (int n = 0; n < N; ++n) C[(int64_t)i * ldc + n] = oracle_f32_to_bf16(Cf[(int64_t)i * N + n]);
  free(Cf);
  return st;
}
