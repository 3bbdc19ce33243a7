// C-ABI shim over the reference's own GEMM launchers.
//
// TEST/BASELINE INFRASTRUCTURE ONLY.  oracle/build.py compiles this file
// together with the reference's unmodified kernel sources
// (src/kernels/kernel_v1.cu ... kernel_v8.cu, read in place) into
// oracle/_ref/libref_gemm.so.  Nothing of the reference is copied here: the
// declarations below restate the launcher signature that the reference's own
// binding declares (src/matmul.cpp:4-23), and ref_gemm() forwards to it the
// way that binding does (src/matmul.cpp:25-39), minus the torch tensors.
//
// The reference checks nothing, so ref_supports() restates each version's
// shape preconditions (tile divisibility: v1 128x256 / BK 128; v2-v3
// 256x256 / BK 128, v3 needs two k-blocks; v4-v8 256x256 / BK 64); callers
// must not launch a version on a shape it does not support.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstring>
#include <exception>

typedef void RefMatmulFn(const nv_bfloat16* A, const nv_bfloat16* B, nv_bfloat16* C, int M,
                         int N, int K);
RefMatmulFn matmul_v1_2d, matmul_v1_3d, matmul_v2, matmul_v3, matmul_v4, matmul_v5, matmul_v6,
    matmul_v7, matmul_v8;

namespace {
struct Entry {
  const char* name;
  RefMatmulFn* fn;
};
const Entry kEntries[] = {
    {"v1_2d", matmul_v1_2d}, {"v1_3d", matmul_v1_3d}, {"v2", matmul_v2},
    {"v3", matmul_v3},       {"v4", matmul_v4},       {"v5", matmul_v5},
    {"v6", matmul_v6},       {"v7", matmul_v7},       {"v8", matmul_v8},
};

RefMatmulFn* lookup(const char* v) {
  for (const Entry& e : kEntries)
    if (std::strcmp(e.name, v) == 0) return e.fn;
  return nullptr;
}
}  // namespace

extern "C" {

// 1 when `version` may run M x N x K, else 0.
int ref_supports(const char* version, int M, int N, int K) {
  if (!version || M <= 0 || N <= 0 || K <= 0) return 0;
  const bool v1 = std::strncmp(version, "v1", 2) == 0;
  const bool v23 = !std::strcmp(version, "v2") || !std::strcmp(version, "v3");
  if (!lookup(version)) return 0;
  if (v1) return (M % 128 == 0) && (N % 256 == 0) && (K % 128 == 0);
  if (M % 256 || N % 256 || K % 64) return 0;
  if (v23 && K % 128) return 0;
  if (!std::strcmp(version, "v3") && K < 256) return 0;
  return 1;
}

// Runs reference version `version` on device pointers (legacy default
// stream, as the reference launches).  0 = launched, 1 = unknown version or
// unsupported shape, 2 = the reference raised, 3 = CUDA launch error.
int ref_gemm(const char* version, const void* A, const void* B, void* C, int M, int N, int K) {
  RefMatmulFn* fn = version ? lookup(version) : nullptr;
  if (!fn || !ref_supports(version, M, N, K)) return 1;
  try {
    fn(static_cast<const nv_bfloat16*>(A), static_cast<const nv_bfloat16*>(B),
       static_cast<nv_bfloat16*>(C), M, N, K);
  } catch (const std::exception&) {
    return 2;
  } catch (...) {
    return 2;
  }
  return cudaGetLastError() == cudaSuccess ? 0 : 3;
}

}  // extern "C"
