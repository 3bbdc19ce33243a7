// Torch extension with the reference binding's API (src/matmul.cpp:25-124):
//   matmul_b200(A, B) -> C
//   profile_matmul_b200(A, B, profiler, num_entries) -> C
// A is an M x K bf16 CUDA tensor, B is the (K, N) view of an N x K row-major
// bf16 buffer (what the reference's harness passes: `randn(N, K).T`,
// src/bench_core.py:110-111), C is a new contiguous M x N bf16 tensor.
//
// Differences from the reference binding, all on the error side: dtype,
// device, rank and shape are checked and raise RuntimeError; a B whose
// memory is not N x K row-major (or any operand whose rows are not 16-byte
// aligned) is first copied into the layout the kernel reads, instead of
// producing garbage; the launch goes on the current torch stream and its
// status is checked.  The math is done by libb200gemm.so through its C ABI.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "b200_gemm.h"

namespace {

void check_status(int st, const char* what) {
  TORCH_CHECK(st == B200_OK, what, " failed: ", b200_gemm_status_string(st), " (status ", st, ")");
}

int64_t round_up8(int64_t x) { return (x + 7) / 8 * 8; }

bool row_major_ok(const at::Tensor& t) {
  // rows x cols with unit column stride, 16-byte aligned rows and base.
  const int64_t rows = t.size(0), cols = t.size(1);
  if (rows == 0 || cols == 0) return true;
  if (cols > 1 && t.stride(1) != 1) return false;
  const int64_t ld = rows > 1 ? t.stride(0) : round_up8(cols);
  if (ld < cols || ld % 8) return false;
  return (reinterpret_cast<uintptr_t>(t.data_ptr()) & 15u) == 0;
}

int64_t leading_dim(const at::Tensor& t) {
  return t.size(0) > 1 ? t.stride(0) : round_up8(t.size(1));
}

// Row-major copy with a 16-byte aligned row stride; returns a view of the
// logical rows x cols region.
at::Tensor to_row_major(const at::Tensor& t) {
  const int64_t rows = t.size(0), cols = t.size(1);
  auto buf = at::empty({rows, round_up8(cols)}, t.options());
  auto view = buf.narrow(1, 0, cols);
  view.copy_(t);
  return view;
}

struct Operands {
  at::Tensor a;   // M x K row-major view
  at::Tensor bt;  // N x K row-major view (= B^T)
  int64_t M, N, K;
};

Operands prepare(const at::Tensor& A, const at::Tensor& B, const char* who) {
  TORCH_CHECK(A.dim() == 2 && B.dim() == 2, who, ": A and B must be 2-D");
  TORCH_CHECK(A.is_cuda() && B.is_cuda(), who, ": A and B must be CUDA tensors");
  TORCH_CHECK(A.device() == B.device(), who, ": A and B must be on the same device");
  TORCH_CHECK(A.scalar_type() == at::kBFloat16 && B.scalar_type() == at::kBFloat16, who,
              ": A and B must be bfloat16");
  Operands o;
  o.M = A.size(0);
  o.K = A.size(1);
  o.N = B.size(1);
  TORCH_CHECK(B.size(0) == o.K, who, ": inner dimensions differ (A is ", o.M, "x", o.K,
              ", B is ", B.size(0), "x", o.N, ")");
  const int64_t lim = std::numeric_limits<int>::max();
  TORCH_CHECK(o.M <= lim && o.N <= lim && o.K <= lim, who, ": dimension exceeds 2^31-1");
  o.a = row_major_ok(A) ? A : to_row_major(A);
  at::Tensor bt = B.t();
  o.bt = row_major_ok(bt) ? bt : to_row_major(bt);
  return o;
}

at::Tensor run(const at::Tensor& A, const at::Tensor& B, const at::Tensor* profiler,
               int64_t num_entries, const char* who) {
  Operands o = prepare(A, B, who);
  const c10::cuda::CUDAGuard guard(A.device());
  const bool pad_c = (o.N % 8) != 0;
  auto C = at::empty({o.M, pad_c ? round_up8(o.N) : o.N}, A.options());
  void* stream = at::cuda::getCurrentCUDAStream().stream();
  const int lda = (int)(o.M && o.K ? leading_dim(o.a) : 8);
  const int ldb = (int)(o.N && o.K ? leading_dim(o.bt) : 8);
  const int ldc = (int)C.size(1);
  int st;
  if (profiler) {
    int rows = 0;
    check_status(b200_gemm_profile_rows((int)o.M, (int)o.N, (int)o.K, &rows), who);
    TORCH_CHECK(profiler->is_cuda() && profiler->scalar_type() == at::kLong &&
                    profiler->is_contiguous() && profiler->device() == A.device(),
                who, ": profiler must be a contiguous int64 CUDA tensor on A's device");
    TORCH_CHECK(num_entries >= 0 && num_entries <= (1 << 24), who, ": bad num_entries");
    TORCH_CHECK(profiler->numel() >= (int64_t)rows * (1 + 4 * num_entries), who,
                ": profiler needs ", rows, " rows of ", 1 + 4 * num_entries, " int64");
    st = b200_gemm_bf16_profile(o.a.data_ptr(), o.bt.data_ptr(), C.data_ptr(), (int)o.M,
                                (int)o.N, (int)o.K, lda, ldb, ldc,
                                reinterpret_cast<int64_t*>(profiler->data_ptr()),
                                (int)num_entries, stream);
  } else {
    st = b200_gemm_bf16(o.a.data_ptr(), o.bt.data_ptr(), C.data_ptr(), (int)o.M, (int)o.N,
                        (int)o.K, lda, ldb, ldc, stream);
  }
  check_status(st, who);
  return pad_c ? C.narrow(1, 0, o.N).contiguous() : C;
}

at::Tensor matmul_b200(const at::Tensor& A, const at::Tensor& B) {
  return run(A, B, nullptr, 0, "matmul_b200");
}

at::Tensor profile_matmul_b200(const at::Tensor& A, const at::Tensor& B,
                               const at::Tensor& profiler, int64_t num_entries) {
  return run(A, B, &profiler, num_entries, "profile_matmul_b200");
}

int64_t profile_rows(int64_t M, int64_t N, int64_t K) {
  int rows = 0;
  check_status(b200_gemm_profile_rows((int)M, (int)N, (int)K, &rows), "profile_rows");
  return rows;
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.def("matmul_b200", &matmul_b200, "C = A @ B for A (M,K) bf16 and B the (K,N) view of an N x K buffer");
  m.def("profile_matmul_b200", &profile_matmul_b200,
        "matmul_b200 with the intra-kernel profiler writing into `profiler`");
  m.def("profile_rows", &profile_rows, "profiler rows needed for an M x N x K call on this device");
}
