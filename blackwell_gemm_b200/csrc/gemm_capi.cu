// C-ABI launcher for the sm_100a BF16 GEMM (declarations: include/b200_gemm.h).
//
// Per call: validate the operands, encode three TMA tensor maps (A, B: 2-D,
// box 64 x 128, 128 B swizzle, zero fill out of bounds; C: 2-D, box
// 64 x 32, 128 B swizzle), then launch the persistent kernel on the caller's
// stream.  The reference does the same three steps per call with 3-D maps and
// without validation (kernel_v8.cu:775-828).
//
// Per device, once: check the architecture, raise the kernel's shared-memory
// limit, ask the occupancy API how many 2-CTA clusters can be resident at
// once (the persistent grid size) and allocate the 4-byte device error word.
// The reference keeps a device-blind static cache instead (kernel_v8.cu:796-820).
#include <cuda.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cstdlib>
#include <mutex>

#include "b200_gemm.h"
#include "gemm_kernel.cuh"

using namespace b200;

namespace {

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_tiled() {
  static EncodeTiledFn fn = []() -> EncodeTiledFn {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) !=
            cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return nullptr;
    return reinterpret_cast<EncodeTiledFn>(p);
  }();
  return fn;
}

constexpr int kMaxDevices = 64;

struct DeviceState {
  bool ready = false;
  int init_status = B200_OK;
  int sms = 0;
  int max_pairs = 0;     // co-resident 2-CTA clusters of the GEMM kernel
  int* status = nullptr; // device error word
};

std::mutex g_mu;
DeviceState g_dev[kMaxDevices];
std::atomic<unsigned long long> g_timeout_ns{2000000000ull};

int env_int(const char* name, int fallback, int lo, int hi) {
  const char* v = std::getenv(name);
  if (!v || !*v) return fallback;
  const int x = std::atoi(v);
  return (x < lo || x > hi) ? fallback : x;
}

// Tuning knobs, process-wide: band height (tile-rows) of the grouped raster
// and K slabs (64 elements each) per pipeline stage.  Initialised from
// B200_GEMM_GROUP / B200_GEMM_SLABS, changeable through b200_gemm_set_tuning.
std::atomic<int> g_group{-1};
std::atomic<int> g_slabs{-1};

int raster_group() {
  int g = g_group.load();
  if (g < 0) {
    g = env_int("B200_GEMM_GROUP", 8, -(1 << 16), 1 << 16);
    if (g == 0) g = 8;
    g_group.store(g);
  }
  return g;
}

int stage_slabs() {
  int s = g_slabs.load();
  if (s < 0) {
    s = env_int("B200_GEMM_SLABS", 1, 1, 2);
    g_slabs.store(s);
  }
  return s;
}

template <typename K>
int max_active_pairs(K kernel, int sms, int smem_bytes, int* out) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * sms, 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = smem_bytes;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, kernel, &cfg) != cudaSuccess) return B200_ERR_LAUNCH;
  *out = n;
  return B200_OK;
}

template <bool kProfile, int kSlabs>
cudaError_t set_smem_limit() {
  return cudaFuncSetAttribute(gemm_bf16_pair_kernel<kProfile, kSlabs>,
                              cudaFuncAttributeMaxDynamicSharedMemorySize,
                              Pipe<kSlabs>::kSmemBytes);
}

int device_state(DeviceState** out) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    cudaGetLastError();
    return B200_ERR_UNSUPPORTED_DEVICE;
  }
  if (dev < 0 || dev >= kMaxDevices) return B200_ERR_UNSUPPORTED_DEVICE;
  std::lock_guard<std::mutex> lock(g_mu);
  DeviceState& d = g_dev[dev];
  if (!d.ready) {
    d.ready = true;
    cudaDeviceProp prop;
    if (cudaGetDeviceProperties(&prop, dev) != cudaSuccess) {
      d.init_status = B200_ERR_UNSUPPORTED_DEVICE;
    } else if (prop.major != 10 || prop.minor != 0) {
      d.init_status = B200_ERR_UNSUPPORTED_DEVICE;  // built for sm_100a only
    } else if (encode_tiled() == nullptr) {
      d.init_status = B200_ERR_TENSOR_MAP;
    } else {
      d.sms = prop.multiProcessorCount;
      int st = B200_OK;
      if (set_smem_limit<false, 1>() != cudaSuccess || set_smem_limit<true, 1>() != cudaSuccess ||
          set_smem_limit<false, 2>() != cudaSuccess || set_smem_limit<true, 2>() != cudaSuccess)
        st = B200_ERR_LAUNCH;
      // Every variant runs one CTA per SM, so one occupancy query sizes all.
      if (st == B200_OK)
        st = max_active_pairs(gemm_bf16_pair_kernel<false, 1>, d.sms, Pipe<1>::kSmemBytes,
                              &d.max_pairs);
      if (st == B200_OK && d.max_pairs < 1) st = B200_ERR_LAUNCH;
      if (st == B200_OK) {
        if (cudaMalloc(&d.status, sizeof(int)) != cudaSuccess ||
            cudaMemset(d.status, 0, sizeof(int)) != cudaSuccess)
          st = B200_ERR_LAUNCH;
      }
      d.init_status = st;
    }
    if (d.init_status != B200_OK) cudaGetLastError();
  }
  if (d.init_status != B200_OK) return d.init_status;
  *out = &d;
  return B200_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// L2 promotion of the operand loads; B200_GEMM_L2_PROMO in {0, 64, 128, 256}
// overrides (the reference exposes the same knob as GEMM_L2_A / GEMM_L2_B,
// kernel_v8.cu:11-31).
CUtensorMapL2promotion l2_promotion() {
  static const CUtensorMapL2promotion p = []() {
    switch (env_int("B200_GEMM_L2_PROMO", 256, 0, 256)) {
      case 0: return CU_TENSOR_MAP_L2_PROMOTION_NONE;
      case 64: return CU_TENSOR_MAP_L2_PROMOTION_L2_64B;
      case 128: return CU_TENSOR_MAP_L2_PROMOTION_L2_128B;
      default: return CU_TENSOR_MAP_L2_PROMOTION_L2_256B;
    }
  }();
  return p;
}

int encode_2d(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer,
              uint64_t row_stride_elems, uint32_t box_inner, uint32_t box_outer) {
  const cuuint64_t dims[2] = {inner, outer};
  const cuuint64_t strides[1] = {row_stride_elems * 2};
  const cuuint32_t box[2] = {box_inner, box_outer};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = encode_tiled()(
      map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
      CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
      l2_promotion(), CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? B200_OK : B200_ERR_TENSOR_MAP;
}

int validate(const void* A, const void* B, void* C, int M, int N, int K, int lda, int ldb,
             int ldc) {
  if (M < 0 || N < 0 || K < 0) return B200_ERR_INVALID_ARGUMENT;
  if (M == 0 || N == 0) return B200_OK;
  if (!C || (K > 0 && (!A || !B))) return B200_ERR_INVALID_ARGUMENT;
  if (ldc < N || (K > 0 && (lda < K || ldb < K))) return B200_ERR_INVALID_ARGUMENT;
  if (!aligned16(C) || (ldc & 7)) return B200_ERR_ALIGNMENT;
  if (K > 0 && (!aligned16(A) || !aligned16(B) || (lda & 7) || (ldb & 7)))
    return B200_ERR_ALIGNMENT;
  return B200_OK;
}

template <bool kProfile>
int run_gemm(const void* A, const void* B, void* C, int M, int N, int K, int lda, int ldb,
             int ldc, long long* prof, int prof_entries, cudaStream_t stream) {
  int st = validate(A, B, C, M, N, K, lda, ldb, ldc);
  if (st != B200_OK) return st;
  if (M == 0 || N == 0) return B200_OK;
  if (kProfile && (prof == nullptr || prof_entries < 0)) return B200_ERR_INVALID_ARGUMENT;
  DeviceState* d = nullptr;
  st = device_state(&d);
  if (st != B200_OK) return st;
  if (K == 0) {
    // Empty reduction: C = 0.
    return cudaMemset2DAsync(C, (size_t)ldc * 2, 0, (size_t)N * 2, M, stream) == cudaSuccess
               ? B200_OK
               : B200_ERR_LAUNCH;
  }
  CUtensorMap ta, tb, tc;
  if (encode_2d(&ta, A, K, M, lda, kSlabK, kCtaM) != B200_OK ||
      encode_2d(&tb, B, K, N, ldb, kSlabK, kCtaN) != B200_OK ||
      encode_2d(&tc, C, N, M, ldc, kStoreCols, 32) != B200_OK)
    return B200_ERR_TENSOR_MAP;

  const int slabs = stage_slabs();
  const int bk = slabs * kSlabK;
  GemmArgs args;
  args.M = M;
  args.N = N;
  args.K = K;
  args.tiles_m = (M + kPairM - 1) / kPairM;
  args.tiles_n = (N + kPairN - 1) / kPairN;
  args.k_blocks = (K + bk - 1) / bk;
  args.group = raster_group();
  args.status = d->status;
  args.timeout_ns = g_timeout_ns.load();
  args.prof = prof;
  args.prof_entries = prof_entries;
  const long long tiles = (long long)args.tiles_m * args.tiles_n;
  const int pairs = (int)(tiles < d->max_pairs ? tiles : d->max_pairs);
  if (slabs == 2)
    gemm_bf16_pair_kernel<kProfile, 2><<<2 * pairs, kThreads, Pipe<2>::kSmemBytes, stream>>>(
        ta, tb, tc, args);
  else
    gemm_bf16_pair_kernel<kProfile, 1><<<2 * pairs, kThreads, Pipe<1>::kSmemBytes, stream>>>(
        ta, tb, tc, args);
  return cudaGetLastError() == cudaSuccess ? B200_OK : B200_ERR_LAUNCH;
}

}  // namespace

extern "C" {

int b200_gemm_bf16(const void* A, const void* B, void* C, int M, int N, int K, int lda, int ldb,
                   int ldc, void* stream) {
  return run_gemm<false>(A, B, C, M, N, K, lda, ldb, ldc, nullptr, 0,
                         static_cast<cudaStream_t>(stream));
}

int b200_gemm_bf16_profile(const void* A, const void* B, void* C, int M, int N, int K, int lda,
                           int ldb, int ldc, int64_t* profiler, int num_entries, void* stream) {
  return run_gemm<true>(A, B, C, M, N, K, lda, ldb, ldc, reinterpret_cast<long long*>(profiler),
                        num_entries, static_cast<cudaStream_t>(stream));
}

int b200_gemm_launch_shape(int M, int N, int K, int* tiles, int* grid, int* smem_bytes,
                           int* threads) {
  if (M < 0 || N < 0 || K < 0) return B200_ERR_INVALID_ARGUMENT;
  const long long t = (long long)((M + kPairM - 1) / kPairM) * ((N + kPairN - 1) / kPairN);
  if (tiles) *tiles = (int)t;
  if (smem_bytes) *smem_bytes = stage_slabs() == 2 ? Pipe<2>::kSmemBytes : Pipe<1>::kSmemBytes;
  if (threads) *threads = kThreads;
  if (grid) {
    *grid = 0;
    DeviceState* d = nullptr;
    if (t > 0 && K > 0 && device_state(&d) == B200_OK)
      *grid = 2 * (int)(t < d->max_pairs ? t : d->max_pairs);
  }
  return B200_OK;
}

int b200_gemm_profile_rows(int M, int N, int K, int* rows) {
  if (!rows) return B200_ERR_INVALID_ARGUMENT;
  int grid = 0;
  const int st = b200_gemm_launch_shape(M, N, K, nullptr, &grid, nullptr, nullptr);
  if (st != B200_OK) return st;
  *rows = grid * kWarps;
  return B200_OK;
}

int b200_gemm_device_status(int clear, int* status_out) {
  if (!status_out) return B200_ERR_INVALID_ARGUMENT;
  DeviceState* d = nullptr;
  const int st = device_state(&d);
  if (st != B200_OK) return st;
  if (cudaDeviceSynchronize() != cudaSuccess) return B200_ERR_LAUNCH;
  int v = 0;
  if (cudaMemcpy(&v, d->status, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess)
    return B200_ERR_LAUNCH;
  if (clear && v != 0 && cudaMemset(d->status, 0, sizeof(int)) != cudaSuccess)
    return B200_ERR_LAUNCH;
  *status_out = v;
  return B200_OK;
}

int b200_gemm_set_tuning(int stage_slabs, int raster_group) {
  if (stage_slabs < 0 || stage_slabs > 2) return B200_ERR_INVALID_ARGUMENT;
  if (stage_slabs > 0) g_slabs.store(stage_slabs);
  if (raster_group != 0) g_group.store(raster_group);
  return B200_OK;
}

int b200_gemm_get_tuning(int* stage_slabs_out, int* raster_group_out) {
  if (stage_slabs_out) *stage_slabs_out = stage_slabs();
  if (raster_group_out) *raster_group_out = raster_group();
  return B200_OK;
}

int b200_gemm_set_wait_timeout_ns(unsigned long long timeout_ns) {
  if (timeout_ns == 0) return B200_ERR_INVALID_ARGUMENT;
  g_timeout_ns.store(timeout_ns);
  return B200_OK;
}

int b200_gemm_wait_probe(unsigned long long timeout_ns, void* stream) {
  if (timeout_ns == 0 || timeout_ns > 10000000000ull) return B200_ERR_INVALID_ARGUMENT;
  DeviceState* d = nullptr;
  const int st = device_state(&d);
  if (st != B200_OK) return st;
  wait_probe_kernel<<<2, 32, 0, static_cast<cudaStream_t>(stream)>>>(d->status, timeout_ns);
  return cudaGetLastError() == cudaSuccess ? B200_OK : B200_ERR_LAUNCH;
}

const char* b200_gemm_status_string(int status) {
  switch (status) {
    case B200_OK: return "ok";
    case B200_ERR_INVALID_ARGUMENT: return "invalid argument (null pointer, negative size or ld < width)";
    case B200_ERR_ALIGNMENT: return "operand not 16-byte aligned (pointers and leading dimensions must be multiples of 8 bf16)";
    case B200_ERR_UNSUPPORTED_DEVICE: return "current CUDA device is not an sm_100 (B200) GPU";
    case B200_ERR_TENSOR_MAP: return "cuTensorMapEncodeTiled rejected an operand";
    case B200_ERR_LAUNCH: return "CUDA error at kernel launch";
    case B200_ERR_DEVICE_TIMEOUT: return "a GEMM pipeline wait ran out of time on the device";
    case B200_ERR_TOO_LARGE: return "size exceeds the entry point's limit";
    default: return "unknown status";
  }
}

void b200_gemm_tile_coord(int t, int tiles_m, int tiles_n, int group, int* tm, int* tn) {
  tile_coord(t, tiles_m, tiles_n, group, tm, tn);
}

uint32_t b200_gemm_idesc(int mma_m, int mma_n) { return make_idesc_bf16_f32(mma_m, mma_n); }

uint64_t b200_gemm_smem_desc(uint32_t smem_addr) { return make_sdesc_k128(smem_addr); }

}  // extern "C"
