// C-ABI launcher for the sm_100a BF16 GEMM (declarations: include/b200_gemm.h).
//
// Per call: validate the operands, pick a kernel configuration (pair tile
// 256 x 256 or 256 x 512, stage depth), encode three TMA tensor maps (A, B:
// 2-D, box 64 x 128, 128 B swizzle, zero fill out of bounds; C: 2-D, box
// 64 x 32, 128 B swizzle), then launch the persistent kernel on the caller's
// stream.  The reference does the same three steps per call with 3-D maps and
// without validation (kernel_v8.cu:775-828).
//
// Per device, once: check the architecture, raise each configuration's
// shared-memory limit, ask the occupancy API how many 2-CTA clusters can be
// resident at once (the persistent grid size) and allocate the 4-byte device
// error word.  The reference keeps a device-blind static cache instead
// (kernel_v8.cu:796-820).
#include <cuda.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "b200_gemm.h"
#include "gemm_kernel.cuh"
#include "gemm_skinny.cuh"

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

// Kernel configurations, named pair-tile width x stage K: {K slabs per
// stage, N sub-tiles per pair tile, sub-tile width}.
enum Variant {
  kV256x64 = 0, kV256x128 = 1, kV512x64 = 2, kV128x64 = 3, kV64x64 = 4, kNumVariants = 5
};
constexpr int kVariantSlabs[kNumVariants] = {1, 2, 1, 1, 1};
constexpr int kVariantNSub[kNumVariants] = {1, 1, 2, 1, 1};
constexpr int kVariantSubW[kNumVariants] = {256, 256, 256, 128, 64};

template <int V>
struct VariantCfg {
  using C = Cfg<kVariantSlabs[V], kVariantNSub[V], kVariantSubW[V]>;
};

template <bool kProfile, int V, int kOut, bool kSK = false>
constexpr auto pair_kernel =
    gemm_bf16_pair_kernel<kProfile, kVariantSlabs[V], kVariantNSub[V], kOut, kVariantSubW[V], kSK>;

constexpr int kMaxDevices = 64;

struct DeviceState {
  bool ready = false;
  int init_status = B200_OK;
  int sms = 0;
  int max_pairs[kNumVariants] = {};         // co-resident 2-CTA clusters per variant
  int* status = nullptr;                    // device error word
  cudaMemPool_t pool = nullptr;             // stream-ordered split-K workspaces
  int sk_clusters[16][4] = {};              // skinny-cluster kernels: resident clusters of 1,2,4,8
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

// Tuning knobs, process-wide: pair-tile width (0 = chosen per shape, 256,
// 512), K slabs per stage for 256-wide tiles (1 or 2) and the raster band
// width.  Initialised from B200_GEMM_TILE_N / B200_GEMM_SLABS /
// B200_GEMM_GROUP, changeable through b200_gemm_set_tuning.
std::atomic<int> g_tile_n{-1};
std::atomic<int> g_slabs{-1};
std::atomic<int> g_group{0};
std::atomic<int> g_splits{-1};
std::atomic<int> g_skinny{-1};
std::atomic<int> g_streamk{-1};
std::atomic<int> g_dynamic{-1};

// Dynamic dealing of the pair kernels' data-parallel units (1) or the
// static deal pair p -> units p, p + P, ... (0, default).  Measured same
// process, cold L2 (TFLOP/s static / dynamic): 8192^3 1597 / 1593, 16384^3
// 1375 / 1375, 8192x6144x4096 1553 / 1496, 8192x4096x4096 1584 / 1542,
// 8192x28672x4096 1547 / 1550, 8192x4096x14336 1535 / 1523, 4096^3 1502 /
// 1465: the static deal is kept.  Initialised from B200_GEMM_DYNAMIC,
// changeable through b200_gemm_set_dynamic.
int dynamic_mode() {
  int v = g_dynamic.load();
  if (v < 0) {
    v = env_int("B200_GEMM_DYNAMIC", 0, 0, 1);
    g_dynamic.store(v);
  }
  return v;
}

// Below this wave efficiency a 256 x 256 grid gets a stream-K tail (mode 1).
constexpr double kStreamKWaveEfficiency = 0.97;

// ... and only from this K up (mode 1): the tail's split tiles meet in a
// fix-up whose cost a short tile does not repay.  Measured (cold L2,
// TFLOP/s, 256-wide tiles with / without the tail): K = 1024: 4096 x 2048
// 533 / 763, 4096 x 4096 795 / 1047, 8192 x 2048 791 / 1042; K = 2048: 2048
// x 4096 878 / 1047; K = 3072: 4096 x 4096 1335 / 1360; K = 4096: 4096 x
// 4096 1500 / 1457, 4096 x 2048 1305 / 1270, 8192 x 2048 1534 / 1457; K =
// 8192: 4096 x 4096 1567 / 1491, 2048 x 4096 1503 / 1428.
constexpr int kStreamKMinK = 4096;

// Stream-K tail of the pair kernel: 0 = off, 1 = when the last wave of tiles
// would leave pairs idle (default), 2 = whenever the tiles are not a whole
// number of waves.  Initialised from B200_GEMM_STREAMK, changeable through
// b200_gemm_set_stream_k.
int stream_k_mode() {
  int v = g_streamk.load();
  if (v < 0) {
    v = env_int("B200_GEMM_STREAMK", 1, 0, 2);
    g_streamk.store(v);
  }
  return v;
}

// L2 cache hints of the skinny kernels' loads (B200_GEMM_L2_HINT, default 1):
// B, read once, evict-first; A, read by every CTA, evict-last.
int skinny_l2_hint() {
  static const int h = env_int("B200_GEMM_L2_HINT", 1, 0, 1);
  return h;
}

std::atomic<int> g_skinny_tiles{-1};

// 128-row blocks of B per tile of the skinny stream-K kernel (blocks of a
// tile share each A slab, so A's share of every SM's L2 inflow falls
// with their number): 1, 2 (M <= 128 only), or 0 = chosen: one.  Two were
// measured slower at every shape (cold-L2 medians, us, one / two blocks):
// N = K = 8192: M = 16 36.2 / 38.1, 64 38.1 / 40.2, 128 42.3 / 46.4;
// N = K = 4096: M = 128 25.9 / 32.0; N = 28672, K = 4096: M = 128 58.6 /
// 68.9 -- each CTA range then cuts twice as many rows of B into partial
// tiles, so the in-kernel fix-up moves twice the slot bytes at the end.
// Initialised from B200_GEMM_SKINNY_TILES, changeable through
// b200_gemm_set_skinny_tiles.
int skinny_stream_tiles(int M) {
  int v = g_skinny_tiles.load();
  if (v < 0) {
    v = env_int("B200_GEMM_SKINNY_TILES", 0, 0, 2);
    g_skinny_tiles.store(v);
  }
  if (M > 128) return 1;
  return v == 0 ? 1 : v;
}

// Skinny-M path (M <= 256): 0 = off, 1 = chosen per shape, 2 = the cluster
// kernel for every M, 3 = the stream-K kernel for every M, 4 = the stream-K
// kernel on 2-CTA pairs, 5 = the cluster kernel on 2-CTA pairs.  Initialised
// from B200_GEMM_SKINNY, changeable through b200_gemm_set_skinny_mode.
int skinny_mode() {
  int v = g_skinny.load();
  if (v < 0) {
    v = env_int("B200_GEMM_SKINNY", 1, 0, 5);
    g_skinny.store(v);
  }
  return v;
}

// Split-K slices: 0 = chosen per shape, 1 = never split, n = n slices.
int tuning_splits() {
  int v = g_splits.load();
  if (v < 0) {
    v = env_int("B200_GEMM_SPLITS", 0, 0, 64);
    g_splits.store(v);
  }
  return v;
}

int tuning_tile_n() {
  int v = g_tile_n.load();
  if (v < 0) {
    v = env_int("B200_GEMM_TILE_N", 0, 0, 512);
    if (v != 64 && v != 128 && v != 256 && v != 512) v = 0;
    g_tile_n.store(v);
  }
  return v;
}

int stage_slabs() {
  int s = g_slabs.load();
  if (s < 0) {
    s = env_int("B200_GEMM_SLABS", 1, 1, 2);
    g_slabs.store(s);
  }
  return s;
}

int raster_group() {
  int g = g_group.load();
  if (g == 0) {
    g = env_int("B200_GEMM_GROUP", -8, -(1 << 16), 1 << 16);
    if (g == 0) g = -8;
    g_group.store(g);
  }
  return g;
}

template <int V>
int query_pairs(int sms, int* out) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * sms, 1, 1);
  cfg.blockDim = dim3(VariantCfg<V>::C::kThreads, 1, 1);
  cfg.dynamicSmemBytes = VariantCfg<V>::C::kSmemBytes;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, pair_kernel<false, V, kOutBf16>, &cfg) != cudaSuccess)
    return B200_ERR_LAUNCH;
  *out = n;
  return B200_OK;
}

template <bool kProfile, int V, int kOut, bool kSK = false>
bool set_smem_limit() {
  return cudaFuncSetAttribute(pair_kernel<kProfile, V, kOut, kSK>,
                              cudaFuncAttributeMaxDynamicSharedMemorySize,
                              VariantCfg<V>::C::kSmemBytes) == cudaSuccess;
}

template <int V>
bool set_smem_limits() {
  return set_smem_limit<false, V, kOutBf16>() && set_smem_limit<true, V, kOutBf16>();
}

// bf16-output limits (with and without the profiler) and resident pairs of
// every configuration.
int init_variants(int sms, int* max_pairs) {
  if (!set_smem_limits<kV256x64>() || !set_smem_limits<kV256x128>() ||
      !set_smem_limits<kV512x64>() || !set_smem_limits<kV128x64>() ||
      !set_smem_limits<kV64x64>() || !set_smem_limit<false, kV256x64, kOutBf16, true>() ||
      !set_smem_limit<false, kV256x128, kOutBf16, true>())
    return B200_ERR_LAUNCH;
  if (query_pairs<kV256x64>(sms, &max_pairs[kV256x64]) != B200_OK ||
      query_pairs<kV256x128>(sms, &max_pairs[kV256x128]) != B200_OK ||
      query_pairs<kV512x64>(sms, &max_pairs[kV512x64]) != B200_OK ||
      query_pairs<kV128x64>(sms, &max_pairs[kV128x64]) != B200_OK ||
      query_pairs<kV64x64>(sms, &max_pairs[kV64x64]) != B200_OK)
    return B200_ERR_LAUNCH;
  for (int v = 0; v < kNumVariants; ++v)
    if (max_pairs[v] < 1) return B200_ERR_LAUNCH;
  return B200_OK;
}

// 128-row blocks of B per unit of the persistent skinny kernel: two (for Mp =
// 256 with a single accumulator, as two no longer fit in TMEM).  Four blocks
// per unit were measured slower at Mp = 128: the ring shrinks to two stages.
constexpr int skinny_tiles(int mp) { return mp > 0 ? 2 : 1; }

// kSlabs: K slabs per stage asked for; each kernel gets the most that fit.
// Largest stream-K tile (128-row blocks of B sharing each A slab) whose
// double-buffered accumulator fits in TMEM: two blocks up to Mp = 128.
constexpr int skinny_stream_max_tiles(int mp) { return 2 * 2 * mp <= 512 ? 2 : 1; }

template <int kMp, int kSlabs, int kTiles, bool kPair = false>
bool set_skinny_stream_limit() {
  constexpr int kSs = skinny_fit_slabs(kMp, kSlabs, kTiles);
  return cudaFuncSetAttribute(gemm_skinny_stream_kernel<kMp, kSs, kTiles, kPair>,
                              cudaFuncAttributeMaxDynamicSharedMemorySize,
                              SkinnyCfg<kMp, kSs, kTiles, kPair>::kSmemBytes) == cudaSuccess;
}

template <int kMp, int kSlabs>
bool set_skinny_limit() {
  constexpr int kT = skinny_tiles(kMp);
  constexpr int kSp = skinny_fit_slabs(kMp, kSlabs, kT);
  return cudaFuncSetAttribute(gemm_skinny_kernel<kMp, kSp, kT>,
                              cudaFuncAttributeMaxDynamicSharedMemorySize,
                              SkinnyCfg<kMp, kSp, kT>::kSmemBytes) == cudaSuccess &&
         set_skinny_stream_limit<kMp, kSlabs, 1>() &&
         set_skinny_stream_limit<kMp, kSlabs, skinny_stream_max_tiles(kMp)>() &&
         (kMp < 32 || set_skinny_stream_limit<(kMp < 32 ? 32 : kMp), kSlabs, 1, true>());
}

template <int kSlabs>
bool set_skinny_limits_for() {
  return set_skinny_limit<16, kSlabs>() && set_skinny_limit<32, kSlabs>() &&
         set_skinny_limit<64, kSlabs>() && set_skinny_limit<128, kSlabs>() &&
         set_skinny_limit<256, kSlabs>();
}

bool set_skinny_limits() {
  return set_skinny_limits_for<1>() && set_skinny_limits_for<2>() && set_skinny_limits_for<4>();
}

// Skinny cluster kernels: (Mp, ring depth, pair slices) per slot of
// DeviceState::sk_clusters.  Shallow rings let two CTAs share an SM, deep
// ones keep one CTA per SM; slots 8-11 are the 2-CTA-pair kernels.
constexpr int kSkc[][3] = {{16, 5, 0},  {16, 10, 0}, {32, 3, 0},  {32, 9, 0},
                           {64, 3, 0},  {64, 8, 0},  {128, 6, 0}, {256, 4, 0},
                           {32, 10, 1}, {64, 9, 1},  {128, 8, 1}, {256, 6, 1}};
constexpr int kNumSkc = 12;
constexpr int kSkcPair0 = 8;  // first pair slot

template <int I>
struct Skc {
  static constexpr int kMp = kSkc[I][0], kStages = kSkc[I][1];
  static constexpr bool kPair = kSkc[I][2] != 0;
  using P = SkinnyClusterCfg<kMp, kStages, kPair>;
  static constexpr auto kernel = gemm_skinny_cluster_kernel<kMp, kStages, kPair>;
};

template <int I>
bool skc_init(DeviceState& d) {
  using S = Skc<I>;
  if (cudaFuncSetAttribute(S::kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           S::P::kSmemBytes) != cudaSuccess)
    return false;
  for (int ci = S::kPair ? 1 : 0; ci < 4; ++ci) {  // pairs: clusters of 2, 4, 8
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(8 * d.sms, 1, 1);
    cfg.blockDim = dim3(S::P::kThreads, 1, 1);
    cfg.dynamicSmemBytes = S::P::kSmemBytes;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 1u << ci;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, S::kernel, &cfg) != cudaSuccess) {
      cudaGetLastError();
      n = 0;
    }
    d.sk_clusters[I][ci] = n;
  }
  return true;
}

bool skc_init_all(DeviceState& d) {
  return skc_init<0>(d) && skc_init<1>(d) && skc_init<2>(d) && skc_init<3>(d) &&
         skc_init<4>(d) && skc_init<5>(d) && skc_init<6>(d) && skc_init<7>(d) &&
         skc_init<8>(d) && skc_init<9>(d) && skc_init<10>(d) && skc_init<11>(d);
}

int init_device(DeviceState& d, int dev) {
  cudaDeviceProp prop;
  if (cudaGetDeviceProperties(&prop, dev) != cudaSuccess) return B200_ERR_UNSUPPORTED_DEVICE;
  if (prop.major != 10 || prop.minor != 0) return B200_ERR_UNSUPPORTED_DEVICE;  // sm_100a only
  if (encode_tiled() == nullptr) return B200_ERR_TENSOR_MAP;
  d.sms = prop.multiProcessorCount;
  if (!set_smem_limit<false, kV256x64, kOutF32>() ||
      !set_smem_limit<false, kV256x64, kOutF32Add>() ||
      !set_smem_limit<false, kV256x64, kOutBf16Epi>() || !set_skinny_limits())
    return B200_ERR_LAUNCH;
  const int vst = init_variants(d.sms, d.max_pairs);
  if (vst != B200_OK) return vst;
  if (!skc_init_all(d)) return B200_ERR_LAUNCH;
  if (cudaMalloc(&d.status, sizeof(int)) != cudaSuccess ||
      cudaMemset(d.status, 0, sizeof(int)) != cudaSuccess)
    return B200_ERR_LAUNCH;
  // Split-K workspaces come from a pool of our own, allocated and freed in
  // stream order, so concurrent calls on different streams never share one;
  // the pool keeps up to 512 MiB mapped between calls (the host-operand
  // entry point holds A, B and C blocks at once).
  cudaMemPoolProps props = {};
  props.allocType = cudaMemAllocationTypePinned;
  props.location.type = cudaMemLocationTypeDevice;
  props.location.id = dev;
  if (cudaMemPoolCreate(&d.pool, &props) != cudaSuccess) return B200_ERR_LAUNCH;
  unsigned long long keep = 512ull << 20;
  if (cudaMemPoolSetAttribute(d.pool, cudaMemPoolAttrReleaseThreshold, &keep) != cudaSuccess)
    return B200_ERR_LAUNCH;
  return B200_OK;
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
    d.init_status = init_device(d, dev);
    if (d.init_status != B200_OK) cudaGetLastError();
  }
  if (d.init_status != B200_OK) return d.init_status;
  *out = &d;
  return B200_OK;
}

long long ceil_div(long long a, long long b) { return (a + b - 1) / b; }

// Scratch memory given to a call instead of the device's pool (the
// allocation-free entry point passes its fixed array).  flags: a region that
// holds only epoch flags, so values left there by earlier calls are always
// older epochs; epoch: the value this call's flags are raised to (each call
// takes a new one), or 0 under stream capture, where the used flags are
// cleared on the stream and the call raises them to 1.  work: workspaces
// (fp32 split-K accumulators, stream-K slots), reused by every call.
struct Scratch {
  unsigned int* flags = nullptr;
  size_t flag_count = 0;
  unsigned int epoch = 0;
  char* work = nullptr;
  size_t work_bytes = 0;
};

// Fraction of pair-slots doing useful work over the persistent waves.
double wave_efficiency(long long tiles, int pairs) {
  const long long waves = ceil_div(tiles, pairs);
  return waves > 0 ? (double)tiles / (double)(waves * pairs) : 0.0;
}

// Configuration for an M x N problem.  512-wide pair tiles read 25% fewer
// operand bytes per FLOP through L2 (one A slab feeds two MMAs), which under
// the 1 kW power cap turns into clock; they are chosen unless halving the
// tile count costs wave efficiency or leaves pairs idle.  Grids of fewer
// 256-wide tiles than pairs leave SMs idle while each pair walks the whole
// K; 128- or 64-wide tiles then finish sooner: the width minimising
// waves x width wins, the wider one on a tie.  Up to K = 1024 the 256-wide
// tile is kept unless the 512-wide one is 2 % more wave-efficient: each
// tile's mainloop is short, and only the 256-wide kernel hides a tile's
// epilogue behind the next tile's MMAs (TFLOP/s, 256 / 512 wide at equal
// wave counts: 4096 x 4096 x 1024 1047 / 982, 8192 x 2048 x 1024 1042 /
// 960; at K = 2048, 8192 x 8192: 1616 / 1636).
int choose_variant(int M, int N, int K, const int* max_pairs) {
  const int tn = tuning_tile_n();
  if (tn == 512) return kV512x64;
  if (tn == 128) return kV128x64;
  if (tn == 64) return kV64x64;
  const int v256 = stage_slabs() == 2 ? kV256x128 : kV256x64;
  if (tn == 256) return v256;
  auto pairs = [&](int v) { return max_pairs ? max_pairs[v] : 74; };
  const long long rows = ceil_div(M, kPairM);
  const long long t256 = rows * ceil_div(N, kSubN);
  const long long t512 = rows * ceil_div(N, 2 * kSubN);
  if (t256 < pairs(v256)) {
    int best = v256;
    long long best_cost = kSubN;  // one wave
    for (const int v : {kV128x64, kV64x64}) {
      const long long t = rows * ceil_div(N, kVariantSubW[v]);
      const long long cost = ceil_div(t, pairs(v)) * kVariantSubW[v];
      if (cost < best_cost) {
        best = v;
        best_cost = cost;
      }
    }
    return best;
  }
  if (t512 < pairs(kV512x64)) return v256;
  // A 256-wide grid whose last wave would run a stream-K tail keeps every
  // pair busy to the end: count it as (nearly) full.
  double eff256 = wave_efficiency(t256, pairs(v256));
  if (stream_k_mode() != 0 && t256 > pairs(v256) && t256 % pairs(v256) != 0 &&
      (stream_k_mode() == 2 || (eff256 < kStreamKWaveEfficiency && K >= kStreamKMinK)))
    eff256 = 0.99;
  const double bias = K <= 1024 ? -0.02 : 0.02;
  return wave_efficiency(t512, pairs(kV512x64)) + bias >= eff256 ? kV512x64 : v256;
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
              uint64_t row_stride_elems, uint32_t box_inner, uint32_t box_outer,
              bool fp32 = false, bool swizzle = true) {
  const cuuint64_t dims[2] = {inner, outer};
  const cuuint64_t strides[1] = {row_stride_elems * (fp32 ? 4 : 2)};
  const cuuint32_t box[2] = {box_inner, box_outer};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = encode_tiled()(
      map, fp32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
      const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
      swizzle ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE, l2_promotion(),
      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? B200_OK : B200_ERR_TENSOR_MAP;
}

int validate(const void* A, const void* B, void* C, int M, int N, int K, int lda, int ldb,
             int ldc, bool c_fp32 = false) {
  if (M < 0 || N < 0 || K < 0) return B200_ERR_INVALID_ARGUMENT;
  if (M == 0 || N == 0) return B200_OK;
  if (!C || (K > 0 && (!A || !B))) return B200_ERR_INVALID_ARGUMENT;
  if (ldc < N || (K > 0 && (lda < K || ldb < K))) return B200_ERR_INVALID_ARGUMENT;
  if (!aligned16(C) || (ldc & (c_fp32 ? 3 : 7))) return B200_ERR_ALIGNMENT;
  if (K > 0 && (!aligned16(A) || !aligned16(B) || (lda & 7) || (ldb & 7)))
    return B200_ERR_ALIGNMENT;
  return B200_OK;
}

// Slices for split-K (units of 256 x 256 tiles x K slices; the fp32
// workspace is cleared, reduce-added into and rounded: two extra passes).
// It pays only when even 64-wide pair tiles would leave more than half the
// pairs idle and K is deep: then K is cut into up to 16 slices of at least 8
// K-blocks.  Shallow problems (fewer than 32 K-blocks) are never split.
int choose_splits(int M, int N, int k_blocks, int pairs) {
  const int forced = tuning_splits();
  int s;
  if (forced > 0) {
    s = forced;
  } else {
    const long long narrow = ceil_div(M, kPairM) * ceil_div(N, kVariantSubW[kV64x64]);
    if (narrow * 2 > pairs || k_blocks < 32) return 1;
    s = k_blocks / 8;
    if (s > 16) s = 16;
  }
  if (s > k_blocks) s = k_blocks;
  return s < 1 ? 1 : s;
}

// Per-(device, stream) counters of the dynamic dealing (GemmArgs::sched):
// two words, zero at every launch -- each launch's last pair sets them back
// to zero -- so consecutive launches on one stream share them and launches
// on different streams never do.  Created on a stream's first call
// (cudaMalloc, cleared on the stream itself); null when none can be made.
struct StreamSched {
  int device;
  cudaStream_t stream;
  unsigned int* words;
};
constexpr int kMaxStreamScheds = 256;
StreamSched g_stream_sched[kMaxStreamScheds];
int g_num_stream_sched = 0;

unsigned int* stream_sched(cudaStream_t stream) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    cudaGetLastError();
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(g_mu);
  for (int i = 0; i < g_num_stream_sched; ++i)
    if (g_stream_sched[i].device == dev && g_stream_sched[i].stream == stream)
      return g_stream_sched[i].words;
  if (g_num_stream_sched == kMaxStreamScheds) return nullptr;
  unsigned int* p = nullptr;
  if (cudaMalloc(&p, 256) != cudaSuccess || cudaMemsetAsync(p, 0, 256, stream) != cudaSuccess) {
    cudaGetLastError();
    if (p) cudaFree(p);
    return nullptr;
  }
  g_stream_sched[g_num_stream_sched++] = {dev, stream, p};
  return p;
}

template <bool kProfile, int V, int kOut, bool kSK = false>
int launch(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc, GemmArgs args,
           int splits, const DeviceState& d, cudaStream_t stream) {
  using C = typename VariantCfg<V>::C;
  args.tiles_n = (int)ceil_div(args.N, C::kTileN);
  args.k_blocks = (int)ceil_div(args.K, C::kBK);
  if (splits > args.k_blocks) splits = args.k_blocks;
  args.kb_per_split = (int)ceil_div(args.k_blocks, splits);
  args.splits = (int)ceil_div(args.k_blocks, args.kb_per_split);  // every slice non-empty
  if (args.sk_tiles <= 0) {
    args.sk_tiles = 0;
    args.dp_tiles = args.tiles_m * args.tiles_n;
  }
  const long long units =
      args.sk_tiles > 0 ? d.max_pairs[V] : (long long)args.dp_tiles * args.splits;
  const int pairs = (int)(units < d.max_pairs[V] ? units : d.max_pairs[V]);
  // Dynamic dealing pays only past the first wave.  Counters: the stream's
  // own outside capture; under capture (a graph may be replayed on another
  // stream) a pair of words from the pool, cleared in the graph.  A caller
  // that set args.sched (the allocation-free entry point) keeps its own.
  char* sched_ws = nullptr;
  if (args.sched == nullptr && dynamic_mode() != 0 && args.dp_tiles * (long long)args.splits > pairs) {
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(stream, &cap) != cudaSuccess) {
      cudaGetLastError();
      cap = cudaStreamCaptureStatusActive;
    }
    if (cap == cudaStreamCaptureStatusNone) {
      args.sched = stream_sched(stream);
    } else if (d.pool != nullptr) {
      if (cudaMallocFromPoolAsync(reinterpret_cast<void**>(&sched_ws), 256, d.pool, stream) ==
              cudaSuccess &&
          cudaMemsetAsync(sched_ws, 0, 256, stream) == cudaSuccess) {
        args.sched = reinterpret_cast<unsigned int*>(sched_ws);
      } else {
        cudaGetLastError();
        return B200_ERR_LAUNCH;
      }
    }
  }
  pair_kernel<kProfile, V, kOut, kSK><<<2 * pairs, C::kThreads, C::kSmemBytes, stream>>>(
      ta, tb, tc, args);
  const int st = cudaGetLastError() == cudaSuccess ? B200_OK : B200_ERR_LAUNCH;
  if (sched_ws != nullptr) cudaFreeAsync(sched_ws, stream);
  return st;
}

// bf16 GEMM with configuration v.  tb maps B with 128-row boxes (the
// 256-wide sub-tiles); narrower sub-tiles load kSubW / 2 rows of B per CTA,
// so their map is encoded here.
// Per-(device, stream) stream-K flag arrays and their epochs.  Returns the
// array (at least `count` flags, zeroed when created) and the next epoch in
// *epoch, or null when one cannot be made (the caller then clears flags of
// its own).  Arrays live until exit.
struct StreamFlags {
  int device;
  cudaStream_t stream;
  unsigned int* flags;
  size_t count;
  unsigned int epoch;
};
constexpr int kMaxStreamFlags = 256;
StreamFlags g_stream_flags[kMaxStreamFlags];
int g_num_stream_flags = 0;

unsigned int* stream_flags(cudaStream_t stream, size_t count, unsigned int* epoch) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    cudaGetLastError();
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(g_mu);
  for (int i = 0; i < g_num_stream_flags; ++i) {
    StreamFlags& f = g_stream_flags[i];
    if (f.device == dev && f.stream == stream && f.count >= count) {
      if (++f.epoch == 0) return nullptr;  // 2^32 calls: fall back to cleared flags
      *epoch = f.epoch;
      return f.flags;
    }
  }
  if (g_num_stream_flags == kMaxStreamFlags) return nullptr;
  const size_t n = count < 4096 ? 4096 : count;
  unsigned int* p = nullptr;
  // Once per (device, stream): cudaMalloc, then a clear queued on the stream
  // itself -- every kernel that reads the array runs on that stream, after
  // the clear, so nothing waits on the host or on other streams.
  if (cudaMalloc(&p, n * sizeof(unsigned int)) != cudaSuccess ||
      cudaMemsetAsync(p, 0, n * sizeof(unsigned int), stream) != cudaSuccess) {
    cudaGetLastError();
    if (p) cudaFree(p);
    return nullptr;
  }
  g_stream_flags[g_num_stream_flags++] = {dev, stream, p, n, 1u};
  *epoch = 1u;
  return p;
}

// Data-parallel waves plus a stream-K tail (see GemmArgs): applies to the
// 256 x 256 pair-tile configurations (their second TMEM accumulator lets a
// tile's finishing epilogue overlap the next tile's MMAs) when the tiles are
// more than one wave and not a whole number of waves (mode 1: only when the last wave would leave
// at least 3 % of the pair-slots idle).  Sets *used; the workspace (one
// piece per epilogue warp per pair, and their flags) comes from the pool.
template <int V>
int launch_streamk(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc,
                   GemmArgs args, const DeviceState& d, cudaStream_t stream, bool* used) {
  using C = typename VariantCfg<V>::C;
  *used = false;
  const int mode = stream_k_mode();
  if (mode == 0) return B200_OK;
  const long long tiles = (long long)args.tiles_m * ceil_div(args.N, C::kTileN);
  const int P = d.max_pairs[V];
  if (tiles <= P || tiles % P == 0) return B200_OK;
  if (mode == 1 && (wave_efficiency(tiles, P) >= kStreamKWaveEfficiency || args.K < kStreamKMinK))
    return B200_OK;
  const long long k_blocks = ceil_div(args.K, C::kBK);
  args.dp_tiles = (int)(tiles / P * P);
  args.sk_tiles = (int)(tiles - args.dp_tiles);
  args.sk_items = args.sk_tiles * k_blocks;
  const long long slots = (long long)P * 2 * C::kEpiWarps;  // one piece per epilogue warp per pair
  const size_t flag_bytes = (size_t)ceil_div(slots * 4, 256) * 256;
  const size_t slot_bytes = (size_t)slots * kPieceFloats * sizeof(float);
  char* ws = nullptr;
  if (cudaMallocFromPoolAsync(reinterpret_cast<void**>(&ws), flag_bytes + slot_bytes, d.pool,
                              stream) != cudaSuccess) {
    cudaGetLastError();
    return B200_ERR_LAUNCH;
  }
  args.sk_slots = reinterpret_cast<float*>(ws + flag_bytes);
  // Flags: outside stream capture, a per-(device, stream) array that keeps
  // its values between calls, each call raising flags to a new epoch (stale
  // flags hold older epochs, so nothing needs clearing and no extra
  // operation precedes the kernel; calls on one stream are ordered, calls on
  // different streams use different arrays).  Under capture the graph may be
  // replayed with the same epoch, so the workspace's own flags are cleared
  // in the graph instead.
  int st = B200_OK;
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(stream, &cap) != cudaSuccess) {
    cudaGetLastError();
    cap = cudaStreamCaptureStatusActive;
  }
  unsigned int* persistent = nullptr;
  if (cap == cudaStreamCaptureStatusNone)
    persistent = stream_flags(stream, (size_t)slots, &args.sk_epoch);
  if (persistent != nullptr) {
    args.sk_flags = persistent;
  } else {
    args.sk_flags = reinterpret_cast<unsigned int*>(ws);
    args.sk_epoch = 1;
    if (cudaMemsetAsync(ws, 0, flag_bytes, stream) != cudaSuccess) st = B200_ERR_LAUNCH;
  }
  if (st == B200_OK) st = launch<false, V, kOutBf16, true>(ta, tb, tc, args, 1, d, stream);
  cudaFreeAsync(ws, stream);
  *used = true;
  return st;
}

template <bool kProfile>
int launch_bf16(int v, const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc,
                const void* B, int ldb, const GemmArgs& args, const DeviceState& d,
                cudaStream_t stream, bool may_allocate = true) {
  if (!kProfile && may_allocate && (v == kV256x64 || v == kV256x128)) {
    bool used = false;
    const int st = v == kV256x128 ? launch_streamk<kV256x128>(ta, tb, tc, args, d, stream, &used)
                                  : launch_streamk<kV256x64>(ta, tb, tc, args, d, stream, &used);
    if (used || st != B200_OK) return st;
  }
  if (v == kV128x64 || v == kV64x64) {
    CUtensorMap tbn;
    if (encode_2d(&tbn, B, args.K, args.N, ldb, kSlabK, kVariantSubW[v] / 2) != B200_OK)
      return B200_ERR_TENSOR_MAP;
    return v == kV128x64 ? launch<kProfile, kV128x64, kOutBf16>(ta, tbn, tc, args, 1, d, stream)
                         : launch<kProfile, kV64x64, kOutBf16>(ta, tbn, tc, args, 1, d, stream);
  }
  switch (v) {
    case kV256x128: return launch<kProfile, kV256x128, kOutBf16>(ta, tb, tc, args, 1, d, stream);
    case kV512x64: return launch<kProfile, kV512x64, kOutBf16>(ta, tb, tc, args, 1, d, stream);
    default: return launch<kProfile, kV256x64, kOutBf16>(ta, tb, tc, args, 1, d, stream);
  }
}

int cast_to_bf16(const float* W, int ldw, void* C, int ldc, int M, int N, int sms,
                 cudaStream_t stream, const EpiArgs* epi = nullptr) {
  const EpiArgs none = {1.0f, 0.0f, nullptr, nullptr, 0};
  const long long groups = (long long)M * ((N + 7) / 8);
  long long blocks = ceil_div(groups, 256);
  if (blocks > 8LL * sms) blocks = 8LL * sms;
  cast_f32_to_bf16_kernel<<<(int)blocks, 256, 0, stream>>>(
      W, ldw, static_cast<__nv_bfloat16*>(C), ldc, M, N, epi ? *epi : none, epi != nullptr);
  return cudaGetLastError() == cudaSuccess ? B200_OK : B200_ERR_LAUNCH;
}

// Skinny-M path (M <= 256): C^T = B A^T with B streamed by every SM (see
// gemm_skinny.cuh).  K is cut into slices so the (128-row block, K slice)
// units fill the SMs, but every slice adds M x N fp32 of reduce-add traffic:
// the slice count minimises (B bytes + slices x workspace bytes) / wave
// efficiency, with at least 2 K-blocks per slice (at N = K = 8192: 9 slices
// up to M = 64, 2 above).
int choose_skinny_splits(long long tiles, int k_blocks, int ctas, int M, int N, int K) {
  const int forced = tuning_splits();
  if (forced > 0) return forced < k_blocks ? forced : k_blocks;
  const double b_bytes = 2.0 * N * K, w_bytes = 4.0 * M * N;
  int best = 1;
  double best_cost = b_bytes / wave_efficiency(tiles, ctas);
  const int max_s = k_blocks / 2 < 64 ? k_blocks / 2 : 64;
  for (int s2 = 2; s2 <= max_s; ++s2) {
    const double cost = (b_bytes + s2 * w_bytes) / wave_efficiency(tiles * s2, ctas);
    if (cost < best_cost) {
      best_cost = cost;
      best = s2;
    }
  }
  return best;
}

constexpr int kSkinnyMaxM = 256;

int skinny_occupancy();
int skc_choose(const DeviceState& d, int I, bool pair, long long tiles, int k_blocks);

// Cluster-kernel slot (kSkc) that run_skinny_cluster takes for M rows of A
// with one-CTA slices.
int skc_slot(int M) {
  const bool two = skinny_occupancy() == 2;
  return M <= 16 ? (two ? 0 : 1) : M <= 32 ? (two ? 2 : 3) : M <= 64 ? (two ? 4 : 5)
                                                            : M <= 128 ? 6 : 7;
}

// The cluster kernel (mode 1) wherever its grid of 128-row blocks x S
// slices fits in one wave.  It ends with one distributed-shared-memory
// reduction where the stream-K kernel ends with a global-memory fix-up of
// the blocks split between CTAs, and it needs no workspace.  Measured (cold
// L2, median us, after a flush that leaves L2 clean / after the written
// flush; cluster, stream-K or split-K as chosen before, cuBLAS): N = K =
// 8192: M = 16 30.7 / 32.9, 32.1 / 36.2, 28.7 / 37.0; M = 64 30.8 / 34.9,
// 34.6 / 38.2, 29.2 / 37.8; M = 128 34.9 / 38.9, 40.1 / 42.3, 28.7 / 37.0;
// N = K = 4096: M = 64 18.4 / 18.5, 21.7 / 22.7, 14.4 / 16.5; M = 256 28.7 /
// 28.7, 30.9 / 33.0, 14.4 / 18.5; N = 4096, K = 14336: M = 128 32.9 / 35.0,
// 38.1 / 40.2, 28.7 / 37.0.  Where the grid needs more than one wave (N =
// 28672) the stream-K kernels stay ahead (M = 128: 61.4 / 65.6 against
// 52.5 / 58.6).  With a forced slice count (b200_gemm_set_splits) only M <= 8
// takes it, as the split-K kernels do.
bool skinny_use_cluster(int M, int N, int K, const DeviceState* d) {
  if (tuning_splits() > 0) return M <= 8;
  const int I = skc_slot(M);
  const long long tiles = ceil_div(N, 128);
  const int k_blocks = (int)ceil_div(K, kSlabK);
  int ci = 0;
  long long fit = 0;
  if (d != nullptr) {
    ci = skc_choose(*d, I, false, tiles, k_blocks);
    fit = d->sk_clusters[I][ci];
  } else {
    // no device: 148 SMs, one CTA each (GPC limits ignored)
    for (int c = 3; c >= 1; --c)
      if (tiles <= (148 >> c) && k_blocks >= (8 << c)) {
        ci = c;
        break;
      }
    fit = 148 >> ci;
  }
  return tiles <= fit;
}

// Above M = 128, the cluster kernel on 2-CTA pairs (each CTA loads half of
// A's rows) where its grid of 256-row blocks fits in one wave on at least as
// many CTAs as the one-CTA kernel's grid would use.  Measured as above (us):
// M = 256, N = K = 8192 (both on 128 CTAs): pairs 42.1 / 43.1, one-CTA 45.0 /
// 45.2, split-K 51.3 / 51.6, cuBLAS 34.7 / 43.1; N = 4096, K = 14336 (8-CTA
// clusters of pairs do not fit: pairs on 64 CTAs, one-CTA on 128): pairs 53.2
// / 55.3, one-CTA 45.1 / 47.1.
bool skinny_use_pair_cluster(int M, int N, int K, const DeviceState* d) {
  if (tuning_splits() > 0 || M <= 128 || d == nullptr) return false;
  const int k_blocks = (int)ceil_div(K, kSlabK);
  const int I = kSkcPair0 + 3;  // M > 128: Mp = 256
  const long long tiles = ceil_div(N, 256);
  const int ci = skc_choose(*d, I, true, tiles, k_blocks);
  if (tiles > d->sk_clusters[I][ci]) return false;
  const int I1 = skc_slot(M);
  const long long tiles1 = ceil_div(N, 128);
  const int ci1 = skc_choose(*d, I1, false, tiles1, k_blocks);
  if (tiles1 > d->sk_clusters[I1][ci1]) return true;
  return (tiles << ci) >= (tiles1 << ci1);
}

// Per shape (mode 1), without a forced slice count: the stream-K kernel
// from the cluster kernel's bound up to M = 128 (measured faster than the
// persistent split-K kernel there at N, K = 4096..28672), the split-K kernel
// above (its units of two blocks of B share A's slab; the stream-K kernel
// re-reads A per block, twice B's bytes at M = 256).
bool skinny_use_stream(int M, int N, int K, const DeviceState* d) {
  return tuning_splits() == 0 && !skinny_use_cluster(M, N, K, d) && M <= 128;
}

// Above M = 128, the stream-K kernel on 2-CTA pairs where the split-K
// kernel's fp32 workspace (cleared, reduce-added into, rounded: three passes
// and two more launches) reaches 16 MB.  Measured (cold-L2 medians, us,
// split-K / pair stream-K / cuBLAS): M = 256, N = 28672, K = 4096: 80.2 / 69.5
// / 66.7; N = K = 8192: 51.5 / 52.4 / 43.1; N = 4096, K = 14336: 47.4 / 48.5 /
// 41.4.  At M <= 128 the pair kernel was ~2 us slower than the one-CTA
// stream-K kernel at every shape (the pair TMEM allocation's launch cost).
bool skinny_use_pair_stream(int M, int N, int K) {
  return tuning_splits() == 0 && M > 128 && (long long)M * N >= (4LL << 20);
}

template <int kMp, int kSlabsWanted>
int launch_skinny(const void* A, const void* B, void* C, int M, int N, int K, int lda, int ldb,
                  int ldc, DeviceState& d, cudaStream_t stream, const EpiArgs* epi,
                  const Scratch* scratch) {
  constexpr int kTiles = skinny_tiles(kMp);
  constexpr int kSlabs = skinny_fit_slabs(kMp, kSlabsWanted, kTiles);
  using P = SkinnyCfg<kMp, kSlabs, kTiles>;
  CUtensorMap tb, ta, tw;
  if (encode_2d(&tb, B, K, N, ldb, kSlabK, P::kRowsB) != B200_OK ||
      encode_2d(&ta, A, K, M, lda, kSlabK, kMp) != B200_OK)
    return B200_ERR_TENSOR_MAP;
  SkinnyArgs args;
  args.l2_hint = skinny_l2_hint();
  args.M = M;
  args.N = N;
  args.K = K;
  args.tiles = (int)ceil_div(N, P::kRowsB);
  args.groups = (int)ceil_div(args.tiles, kTiles);
  args.k_blocks = (int)ceil_div(K, P::kBK);
  int splits = choose_skinny_splits(args.groups, args.k_blocks, d.sms, M, N, K);
  args.kb_per_split = (int)ceil_div(args.k_blocks, splits);
  args.splits = (int)ceil_div(args.k_blocks, args.kb_per_split);
  args.status = d.status;
  args.timeout_ns = g_timeout_ns.load();
  const int ldw = (int)ceil_div(N, 8) * 8;
  const size_t bytes = (size_t)M * ldw * sizeof(float);
  float* W = nullptr;
  if (scratch != nullptr) {
    if (bytes > scratch->work_bytes) return B200_ERR_TOO_LARGE;
    W = reinterpret_cast<float*>(scratch->work);
  } else if (cudaMallocFromPoolAsync(reinterpret_cast<void**>(&W), bytes, d.pool, stream) !=
             cudaSuccess) {
    cudaGetLastError();
    return B200_ERR_LAUNCH;
  }
  int st = encode_2d(&tw, W, N, M, ldw, 32, P::kChunk, true, false);
  if (st == B200_OK && cudaMemsetAsync(W, 0, bytes, stream) != cudaSuccess) st = B200_ERR_LAUNCH;
  if (st == B200_OK) {
    const long long units = (long long)args.groups * args.splits;
    const int grid = (int)(units < d.sms ? units : d.sms);
    gemm_skinny_kernel<kMp, kSlabs, kTiles><<<grid, P::kThreads, P::kSmemBytes, stream>>>(
        tb, ta, tw, args);
    if (cudaGetLastError() != cudaSuccess) st = B200_ERR_LAUNCH;
  }
  if (st == B200_OK) st = cast_to_bf16(W, ldw, C, ldc, M, N, d.sms, stream, epi);
  if (scratch == nullptr) cudaFreeAsync(W, stream);
  return st;
}

// Stream-K skinny kernel (gemm_skinny_stream_kernel): G = min(SMs, work
// items) CTAs, equal contiguous ranges of (tile, K block) items, one
// cooperative launch; partial tiles meet in a per-call slot workspace.
long long stream_owner_host(long long x, long long total, int G) {
  return ((x + 1) * G + total - 1) / total - 1;
}

template <int kMp, int kSlabs, int kTiles, bool kPair = false>
int launch_skinny_stream(const void* A, const void* B, void* C, int M, int N, int K, int lda,
                         int ldb, int ldc, DeviceState& d, cudaStream_t stream,
                         const Scratch* scratch) {
  using P = SkinnyCfg<kMp, kSlabs, kTiles, kPair>;
  // flag / slot units per tile: one, or a pair tile's two CTA halves
  constexpr int kUnits = kPair ? 2 : 1;
  CUtensorMap tb, ta, tc;
  if (encode_2d(&tb, B, K, N, ldb, kSlabK, P::kRowsB) != B200_OK ||
      encode_2d(&ta, A, K, M, lda, kSlabK, P::kRowsA) != B200_OK ||
      encode_2d(&tc, C, N, M, ldc, 32, P::kChunk, false, false) != B200_OK)
    return B200_ERR_TENSOR_MAP;
  SkinnyStreamArgs args;
  args.l2_hint = skinny_l2_hint();
  args.M = M;
  args.N = N;
  args.K = K;
  args.tiles = (int)ceil_div(N, (kPair ? 2 : kTiles) * P::kRowsB);
  args.k_blocks = (int)ceil_div(K, P::kBK);
  args.total = (long long)args.tiles * args.k_blocks;
  const int workers = kPair ? d.sms / 2 : d.sms;  // pairs or CTAs, one per SM (pair)
  const int G = (int)(args.total < workers ? args.total : workers);
  int max_seg = 1;
  for (int t = 0; t < args.tiles; ++t) {
    const long long x0 = (long long)t * args.k_blocks;
    const long long segs = stream_owner_host(x0 + args.k_blocks - 1, args.total, G) -
                           stream_owner_host(x0, args.total, G) + 1;
    if (segs > max_seg) max_seg = (int)segs;
  }
  args.max_seg = max_seg;
  args.status = d.status;
  args.timeout_ns = g_timeout_ns.load();
  const size_t nflags = (size_t)kUnits * args.tiles * max_seg * 4;
  const size_t flag_bytes = (size_t)ceil_div((long long)nflags * 4, 256) * 256;
  const size_t slot_bytes =
      (size_t)kUnits * args.tiles * max_seg * kTiles * kMp * P::kRowsB * sizeof(float);
  char* ws = nullptr;
  int st = B200_OK;
  if (scratch != nullptr) {
    // The caller's scratch: slots in its workspace, flags in its flag region
    // (a new epoch per call, or cleared flags under capture).
    if (slot_bytes > scratch->work_bytes || nflags > scratch->flag_count)
      return B200_ERR_TOO_LARGE;
    args.slots = reinterpret_cast<float*>(scratch->work);
    args.flags = scratch->flags;
    args.epoch = scratch->epoch;
    if (args.epoch == 0) {
      args.epoch = 1;
      if (cudaMemsetAsync(scratch->flags, 0, nflags * 4, stream) != cudaSuccess)
        st = B200_ERR_LAUNCH;
    }
  } else {
    if (cudaMallocFromPoolAsync(reinterpret_cast<void**>(&ws), flag_bytes + slot_bytes, d.pool,
                                stream) != cudaSuccess) {
      cudaGetLastError();
      return B200_ERR_LAUNCH;
    }
    args.slots = reinterpret_cast<float*>(ws + flag_bytes);
    // Flags: the stream's epoch-numbered array outside capture (no clearing
    // operation before the kernel), cleared workspace flags under capture.
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(stream, &cap) != cudaSuccess) {
      cudaGetLastError();
      cap = cudaStreamCaptureStatusActive;
    }
    unsigned int* persistent = nullptr;
    if (cap == cudaStreamCaptureStatusNone)
      persistent = stream_flags(stream, nflags, &args.epoch);
    if (persistent != nullptr) {
      args.flags = persistent;
    } else {
      args.flags = reinterpret_cast<unsigned int*>(ws);
      args.epoch = 1;
      if (cudaMemsetAsync(ws, 0, flag_bytes, stream) != cudaSuccess) st = B200_ERR_LAUNCH;
    }
  }
  if (st == B200_OK) {
    // Cooperative: the fix-up waits on CTAs of higher index, so all of the
    // grid (one CTA per SM) must be resident together.  Pairs: 2-CTA clusters.
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(kUnits * G), 1, 1);
    cfg.blockDim = dim3(P::kThreads, 1, 1);
    cfg.dynamicSmemBytes = P::kSmemBytes;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = kUnits;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = kPair ? 2 : 1;
    if (cudaLaunchKernelEx(&cfg, gemm_skinny_stream_kernel<kMp, kSlabs, kTiles, kPair>, tb, ta,
                           tc, args) != cudaSuccess) {
      cudaGetLastError();
      st = B200_ERR_LAUNCH;
    }
  }
  if (ws != nullptr) cudaFreeAsync(ws, stream);
  return st;
}

template <int kSlabs>
int run_skinny_stream_slabs(const void* A, const void* B, void* C, int M, int N, int K, int lda,
                            int ldb, int ldc, DeviceState& d, cudaStream_t stream,
                            const Scratch* scratch, bool pair = false) {
#define B200_SKS(MP, T)                                                                    \
  launch_skinny_stream<MP, skinny_fit_slabs(MP, kSlabs, T), T>(A, B, C, M, N, K, lda, ldb, ldc, \
                                                               d, stream, scratch)
  if (pair) {
#define B200_SKP(MP)                                                                         \
  launch_skinny_stream<MP, skinny_fit_slabs(MP, kSlabs), 1, true>(A, B, C, M, N, K, lda, ldb, \
                                                                  ldc, d, stream, scratch)
    if (M <= 32) return B200_SKP(32);
    if (M <= 64) return B200_SKP(64);
    if (M <= 128) return B200_SKP(128);
    return B200_SKP(256);
#undef B200_SKP
  }
  const bool two = skinny_stream_tiles(M) == 2;
  if (M <= 16) return two ? B200_SKS(16, 2) : B200_SKS(16, 1);
  if (M <= 32) return two ? B200_SKS(32, 2) : B200_SKS(32, 1);
  if (M <= 64) return two ? B200_SKS(64, 2) : B200_SKS(64, 1);
  if (M <= 128) return two ? B200_SKS(128, 2) : B200_SKS(128, 1);
  return B200_SKS(256, 1);
#undef B200_SKS
}

template <int kSlabs>
int run_skinny_slabs(const void* A, const void* B, void* C, int M, int N, int K, int lda, int ldb,
                     int ldc, DeviceState& d, cudaStream_t stream, const EpiArgs* epi,
                     const Scratch* scratch) {
#define B200_SKW(MP) \
  launch_skinny<MP, kSlabs>(A, B, C, M, N, K, lda, ldb, ldc, d, stream, epi, scratch)
  if (M <= 16) return B200_SKW(16);
  if (M <= 32) return B200_SKW(32);
  if (M <= 64) return B200_SKW(64);
  if (M <= 128) return B200_SKW(128);
  return B200_SKW(256);
#undef B200_SKW
}

// K slabs per stage of the skinny kernel (B200_GEMM_SKINNY_SLABS: 1, 2, 4).
int skinny_slabs() {
  static const int s = env_int("B200_GEMM_SKINNY_SLABS", 2, 1, 4);
  return s;
}

// Cluster split-K: the largest cluster (8, 4, 2, 1 CTAs; pair kernels 8, 4,
// 2) whose grid of tiles x cluster-size CTAs fits in one wave, keeping >= 8
// K blocks per slice; a forced slice count (b200_gemm_set_splits) picks the
// cluster whose slice count is the largest power of two not above it.
// Returns log2 of the cluster size.
int skc_choose(const DeviceState& d, int I, bool pair, long long tiles, int k_blocks) {
  const int lo = pair ? 1 : 0;
  const int forced = tuning_splits();
  if (forced > 0) {
    int ci = lo;
    while (ci < 3 && ((2 << ci) >> lo) <= forced) ++ci;
    return ci;
  }
  for (int c = 3; c > lo; --c) {
    const long long clusters = d.sk_clusters[I][c];
    if (clusters > 0 && tiles <= clusters && k_blocks >= 8 * ((1 << c) >> lo)) return c;
  }
  return lo;
}

template <int I>
int launch_skinny_cluster(const void* A, const void* B, void* C, int M, int N, int K, int lda,
                          int ldb, int ldc, DeviceState& d, cudaStream_t stream) {
  using S = Skc<I>;
  const long long tiles = ceil_div(N, S::P::kBlockRows);
  const int k_blocks = (int)ceil_div(K, kSlabK);
  const int ci = skc_choose(d, I, S::kPair, tiles, k_blocks);
  if (d.sk_clusters[I][ci] < 1) return B200_ERR_LAUNCH;
  const int csize = 1 << ci;
  const int slices = S::kPair ? csize / 2 : csize;
  CUtensorMap tb, ta;
  if (encode_2d(&tb, B, K, N, ldb, kSlabK, S::P::kRowsB) != B200_OK ||
      encode_2d(&ta, A, K, M, lda, kSlabK, S::P::kRowsA) != B200_OK)
    return B200_ERR_TENSOR_MAP;
  SkinnyClusterArgs args;
  args.l2_hint = skinny_l2_hint();
  args.M = M;
  args.N = N;
  args.K = K;
  args.k_blocks = k_blocks;
  args.kb_per = (int)ceil_div(k_blocks, slices);
  args.ldc = ldc;
  args.C = static_cast<__nv_bfloat16*>(C);
  args.status = d.status;
  args.timeout_ns = g_timeout_ns.load();
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(tiles * csize), 1, 1);
  cfg.blockDim = dim3(S::P::kThreads, 1, 1);
  cfg.dynamicSmemBytes = S::P::kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = (unsigned)csize;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, S::kernel, tb, ta, args) != cudaSuccess) {
    cudaGetLastError();
    return B200_ERR_LAUNCH;
  }
  return B200_OK;
}

// Ring-depth preference of the cluster kernels: 1 = one deep ring per SM
// (default, measured faster), 2 = two CTAs per SM where the M bucket allows.
int skinny_occupancy() {
  static const int o = env_int("B200_GEMM_SKINNY_OCC", 1, 1, 2);
  return o;
}

int run_skinny_cluster(const void* A, const void* B, void* C, int M, int N, int K, int lda,
                       int ldb, int ldc, DeviceState& d, cudaStream_t stream, bool pair = false) {
#define B200_SKC(I) launch_skinny_cluster<I>(A, B, C, M, N, K, lda, ldb, ldc, d, stream)
  if (pair) {
    if (M <= 32) return B200_SKC(kSkcPair0);
    if (M <= 64) return B200_SKC(kSkcPair0 + 1);
    if (M <= 128) return B200_SKC(kSkcPair0 + 2);
    return B200_SKC(kSkcPair0 + 3);
  }
  switch (skc_slot(M)) {
    case 0: return B200_SKC(0);
    case 1: return B200_SKC(1);
    case 2: return B200_SKC(2);
    case 3: return B200_SKC(3);
    case 4: return B200_SKC(4);
    case 5: return B200_SKC(5);
    case 6: return B200_SKC(6);
    default: return B200_SKC(7);
  }
#undef B200_SKC
}

int run_skinny(const void* A, const void* B, void* C, int M, int N, int K, int lda, int ldb,
               int ldc, DeviceState& d, cudaStream_t stream, const EpiArgs* epi = nullptr,
               const Scratch* scratch = nullptr) {
  // Per shape (mode 1): the single-launch cluster kernel, on 2-CTA pairs
  // above 128 rows of A where that fits with two slices at most
  // (skinny_use_pair_cluster), else on single CTAs where its grid fits one
  // wave (skinny_use_cluster); otherwise up to 128 rows the stream-K kernel
  // (all SMs, no workspace clear or rounding pass), above it the stream-K
  // kernel on 2-CTA pairs for wide B, else the persistent split-K kernel.
  // B200_GEMM_SKINNY = 2..5 forces one kernel for every M.  (The cluster
  // kernel writes C directly, so fused epilogues take the workspace kernel,
  // whose rounding pass applies them.)
  const int mode = skinny_mode();
  if (epi == nullptr && mode == 1) {
    if (skinny_use_pair_cluster(M, N, K, &d))
      return run_skinny_cluster(A, B, C, M, N, K, lda, ldb, ldc, d, stream, true);
    if (skinny_use_cluster(M, N, K, &d))
      return run_skinny_cluster(A, B, C, M, N, K, lda, ldb, ldc, d, stream);
  }
  // (a forced slice count, b200_gemm_set_splits, takes the split-K kernels)
  const bool pair = mode == 4 || (mode == 1 && skinny_use_pair_stream(M, N, K));
  if (epi == nullptr && (mode == 3 || pair || (mode == 1 && skinny_use_stream(M, N, K, &d)))) {
    switch (skinny_slabs()) {
      case 1: return run_skinny_stream_slabs<1>(A, B, C, M, N, K, lda, ldb, ldc, d, stream, scratch, pair);
      case 4: return run_skinny_stream_slabs<4>(A, B, C, M, N, K, lda, ldb, ldc, d, stream, scratch, pair);
      default: return run_skinny_stream_slabs<2>(A, B, C, M, N, K, lda, ldb, ldc, d, stream, scratch, pair);
    }
  }
  if (epi == nullptr && mode == 5)
    return run_skinny_cluster(A, B, C, M, N, K, lda, ldb, ldc, d, stream, true);
  if (epi == nullptr && mode == 2)
    return run_skinny_cluster(A, B, C, M, N, K, lda, ldb, ldc, d, stream);
  switch (skinny_slabs()) {
    case 1: return run_skinny_slabs<1>(A, B, C, M, N, K, lda, ldb, ldc, d, stream, epi, scratch);
    case 4: return run_skinny_slabs<4>(A, B, C, M, N, K, lda, ldb, ldc, d, stream, epi, scratch);
    default: return run_skinny_slabs<2>(A, B, C, M, N, K, lda, ldb, ldc, d, stream, epi, scratch);
  }
}

// Skinny path for M <= 256 when B is large enough to need every SM and K
// deep enough to be worth streaming (B200_GEMM_SKINNY=0 disables it).
bool use_skinny(int M, int N, int K) {
  return skinny_mode() != 0 && M <= kSkinnyMaxM && N >= 1024 && K >= 512;
}

// K slices a skinny call uses (for reporting): the cluster size of the
// cluster kernel (M <= 16), else the persistent kernel's slice count.  Without
// a device, 148 SMs are assumed and the persistent kernel is reported.
int skinny_slices(int M, int N, int K, const DeviceState* d) {
  const int mode = skinny_mode();
  const int forced = tuning_splits();
  const long long tiles = ceil_div(N, 128);
  if (d && (mode == 5 || (mode == 1 && skinny_use_pair_cluster(M, N, K, d)))) {
    const int I = kSkcPair0 + (M <= 32 ? 0 : M <= 64 ? 1 : M <= 128 ? 2 : 3);
    return (1 << skc_choose(*d, I, true, ceil_div(N, 256), (int)ceil_div(K, kSlabK))) / 2;
  }
  if (d && (mode == 2 || (mode == 1 && skinny_use_cluster(M, N, K, d))))
    return 1 << skc_choose(*d, skc_slot(M), false, tiles, (int)ceil_div(K, kSlabK));
  const int mp = M <= 16 ? 16 : M <= 32 ? 32 : M <= 64 ? 64 : M <= 128 ? 128 : 256;
  const bool pair_stream = mode == 4 || (mode == 1 && skinny_use_pair_stream(M, N, K));
  if (mode == 3 || pair_stream || (mode == 1 && skinny_use_stream(M, N, K, d))) {
    // stream-K: the most CTAs (pairs) any one tile of B is cut between
    const bool pair = pair_stream;
    const int st = pair ? 2 : skinny_stream_tiles(M);
    const int pmp = pair && mp < 32 ? 32 : mp;
    const long long kb = ceil_div(K, skinny_fit_slabs(pmp, skinny_slabs(), pair ? 1 : st) * kSlabK);
    const long long stiles = ceil_div(N, 128LL * st);
    const long long total = stiles * kb;
    const int workers = (d ? d->sms : 148) / (pair ? 2 : 1);
    const int G = (int)(total < workers ? total : workers);
    long long most = 1;
    for (long long t = 0; t < stiles; ++t) {
      const long long c = stream_owner_host(t * kb + kb - 1, total, G) -
                          stream_owner_host(t * kb, total, G) + 1;
      if (c > most) most = c;
    }
    return (int)most;
  }
  const int nt = skinny_tiles(mp);
  const int k_blocks = (int)ceil_div(K, skinny_fit_slabs(mp, skinny_slabs(), nt) * kSlabK);
  const int s = choose_skinny_splits(ceil_div(tiles, nt), k_blocks, d ? d->sms : 148, M, N, K);
  return (int)ceil_div(k_blocks, ceil_div(k_blocks, s));
}

GemmArgs base_args(int M, int N, int K, const DeviceState& d, long long* prof, int entries) {
  GemmArgs args;
  args.M = M;
  args.N = N;
  args.K = K;
  args.tiles_m = (int)ceil_div(M, kPairM);
  args.tiles_n = 0;
  args.k_blocks = 0;
  args.group = raster_group();
  args.splits = 1;
  args.kb_per_split = 0;
  args.status = d.status;
  args.timeout_ns = g_timeout_ns.load();
  args.prof = prof;
  args.prof_entries = entries;
  args.epi = {1.0f, 0.0f, nullptr, nullptr, 0};
  args.dp_tiles = 0;
  args.sk_tiles = 0;
  args.sk_items = 0;
  args.sk_slots = nullptr;
  args.sk_flags = nullptr;
  args.sk_epoch = 0;
  args.sched = nullptr;
  // Operand loads are marked evict-last: at 8192^3 (and the projection
  // shapes) that keeps A and B ahead of the output and of other data in L2
  // and was measured ~2% faster, at equal power, than the default policy.
  // B200_GEMM_L2_A / B200_GEMM_L2_B = 0 (normal), 1 (evict-first), 2 (evict-last).
  static const int l2_a = env_int("B200_GEMM_L2_A", 2, 0, 2);
  static const int l2_b = env_int("B200_GEMM_L2_B", 2, 0, 2);
  args.l2_a = l2_a;
  args.l2_b = l2_b;
  return args;
}

template <bool kProfile>
int run_gemm(const void* A, const void* B, void* C, int M, int N, int K, int lda, int ldb,
             int ldc, long long* prof, int prof_entries, cudaStream_t stream,
             const EpiArgs* epi = nullptr) {
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

  if (!kProfile && use_skinny(M, N, K))
    return run_skinny(A, B, C, M, N, K, lda, ldb, ldc, *d, stream, epi);
  GemmArgs args = base_args(M, N, K, *d, prof, prof_entries);
  if (epi) args.epi = *epi;
  // Split-K (not with the profiler): tiles accumulate their K slices into a
  // zeroed fp32 workspace by TMA reduce-add, then one pass rounds to bf16.
  if (!kProfile) {
    const int splits = choose_splits(M, N, (int)ceil_div(K, kSlabK), d->max_pairs[kV256x64]);
    if (splits > 1) {
      const int ldw = (int)ceil_div(N, 8) * 8;
      const size_t bytes = (size_t)M * ldw * sizeof(float);
      float* W = nullptr;
      if (cudaMallocFromPoolAsync(reinterpret_cast<void**>(&W), bytes, d->pool, stream) !=
          cudaSuccess) {
        cudaGetLastError();
        return B200_ERR_LAUNCH;
      }
      st = encode_2d(&tc, W, N, M, ldw, 32, 32, true);
      if (st == B200_OK && cudaMemsetAsync(W, 0, bytes, stream) != cudaSuccess)
        st = B200_ERR_LAUNCH;
      if (st == B200_OK) st = launch<false, kV256x64, kOutF32Add>(ta, tb, tc, args, splits, *d,
                                                                   stream);
      if (st == B200_OK) st = cast_to_bf16(W, ldw, C, ldc, M, N, d->sms, stream, epi);
      cudaFreeAsync(W, stream);
      return st;
    }
  }
  if (!kProfile && epi) return launch<false, kV256x64, kOutBf16Epi>(ta, tb, tc, args, 1, *d, stream);
  return launch_bf16<kProfile>(choose_variant(M, N, K, d->max_pairs), ta, tb, tc, B, ldb, args, *d,
                               stream);
}

// fp32 C = A * B^T (no rounding), 256 x 256 tiles: the K-split partials.
int run_gemm_f32out(const void* A, const void* B, float* C, int M, int N, int K, int lda,
                    int ldb, int ldc, cudaStream_t stream) {
  int st = validate(A, B, C, M, N, K, lda, ldb, ldc, true);
  if (st != B200_OK) return st;
  if (M == 0 || N == 0) return B200_OK;
  DeviceState* d = nullptr;
  st = device_state(&d);
  if (st != B200_OK) return st;
  if (K == 0)
    return cudaMemset2DAsync(C, (size_t)ldc * 4, 0, (size_t)N * 4, M, stream) == cudaSuccess
               ? B200_OK
               : B200_ERR_LAUNCH;
  CUtensorMap ta, tb, tc;
  if (encode_2d(&ta, A, K, M, lda, kSlabK, kCtaM) != B200_OK ||
      encode_2d(&tb, B, K, N, ldb, kSlabK, kCtaN) != B200_OK ||
      encode_2d(&tc, C, N, M, ldc, 32, 32, true) != B200_OK)
    return B200_ERR_TENSOR_MAP;
  GemmArgs args = base_args(M, N, K, *d, nullptr, 0);
  return launch<false, kV256x64, kOutF32>(ta, tb, tc, args, 1, *d, stream);
}

// ---------------------------------------------------------------------------
// Host-resident operands.  A and B go up in blocks of rows, alternately
// (A_0, B_0, A_1, B_1, ...), into full device copies; the GEMM of C block
// (i, j) = A_i B_j^T goes out as soon as both blocks are up, and that block of
// C comes back as soon as it is done.  Uploads, GEMMs and downloads run on
// three streams of their own (events order them and the reuse of four
// rotating C buffers), so the link carries data both ways from the first
// blocks on and the GEMMs hide under the transfers.  The pipeline is ordered
// after the caller's stream at entry and the caller's stream waits for its
// end, so the call is asynchronous like the others.
struct HostPipe {
  bool ready = false;
  cudaStream_t up = nullptr, mm = nullptr, down = nullptr;
};
HostPipe g_pipe[kMaxDevices];

int host_pipe(HostPipe** out) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    cudaGetLastError();
    return B200_ERR_UNSUPPORTED_DEVICE;
  }
  std::lock_guard<std::mutex> lock(g_mu);
  HostPipe& p = g_pipe[dev];
  if (!p.ready) {
    if (cudaStreamCreateWithFlags(&p.up, cudaStreamNonBlocking) != cudaSuccess ||
        cudaStreamCreateWithFlags(&p.mm, cudaStreamNonBlocking) != cudaSuccess ||
        cudaStreamCreateWithFlags(&p.down, cudaStreamNonBlocking) != cudaSuccess) {
      cudaGetLastError();
      return B200_ERR_LAUNCH;
    }
    p.ready = true;
  }
  *out = &p;
  return B200_OK;
}

// rows x width bytes between pitched buffers: one linear copy where both
// sides are contiguous, else a pitched copy.  (Measured the same as pitched
// copies throughout: 8192^3 with one block, 7.97 ms per call on one GPU, 22.2
// ms with eight GPUs sharing the host, both before and after.)
cudaError_t copy_rows(void* dst, size_t dpitch, const void* src, size_t spitch, size_t width,
                      size_t rows, cudaMemcpyKind kind, cudaStream_t stream) {
  if ((dpitch == width && spitch == width) || rows == 1)
    return cudaMemcpyAsync(dst, src, width * rows, kind, stream);
  return cudaMemcpy2DAsync(dst, dpitch, src, spitch, width, rows, kind, stream);
}

int run_gemm_host(const void* A, const void* B, void* C, int M, int N, int K, int lda, int ldb,
                  int ldc, int block_rows, cudaStream_t stream) {
  if (M < 0 || N < 0 || K < 0 || block_rows < 0) return B200_ERR_INVALID_ARGUMENT;
  if (M == 0 || N == 0) return B200_OK;
  if (!C || (K > 0 && (!A || !B)) || ldc < N || (K > 0 && (lda < K || ldb < K)))
    return B200_ERR_INVALID_ARGUMENT;
  DeviceState* d = nullptr;
  int st = device_state(&d);
  if (st != B200_OK) return st;
  HostPipe* p = nullptr;
  st = host_pipe(&p);
  if (st != B200_OK) return st;
  if (block_rows == 0) {
    const int big = M > N ? M : N;
    block_rows = (int)(ceil_div(ceil_div(big, 4), kPairM) * kPairM);
  }
  const int br = block_rows < M ? block_rows : M;                      // rows of A per block
  const int bc = (int)(ceil_div(block_rows < N ? block_rows : N, 8) * 8);  // rows of B per block
  const int mb = (int)ceil_div(M, br), nb = (int)ceil_div(N, bc);
  const int pairs = mb * nb;
  constexpr int kCBufs = 4;
  const int ncb = pairs < kCBufs ? pairs : kCBufs;
  const int kd = (int)ceil_div(K > 0 ? K : 1, 8) * 8;  // device row strides: 16-byte multiples
  const int cld = (int)ceil_div(bc, 8) * 8;
  const size_t a_bytes = (size_t)M * kd * 2, b_bytes = (size_t)N * kd * 2;
  const size_t c_bytes = (size_t)br * cld * 2;
  const size_t total = a_bytes + b_bytes + ncb * c_bytes;

  const int nev = 2 + mb + nb + 2 * pairs;
  cudaEvent_t* ev = new cudaEvent_t[nev];
  int made = 0;
  for (; made < nev; ++made)
    if (cudaEventCreateWithFlags(&ev[made], cudaEventDisableTiming) != cudaSuccess) break;
  auto finish = [&](int status) {
    for (int i = 0; i < made; ++i) cudaEventDestroy(ev[i]);
    delete[] ev;
    if (status != B200_OK) cudaGetLastError();
    return status;
  };
  if (made < nev) return finish(B200_ERR_LAUNCH);
  cudaEvent_t ev_start = ev[0], ev_end = ev[1];
  cudaEvent_t* ev_a = ev + 2;                 // A block i uploaded
  cudaEvent_t* ev_b = ev_a + mb;              // B block j uploaded
  cudaEvent_t* ev_mm = ev_b + nb;             // GEMM q done
  cudaEvent_t* ev_down = ev_mm + pairs;       // C block q downloaded

  bool ok = cudaEventRecord(ev_start, stream) == cudaSuccess &&
            cudaStreamWaitEvent(p->up, ev_start, 0) == cudaSuccess &&
            cudaStreamWaitEvent(p->mm, ev_start, 0) == cudaSuccess &&
            cudaStreamWaitEvent(p->down, ev_start, 0) == cudaSuccess;
  char* ws = nullptr;
  if (ok) ok = cudaMallocFromPoolAsync(reinterpret_cast<void**>(&ws), total, d->pool, p->up) ==
               cudaSuccess;
  if (!ok) return finish(B200_ERR_LAUNCH);
  char* dA = ws;
  char* dB = ws + a_bytes;
  char* dC = dB + b_bytes;
  int q = 0;  // GEMMs issued so far
  // GEMM of C block (i, j) and the download of its rows and columns.
  auto issue = [&](int i, int j) {
    const int r0 = i * br, rows = M - r0 < br ? M - r0 : br;
    const int c0 = j * bc, cols = N - c0 < bc ? N - c0 : bc;
    char* cb = dC + (size_t)(q % ncb) * c_bytes;
    bool good = cudaStreamWaitEvent(p->mm, ev_a[i], 0) == cudaSuccess &&
                cudaStreamWaitEvent(p->mm, ev_b[j], 0) == cudaSuccess;
    if (good && q >= ncb) good = cudaStreamWaitEvent(p->mm, ev_down[q - ncb], 0) == cudaSuccess;
    if (good)
      good = run_gemm<false>(dA + (size_t)r0 * kd * 2, dB + (size_t)c0 * kd * 2, cb, rows, cols, K,
                             kd, kd, cld, nullptr, 0, p->mm) == B200_OK;
    good = good && cudaEventRecord(ev_mm[q], p->mm) == cudaSuccess &&
           cudaStreamWaitEvent(p->down, ev_mm[q], 0) == cudaSuccess &&
           copy_rows(static_cast<char*>(C) + ((size_t)r0 * ldc + c0) * 2, (size_t)ldc * 2, cb,
                     (size_t)cld * 2, (size_t)cols * 2, rows, cudaMemcpyDeviceToHost,
                     p->down) == cudaSuccess &&
           cudaEventRecord(ev_down[q], p->down) == cudaSuccess;
    ++q;
    return good;
  };
  // Upload A_0, B_0, A_1, B_1, ...; each GEMM goes out once its two blocks are up.
  const int steps = mb > nb ? mb : nb;
  for (int s2 = 0; ok && s2 < steps; ++s2) {
    if (s2 < mb) {
      const int r0 = s2 * br, rows = M - r0 < br ? M - r0 : br;
      if (K > 0)
        ok = copy_rows(dA + (size_t)r0 * kd * 2, (size_t)kd * 2,
                       static_cast<const char*>(A) + (size_t)r0 * lda * 2, (size_t)lda * 2,
                       (size_t)K * 2, rows, cudaMemcpyHostToDevice, p->up) == cudaSuccess;
      ok = ok && cudaEventRecord(ev_a[s2], p->up) == cudaSuccess;
      for (int j = 0; ok && j < s2 && j < nb; ++j) ok = issue(s2, j);
    }
    if (ok && s2 < nb) {
      const int c0 = s2 * bc, cols = N - c0 < bc ? N - c0 : bc;
      if (K > 0)
        ok = copy_rows(dB + (size_t)c0 * kd * 2, (size_t)kd * 2,
                       static_cast<const char*>(B) + (size_t)c0 * ldb * 2, (size_t)ldb * 2,
                       (size_t)K * 2, cols, cudaMemcpyHostToDevice, p->up) == cudaSuccess;
      ok = ok && cudaEventRecord(ev_b[s2], p->up) == cudaSuccess;
      for (int i = 0; ok && i <= s2 && i < mb; ++i) ok = issue(i, s2);
    }
  }
  // Join, after an error too (work already queued may still use the device
  // buffers and the caller's host memory): the download stream follows the
  // other two, frees the buffers and releases the caller's stream.  Where an
  // ordering step itself fails, the pipeline's streams are drained instead,
  // so nothing of this call is in flight when it returns an error.
  const bool joined = cudaEventRecord(ev_start, p->up) == cudaSuccess &&
                      cudaStreamWaitEvent(p->down, ev_start, 0) == cudaSuccess &&
                      cudaEventRecord(ev_mm[pairs - 1], p->mm) == cudaSuccess &&
                      cudaStreamWaitEvent(p->down, ev_mm[pairs - 1], 0) == cudaSuccess;
  if (!joined) {
    cudaGetLastError();
    cudaStreamSynchronize(p->up);
    cudaStreamSynchronize(p->mm);
  }
  cudaFreeAsync(ws, p->down);
  const bool released = cudaEventRecord(ev_end, p->down) == cudaSuccess &&
                        cudaStreamWaitEvent(stream, ev_end, 0) == cudaSuccess;
  if (!released) {
    cudaGetLastError();
    cudaStreamSynchronize(p->down);
  }
  return finish(ok && joined && released ? B200_OK : B200_ERR_LAUNCH);
}

// ---------------------------------------------------------------------------
// Fused K-split over NVLink (device side: ksplit_fused.cuh).
//
// Exchange blob (B200_KSPLIT_HANDLE_BYTES) that each rank publishes: the IPC
// handle of its receive area plus what the peers check before mapping it.
struct KsplitBlob {
  uint32_t magic;
  int32_t rank, nranks, device;
  int64_t cap_pieces;
  uint64_t bytes, flag_bytes;
  cudaIpcMemHandle_t handle;
};
constexpr uint32_t kKsplitMagic = 0x4b533230u;  // "02SK"
static_assert(sizeof(KsplitBlob) <= B200_KSPLIT_HANDLE_BYTES, "exchange blob too large");

// Pieces (32 x 256 fp32 epilogue-warp slices) per owner for an M x N call
// with pair tiles `tile_n` wide (the last tile's sub-tiles all count).
long long ks_pieces(long long M, long long N, int nranks, int tile_n) {
  return M / nranks / kPairM * ceil_div(N, tile_n) * (tile_n / kSubN) * 8;
}

}  // namespace

struct b200_ksplit_comm {
  int device = -1, rank = 0, nranks = 1;
  long long cap_pieces = 0;
  size_t bytes = 0, flag_bytes = 0;
  char* base = nullptr;                 // this rank's receive area
  char* mapped[kMaxRanks] = {};         // every rank's receive area as mapped here
  unsigned int epoch = 0;               // calls made so far
  bool connected = false;
};

namespace {

// Run `fn` with `dev` as the current device, restoring the caller's.
template <class F>
int on_device(int dev, F fn) {
  int prev = -1;
  if (cudaGetDevice(&prev) != cudaSuccess) {
    cudaGetLastError();
    return B200_ERR_UNSUPPORTED_DEVICE;
  }
  if (prev != dev && cudaSetDevice(dev) != cudaSuccess) {
    cudaGetLastError();
    return B200_ERR_UNSUPPORTED_DEVICE;
  }
  const int st = fn();
  if (prev != dev) cudaSetDevice(prev);
  return st;
}

int run_ksplit(b200_ksplit_comm* c, const void* A, const void* B, void* C, int M, int N, int K,
               int lda, int ldb, int ldc, cudaStream_t stream) {
  if (!c || !c->connected) return B200_ERR_INVALID_ARGUMENT;
  if (M <= 0 || N <= 0 || K <= 0 || M % (kPairM * c->nranks) != 0) return B200_ERR_INVALID_ARGUMENT;
  const int rows = M / c->nranks;
  int st = validate(A, B, C, rows, N, K, lda, ldb, ldc);
  if (st != B200_OK) return st;
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev != c->device) {
    cudaGetLastError();
    return B200_ERR_INVALID_ARGUMENT;
  }
  // Pair tiles: 512 wide unless that costs wave efficiency (as for the plain
  // GEMM); the 256-wide kernel overlaps each tile's epilogue with the next
  // tile's MMAs, the 512-wide one reads 25% fewer operand bytes per FLOP.
  DeviceState* d = nullptr;
  st = device_state(&d);
  if (st != B200_OK) return st;
  const bool wide = choose_variant(M, N, K, d->max_pairs) == kV512x64;
  const long long pieces = ks_pieces(M, N, c->nranks, wide ? 2 * kSubN : kSubN);
  if (pieces > c->cap_pieces) return B200_ERR_TOO_LARGE;
  CUtensorMap ta, tb, tc;
  if (encode_2d(&ta, A, K, M, lda, kSlabK, kCtaM) != B200_OK ||
      encode_2d(&tb, B, K, N, ldb, kSlabK, kCtaN) != B200_OK ||
      encode_2d(&tc, C, N, rows, ldc, kStoreCols, 32) != B200_OK)
    return B200_ERR_TENSOR_MAP;
  GemmArgs args = base_args(M, N, K, *d, nullptr, 0);
  KsArgs& ks = args.ks;
  ks.rank = c->rank;
  ks.nranks = c->nranks;
  ks.tiles_m_own = rows / kPairM;
  ks.pieces = (int)pieces;
  ks.epoch = c->epoch + 1;
  ks.parity = (int)(ks.epoch & 1u);
  // Peers may reach the call later than this rank (host skew, first-call
  // set-up): their pieces get five times the pipeline's bound (10 s by
  // default).
  ks.peer_timeout_ns = 5ull * g_timeout_ns.load();
  for (int q = 0; q < kMaxRanks; ++q) {
    ks.recv[q] = nullptr;
    ks.flags[q] = nullptr;
  }
  for (int q = 0; q < c->nranks; ++q) {
    ks.flags[q] = reinterpret_cast<unsigned int*>(c->mapped[q]);
    ks.recv[q] = reinterpret_cast<float*>(c->mapped[q] + c->flag_bytes);
  }
  st = wide ? launch<false, kV512x64, kOutKsplit>(ta, tb, tc, args, 1, *d, stream)
            : launch<false, kV256x64, kOutKsplit>(ta, tb, tc, args, 1, *d, stream);
  if (st == B200_OK) c->epoch = ks.epoch;  // the epoch is spent once the kernel is queued
  return st;
}

template <int V>
void shape_of(long long* tile_n, int* smem, int* threads) {
  using C = typename VariantCfg<V>::C;
  *tile_n = C::kTileN;
  *smem = C::kSmemBytes;
  *threads = C::kThreads;
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

int b200_gemm_bf16_f32out(const void* A, const void* B, float* C, int M, int N, int K, int lda,
                          int ldb, int ldc, void* stream) {
  return run_gemm_f32out(A, B, C, M, N, K, lda, ldb, ldc, static_cast<cudaStream_t>(stream));
}

int b200_gemm_bf16_epilogue(const void* A, const void* B, void* C, int M, int N, int K, int lda,
                            int ldb, int ldc, float alpha, const void* bias, float beta,
                            const void* residual, int ldr, void* stream) {
  if (bias && !aligned16(bias)) return B200_ERR_ALIGNMENT;
  if (residual && (!aligned16(residual) || (ldr & 7))) return B200_ERR_ALIGNMENT;
  if (residual && ldr < N) return B200_ERR_INVALID_ARGUMENT;
  const EpiArgs epi = {alpha, beta, static_cast<const __nv_bfloat16*>(bias),
                       static_cast<const __nv_bfloat16*>(residual), ldr};
  return run_gemm<false>(A, B, C, M, N, K, lda, ldb, ldc, nullptr, 0,
                         static_cast<cudaStream_t>(stream), &epi);
}

int b200_gemm_bf16_host(const void* A, const void* B, void* C, int M, int N, int K, int lda,
                        int ldb, int ldc, int block_rows, void* stream) {
  return run_gemm_host(A, B, C, M, N, K, lda, ldb, ldc, block_rows,
                       static_cast<cudaStream_t>(stream));
}

int b200_cast_f32_bf16(const float* W, int ldw, void* C, int ldc, int M, int N, void* stream) {
  if (M < 0 || N < 0 || ldw < N || ldc < N) return B200_ERR_INVALID_ARGUMENT;
  if (M == 0 || N == 0) return B200_OK;
  if (!W || !C) return B200_ERR_INVALID_ARGUMENT;
  if (!aligned16(W) || !aligned16(C) || (ldw & 3) || (ldc & 7)) return B200_ERR_ALIGNMENT;
  DeviceState* d = nullptr;
  const int st = device_state(&d);
  if (st != B200_OK) return st;
  return cast_to_bf16(W, ldw, C, ldc, M, N, d->sms, static_cast<cudaStream_t>(stream));
}

int b200_gemm_launch_shape(int M, int N, int K, int* tiles, int* grid, int* smem_bytes,
                           int* threads) {
  if (M < 0 || N < 0 || K < 0) return B200_ERR_INVALID_ARGUMENT;
  DeviceState* d = nullptr;
  const bool have_dev = device_state(&d) == B200_OK;
  const int v = choose_variant(M, N, K, have_dev ? d->max_pairs : nullptr);
  long long tile_n;
  int smem, thr;
  if (v == kV512x64) shape_of<kV512x64>(&tile_n, &smem, &thr);
  else if (v == kV256x128) shape_of<kV256x128>(&tile_n, &smem, &thr);
  else if (v == kV128x64) shape_of<kV128x64>(&tile_n, &smem, &thr);
  else if (v == kV64x64) shape_of<kV64x64>(&tile_n, &smem, &thr);
  else shape_of<kV256x64>(&tile_n, &smem, &thr);
  const long long t = ceil_div(M, kPairM) * ceil_div(N, tile_n);
  if (tiles) *tiles = (int)t;
  if (smem_bytes) *smem_bytes = smem;
  if (threads) *threads = thr;
  if (grid) {
    *grid = 0;
    if (t > 0 && K > 0 && have_dev) *grid = 2 * (int)(t < d->max_pairs[v] ? t : d->max_pairs[v]);
  }
  return B200_OK;
}

int b200_gemm_profile_rows(int M, int N, int K, int* rows) {
  if (!rows) return B200_ERR_INVALID_ARGUMENT;
  int grid = 0, threads = 0;
  const int st = b200_gemm_launch_shape(M, N, K, nullptr, &grid, nullptr, &threads);
  if (st != B200_OK) return st;
  *rows = grid * (threads / 32);
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

int b200_gemm_set_tuning(int tile_n, int stage_slabs, int raster_group) {
  if ((tile_n != 0 && tile_n != -1 && tile_n != 64 && tile_n != 128 && tile_n != 256 &&
       tile_n != 512) ||
      stage_slabs < 0 ||
      stage_slabs > 2)
    return B200_ERR_INVALID_ARGUMENT;
  if (tile_n == -1) g_tile_n.store(0);
  else if (tile_n != 0) g_tile_n.store(tile_n);
  if (stage_slabs > 0) g_slabs.store(stage_slabs);
  if (raster_group != 0) g_group.store(raster_group);
  return B200_OK;
}

int b200_gemm_set_stream_k(int mode) {
  if (mode < 0 || mode > 2) return B200_ERR_INVALID_ARGUMENT;
  g_streamk.store(mode);
  return B200_OK;
}

int b200_gemm_set_dynamic(int mode) {
  if (mode < 0 || mode > 1) return B200_ERR_INVALID_ARGUMENT;
  g_dynamic.store(mode);
  return B200_OK;
}

int b200_gemm_set_skinny_tiles(int tiles) {
  if (tiles < 0 || tiles > 2) return B200_ERR_INVALID_ARGUMENT;
  g_skinny_tiles.store(tiles);
  return B200_OK;
}

int b200_gemm_set_skinny_mode(int mode) {
  if (mode < 0 || mode > 5) return B200_ERR_INVALID_ARGUMENT;
  g_skinny.store(mode);
  return B200_OK;
}

int b200_gemm_set_splits(int splits) {
  if (splits < 0 || splits > 64) return B200_ERR_INVALID_ARGUMENT;
  g_splits.store(splits);
  return B200_OK;
}

int b200_gemm_get_splits(int M, int N, int K, int* splits) {
  if (!splits || M < 0 || N < 0 || K < 0) return B200_ERR_INVALID_ARGUMENT;
  DeviceState* d = nullptr;
  const bool have_dev = device_state(&d) == B200_OK;
  if (M == 0 || N == 0 || K == 0) *splits = 1;
  else if (use_skinny(M, N, K)) *splits = skinny_slices(M, N, K, have_dev ? d : nullptr);
  else *splits = choose_splits(M, N, (int)ceil_div(K, kSlabK), have_dev ? d->max_pairs[kV256x64] : 74);
  return B200_OK;
}

int b200_gemm_get_tuning(int* tile_n, int* stage_slabs_out, int* raster_group_out) {
  if (tile_n) *tile_n = tuning_tile_n();
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

int b200_gemm_sk_range_pairs(long long items, int pairs) { return sk_range_pairs(items, pairs); }

void b200_gemm_sk_range(int pair, long long items, int range_pairs, long long* lo,
                        long long* hi) {
  sk_range(pair, items, range_pairs, lo, hi);
}

int b200_gemm_sk_owner(long long x, long long items, int range_pairs) {
  return sk_owner(x, items, range_pairs);
}

void b200_gemm_sk_next_segment(long long lo, long long* pos, int k_blocks, int* t, int* kb0,
                               int* kb1) {
  sk_next_segment(lo, pos, k_blocks, t, kb0, kb1);
}

uint64_t b200_gemm_smem_desc(uint32_t smem_addr) { return make_sdesc_k128(smem_addr); }

int b200_ksplit_create(int rank, int nranks, int max_m, int max_n, b200_ksplit_comm** comm,
                       void* handle) {
  if (!comm || !handle) return B200_ERR_INVALID_ARGUMENT;
  *comm = nullptr;
  if (nranks < 1 || nranks > kMaxRanks || rank < 0 || rank >= nranks || max_n <= 0 ||
      max_m <= 0 || max_m % (kPairM * nranks) != 0)
    return B200_ERR_INVALID_ARGUMENT;
  DeviceState* d = nullptr;
  int st = device_state(&d);
  if (st != B200_OK) return st;
  if (!set_smem_limit<false, kV256x64, kOutKsplit>() ||
      !set_smem_limit<false, kV512x64, kOutKsplit>())
    return B200_ERR_LAUNCH;
  b200_ksplit_comm* c = new b200_ksplit_comm();
  cudaGetDevice(&c->device);
  c->rank = rank;
  c->nranks = nranks;
  c->cap_pieces = ks_pieces(max_m, max_n, nranks, 2 * kSubN);  // fits either tile width
  c->flag_bytes = (size_t)ceil_div((long long)nranks * c->cap_pieces * 4, 4096) * 4096;
  c->bytes = c->flag_bytes + (size_t)2 * nranks * c->cap_pieces * kPieceFloats * sizeof(float);
  KsplitBlob blob = {};
  if (cudaMalloc(&c->base, c->bytes) != cudaSuccess ||
      cudaMemset(c->base, 0, c->flag_bytes) != cudaSuccess ||
      cudaDeviceSynchronize() != cudaSuccess ||
      cudaIpcGetMemHandle(&blob.handle, c->base) != cudaSuccess) {
    cudaGetLastError();
    if (c->base) cudaFree(c->base);
    delete c;
    return B200_ERR_LAUNCH;
  }
  c->mapped[rank] = c->base;
  blob.magic = kKsplitMagic;
  blob.rank = rank;
  blob.nranks = nranks;
  blob.device = c->device;
  blob.cap_pieces = c->cap_pieces;
  blob.bytes = c->bytes;
  blob.flag_bytes = c->flag_bytes;
  std::memset(handle, 0, B200_KSPLIT_HANDLE_BYTES);
  std::memcpy(handle, &blob, sizeof(blob));
  *comm = c;
  return B200_OK;
}

int b200_ksplit_connect(b200_ksplit_comm* c, const void* handles) {
  if (!c || !handles || c->connected) return B200_ERR_INVALID_ARGUMENT;
  const char* h = static_cast<const char*>(handles);
  for (int q = 0; q < c->nranks; ++q) {
    KsplitBlob b;
    std::memcpy(&b, h + (size_t)q * B200_KSPLIT_HANDLE_BYTES, sizeof(b));
    if (b.magic != kKsplitMagic || b.rank != q || b.nranks != c->nranks ||
        b.cap_pieces != c->cap_pieces || b.bytes != c->bytes || b.flag_bytes != c->flag_bytes)
      return B200_ERR_INVALID_ARGUMENT;
  }
  return on_device(c->device, [&]() {
    for (int q = 0; q < c->nranks; ++q) {
      if (q == c->rank) continue;
      KsplitBlob b;
      std::memcpy(&b, h + (size_t)q * B200_KSPLIT_HANDLE_BYTES, sizeof(b));
      void* p = nullptr;
      if (cudaIpcOpenMemHandle(&p, b.handle, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
        cudaGetLastError();
        for (int r = 0; r < q; ++r)
          if (r != c->rank && c->mapped[r]) {
            cudaIpcCloseMemHandle(c->mapped[r]);
            c->mapped[r] = nullptr;
          }
        return B200_ERR_LAUNCH;
      }
      c->mapped[q] = static_cast<char*>(p);
    }
    c->connected = true;
    return B200_OK;
  });
}

int b200_ksplit_gemm_bf16(b200_ksplit_comm* comm, const void* A, const void* B, void* C, int M,
                          int N, int K, int lda, int ldb, int ldc, void* stream) {
  return run_ksplit(comm, A, B, C, M, N, K, lda, ldb, ldc, static_cast<cudaStream_t>(stream));
}

int b200_ksplit_epoch(const b200_ksplit_comm* comm, unsigned int* epoch) {
  if (!comm || !epoch) return B200_ERR_INVALID_ARGUMENT;
  *epoch = comm->epoch;
  return B200_OK;
}

int b200_ksplit_destroy(b200_ksplit_comm* c) {
  if (!c) return B200_OK;
  const int st = on_device(c->device, [&]() {
    int r = cudaDeviceSynchronize() == cudaSuccess ? B200_OK : B200_ERR_LAUNCH;
    for (int q = 0; q < c->nranks; ++q)
      if (q != c->rank && c->mapped[q] && cudaIpcCloseMemHandle(c->mapped[q]) != cudaSuccess)
        r = B200_ERR_LAUNCH;
    if (c->base && cudaFree(c->base) != cudaSuccess) r = B200_ERR_LAUNCH;
    cudaGetLastError();
    return r;
  });
  delete c;
  return st;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Allocation-free entry point.
//
// Some callers cannot let a library allocate device memory: processes that
// reserve the GPU's memory up front through their own allocator or arena (a
// serving engine that sizes its caches to fill HBM leaves nothing for a
// later cudaMalloc, and a stream-ordered pool growing behind its back breaks
// its accounting), and latency-critical loops in which cudaMalloc/cudaFree
// would synchronize the device.  b200_gemm_bf16 allocates on a device's
// first call (its error word and its split-K pool) and may grow the pool on
// any split-K call; b200_gemm_bf16_noalloc computes the same GEMM with all
// of its scratch in the fixed array below, which every GPU that loads this
// library holds until exit.
//
// Layout of the scratch array (16 MiB):
//   [0, 4)            error word of the kernels this entry point launches
//                     (sticky: read and cleared by b200_gemm_noalloc_status)
//   [128, 136)        counters of the pair kernels' dynamic dealing (zero
//                     between launches: each launch's last pair resets them)
//   [256, 64 KiB)     epoch flags of the skinny stream-K kernel (only flags
//                     live here, so values left by earlier calls are older
//                     epochs and nothing needs clearing between calls)
//   [64 KiB, 16 MiB)  workspace: split-K fp32 accumulators, stream-K slots
// Split-K slice counts chosen per shape always fit (the pair kernel splits
// only grids of at most ~600 K outputs, 2.4 MB of fp32; a skinny call whose
// workspace would not fit runs the cluster kernel, which needs none); only a
// forced slice count (b200_gemm_set_splits) can need more than the
// workspace, and such a call returns B200_ERR_TOO_LARGE.
namespace {

constexpr size_t kNoAllocScratchBytes = 16u << 20;
constexpr size_t kNoAllocSchedOffset = 128;
constexpr size_t kNoAllocFlagsOffset = 256;
constexpr size_t kNoAllocWorkspaceOffset = 64u << 10;
constexpr size_t kNoAllocFlagCount = (kNoAllocWorkspaceOffset - kNoAllocFlagsOffset) / 4;
constexpr size_t kNoAllocWorkspaceBytes = kNoAllocScratchBytes - kNoAllocWorkspaceOffset;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

struct NoAllocDevice {
  bool ready = false;
  int init_status = B200_OK;
  DeviceState launch;           // sms, max_pairs, sk_clusters; status = the array's error word
  unsigned char* scratch = nullptr;  // device address of g_noalloc_scratch
  unsigned int epoch = 0;       // flag epochs handed out so far
};

std::mutex g_noalloc_mu;
NoAllocDevice g_noalloc_dev[kMaxDevices];

// Once per device, with that device current: the same architecture checks,
// shared-memory limits and occupancy queries as the allocating path (which
// also load every kernel this entry point launches), plus the device address
// of the scratch array.  None of these calls allocate.
int noalloc_setup(NoAllocDevice& nd, int dev) {
  cudaDeviceProp prop;
  if (cudaGetDeviceProperties(&prop, dev) != cudaSuccess) return B200_ERR_UNSUPPORTED_DEVICE;
  if (prop.major != 10 || prop.minor != 0) return B200_ERR_UNSUPPORTED_DEVICE;
  if (encode_tiled() == nullptr) return B200_ERR_TENSOR_MAP;
  nd.launch.sms = prop.multiProcessorCount;
  if (!set_smem_limit<false, kV256x64, kOutF32Add>() || !set_skinny_limits())
    return B200_ERR_LAUNCH;
  const int vst = init_variants(nd.launch.sms, nd.launch.max_pairs);
  if (vst != B200_OK) return vst;
  if (!skc_init_all(nd.launch)) return B200_ERR_LAUNCH;
  cudaFuncAttributes fa;
  if (cudaFuncGetAttributes(&fa, cast_f32_to_bf16_kernel) != cudaSuccess ||
      cudaFuncGetAttributes(&fa, wait_probe_kernel) != cudaSuccess)
    return B200_ERR_LAUNCH;
  // In host code g_noalloc_scratch names a host-side stand-in; the kernels
  // must be given the device address.
  void* p = nullptr;
  if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || p == nullptr)
    return B200_ERR_LAUNCH;
  nd.scratch = static_cast<unsigned char*>(p);
  nd.launch.status = reinterpret_cast<int*>(nd.scratch);
  nd.launch.pool = nullptr;
  return B200_OK;
}

int noalloc_device(NoAllocDevice** out) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    cudaGetLastError();
    return B200_ERR_UNSUPPORTED_DEVICE;
  }
  if (dev < 0 || dev >= kMaxDevices) return B200_ERR_UNSUPPORTED_DEVICE;
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  NoAllocDevice& nd = g_noalloc_dev[dev];
  if (!nd.ready) {
    nd.ready = true;
    nd.init_status = noalloc_setup(nd, dev);
    if (nd.init_status != B200_OK) cudaGetLastError();
  }
  if (nd.init_status != B200_OK) return nd.init_status;
  *out = &nd;
  return B200_OK;
}

// The scratch of one call: a new flag epoch (2, 3, ...) outside stream
// capture; under capture (a graph may be replayed with the same epoch) epoch
// 0, which makes the skinny stream-K launch clear the flags it uses on the
// stream and raise them to 1, below every epoch handed out here.  Flags are
// compared by signed difference, so a wrap of the counter keeps older epochs
// older.
Scratch noalloc_scratch(NoAllocDevice& nd, cudaStream_t stream) {
  Scratch sc;
  sc.flags = reinterpret_cast<unsigned int*>(nd.scratch + kNoAllocFlagsOffset);
  sc.flag_count = kNoAllocFlagCount;
  sc.work = reinterpret_cast<char*>(nd.scratch + kNoAllocWorkspaceOffset);
  sc.work_bytes = kNoAllocWorkspaceBytes;
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(stream, &cap) != cudaSuccess) {
    cudaGetLastError();
    cap = cudaStreamCaptureStatusActive;
  }
  if (cap == cudaStreamCaptureStatusNone) {
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (++nd.epoch < 2) nd.epoch = 2;
    sc.epoch = nd.epoch;
  }
  return sc;
}

int run_gemm_noalloc(const void* A, const void* B, void* C, int M, int N, int K, int lda,
                     int ldb, int ldc, cudaStream_t stream) {
  int st = validate(A, B, C, M, N, K, lda, ldb, ldc);
  if (st != B200_OK) return st;
  if (M == 0 || N == 0) return B200_OK;
  NoAllocDevice* nd = nullptr;
  st = noalloc_device(&nd);
  if (st != B200_OK) return st;
  if (K == 0)
    return cudaMemset2DAsync(C, (size_t)ldc * 2, 0, (size_t)N * 2, M, stream) == cudaSuccess
               ? B200_OK
               : B200_ERR_LAUNCH;
  // Skinny M: the same per-shape kernel as the allocating path, its workspace
  // (if any) in the array; where that does not fit, the cluster kernel, which
  // adds its K slices in distributed shared memory and needs no workspace.
  if (use_skinny(M, N, K)) {
    const Scratch sc = noalloc_scratch(*nd, stream);
    st = run_skinny(A, B, C, M, N, K, lda, ldb, ldc, nd->launch, stream, nullptr, &sc);
    if (st == B200_ERR_TOO_LARGE)
      st = run_skinny_cluster(A, B, C, M, N, K, lda, ldb, ldc, nd->launch, stream);
    return st;
  }
  const int splits =
      choose_splits(M, N, (int)ceil_div(K, kSlabK), nd->launch.max_pairs[kV256x64]);
  const int ldw = (int)ceil_div(N, 8) * 8;
  const size_t ws_bytes = (size_t)M * ldw * sizeof(float);
  if (splits > 1 && ws_bytes > kNoAllocWorkspaceBytes) return B200_ERR_TOO_LARGE;

  CUtensorMap ta, tb, tc;
  if (encode_2d(&ta, A, K, M, lda, kSlabK, kCtaM) != B200_OK ||
      encode_2d(&tb, B, K, N, ldb, kSlabK, kCtaN) != B200_OK)
    return B200_ERR_TENSOR_MAP;
  GemmArgs args = base_args(M, N, K, nd->launch, nullptr, 0);
  // Dynamic dealing's counters: two words of the array, zero when the
  // library is loaded and set back to zero by every launch's last pair.
  if (dynamic_mode() != 0) args.sched = reinterpret_cast<unsigned int*>(nd->scratch + kNoAllocSchedOffset);
  if (splits > 1) {
    // The split-K accumulator must start at zero: the array keeps the
    // previous call's contents.
    float* W = reinterpret_cast<float*>(nd->scratch + kNoAllocWorkspaceOffset);
    if (encode_2d(&tc, W, N, M, ldw, 32, 32, true) != B200_OK) return B200_ERR_TENSOR_MAP;
    if (cudaMemsetAsync(W, 0, ws_bytes, stream) != cudaSuccess) return B200_ERR_LAUNCH;
    st = launch<false, kV256x64, kOutF32Add>(ta, tb, tc, args, splits, nd->launch, stream);
    if (st != B200_OK) return st;
    return cast_to_bf16(W, ldw, C, ldc, M, N, nd->launch.sms, stream);
  }
  if (encode_2d(&tc, C, N, M, ldc, kStoreCols, 32) != B200_OK) return B200_ERR_TENSOR_MAP;
  // (no stream-K tail here: its slots, 74 pairs x 8 pieces x 32 KiB, exceed
  // the array's workspace)
  return launch_bf16<false>(choose_variant(M, N, K, nd->launch.max_pairs), ta, tb, tc, B, ldb, args,
                            nd->launch, stream, false);
}

}  // namespace

extern "C" int b200_gemm_bf16_noalloc(const void* A, const void* B, void* C, int M, int N,
                                      int K, int lda, int ldb, int ldc, void* stream) {
  return run_gemm_noalloc(A, B, C, M, N, K, lda, ldb, ldc, static_cast<cudaStream_t>(stream));
}

extern "C" int b200_gemm_noalloc_status(int clear, int* status_out) {
  if (!status_out) return B200_ERR_INVALID_ARGUMENT;
  NoAllocDevice* nd = nullptr;
  const int st = noalloc_device(&nd);
  if (st != B200_OK) return st;
  if (cudaDeviceSynchronize() != cudaSuccess) return B200_ERR_LAUNCH;
  int v = 0;
  if (cudaMemcpy(&v, nd->scratch, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess)
    return B200_ERR_LAUNCH;
  if (clear && v != 0 && cudaMemset(nd->scratch, 0, sizeof(int)) != cudaSuccess)
    return B200_ERR_LAUNCH;
  *status_out = v;
  return B200_OK;
}

extern "C" int b200_gemm_noalloc_wait_probe(unsigned long long timeout_ns, void* stream) {
  if (timeout_ns == 0 || timeout_ns > 10000000000ull) return B200_ERR_INVALID_ARGUMENT;
  NoAllocDevice* nd = nullptr;
  const int st = noalloc_device(&nd);
  if (st != B200_OK) return st;
  wait_probe_kernel<<<2, 32, 0, static_cast<cudaStream_t>(stream)>>>(nd->launch.status, timeout_ns);
  return cudaGetLastError() == cudaSuccess ? B200_OK : B200_ERR_LAUNCH;
}
