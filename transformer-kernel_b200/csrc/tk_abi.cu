// C ABI of libtk_b200: argument checks, TMA tensor-map encoding, launch
// configuration, and the device error word. One translation unit holds all
// kernels so they share the error word (tk::g_error).
#include <cuda.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cmath>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <vector>

#include "tk_attn.cuh"
#include "tk_attn_wide.cuh"
#include "tk_gemm.cuh"
#include "tk_layernorm.cuh"
#include "tk_stack_small.cuh"
#include "tk_ptx.cuh"
#include "../../include/tk_b200.h"

namespace {

thread_local std::string g_last_error;
std::atomic<uint64_t> g_wait_limit_ns{2000000000ull};
std::atomic<int> g_programmatic_launch{1};

// Launch-bound (small) kernels are launched with programmatic stream
// serialization (when enabled): such a kernel may be scheduled while the
// previous kernel in the stream drains, runs its prologue (barrier init,
// TMEM allocation, tensor-map prefetch), then waits in griddepcontrol.wait
// for that kernel's results. Inside a CUDA graph the dependency becomes a
// programmatic edge. Measured on one B200: C2 (batch 1, seq 512) forward
// -10%; applied to the large C3 kernels it cost ~2% (early-scheduled CTAs
// share SMs with the previous kernel's tail), so large kernels launch plainly.
constexpr double kSmallGemmMNK = 8.6e9;        // M * N * K
constexpr double kSmallAttnWork = 2.2e9;       // B * H * S * S * hd
constexpr double kSmallLnElements = 4.2e6;     // rows * d

template <typename... KArgs, typename... Args>
cudaError_t launch(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream, bool small,
                   Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = (small && g_programmatic_launch.load()) ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

int fail(int status, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return status;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(e == cudaErrorLaunchFailure || e == cudaErrorInvalidConfiguration ? TK_ERR_LAUNCH : TK_ERR_CUDA,
              "%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}

// --- driver entry point for cuTensorMapEncodeTiled (no -lcuda needed) --------
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// Tensor map over a row-major fp16 (or fp32) tensor: dims innermost first.
int make_map(CUtensorMap* map, CUtensorMapDataType dtype, const void* base, int rank, const cuuint64_t* dims,
             const cuuint64_t* strides_bytes, const cuuint32_t* box, CUtensorMapSwizzle swz) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) return fail(TK_ERR_LAUNCH, "cuTensorMapEncodeTiled unavailable from the driver");
  cuuint32_t estr[5] = {1, 1, 1, 1, 1};
  if (rank < 1 || rank > 5) return fail(TK_ERR_INVALID, "tensor map rank %d", rank);
  CUresult r = fn(map, dtype, rank, const_cast<void*>(base), dims, strides_bytes, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(TK_ERR_LAUNCH, "cuTensorMapEncodeTiled failed (CUresult %d)", static_cast<int>(r));
  return TK_OK;
}

int make_map_f16(CUtensorMap* map, const void* base, int rank, const cuuint64_t* dims, const cuuint64_t* strides_bytes,
                 const cuuint32_t* box, CUtensorMapSwizzle swz) {
  return make_map(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, base, rank, dims, strides_bytes, box, swz);
}

struct DeviceInfo {
  int sms = 0;
  bool gemm_attr_set[4][5] = {};
  bool attn_attr_set[5] = {};
  bool small_attr_set[2] = {};
};
std::mutex g_dev_mu;
DeviceInfo g_dev[64];

int current_device(int* dev, DeviceInfo** info) {
  cudaError_t e = cudaGetDevice(dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (*dev < 0 || *dev >= 64) return fail(TK_ERR_CUDA, "device ordinal %d out of range", *dev);
  std::lock_guard<std::mutex> lk(g_dev_mu);
  DeviceInfo& d = g_dev[*dev];
  if (d.sms == 0) {
    int major = 0, minor = 0;
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, *dev);
    cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, *dev);
    if (major != 10 || minor != 0)
      return fail(TK_ERR_UNSUPPORTED, "libtk_b200 is built for sm_100a; device %d is sm_%d%d", *dev, major, minor);
    e = cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, *dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceGetAttribute");
  }
  *info = &d;
  return TK_OK;
}

bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// Base and size of the device allocation that contains `ptr` (driver API
// cuMemGetAddressRange, reached like cuTensorMapEncodeTiled).
int allocation_range(const void* ptr, CUdeviceptr* base, size_t* size) {
  using RangeFn = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);
  static RangeFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<RangeFn>(p);
  });
  if (fn == nullptr) return fail(TK_ERR_CUDA, "cuMemGetAddressRange unavailable from the driver");
  CUresult r = fn(base, size, reinterpret_cast<CUdeviceptr>(ptr));
  if (r != CUDA_SUCCESS) return fail(TK_ERR_INVALID, "no device allocation holds %p (CUresult %d)", ptr, static_cast<int>(r));
  return TK_OK;
}

// Imported peer allocations: one mapping per exported allocation, counted.
struct PeerMap {
  void* base;
  size_t size;
  int refs;
};
std::mutex g_peer_mu;
std::map<std::string, PeerMap> g_peer_maps;

// ----------------------------------------------------------------------------
// GEMM dispatch
// ----------------------------------------------------------------------------
template <int BN, int EPI>
int launch_gemm(const CUtensorMap& ma, const CUtensorMap& mw, const tk::gemm::Params& p, DeviceInfo* info,
                cudaStream_t stream) {
  using C = tk::gemm::Cfg<BN>;
  auto kern = tk::gemm::gemm_kernel<BN, EPI>;
  const int bi = BN == 64 ? 0 : BN == 128 ? 1 : 2;
  {
    std::lock_guard<std::mutex> lk(g_dev_mu);
    if (!info->gemm_attr_set[bi][EPI]) {
      cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES);
      if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(gemm smem)");
      info->gemm_attr_set[bi][EPI] = true;
    }
  }
  const int tiles = ((p.M + tk::gemm::kBM - 1) / tk::gemm::kBM) * ((p.N + BN - 1) / BN);
  const int grid = tiles < info->sms ? tiles : info->sms;
  const bool small = static_cast<double>(p.M) * p.N * p.K <= kSmallGemmMNK;
  cudaError_t e = launch(kern, dim3(grid), dim3(tk::gemm::kThreads), C::SMEM_BYTES, stream, small, ma, mw, p);
  if (e != cudaSuccess) return cuda_fail(e, "gemm launch");
  return TK_OK;
}

template <int BN>
int launch_gemm_epi(int epi, const CUtensorMap& ma, const CUtensorMap& mw, const tk::gemm::Params& p,
                    DeviceInfo* info, cudaStream_t s) {
  switch (epi) {
    case TK_EPI_BIAS: return launch_gemm<BN, tk::gemm::kBias>(ma, mw, p, info, s);
    case TK_EPI_BIAS_GELU: return launch_gemm<BN, tk::gemm::kBiasGelu>(ma, mw, p, info, s);
    case TK_EPI_BIAS_RESID: return launch_gemm<BN, tk::gemm::kBiasResid>(ma, mw, p, info, s);
    case TK_EPI_BIAS_RESID_LN: return launch_gemm<BN, tk::gemm::kBiasResidLn>(ma, mw, p, info, s);
  }
  return fail(TK_ERR_INVALID, "unknown epilogue %d", epi);
}

template <int EPI>
int launch_gemm_pair(const CUtensorMap& ma, const CUtensorMap& mw, const CUtensorMap& mo, const tk::gemm::Params& p,
                     DeviceInfo* info, cudaStream_t stream) {
  using C = tk::gemm::PairCfg;
  auto kern = tk::gemm::gemm_pair_kernel<EPI>;
  {
    std::lock_guard<std::mutex> lk(g_dev_mu);
    if (!info->gemm_attr_set[3][EPI]) {
      cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES);
      if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(gemm pair smem)");
      info->gemm_attr_set[3][EPI] = true;
    }
  }
  const int tiles = ((p.M + 255) / 256) * (p.N / 256);
  const int pairs = tiles < info->sms / 2 ? tiles : info->sms / 2;
  const bool small = static_cast<double>(p.M) * p.N * p.K <= kSmallGemmMNK;
  cudaError_t e = launch(kern, dim3(2 * pairs), dim3(tk::gemm::kThreads), C::SMEM_BYTES, stream, small, ma, mw, mo, p);
  if (e != cudaSuccess) return cuda_fail(e, "gemm pair launch");
  return TK_OK;
}

// The CTA-pair kernel (256 x 256 tiles over two SMs) for non-LN epilogues
// with N % 256 == 0 and at least two waves of pair tiles.
bool use_pair(int epi, int64_t M, int64_t N, int sms) {
  if (epi == TK_EPI_BIAS_RESID_LN || N % 256 != 0) return false;
  const int64_t tiles = ((M + 255) / 256) * (N / 256);
  return tiles >= sms;
}

// Tile width: the fused-LN epilogue needs the whole row in one tile; else the
// widest tile that still gives every SM at least one tile.
int pick_bn(int epi, int64_t M, int64_t N, int sms) {
  if (epi == TK_EPI_BIAS_RESID_LN) return static_cast<int>(N);
  const int64_t m_tiles = (M + 127) / 128;
  for (int bn : {256, 128}) {
    if (N % bn == 0 && m_tiles * (N / bn) >= sms) return bn;
  }
  return N % 32 == 0 ? 64 : 0;  // a 64-wide tile masks a trailing half tile
}

// Measured tile configurations (tk_gemm_tiles_set): for a GEMM's (N, K,
// epilogue), the entry whose M is nearest on a log scale names the variant;
// a variant the shape cannot take is ignored, as is an empty table.
struct TileEntry {
  int64_t M, N, K;
  int epi, variant;
};
std::mutex g_tiles_mu;
std::vector<TileEntry> g_tiles;

int table_variant(int epi, int64_t M, int64_t N, int64_t K) {
  std::lock_guard<std::mutex> lk(g_tiles_mu);
  int best = TK_TILES_AUTO;
  double best_d = 1e30;
  for (const TileEntry& t : g_tiles) {
    if (t.N != N || t.K != K || t.epi != epi) continue;
    const double dd = std::fabs(std::log(static_cast<double>(t.M)) - std::log(static_cast<double>(M)));
    if (dd < best_d) {
      best_d = dd;
      best = t.variant;
    }
  }
  return best;
}

// (pair, tile width) for a GEMM: the table's variant when it applies, else
// the built-in rules.
void choose_tiles(int epi, int64_t M, int64_t N, int64_t K, int sms, bool* pair, int* bn) {
  const int v = epi == TK_EPI_BIAS_RESID_LN ? TK_TILES_AUTO : table_variant(epi, M, N, K);
  if (v == TK_TILES_PAIR && N % 256 == 0) {
    *pair = true;
    *bn = 128;
    return;
  }
  if ((v == TK_TILES_256 && N % 256 == 0) || (v == TK_TILES_128 && N % 128 == 0) || v == TK_TILES_64) {
    *pair = false;
    *bn = v == TK_TILES_256 ? 256 : v == TK_TILES_128 ? 128 : 64;
    return;
  }
  *pair = use_pair(epi, M, N, sms);
  *bn = *pair ? 128 : pick_bn(epi, M, N, sms);  // pair: each CTA stages 128 rows of W
}

}  // namespace

extern "C" {

const char* tk_last_error(void) { return g_last_error.c_str(); }

int tk_gemm_tiles_set(int64_t M, int64_t N, int64_t K, int epilogue, int variant) {
  g_last_error.clear();
  if (M <= 0 || N <= 0 || K <= 0 || epilogue < TK_EPI_BIAS || epilogue > TK_EPI_BIAS_RESID_LN ||
      variant < TK_TILES_AUTO || variant > TK_TILES_64)
    return fail(TK_ERR_INVALID, "tk_gemm_tiles_set: bad entry M=%lld N=%lld K=%lld epilogue=%d variant=%d",
                (long long)M, (long long)N, (long long)K, epilogue, variant);
  std::lock_guard<std::mutex> lk(g_tiles_mu);
  for (TileEntry& t : g_tiles) {
    if (t.M == M && t.N == N && t.K == K && t.epi == epilogue) {
      t.variant = variant;
      return TK_OK;
    }
  }
  if (g_tiles.size() >= 4096) return fail(TK_ERR_UNSUPPORTED, "tk_gemm_tiles_set: table full (4096 entries)");
  g_tiles.push_back(TileEntry{M, N, K, epilogue, variant});
  return TK_OK;
}

int tk_gemm_tiles_clear(void) {
  std::lock_guard<std::mutex> lk(g_tiles_mu);
  g_tiles.clear();
  return TK_OK;
}

int tk_gemm_tiles_chosen(int64_t M, int64_t N, int64_t K, int epilogue) {
  g_last_error.clear();
  int dev;
  DeviceInfo* info;
  if (int st = current_device(&dev, &info)) return st;
  bool pair = false;
  int bn = 0;
  choose_tiles(epilogue, M, N, K, info->sms, &pair, &bn);
  return pair ? TK_TILES_PAIR : bn == 256 ? TK_TILES_256 : bn == 128 ? TK_TILES_128 : bn == 64 ? TK_TILES_64 : 0;
}

const char* tk_version(void) { return "tk_b200 0.1 (sm_100a)"; }

uint64_t tk_set_wait_limit_ns(uint64_t ns) { return g_wait_limit_ns.exchange(ns); }

int tk_set_programmatic_launch(int enable) { return g_programmatic_launch.exchange(enable ? 1 : 0); }

int tk_layernorm_supported(int64_t d) { return d >= 1 && d <= 8192 ? 1 : 0; }

int tk_attn_supported(int64_t head_dim) {
  return head_dim == 8 || head_dim == 16 || head_dim == 32 || head_dim == 64 || head_dim == 128 || head_dim == 256
             ? 1
             : 0;
}

int tk_layernorm(const void* x, int x_dtype, int64_t ld_x, const void* y, int y_dtype, int64_t ld_y, void* sum_out,
                 int64_t ld_sum, const float* gamma, const float* beta, float eps, void* out, int out_dtype,
                 int64_t ld_out, const int32_t* row_len, int64_t seq_len, int64_t rows, int64_t d, void* stream) {
  g_last_error.clear();
  if (rows < 0 || d < 1) return fail(TK_ERR_INVALID, "tk_layernorm: rows=%lld d=%lld", (long long)rows, (long long)d);
  if (!tk_layernorm_supported(d)) return fail(TK_ERR_UNSUPPORTED, "tk_layernorm: d=%lld > 8192", (long long)d);
  if (x == nullptr || gamma == nullptr || beta == nullptr || out == nullptr)
    return fail(TK_ERR_INVALID, "tk_layernorm: null pointer");
  auto dt_ok = [](int t) { return t == TK_F32 || t == TK_F16; };
  if (!dt_ok(x_dtype) || !dt_ok(out_dtype) || (y != nullptr && !dt_ok(y_dtype)))
    return fail(TK_ERR_INVALID, "tk_layernorm: dtype must be TK_F32 or TK_F16");
  if (ld_x < d || ld_out < d || (y != nullptr && ld_y < d) || (sum_out != nullptr && ld_sum < d))
    return fail(TK_ERR_INVALID, "tk_layernorm: row stride smaller than d");
  if (row_len != nullptr && (seq_len <= 0 || rows % seq_len != 0))
    return fail(TK_ERR_INVALID, "tk_layernorm: row_len needs seq_len dividing rows");
  if (rows == 0) return TK_OK;
  int dev;
  DeviceInfo* info;
  if (int st = current_device(&dev, &info)) return st;

  tk::ln::Args a;
  a.row_len = row_len;
  a.seq_len = seq_len > 0 ? seq_len : 1;
  a.x = x; a.y = y; a.s = sum_out; a.gamma = gamma; a.beta = beta; a.h = out;
  a.rows = rows; a.d = d; a.ld_x = ld_x; a.ld_y = ld_y; a.ld_s = ld_sum; a.ld_h = ld_out; a.eps = eps;
  auto vec_ok = [&](const void* p, int64_t ld, int t) {
    const size_t es = t == TK_F32 ? 4 : 2;
    return p == nullptr || (aligned(p, 4 * es) && (ld * es) % (4 * es) == 0);
  };
  a.vec = (d % 4 == 0) && vec_ok(x, ld_x, x_dtype) && vec_ok(out, ld_out, out_dtype) &&
          (y == nullptr || vec_ok(y, ld_y, y_dtype)) && (sum_out == nullptr || vec_ok(sum_out, ld_sum, x_dtype)) &&
          aligned(gamma, 16) && aligned(beta, 16);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool xf = x_dtype == TK_F32, yf = (y == nullptr) || y_dtype == TK_F32, of = out_dtype == TK_F32;

#define TK_LN_DISPATCH(KERNEL, GRID, ...)                                                    \
  do {                                                                                     \
    if (xf && yf && of) e = launch(KERNEL<__VA_ARGS__ float, float, float, float>, dim3(GRID), dim3(256), 0, s, small, a); \
    else if (xf && yf && !of) e = launch(KERNEL<__VA_ARGS__ float, float, float, __half>, dim3(GRID), dim3(256), 0, s, small, a); \
    else if (xf && !yf && of) e = launch(KERNEL<__VA_ARGS__ float, __half, float, float>, dim3(GRID), dim3(256), 0, s, small, a); \
    else if (xf && !yf && !of) e = launch(KERNEL<__VA_ARGS__ float, __half, float, __half>, dim3(GRID), dim3(256), 0, s, small, a); \
    else if (!xf && yf && of) e = launch(KERNEL<__VA_ARGS__ __half, float, __half, float>, dim3(GRID), dim3(256), 0, s, small, a); \
    else if (!xf && yf && !of) e = launch(KERNEL<__VA_ARGS__ __half, float, __half, __half>, dim3(GRID), dim3(256), 0, s, small, a); \
    else if (!xf && !yf && of) e = launch(KERNEL<__VA_ARGS__ __half, __half, __half, float>, dim3(GRID), dim3(256), 0, s, small, a); \
    else e = launch(KERNEL<__VA_ARGS__ __half, __half, __half, __half>, dim3(GRID), dim3(256), 0, s, small, a); \
  } while (0)

  cudaError_t e = cudaSuccess;
  const bool small = static_cast<double>(rows) * d <= kSmallLnElements;
  if (d <= 1024 && y == nullptr && a.vec && x_dtype == TK_F32 && rows >= 8 * info->sms) {
    // the forward's LayerNorm (fp32 rows in, no residual branch): persistent
    // grid, each warp prefetching its next row (two 256-thread CTAs per SM)
    const int64_t cap = static_cast<int64_t>(info->sms) * 2;
    const int64_t blocks = (rows + 7) / 8;
    const int grid = static_cast<int>(blocks < cap ? blocks : cap);
    auto go = [&](auto kern) { return launch(kern, dim3(grid), dim3(256), 0, s, small, a); };
    if (of) {
      if (d <= 128) e = go(tk::ln::ln_warp_rows_prefetch<1, float, float, float>);
      else if (d <= 256) e = go(tk::ln::ln_warp_rows_prefetch<2, float, float, float>);
      else if (d <= 512) e = go(tk::ln::ln_warp_rows_prefetch<4, float, float, float>);
      else e = go(tk::ln::ln_warp_rows_prefetch<8, float, float, float>);
    } else {
      if (d <= 128) e = go(tk::ln::ln_warp_rows_prefetch<1, float, float, __half>);
      else if (d <= 256) e = go(tk::ln::ln_warp_rows_prefetch<2, float, float, __half>);
      else if (d <= 512) e = go(tk::ln::ln_warp_rows_prefetch<4, float, float, __half>);
      else e = go(tk::ln::ln_warp_rows_prefetch<8, float, float, __half>);
    }
  } else if (d <= 1024) {
    const int64_t warps_needed = rows;
    int64_t blocks = (warps_needed + 7) / 8;
    const int64_t cap = static_cast<int64_t>(info->sms) * 16;
    const int grid = static_cast<int>(blocks < cap ? blocks : cap);
    if (d <= 128) TK_LN_DISPATCH(tk::ln::ln_warp_rows, grid, 1,);
    else if (d <= 256) TK_LN_DISPATCH(tk::ln::ln_warp_rows, grid, 2,);
    else if (d <= 512) TK_LN_DISPATCH(tk::ln::ln_warp_rows, grid, 4,);
    else TK_LN_DISPATCH(tk::ln::ln_warp_rows, grid, 8,);
  } else {
    const int64_t cap = static_cast<int64_t>(info->sms) * 8;
    const int grid = static_cast<int>(rows < cap ? rows : cap);
    TK_LN_DISPATCH(tk::ln::ln_cta_rows, grid, );
  }
#undef TK_LN_DISPATCH
  if (e != cudaSuccess) return cuda_fail(e, "tk_layernorm launch");
  return TK_OK;
}

int tk_gemm(const void* A, int64_t lda, const void* W, int64_t ldw, const float* bias, int epilogue,
            const float* resid, int64_t ld_resid, float* sum_out, int64_t ld_sum, const float* gamma,
            const float* beta, float eps, void* out, int out_dtype, int64_t ldo, const int32_t* row_len,
            int64_t seq_len, int64_t M, int64_t N, int64_t K, void* stream) {
  g_last_error.clear();
  if (A == nullptr || W == nullptr || bias == nullptr) return fail(TK_ERR_INVALID, "tk_gemm: null A/W/bias");
  if (M < 0 || N <= 0 || K <= 0 || M > (1ll << 31) - 1 || N > 65536 || K > 65536)
    return fail(TK_ERR_INVALID, "tk_gemm: bad sizes M=%lld N=%lld K=%lld", (long long)M, (long long)N, (long long)K);
  if (N % 32 != 0 || K % 8 != 0)
    return fail(TK_ERR_UNSUPPORTED, "tk_gemm: needs N %% 32 == 0 and K %% 8 == 0 (N=%lld K=%lld)", (long long)N,
                (long long)K);
  if (lda < K || ldw < K || lda % 8 != 0 || ldw % 8 != 0 || !aligned(A, 16) || !aligned(W, 16))
    return fail(TK_ERR_INVALID, "tk_gemm: A/W need 16-byte aligned rows (ld %% 8 == 0, ld >= K)");
  if (!aligned(bias, 16)) return fail(TK_ERR_INVALID, "tk_gemm: bias must be 16-byte aligned");
  const bool resid_epi = epilogue == TK_EPI_BIAS_RESID || epilogue == TK_EPI_BIAS_RESID_LN;
  if (resid_epi) {
    if (resid == nullptr || sum_out == nullptr || ld_resid < N || ld_sum < N || ld_resid % 4 || ld_sum % 4 ||
        !aligned(resid, 16) || !aligned(sum_out, 16))
      return fail(TK_ERR_INVALID, "tk_gemm: residual epilogue needs 16-byte aligned fp32 resid/sum_out rows");
  }
  const bool ln_epi = epilogue == TK_EPI_BIAS_RESID_LN;
  if (ln_epi) {
    if (gamma == nullptr || beta == nullptr || !aligned(gamma, 16) || !aligned(beta, 16))
      return fail(TK_ERR_INVALID, "tk_gemm: LN epilogue needs aligned gamma/beta");
    if (!(N == 64 || N == 128 || N == 256))
      return fail(TK_ERR_UNSUPPORTED, "tk_gemm: fused LN epilogue needs N in {64,128,256} (N=%lld)", (long long)N);
  }
  const bool writes_out = epilogue != TK_EPI_BIAS_RESID;
  if (writes_out) {
    const bool f32 = ln_epi && out_dtype == TK_F32;
    if (!ln_epi && out_dtype != TK_F16) return fail(TK_ERR_INVALID, "tk_gemm: this epilogue writes fp16");
    if (out == nullptr || ldo < N || (f32 ? ldo % 4 : ldo % 8) != 0 || !aligned(out, 16))
      return fail(TK_ERR_INVALID, "tk_gemm: out needs 16-byte aligned rows");
  }
  if (row_len != nullptr && (seq_len <= 0 || M % seq_len != 0))
    return fail(TK_ERR_INVALID, "tk_gemm: row_len needs seq_len dividing M");
  if (M == 0) return TK_OK;
  int dev;
  DeviceInfo* info;
  if (int st = current_device(&dev, &info)) return st;
  bool pair = false;
  int bn = 0;
  choose_tiles(epilogue, M, N, K, info->sms, &pair, &bn);
  if (bn == 0) return fail(TK_ERR_UNSUPPORTED, "tk_gemm: N=%lld has no tile width", (long long)N);

  CUtensorMap ma, mw;
  {
    cuuint64_t dims[2] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(M)};
    cuuint64_t strides[1] = {static_cast<cuuint64_t>(lda) * 2};
    cuuint32_t box[2] = {64, 128};
    if (int st = make_map_f16(&ma, A, 2, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B)) return st;
  }
  {
    cuuint64_t dims[2] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(N)};
    cuuint64_t strides[1] = {static_cast<cuuint64_t>(ldw) * 2};
    cuuint32_t box[2] = {64, static_cast<cuuint32_t>(bn)};
    if (int st = make_map_f16(&mw, W, 2, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B)) return st;
  }
  tk::gemm::Params p;
  p.M = static_cast<int>(M); p.N = static_cast<int>(N); p.K = static_cast<int>(K);
  p.bias = bias; p.resid = resid; p.ld_resid = ld_resid; p.sum_out = sum_out; p.ld_sum = ld_sum;
  p.out = out; p.ldo = ldo; p.out_f32 = (ln_epi && out_dtype == TK_F32) ? 1 : 0;
  p.gamma = gamma; p.beta = beta; p.eps = eps;
  p.row_len = row_len; p.seq_len = static_cast<int>(seq_len > 0 ? seq_len : 1);
  p.reduce_add = 0;
  p.wait_limit_ns = g_wait_limit_ns.load();
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (pair) {
    // fp16 outputs leave through TMA stores of 32 x 32 tiles (64-byte swizzle)
    CUtensorMap mo = ma;  // unused by the staged residual epilogue
    p.reduce_add = (epilogue == TK_EPI_BIAS_RESID && resid == sum_out && ld_resid == ld_sum && row_len == nullptr);
    if (p.reduce_add) {
      // in-place residual update: TMA reduce-add of 32 x 32 fp32 tiles (128-byte swizzle) into sum_out
      cuuint64_t dims[2] = {static_cast<cuuint64_t>(N), static_cast<cuuint64_t>(M)};
      cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld_sum) * 4};
      cuuint32_t box[2] = {32, 32};
      if (int st = make_map(&mo, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, sum_out, 2, dims, strides, box,
                            CU_TENSOR_MAP_SWIZZLE_128B))
        return st;
    } else if (epilogue != TK_EPI_BIAS_RESID) {
      cuuint64_t dims[2] = {static_cast<cuuint64_t>(N), static_cast<cuuint64_t>(M)};
      cuuint64_t strides[1] = {static_cast<cuuint64_t>(ldo) * 2};
      cuuint32_t box[2] = {32, 32};
      if (int st = make_map_f16(&mo, out, 2, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_64B)) return st;
    }
    switch (epilogue) {
      case TK_EPI_BIAS: return launch_gemm_pair<tk::gemm::kBias>(ma, mw, mo, p, info, s);
      case TK_EPI_BIAS_GELU: return launch_gemm_pair<tk::gemm::kBiasGelu>(ma, mw, mo, p, info, s);
      case TK_EPI_BIAS_RESID: return launch_gemm_pair<tk::gemm::kBiasResid>(ma, mw, mo, p, info, s);
    }
  }
  switch (bn) {
    case 64: return launch_gemm_epi<64>(epilogue, ma, mw, p, info, s);
    case 128: return launch_gemm_epi<128>(epilogue, ma, mw, p, info, s);
    case 256: return launch_gemm_epi<256>(epilogue, ma, mw, p, info, s);
  }
  return fail(TK_ERR_UNSUPPORTED, "tk_gemm: no kernel for tile width %d", bn);
}

// --- GEMM + residual + LayerNorm over rows wider than a tile -----------------
namespace {
bool wide_ln_shape(int64_t N) { return N % 256 == 0 && N >= 512 && N <= 4096; }
int64_t align256(int64_t v) { return (v + 255) / 256 * 256; }
}  // namespace

int64_t tk_gemm_resid_ln_workspace_bytes(int64_t M, int64_t N) {
  if (M <= 0 || !wide_ln_shape(N)) return 0;
  return align256(M * 8) + align256(M * (N / 128) * 8);  // state words [M] u64, partials [M, N/128] float2
}

int tk_gemm_resid_ln_supported(int64_t M, int64_t N, int64_t K) {
  if (M < 0 || K <= 0 || K % 8 != 0) return 0;
  return (N == 64 || N == 128 || N == 256 || wide_ln_shape(N)) ? 1 : 0;
}

int tk_gemm_resid_ln(const void* A, int64_t lda, const void* W, int64_t ldw, const float* bias, const float* resid,
                     int64_t ld_resid, float* sum_out, int64_t ld_sum, const float* gamma, const float* beta, float eps,
                     void* out, int out_dtype, int64_t ldo, const int32_t* row_len, int64_t seq_len, int64_t M,
                     int64_t N, int64_t K, void* workspace, int64_t workspace_bytes, void* stream) {
  g_last_error.clear();
  if (N == 64 || N == 128 || N == 256)  // one tile holds the whole row: no workspace
    return tk_gemm(A, lda, W, ldw, bias, TK_EPI_BIAS_RESID_LN, resid, ld_resid, sum_out, ld_sum, gamma, beta, eps,
                   out, out_dtype, ldo, row_len, seq_len, M, N, K, stream);
  if (A == nullptr || W == nullptr || bias == nullptr || resid == nullptr || sum_out == nullptr || gamma == nullptr ||
      beta == nullptr || out == nullptr)
    return fail(TK_ERR_INVALID, "tk_gemm_resid_ln: null pointer");
  if (M < 0 || K <= 0 || M > (1ll << 31) - 1 || K > 65536)
    return fail(TK_ERR_INVALID, "tk_gemm_resid_ln: bad sizes M=%lld N=%lld K=%lld", (long long)M, (long long)N,
                (long long)K);
  if (!wide_ln_shape(N) || K % 8 != 0)
    return fail(TK_ERR_UNSUPPORTED, "tk_gemm_resid_ln: needs N in {64,128,256} or N %% 256 == 0 with "
                "512 <= N <= 4096, and K %% 8 == 0 (N=%lld K=%lld)", (long long)N, (long long)K);
  if (lda < K || ldw < K || lda % 8 != 0 || ldw % 8 != 0 || !aligned(A, 16) || !aligned(W, 16))
    return fail(TK_ERR_INVALID, "tk_gemm_resid_ln: A/W need 16-byte aligned rows (ld %% 8 == 0, ld >= K)");
  if (!aligned(bias, 16) || !aligned(gamma, 16) || !aligned(beta, 16))
    return fail(TK_ERR_INVALID, "tk_gemm_resid_ln: bias/gamma/beta must be 16-byte aligned");
  if (ld_resid < N || ld_sum < N || ld_resid % 4 || ld_sum % 4 || !aligned(resid, 16) || !aligned(sum_out, 16))
    return fail(TK_ERR_INVALID, "tk_gemm_resid_ln: resid/sum_out need 16-byte aligned fp32 rows");
  if (out_dtype != TK_F16 && out_dtype != TK_F32) return fail(TK_ERR_INVALID, "tk_gemm_resid_ln: out dtype");
  if (ldo < N || (out_dtype == TK_F32 ? ldo % 4 : ldo % 8) != 0 || !aligned(out, 16))
    return fail(TK_ERR_INVALID, "tk_gemm_resid_ln: out needs 16-byte aligned rows");
  if (row_len != nullptr && (seq_len <= 0 || M % seq_len != 0))
    return fail(TK_ERR_INVALID, "tk_gemm_resid_ln: row_len needs seq_len dividing M");
  const int64_t need = tk_gemm_resid_ln_workspace_bytes(M, N);
  if (workspace == nullptr || workspace_bytes < need || !aligned(workspace, 256))
    return fail(TK_ERR_INVALID, "tk_gemm_resid_ln: needs a 256-byte aligned workspace of %lld bytes (got %lld)",
                (long long)need, (long long)workspace_bytes);
  if (M == 0) return TK_OK;
  int dev;
  DeviceInfo* info;
  if (int st = current_device(&dev, &info)) return st;
  CUtensorMap ma, mw;
  {
    cuuint64_t dims[2] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(M)};
    cuuint64_t strides[1] = {static_cast<cuuint64_t>(lda) * 2};
    cuuint32_t box[2] = {64, 128};
    if (int st = make_map_f16(&ma, A, 2, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B)) return st;
  }
  {
    cuuint64_t dims[2] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(N)};
    cuuint64_t strides[1] = {static_cast<cuuint64_t>(ldw) * 2};
    cuuint32_t box[2] = {64, 128};
    if (int st = make_map_f16(&mw, W, 2, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B)) return st;
  }
  tk::gemm::Params p;
  p.M = static_cast<int>(M); p.N = static_cast<int>(N); p.K = static_cast<int>(K);
  p.bias = bias; p.resid = resid; p.ld_resid = ld_resid; p.sum_out = sum_out; p.ld_sum = ld_sum;
  p.out = out; p.ldo = ldo; p.out_f32 = out_dtype == TK_F32 ? 1 : 0;
  p.gamma = gamma; p.beta = beta; p.eps = eps;
  p.row_len = row_len; p.seq_len = static_cast<int>(seq_len > 0 ? seq_len : 1);
  p.reduce_add = 0;
  p.wait_limit_ns = g_wait_limit_ns.load();
  // State words at the front, partials at the back: a workspace sized for M
  // rows serves every M' <= M without the two regions ever overlapping, so
  // the words a completed call leaves at zero stay zero.
  p.ln_parts = static_cast<int>(N / 128);
  p.ln_state = static_cast<unsigned long long*>(workspace);
  p.ln_part = reinterpret_cast<float2*>(static_cast<char*>(workspace) + (workspace_bytes / 256) * 256 -
                                        align256(M * (N / 128) * 8));
  return launch_gemm_pair<tk::gemm::kBiasResidLnX>(ma, mw, ma, p, info, static_cast<cudaStream_t>(stream));
}

// --- the same GEMM + residual + LayerNorm, with no workspace argument ---------
// For callers that cannot allocate device memory (see include/tk_b200.h):
// the scratch is a file-scope device array of fixed size, which every GPU
// that loads this library holds until the process exits. Host code cannot
// use the array's name as a device address, so the entry point looks the
// address up once per device with cudaGetSymbolAddress.
namespace {
constexpr int64_t kStaticLnScratchBytes = int64_t(8) << 20;  // 8 MiB
static __device__ __align__(256) unsigned char g_ln_static_scratch[kStaticLnScratchBytes];
std::mutex g_static_mu;
void* g_static_scratch_ptr[64] = {};
}  // namespace

int tk_gemm_resid_ln_static(const void* A, int64_t lda, const void* W, int64_t ldw, const float* bias,
                            const float* resid, int64_t ld_resid, float* sum_out, int64_t ld_sum, const float* gamma,
                            const float* beta, float eps, void* out, int out_dtype, int64_t ldo,
                            const int32_t* row_len, int64_t seq_len, int64_t M, int64_t N, int64_t K, void* stream) {
  g_last_error.clear();
  if (N == 64 || N == 128 || N == 256)  // one tile holds the whole row: no scratch at all
    return tk_gemm(A, lda, W, ldw, bias, TK_EPI_BIAS_RESID_LN, resid, ld_resid, sum_out, ld_sum, gamma, beta, eps,
                   out, out_dtype, ldo, row_len, seq_len, M, N, K, stream);
  if (!wide_ln_shape(N))
    return fail(TK_ERR_UNSUPPORTED, "tk_gemm_resid_ln_static: needs N in {64,128,256} or N %% 256 == 0 with "
                "512 <= N <= 4096 (N=%lld)", (long long)N);
  if (M < 0) return fail(TK_ERR_INVALID, "tk_gemm_resid_ln_static: M=%lld", (long long)M);
  const int64_t need = tk_gemm_resid_ln_workspace_bytes(M, N);
  if (need > kStaticLnScratchBytes)
    return fail(TK_ERR_UNSUPPORTED, "tk_gemm_resid_ln_static: M=%lld rows of N=%lld need %lld bytes of scratch; the "
                "built-in scratch holds %lld bytes (at most %lld rows at this N); use tk_gemm_resid_ln with a "
                "workspace", (long long)M, (long long)N, (long long)need, (long long)kStaticLnScratchBytes,
                (long long)(kStaticLnScratchBytes / (8 + (N / 128) * 8) - 64));
  int dev;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= 64) return fail(TK_ERR_CUDA, "device ordinal %d out of range", dev);
  void* scratch = nullptr;
  {
    // set-up, once per device, with that device current (the caller's)
    std::lock_guard<std::mutex> lk(g_static_mu);
    if (g_static_scratch_ptr[dev] == nullptr) {
      void* ptr = nullptr;
      e = cudaGetSymbolAddress(&ptr, g_ln_static_scratch);
      if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(scratch)");
      g_static_scratch_ptr[dev] = ptr;
    }
    scratch = g_static_scratch_ptr[dev];
  }
  // The array keeps the last call's contents, whatever its shape: zero the
  // per-row state words this call counts in (front of the array) first.
  e = cudaMemsetAsync(scratch, 0, static_cast<size_t>(align256(M * 8)), static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync(scratch)");
  return tk_gemm_resid_ln(A, lda, W, ldw, bias, resid, ld_resid, sum_out, ld_sum, gamma, beta, eps, out, out_dtype,
                          ldo, row_len, seq_len, M, N, K, scratch, kStaticLnScratchBytes, stream);
}

int tk_stack_small_supported(int64_t d, int64_t heads, int64_t ffn, int64_t seq_len) {
  return d == 128 && ffn == 128 && (heads == 2 || heads == 4) && seq_len >= 1 && seq_len <= 128 ? 1 : 0;
}

int tk_stack_small(const float* x, float* out, const void* w_packed, const float* vec_packed, const float* final_gamma,
                   const float* final_beta, float eps, const int32_t* row_len, int64_t B, int64_t S, int64_t d,
                   int64_t heads, int64_t ffn, int64_t L, int causal, float scale, void* stream) {
  g_last_error.clear();
  if (x == nullptr || out == nullptr || w_packed == nullptr || vec_packed == nullptr || final_gamma == nullptr ||
      final_beta == nullptr)
    return fail(TK_ERR_INVALID, "tk_stack_small: null pointer");
  if (B < 0 || L < 1) return fail(TK_ERR_INVALID, "tk_stack_small: B=%lld L=%lld", (long long)B, (long long)L);
  if (!tk_stack_small_supported(d, heads, ffn, S))
    return fail(TK_ERR_UNSUPPORTED, "tk_stack_small: needs d = ffn = 128, 2 or 4 heads, 1 <= S <= 128 (d=%lld "
                "heads=%lld ffn=%lld S=%lld)", (long long)d, (long long)heads, (long long)ffn, (long long)S);
  if (!aligned(x, 16) || !aligned(out, 16) || !aligned(w_packed, 16) || !aligned(vec_packed, 16))
    return fail(TK_ERR_INVALID, "tk_stack_small: x / out / packed weights need 16-byte alignment");
  if (B > (1ll << 31) - 1 || L * tk::small::kWRowsPerLayer > (1ll << 31) - 1)
    return fail(TK_ERR_UNSUPPORTED, "tk_stack_small: too large");
  if (B == 0) return TK_OK;
  int dev;
  DeviceInfo* info;
  if (int st = current_device(&dev, &info)) return st;
  CUtensorMap mw;
  {
    cuuint64_t dims[2] = {128, static_cast<cuuint64_t>(L * tk::small::kWRowsPerLayer)};
    cuuint64_t strides[1] = {256};
    cuuint32_t box[2] = {64, 128};
    if (int st = make_map_f16(&mw, w_packed, 2, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B)) return st;
  }
  tk::small::Params p;
  p.x = x;
  p.out = out;
  p.vec = vec_packed;
  p.final_g = final_gamma;
  p.final_b = final_beta;
  p.row_len = row_len;
  p.B = static_cast<int>(B);
  p.S = static_cast<int>(S);
  p.H = static_cast<int>(heads);
  p.L = static_cast<int>(L);
  p.causal = causal ? 1 : 0;
  p.eps = eps;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.wait_limit_ns = g_wait_limit_ns.load();
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  auto run = [&](auto kern, int slot, int smem_bytes) -> cudaError_t {
    {
      std::lock_guard<std::mutex> lk(g_dev_mu);
      if (!info->small_attr_set[slot]) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes);
        if (e != cudaSuccess) return e;
        info->small_attr_set[slot] = true;
      }
    }
    return launch(kern, dim3(static_cast<unsigned>(B)), dim3(tk::small::kThreads), smem_bytes, s, true, mw, p);
  };
  cudaError_t e = heads == 4 ? run(tk::small::stack_small_kernel<32>, 0, tk::small::Cfg<32>::SMEM_BYTES)
                             : run(tk::small::stack_small_kernel<64>, 1, tk::small::Cfg<64>::SMEM_BYTES);
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "tk_stack_small launch");
  return TK_OK;
}

int tk_attn_fwd(const void* q, const void* k, const void* v, int64_t stride_b, int64_t stride_h, int64_t stride_s,
                void* out, int64_t ld_out, int64_t B, int64_t S, int64_t H, int64_t hd, float scale, int causal,
                const int32_t* kv_len, void* stream) {
  g_last_error.clear();
  if (q == nullptr || k == nullptr || v == nullptr || out == nullptr)
    return fail(TK_ERR_INVALID, "tk_attn_fwd: null pointer");
  if (B <= 0 || S <= 0 || H <= 0 || hd <= 0) return fail(TK_ERR_INVALID, "tk_attn_fwd: non-positive size");
  if (!tk_attn_supported(hd))
    return fail(TK_ERR_UNSUPPORTED, "tk_attn_fwd: head_dim %lld not in {8,16,32,64,128,256}", (long long)hd);
  if (stride_b <= 0 || stride_h <= 0 || stride_s <= 0 || stride_b % 8 || stride_h % 8 || stride_s % 8 ||
      !aligned(q, 16) || !aligned(k, 16) || !aligned(v, 16))
    return fail(TK_ERR_INVALID, "tk_attn_fwd: q/k/v need 16-byte aligned bases and strides (multiples of 8 elements)");
  if (ld_out < H * hd || ld_out % 8 || !aligned(out, 16))
    return fail(TK_ERR_INVALID, "tk_attn_fwd: out needs 16-byte aligned rows and ld_out >= H*hd");
  const int64_t q_tiles = (S + 127) / 128;
  if (S > (1ll << 31) - 1 || B * H * q_tiles > (1ll << 31) - 1)
    return fail(TK_ERR_UNSUPPORTED, "tk_attn_fwd: grid too large");
  int dev;
  DeviceInfo* info;
  if (int st = current_device(&dev, &info)) return st;

  CUtensorMap maps[3];
  const void* bases[3] = {q, k, v};
  // Dimensions in increasing stride order (the encoder rejects others).
  const bool heads_inner = stride_h < stride_s;
  const int64_t mid_dim[2] = {heads_inner ? H : S, heads_inner ? S : H};
  const int64_t mid_stride[2] = {heads_inner ? stride_h : stride_s, heads_inner ? stride_s : stride_h};
  if (mid_stride[0] < hd || mid_stride[1] < mid_stride[0] || stride_b < mid_stride[1])
    return fail(TK_ERR_UNSUPPORTED, "tk_attn_fwd: strides (b=%lld, h=%lld, s=%lld) overlap", (long long)stride_b,
                (long long)stride_h, (long long)stride_s);
  cuuint64_t dims[4] = {static_cast<cuuint64_t>(hd), static_cast<cuuint64_t>(mid_dim[0]),
                        static_cast<cuuint64_t>(mid_dim[1]), static_cast<cuuint64_t>(B)};
  cuuint64_t strides[3] = {static_cast<cuuint64_t>(mid_stride[0]) * 2, static_cast<cuuint64_t>(mid_stride[1]) * 2,
                           static_cast<cuuint64_t>(stride_b) * 2};
  // head_dim 8 runs the 16-wide kernel: the box is 16 columns wide and TMA
  // fills the 8 columns past the tensor's inner dimension with zeros.
  // head_dim 128 / 256 run the chunked kernel: boxes of 64 columns.
  const int64_t hd_k = hd < 16 ? 16 : hd;
  const bool wide = hd_k > 64;
  cuuint32_t box[4] = {static_cast<cuuint32_t>(wide ? 64 : hd_k), heads_inner ? 1u : 128u, heads_inner ? 128u : 1u,
                       1};
  const CUtensorMapSwizzle swz = (hd_k == 64 || wide) ? CU_TENSOR_MAP_SWIZZLE_128B
                                 : hd_k == 32 ? CU_TENSOR_MAP_SWIZZLE_64B
                                              : CU_TENSOR_MAP_SWIZZLE_32B;
  for (int i = 0; i < 3; ++i)
    if (int st = make_map_f16(&maps[i], bases[i], 4, dims, strides, box, swz)) return st;
  tk::attn::Params p;
  p.out = static_cast<__half*>(out);
  p.ld_out = ld_out;
  p.B = static_cast<int>(B);
  p.S = static_cast<int>(S);
  p.H = static_cast<int>(H);
  p.scale_log2 = scale * 1.4426950408889634f;
  p.causal = causal ? 1 : 0;
  p.kv_len = kv_len;
  p.heads_inner = heads_inner ? 1 : 0;
  p.hd = static_cast<int>(hd);
  p.wait_limit_ns = g_wait_limit_ns.load();
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // persistent: one CTA per SM over the (b, h, query-tile pair) work items
  const int64_t items = B * H * ((q_tiles + 1) / 2);
  const unsigned grid = static_cast<unsigned>(items < info->sms ? items : info->sms);
  const bool small = static_cast<double>(B) * H * S * S * hd <= kSmallAttnWork;
  int built_regs = 0;  // set when a kernel's register count does not match its register split
  auto run = [&](auto kern, int slot, int smem_bytes, unsigned grid_x, unsigned threads) -> cudaError_t {
    {
      std::lock_guard<std::mutex> lk(g_dev_mu);
      if (!info->attn_attr_set[slot]) {
        if (threads == tk::attn::kThreads) {
          // The in-kernel setmaxnreg split hands out exactly threads x
          // kLaunchRegs registers; with any other launch allocation the
          // softmax warpgroups' increase could never be granted.
          cudaFuncAttributes fa;
          cudaError_t e = cudaFuncGetAttributes(&fa, kern);
          if (e != cudaSuccess) return e;
          if (fa.numRegs != tk::attn::kLaunchRegs) {
            built_regs = fa.numRegs;
            return cudaErrorInvalidConfiguration;
          }
        }
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes);
        if (e != cudaSuccess) return e;
        info->attn_attr_set[slot] = true;
      }
    }
    return launch(kern, dim3(grid_x), dim3(threads), smem_bytes, s, small, maps[0], maps[1], maps[2], p);
  };
  cudaError_t e;
  // chunked kernel: one CTA per (b, h, query tile)
  const unsigned wide_grid = static_cast<unsigned>(B * H * q_tiles);
  constexpr unsigned kT = tk::attn::kThreads, kTw = tk::attn::wide::kThreads;
  if (hd_k == 256)
    e = run(tk::attn::wide::attn_fwd_wide_kernel<256>, 4, tk::attn::wide::Cfg<256>::SMEM_BYTES, wide_grid, kTw);
  else if (hd_k == 128)
    e = run(tk::attn::wide::attn_fwd_wide_kernel<128>, 3, tk::attn::wide::Cfg<128>::SMEM_BYTES, wide_grid, kTw);
  else if (hd_k == 64)
    e = run(tk::attn::attn_fwd_kernel<64>, 2, tk::attn::Cfg<64>::SMEM_BYTES, grid, kT);
  else if (hd_k == 32)
    e = run(tk::attn::attn_fwd_kernel<32>, 1, tk::attn::Cfg<32>::SMEM_BYTES, grid, kT);
  else
    e = run(tk::attn::attn_fwd_kernel<16>, 0, tk::attn::Cfg<16>::SMEM_BYTES, grid, kT);
  if (built_regs != 0)
    return fail(TK_ERR_LAUNCH, "tk_attn_fwd: kernel built with %d registers per thread; its register split needs %d",
                built_regs, tk::attn::kLaunchRegs);
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "tk_attn_fwd launch");
  return TK_OK;
}

// ----------------------------------------------------------------------------
// peer memory (CUDA IPC) and row copies
// ----------------------------------------------------------------------------
int tk_peer_export(const void* ptr, void* handle, int64_t* offset) {
  g_last_error.clear();
  if (ptr == nullptr || handle == nullptr || offset == nullptr) return fail(TK_ERR_INVALID, "tk_peer_export: null pointer");
  CUdeviceptr base = 0;
  size_t size = 0;
  if (int st = allocation_range(ptr, &base, &size)) return st;
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
  if (e != cudaSuccess) return cuda_fail(e, "cudaIpcGetMemHandle");
  static_assert(sizeof(h) == 64, "IPC handle size");
  std::memcpy(handle, &h, sizeof(h));
  *offset = static_cast<int64_t>(reinterpret_cast<uintptr_t>(ptr) - static_cast<uintptr_t>(base));
  return TK_OK;
}

int tk_peer_import(const void* handle, int64_t offset, void** ptr) {
  g_last_error.clear();
  if (handle == nullptr || ptr == nullptr || offset < 0) return fail(TK_ERR_INVALID, "tk_peer_import: bad argument");
  const std::string key(static_cast<const char*>(handle), 64);
  std::lock_guard<std::mutex> lk(g_peer_mu);
  auto it = g_peer_maps.find(key);
  if (it == g_peer_maps.end()) {
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handle, sizeof(h));
    void* base = nullptr;
    cudaError_t e = cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) return cuda_fail(e, "cudaIpcOpenMemHandle");
    CUdeviceptr b = 0;
    size_t size = 0;
    if (int st = allocation_range(base, &b, &size)) {
      cudaIpcCloseMemHandle(base);
      return st;
    }
    it = g_peer_maps.emplace(key, PeerMap{base, size, 0}).first;
  }
  if (static_cast<size_t>(offset) >= it->second.size)
    return fail(TK_ERR_INVALID, "tk_peer_import: offset %lld beyond the %zu-byte allocation", (long long)offset,
                it->second.size);
  ++it->second.refs;
  *ptr = static_cast<char*>(it->second.base) + offset;
  return TK_OK;
}

int tk_peer_release(void* ptr) {
  g_last_error.clear();
  std::lock_guard<std::mutex> lk(g_peer_mu);
  // the mapping whose range holds ptr
  auto best = g_peer_maps.end();
  const uintptr_t q = reinterpret_cast<uintptr_t>(ptr);
  for (auto it = g_peer_maps.begin(); it != g_peer_maps.end(); ++it) {
    const uintptr_t b = reinterpret_cast<uintptr_t>(it->second.base);
    if (q >= b && q < b + it->second.size) best = it;
  }
  if (best == g_peer_maps.end()) return fail(TK_ERR_INVALID, "tk_peer_release: %p is not in an imported mapping", ptr);
  if (--best->second.refs == 0) {
    cudaError_t e = cudaIpcCloseMemHandle(best->second.base);
    g_peer_maps.erase(best);
    if (e != cudaSuccess) return cuda_fail(e, "cudaIpcCloseMemHandle");
  }
  return TK_OK;
}

int tk_copy_rows(void* dst, int64_t dst_ld, const void* src, int64_t src_ld, int64_t row_bytes, int64_t rows,
                 void* stream) {
  g_last_error.clear();
  if (rows < 0 || row_bytes < 0 || (rows > 0 && (dst == nullptr || src == nullptr)))
    return fail(TK_ERR_INVALID, "tk_copy_rows: bad argument");
  if (rows > 1 && (dst_ld < row_bytes || src_ld < row_bytes))
    return fail(TK_ERR_INVALID, "tk_copy_rows: row stride smaller than a row");
  if (rows == 0 || row_bytes == 0) return TK_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e;
  if (dst_ld == row_bytes && src_ld == row_bytes)
    e = cudaMemcpyAsync(dst, src, static_cast<size_t>(row_bytes * rows), cudaMemcpyDeviceToDevice, s);
  else
    e = cudaMemcpy2DAsync(dst, static_cast<size_t>(dst_ld), src, static_cast<size_t>(src_ld),
                          static_cast<size_t>(row_bytes), static_cast<size_t>(rows), cudaMemcpyDeviceToDevice, s);
  if (e != cudaSuccess) return cuda_fail(e, "tk_copy_rows");
  return TK_OK;
}

}  // extern "C"

// ----------------------------------------------------------------------------
// error word + self test
// ----------------------------------------------------------------------------
namespace {
__global__ void selftest_wait_kernel(uint64_t limit_ns) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    tk::mbar_init(&bar, 1);
    tk::fence_barrier_init();
    // Nothing ever arrives on `bar`: the wait must give up after limit_ns.
    if (!tk::mbar_wait(&bar, 0, nullptr, limit_ns)) tk::report_error(tk::kDevWaitTimeout, 0xFF01u);
  }
}
}  // namespace

extern "C" {

int tk_selftest_wait_timeout(void* stream) {
  g_last_error.clear();
  int dev;
  DeviceInfo* info;
  if (int st = current_device(&dev, &info)) return st;
  selftest_wait_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(g_wait_limit_ns.load());
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "selftest launch");
  return TK_OK;
}

int tk_check_device_errors(void* stream) {
  g_last_error.clear();
  cudaError_t e = cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "cudaStreamSynchronize");
  tk::ErrorWord w;
  e = cudaMemcpyFromSymbol(&w, tk::g_error, sizeof(w));
  if (e != cudaSuccess) return cuda_fail(e, "read error word");
  if (w.code == tk::kDevOk) return TK_OK;
  const tk::ErrorWord zero = {0, 0, 0, 0};
  e = cudaMemcpyToSymbol(tk::g_error, &zero, sizeof(zero));
  if (e != cudaSuccess) return cuda_fail(e, "clear error word");
  if (w.code == tk::kDevWaitTimeout)
    return fail(TK_ERR_TIMEOUT, "device wait timed out: site 0x%x, block %u, %u failure(s)", w.where, w.detail, w.count);
  return fail(TK_ERR_DEVICE, "device error %u at site 0x%x, block %u, %u failure(s)", w.code, w.where, w.detail,
              w.count);
}

}  // extern "C"
