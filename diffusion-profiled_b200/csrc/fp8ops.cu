// fp8ops.cu — host side of the C ABI declared in include/fp8ops.h.
//
// One translation unit holds every kernel (quantize.cuh, gemm_kmajor.cuh,
// gemm_wgrad.cuh) so that they share one device error word.  Host code here
// validates arguments, encodes TMA tensor maps, picks tile configurations and
// launches on the caller's stream.  It allocates nothing.
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "fp8ops.h"
#include "gemm_kmajor.cuh"
#include "gemm_wgrad.cuh"
#include "quantize.cuh"
#include "conv_halo.cuh"
#include "conv_halo_t.cuh"
#include "groupnorm.cuh"
#include "layernorm.cuh"
#include "resample.cuh"
#include "optim.cuh"
#include "cast_batch.cuh"
#include "attention.cuh"

using namespace fp8b;

// Device-side error word (one per device that loads this library).
__device__ int g_fp8_device_error = 0;

// Tickets of the last-CTA scale folds (ScaleFold), zero between launches.  Each
// launch that folds gets the next counter of the ring, so launches that can run
// at the same time (other streams) use different counters unless more than
// kFoldCounters folding launches were issued between them.
constexpr int kFoldCounters = 8192;
__device__ unsigned int g_fold_counters[kFoldCounters];

namespace {

constexpr int kMaxDevices = 64;

// Kernels launched through this library since load (graph replays not included).
std::atomic<unsigned long long> g_launches{0};
inline void count_launches(unsigned n) { g_launches.fetch_add(n, std::memory_order_relaxed); }

thread_local int t_last_status = FP8_OK;
thread_local char t_last_msg[512] = {0};

int set_error(int status, const char* fmt, ...) {
  t_last_status = status;
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(t_last_msg, sizeof(t_last_msg), fmt, ap);
  va_end(ap);
  return status;
}

int ok() {
  t_last_status = FP8_OK;
  t_last_msg[0] = 0;
  return FP8_OK;
}

#define FP8_CUDA_TRY(expr)                                                                       \
  do {                                                                                           \
    cudaError_t e_ = (expr);                                                                     \
    if (e_ != cudaSuccess)                                                                       \
      return set_error(FP8_ERR_CUDA, "%s failed: %s (%s:%d)", #expr, cudaGetErrorString(e_),     \
                       __FILE__, __LINE__);                                                      \
  } while (0)

#define FP8_REQUIRE(cond, status, ...)         \
  do {                                         \
    if (!(cond)) return set_error(status, __VA_ARGS__); \
  } while (0)

// ------------------------------------------------------------------ per-device state
struct DeviceState {
  int sm_count = 0;
  int* err_ptr = nullptr;
  unsigned int* fold_base = nullptr;  // g_fold_counters on this device
  std::atomic<unsigned int> fold_next{0};
  // Set (release) after the fields above are written; a reader that sees it
  // (acquire) sees them too.
  std::atomic<bool> init{false};
};
DeviceState g_dev[kMaxDevices];
std::mutex g_dev_mu;

int device_state(DeviceState** out) {
  int dev = 0;
  FP8_CUDA_TRY(cudaGetDevice(&dev));
  FP8_REQUIRE(dev >= 0 && dev < kMaxDevices, FP8_ERR_UNSUPPORTED, "device ordinal %d out of range", dev);
  DeviceState& st = g_dev[dev];
  if (!st.init.load(std::memory_order_acquire)) {
    std::lock_guard<std::mutex> lock(g_dev_mu);
    if (!st.init.load(std::memory_order_relaxed)) {
      FP8_CUDA_TRY(cudaDeviceGetAttribute(&st.sm_count, cudaDevAttrMultiProcessorCount, dev));
      void* p = nullptr;
      FP8_CUDA_TRY(cudaGetSymbolAddress(&p, g_fp8_device_error));
      st.err_ptr = static_cast<int*>(p);
      FP8_CUDA_TRY(cudaGetSymbolAddress(&p, g_fold_counters));
      st.fold_base = static_cast<unsigned int*>(p);
      st.init.store(true, std::memory_order_release);
    }
  }
  *out = &st;
  return FP8_OK;
}

// The counter of the next launch that folds a scale in its last CTA.
unsigned int* fold_counter(DeviceState* st) {
  return st->fold_base + st->fold_next.fetch_add(1, std::memory_order_relaxed) % kFoldCounters;
}

// ------------------------------------------------------------------ TMA tensor maps
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

int get_encode_fn(EncodeTiledFn* out) {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  static cudaError_t status = cudaSuccess;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    status = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
    if (status == cudaSuccess && q == cudaDriverEntryPointSuccess) fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  FP8_REQUIRE(fn != nullptr, FP8_ERR_CUDA, "cuTensorMapEncodeTiled unavailable (%s)", cudaGetErrorString(status));
  *out = fn;
  return FP8_OK;
}

// 2-D byte matrix [rows][cols] (cols contiguous), box = 128 bytes x box_rows, 128B swizzle.
int make_map_2d(CUtensorMap* map, const void* ptr, int64_t rows, int64_t cols, int box_rows) {
  EncodeTiledFn enc = nullptr;
  if (int s = get_encode_fn(&enc)) return s;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(cols)};
  cuuint32_t box[2] = {128u, static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1u, 1u};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  FP8_REQUIRE(r == CUDA_SUCCESS, FP8_ERR_CUDA, "cuTensorMapEncodeTiled(2d %lldx%lld) failed: %d", (long long)rows,
              (long long)cols, (int)r);
  return FP8_OK;
}

// 2-D matrix [rows][cols] of `elem_bytes`-wide elements with row stride `ld`
// elements; box = box_cols x box_rows, 128B swizzle (box_cols * elem_bytes == 128).
// Used for the epilogue TMA stores (bf16 outputs, fp32 split-K partials).
int make_map_2d_store(CUtensorMap* map, const void* ptr, CUtensorMapDataType dtype, int elem_bytes, int64_t rows,
                      int64_t cols, int64_t ld, int box_cols, int box_rows) {
  EncodeTiledFn enc = nullptr;
  if (int s = get_encode_fn(&enc)) return s;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld) * elem_bytes};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(box_cols), static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1u, 1u};
  CUresult r = enc(map, dtype, 2, const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  FP8_REQUIRE(r == CUDA_SUCCESS, FP8_ERR_CUDA, "cuTensorMapEncodeTiled(store %lldx%lld) failed: %d",
              (long long)rows, (long long)cols, (int)r);
  return FP8_OK;
}

int make_map_out_bf16(CUtensorMap* map, const void* ptr, int64_t rows, int64_t cols) {
  return make_map_2d_store(map, ptr, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, rows, cols, cols, 64, 32);
}

// Conv geometry: 128-pixel tiles that cover whole image rows (or whole images).
struct ConvTile {
  int rows;  // image rows per 128-pixel tile
  int imgs;  // images per 128-pixel tile
};

bool conv_tile(int height, int width, ConvTile* t) {
  if (width <= 0 || height <= 0 || width > 128 || 128 % width != 0) return false;
  const int hw = height * width;
  if (hw >= 128) {
    const int rows = 128 / width;
    if (height % rows != 0) return false;
    *t = {rows, 1};
  } else {
    if (128 % hw != 0) return false;
    *t = {height, 128 / hw};
  }
  return true;
}

// 4-D NHWC byte tensor [B][H][W][C]; box = 128 channels x W x rows x imgs, 128B swizzle.
// Out-of-range coordinates (the conv padding ring, images past the batch) read as 0.
int make_map_conv(CUtensorMap* map, const void* ptr, int batch, int height, int width, int channels,
                  const ConvTile& t) {
  EncodeTiledFn enc = nullptr;
  if (int s = get_encode_fn(&enc)) return s;
  cuuint64_t dims[4] = {static_cast<cuuint64_t>(channels), static_cast<cuuint64_t>(width),
                        static_cast<cuuint64_t>(height), static_cast<cuuint64_t>(batch)};
  cuuint64_t strides[3] = {static_cast<cuuint64_t>(channels), static_cast<cuuint64_t>(width) * channels,
                           static_cast<cuuint64_t>(height) * width * channels};
  cuuint32_t box[4] = {128u, static_cast<cuuint32_t>(width), static_cast<cuuint32_t>(t.rows),
                       static_cast<cuuint32_t>(t.imgs)};
  cuuint32_t estr[4] = {1u, 1u, 1u, 1u};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, const_cast<void*>(ptr), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  FP8_REQUIRE(r == CUDA_SUCCESS, FP8_ERR_CUDA, "cuTensorMapEncodeTiled(conv %dx%dx%dx%d) failed: %d", batch,
              height, width, channels, (int)r);
  return FP8_OK;
}

bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// Programmatic dependent launch: 0 = plain stream order (the default), 1 = the
// tensor-core kernels, 2 = every kernel.  Each kernel waits for its predecessor
// (pdl_sync / pdl_wait) before touching global memory, so the attribute only
// lets its CTAs start, and run their prologue, while the previous kernel's CTAs
// drain.  Measured on B200: a conv kernel following another conv kernel gains
// 0.5-1 us, but the quantize -> conv chains of a training step gain nothing
// (their streaming kernels leave no SM free early), so it is off by default.
int g_pdl = 0;

// History entry of an all-zero tensor in the delayed-scaling windows:
// 0 = the reference's (its scale, 1.0), 1 = 0.0 (fp8_set_empty_tensor_history).
int g_empty_zero = 0;

// Current-scaling quantize: 1 = the one-launch shared-memory-resident kernel where it
// applies (default), 0 = always the two passes (fp8_set_quantize_resident).
int g_quant_resident = 1;

// Weight gradient: 1 = the bf16 / fp32 conversion folded into the split-K kernel (a
// cooperative launch) where the grid fits one CTA per SM, 0 = a separate launch (default:
// measured on config 2, the cooperative launch and grid barrier cost more than the
// conversion launch they replace, 25.8 vs 24.6 us for the whole dW).
int g_wgrad_fused = 0;

enum KernelClass { kStreamingKernel = 0, kTensorKernel = 1 };

// Launch `kern` on `stream`, with programmatic stream serialization when enabled
// for its class, optionally as clusters of `cluster_x` CTAs.
template <typename... KArgs, typename... Args>
cudaError_t launch_kernel(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                          int cluster_x, KernelClass cls, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  unsigned n = 0;
  if (g_pdl == 2 || (g_pdl == 1 && cls == kTensorKernel)) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  if (cluster_x > 1) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = static_cast<unsigned>(cluster_x);
    attr[n].val.clusterDim.y = 1;
    attr[n].val.clusterDim.z = 1;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  return cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
}

// Batched byte transpose dst[b][c][r] = src[b][r][c]; whole 16-byte-aligned
// 64x64 tiles take the vectorised kernel.
int launch_transpose(const void* src, void* dst, int64_t rows, int64_t cols, int64_t src_ld, int64_t dst_ld,
                     int64_t src_bstride, int64_t dst_bstride, int batch, cudaStream_t stream) {
  const int64_t gx = (rows + kTransTile - 1) / kTransTile, gy = (cols + kTransTile - 1) / kTransTile;
  FP8_REQUIRE(gx < (1ll << 31) && gy <= 65535 && batch <= 65535, FP8_ERR_UNSUPPORTED, "transpose too large");
  dim3 grid(static_cast<unsigned>(gx), static_cast<unsigned>(gy), static_cast<unsigned>(batch));
  const bool tiles16 = rows % kTransTile == 0 && cols % kTransTile == 0 && src_ld % 16 == 0 && dst_ld % 16 == 0 &&
                       src_bstride % 16 == 0 && dst_bstride % 16 == 0 && aligned(src, 16) && aligned(dst, 16);
  if (tiles16)
    FP8_CUDA_TRY(launch_kernel(transpose_u8_tiles16_kernel, grid, dim3(256), 0, stream, 1, kStreamingKernel,
                               static_cast<const uint8_t*>(src), static_cast<uint8_t*>(dst), src_ld, dst_ld,
                               src_bstride, dst_bstride));
  else
    FP8_CUDA_TRY(launch_kernel(transpose_u8_kernel, grid, dim3(256), 0, stream, 1, kStreamingKernel,
                               static_cast<const uint8_t*>(src), static_cast<uint8_t*>(dst), rows, cols, src_ld, dst_ld,
                               src_bstride, dst_bstride));
  count_launches(1);
  return FP8_OK;
}

// ------------------------------------------------------------------ tuning overrides
int g_override_bm_sub = 0;
int g_override_bn = 0;
int g_override_group = 0;
// 0 auto, 1 tap-by-tap K-major GEMM, 2 halo kernel, 3 CTA-pair halo, 4 transposed halo (where they apply)
int g_conv_algo = 0;

// ------------------------------------------------------------------ halo conv launch
// NHWC map whose box is (128 channels, W, R+2 rows, 1 image): the rows of one
// 128-pixel tile plus one halo row on each side.
int make_map_conv_halo(CUtensorMap* map, const void* ptr, int batch, int height, int width, int channels,
                       int rows_per_tile) {
  EncodeTiledFn enc = nullptr;
  if (int s = get_encode_fn(&enc)) return s;
  cuuint64_t dims[4] = {static_cast<cuuint64_t>(channels), static_cast<cuuint64_t>(width),
                        static_cast<cuuint64_t>(height), static_cast<cuuint64_t>(batch)};
  cuuint64_t strides[3] = {static_cast<cuuint64_t>(channels), static_cast<cuuint64_t>(width) * channels,
                           static_cast<cuuint64_t>(height) * width * channels};
  cuuint32_t box[4] = {128u, static_cast<cuuint32_t>(width), static_cast<cuuint32_t>(rows_per_tile + 2), 1u};
  cuuint32_t estr[4] = {1u, 1u, 1u, 1u};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, const_cast<void*>(ptr), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  FP8_REQUIRE(r == CUDA_SUCCESS, FP8_ERR_CUDA, "cuTensorMapEncodeTiled(conv halo %dx%dx%dx%d) failed: %d", batch,
              height, width, channels, (int)r);
  return FP8_OK;
}

// The halo kernel needs 128-pixel tiles inside one image with 1024-byte aligned
// row shifts: W in {16, 32} (every 32x32 and 16x16 shape of the UNet).
bool halo_applies(int height, int width) {
  return (width == 32 || width == 16) && (height * width) % 128 == 0 && height % (128 / width) == 0;
}

template <int BN, bool RES, int W>
int launch_halo_cfg(const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& mo, const HaloParams& p,
                    int sm_count, cudaStream_t stream) {
  using Cfg = HaloConfig<BN, RES, W>;
  auto kern = conv_halo_fp8_kernel<BN, RES, W>;
  FP8_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmemBytes));
  int grid;
  if (RES) {
    // every CTA owns one column tile (its weights stay in smem)
    const int per_n = std::max(1, std::min(sm_count / p.num_n_tiles, p.num_m_tiles));
    grid = per_n * p.num_n_tiles;
  } else {
    grid = std::min(sm_count, p.num_m_tiles * p.num_n_tiles);
  }
  FP8_CUDA_TRY(launch_kernel(kern, dim3(grid), dim3(kGemmThreads), Cfg::kSmemBytes, stream, 1, kTensorKernel, ma, mb,
                             mo, p));
  count_launches(1);
  return FP8_OK;
}

// Clusters of two CTAs that can be resident at once (cached per device).
std::atomic<int> g_pair_clusters[kMaxDevices] = {};

template <int W>
int launch_halo_pair(const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& mo, const HaloParams& p,
                     int sm_count, cudaStream_t stream) {
  using Cfg = HaloPairConfig<W>;
  auto kern = conv_halo_pair_fp8_kernel<W>;
  FP8_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmemBytes));
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.blockDim = dim3(kGemmThreads, 1, 1);
  cfg.dynamicSmemBytes = Cfg::kSmemBytes;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int dev = 0;
  FP8_CUDA_TRY(cudaGetDevice(&dev));
  int max_pairs = (dev >= 0 && dev < kMaxDevices) ? g_pair_clusters[dev].load(std::memory_order_relaxed) : 0;
  if (max_pairs <= 0) {
    cfg.gridDim = dim3(static_cast<unsigned>(sm_count & ~1), 1, 1);
    FP8_CUDA_TRY(cudaOccupancyMaxActiveClusters(&max_pairs, kern, &cfg));
    if (max_pairs <= 0) max_pairs = sm_count / 2;
    if (dev >= 0 && dev < kMaxDevices) g_pair_clusters[dev].store(max_pairs, std::memory_order_relaxed);
  }
  // Every pair keeps one column tile's weights resident: a whole number of pairs per column tile.
  const int pair_tiles = p.num_m_tiles / 2;
  const int per_n = std::max(1, std::min(max_pairs / p.num_n_tiles, pair_tiles));
  FP8_CUDA_TRY(launch_kernel(kern, dim3(static_cast<unsigned>(2 * per_n * p.num_n_tiles)), dim3(kGemmThreads),
                             Cfg::kSmemBytes, stream, 2, kTensorKernel, ma, mb, mo, p));
  count_launches(1);
  return FP8_OK;
}

template <int W, bool A_MN = false>
int launch_halo_t(const CUtensorMap& ma, const CUtensorMap& mw, HaloTParams p, int sm_count, cudaStream_t stream) {
  using Cfg = HaloTConfig<W>;
  auto kern = conv_halo_t_fp8_kernel<W, A_MN>;
  FP8_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmemBytes));
  // Every CTA keeps one column tile's weights resident: a whole number of CTAs per column tile.
  const int per_n = std::max(1, std::min(sm_count / p.num_n_tiles, p.full_tiles));
  p.whole_tiles = (p.full_tiles / per_n) * per_n;
  FP8_CUDA_TRY(launch_kernel(kern, dim3(per_n * p.num_n_tiles), dim3(kGemmThreads), Cfg::kSmemBytes, stream, 1,
                             kTensorKernel, ma, mw, p));
  count_launches(1);
  return FP8_OK;
}

// The forward's weights [Cout][3][3][Cin] as a 3-D map (Cin, tap, Cout) with box
// (128, 1, 128): one tap's 128 x 128 block, Cout rows of 128 Cin bytes (the
// data-grad's MN-major A operand).
int make_map_weight_taps(CUtensorMap* map, const void* wq, int cout, int cin) {
  EncodeTiledFn enc = nullptr;
  if (int s = get_encode_fn(&enc)) return s;
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(cin), 9u, static_cast<cuuint64_t>(cout)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(cin), static_cast<cuuint64_t>(9) * cin};
  cuuint32_t box[3] = {128u, 1u, 128u};
  cuuint32_t estr[3] = {1u, 1u, 1u};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(wq), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  FP8_REQUIRE(r == CUDA_SUCCESS, FP8_ERR_CUDA, "cuTensorMapEncodeTiled(weight taps %dx9x%d) failed: %d", cout, cin,
              (int)r);
  return FP8_OK;
}

// The transposed halo kernel: 128 reduced channels, whole 128-channel output
// tiles, 256-pixel tiles inside one image, 4-byte aligned output rows.
bool halo_t_applies(int height, int width, int c_red, int n_out, const void* out) {
  return (width == 32 || width == 16) && c_red == 128 && n_out % 128 == 0 && (height * width) % 256 == 0 &&
         aligned(out, 4);
}

// Conv fwd / data-grad with the halo kernel.  act: NHWC e4m3 input of the GEMM
// (X for fwd, dY for data-grad) with `c_red` channels; wmat: K-major weights
// [n_out][9*c_red]; out: NHWC bf16 [B*H*W][n_out].
int launch_conv_halo(const void* act, const void* wmat, void* out, const float* sa, const float* sb,
                     const void* bias, int epilogue, int batch, int height, int width, int c_red, int n_out,
                     bool fwd, int* err, int sm_count, cudaStream_t stream, bool w_natural = false) {
  const int rows = 128 / width;
  const int64_t M = static_cast<int64_t>(batch) * height * width;
  if ((g_conv_algo == 0 || g_conv_algo == 4) && halo_t_applies(height, width, c_red, n_out, out)) {
    CUtensorMap ma, mw;
    if (int s = make_map_conv_halo(&ma, act, batch, height, width, c_red, 2 * rows)) return s;
    if (w_natural) {  // data-grad on the forward's [Cout = c_red][3][3][Cin = n_out] weights
      if (int s = make_map_weight_taps(&mw, wmat, c_red, n_out)) return s;
    } else {
      if (int s = make_map_2d(&mw, wmat, n_out, 9ll * c_red, 128)) return s;
    }
    HaloTParams t{};
    t.num_n_tiles = n_out / 128;
    t.full_tiles = static_cast<int>(M / 256);
    t.HW = height * width;
    t.W = width;
    t.fwd = fwd ? 1 : 0;
    t.N = n_out;
    t.scale_a = sa;
    t.scale_b = sb;
    t.bias = static_cast<const __nv_bfloat16*>(bias);
    t.out = static_cast<__nv_bfloat16*>(out);
    t.epilogue = epilogue;
    t.err = err;
    if (w_natural) {
      if (width == 32) return launch_halo_t<32, true>(ma, mw, t, sm_count, stream);
      return launch_halo_t<16, true>(ma, mw, t, sm_count, stream);
    }
    if (width == 32) return launch_halo_t<32>(ma, mw, t, sm_count, stream);
    return launch_halo_t<16>(ma, mw, t, sm_count, stream);
  }
  FP8_REQUIRE(!w_natural, FP8_ERR_UNSUPPORTED, "natural-layout weights need the transposed halo kernel");
  const bool resident = (c_red == 128);
  // CTA pairs (only on request: measured slower than the single-CTA kernel on
  // config 2): 128 reduced channels, whole 128-column tiles, 256-pixel tiles
  // inside one image.
  const bool pair = resident && g_conv_algo == 3 && n_out % 128 == 0 && (height * width) % 256 == 0;
  const int bn = resident ? 128 : (n_out % 256 == 0 ? 256 : 128);
  CUtensorMap ma, mb, mo;
  if (int s = make_map_conv_halo(&ma, act, batch, height, width, c_red, rows)) return s;
  if (int s = make_map_2d(&mb, wmat, n_out, 9ll * c_red, pair ? 64 : bn)) return s;
  if (int s = make_map_out_bf16(&mo, out, M, n_out)) return s;
  HaloParams p{};
  p.num_n_tiles = n_out / bn;
  p.num_m_tiles = static_cast<int>(M / 128);
  p.cchunks = c_red / 128;
  p.HW = height * width;
  p.W = width;
  p.R = rows;
  p.fwd = fwd ? 1 : 0;
  p.N = n_out;
  p.scale_a = sa;
  p.scale_b = sb;
  p.bias = static_cast<const __nv_bfloat16*>(bias);
  p.epilogue = epilogue;
  p.err = err;
  if (pair) {
    if (width == 32) return launch_halo_pair<32>(ma, mb, mo, p, sm_count, stream);
    return launch_halo_pair<16>(ma, mb, mo, p, sm_count, stream);
  }
  if (width == 32) {
    if (resident) return launch_halo_cfg<128, true, 32>(ma, mb, mo, p, sm_count, stream);
    if (bn == 256) return launch_halo_cfg<256, false, 32>(ma, mb, mo, p, sm_count, stream);
    return launch_halo_cfg<128, false, 32>(ma, mb, mo, p, sm_count, stream);
  }
  if (resident) return launch_halo_cfg<128, true, 16>(ma, mb, mo, p, sm_count, stream);
  if (bn == 256) return launch_halo_cfg<256, false, 16>(ma, mb, mo, p, sm_count, stream);
  return launch_halo_cfg<128, false, 16>(ma, mb, mo, p, sm_count, stream);
}

// ------------------------------------------------------------------ K-major GEMM launch
template <int BM_SUB, int BN, int STAGES, int EPI = kEpiWarps>
int launch_kgemm_cfg(const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& mo, KGemmParams p,
                     int sm_count, cudaStream_t stream) {
  using Cfg = KGemmConfig<BM_SUB, BN, STAGES, EPI>;
  auto kern = kgemm_fp8_kernel<BM_SUB, BN, STAGES, EPI>;
  FP8_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmemBytes));
  const int grid = p.num_tiles < sm_count ? p.num_tiles : sm_count;
  FP8_CUDA_TRY(launch_kernel(kern, dim3(grid), dim3(Cfg::kThreads), Cfg::kSmemBytes, stream, 1, kTensorKernel, ma,
                             mb, mo, p));
  count_launches(1);
  return FP8_OK;
}

struct KGemmShape {
  int64_t M, N;
  int k_blocks;
  bool plain = false;  // plain GEMM (no conv window)
};

// Plain GEMMs with at most this many 128-byte K blocks take the eight-epilogue-warp
// instances (their tile time is the epilogue's) and column tiles of 256 or 128.
constexpr int kShortKBlocks = 8;

void choose_kgemm_tile(const KGemmShape& s, int sm_count, int* bm_sub, int* bn) {
  if (g_override_bn > 0 && s.N % g_override_bn == 0) {
    *bn = g_override_bn;
    *bm_sub = g_override_bm_sub > 0 ? g_override_bm_sub : 1;
    if (*bm_sub == 2 && *bn == 256) *bm_sub = 1;
    if (*bm_sub == 2 && *bn == 64) *bm_sub = 1;
    return;
  }
  // The widest column tile that still gives about a wave of tiles (>= 80 % of the
  // SMs): narrow N = 64 MMAs lose to the per-stage commit bubble, so 128 tiles of
  // N = 128 beat 256 of N = 64 (8x8 convs at B = 128: 11.4 vs 17.3 us); with
  // fewer tiles than that at every width, the narrowest (most tiles).
  const int64_t m_tiles = (s.M + 127) / 128;
  *bm_sub = 1;
  // Short-K plain GEMMs: 256 columns where that gives about a wave, else 128 (their
  // 64-column tiles measured slower: config 1 14.3 vs 11.3 / 9.1 us at 128 / 256, and the
  // time-embedding GEMM 128 x 11264 x 512 5.7 vs 4.8 us at 128).
  if (s.plain && s.k_blocks <= kShortKBlocks && s.N % 128 == 0) {
    *bn = (s.N % 256 == 0 && m_tiles * (s.N / 256) * 5 >= static_cast<int64_t>(sm_count) * 4) ? 256 : 128;
    return;
  }
  for (int cand : {256, 128, 64}) {
    if (s.N % cand != 0 && !(cand == 64 && s.N % 32 == 0)) continue;
    const int64_t tiles = m_tiles * ((s.N + cand - 1) / cand);
    *bn = cand;
    if (tiles * 5 >= static_cast<int64_t>(sm_count) * 4) return;
  }
}

int launch_kgemm(const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& mo, KGemmParams p, int bm_sub,
                 int bn, int sm_count, cudaStream_t stream) {
  const int64_t m_tiles = (static_cast<int64_t>(p.M) + 128 * bm_sub - 1) / (128 * bm_sub);
  p.num_n_tiles = (p.N + bn - 1) / bn;
  const int64_t tiles = m_tiles * p.num_n_tiles;
  FP8_REQUIRE(tiles < (1ll << 31), FP8_ERR_UNSUPPORTED, "too many tiles");
  p.num_tiles = static_cast<int>(tiles);
  // Short reductions (plain GEMMs of a few K blocks): the epilogue, not the MMAs, sets the
  // tile rate, so eight epilogue warps drain the accumulators (tiles of at least two
  // 64-column chunks; a 64-column tile keeps four).
  if (p.a_conv == 0 && p.k_blocks <= kShortKBlocks) {
    if (bm_sub == 1 && bn == 128) return launch_kgemm_cfg<1, 128, 4, 8>(ma, mb, mo, p, sm_count, stream);
    if (bm_sub == 1 && bn == 256) return launch_kgemm_cfg<1, 256, 3, 8>(ma, mb, mo, p, sm_count, stream);
    if (bm_sub == 2 && bn == 128) return launch_kgemm_cfg<2, 128, 3, 8>(ma, mb, mo, p, sm_count, stream);
  }
  if (bm_sub == 1 && bn == 64) return launch_kgemm_cfg<1, 64, 8>(ma, mb, mo, p, sm_count, stream);
  if (bm_sub == 1 && bn == 128) return launch_kgemm_cfg<1, 128, 6>(ma, mb, mo, p, sm_count, stream);
  if (bm_sub == 1 && bn == 256) return launch_kgemm_cfg<1, 256, 4>(ma, mb, mo, p, sm_count, stream);
  if (bm_sub == 2 && bn == 128) return launch_kgemm_cfg<2, 128, 4>(ma, mb, mo, p, sm_count, stream);
  return set_error(FP8_ERR_UNSUPPORTED, "no K-major GEMM instance for bm_sub=%d bn=%d", bm_sub, bn);
}

int check_scale_ptrs(const float* a, const float* b) {
  FP8_REQUIRE(a != nullptr && b != nullptr, FP8_ERR_INVALID_ARGUMENT, "scale pointers must be non-NULL");
  FP8_REQUIRE(aligned(a, 4) && aligned(b, 4), FP8_ERR_INVALID_ARGUMENT, "scale pointers must be 4-byte aligned");
  return FP8_OK;
}

int check_conv_args(int batch, int height, int width, int cin, int cout, ConvTile* t) {
  FP8_REQUIRE(batch > 0 && height > 0 && width > 0 && cin > 0 && cout > 0, FP8_ERR_INVALID_ARGUMENT,
              "conv sizes must be positive (B=%d H=%d W=%d Cin=%d Cout=%d)", batch, height, width, cin, cout);
  FP8_REQUIRE(cin % 128 == 0 && cout % 128 == 0, FP8_ERR_UNSUPPORTED,
              "conv channels must be multiples of 128 (Cin=%d Cout=%d)", cin, cout);
  FP8_REQUIRE(conv_tile(height, width, t), FP8_ERR_UNSUPPORTED,
              "conv spatial %dx%d not tileable into 128-pixel row/image tiles", height, width);
  FP8_REQUIRE(static_cast<int64_t>(batch) * height * width < (1ll << 31), FP8_ERR_UNSUPPORTED,
              "conv pixel count too large");
  return FP8_OK;
}

// ------------------------------------------------------------------ weight-gradient launch
template <int G, bool HALO = false>
int launch_wgrad_cfg(const CUtensorMap& mdy, const CUtensorMap& mb, const CUtensorMap& mp, WGradParams p,
                     cudaStream_t stream) {
  using Cfg = WGradConfig<G, HALO>;
  auto kern = wgrad_fp8_kernel<G, HALO>;
  FP8_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmemBytes));
  if (p.grid_arrive != nullptr) {
    // fused conversion: every CTA must be resident for the grid barrier
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(p.num_tiles * p.splits));
    cfg.blockDim = dim3(kGemmThreads);
    cfg.dynamicSmemBytes = Cfg::kSmemBytes;
    cfg.stream = stream;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeCooperative;
    at[0].val.cooperative = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    FP8_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, mdy, mb, mp, p));
  } else {
    FP8_CUDA_TRY(launch_kernel(kern, dim3(p.num_tiles * p.splits), dim3(kGemmThreads), Cfg::kSmemBytes, stream, 1,
                               kTensorKernel, mdy, mb, mp, p));
  }
  count_launches(1);
  return FP8_OK;
}

struct WGradPlan {
  int group;
  int num_groups;
  int num_tiles;
  int splits;
  int k_blocks;
};

WGradPlan plan_wgrad(int64_t m_rows, int64_t n_cols, int64_t pixels, int split_k, int sm_count) {
  WGradPlan w{};
  const int boxes = static_cast<int>(n_cols / 128);
  // Wider column groups share each dY box among more MMAs (less L2->SMEM traffic
  // per FLOP): 3 boxes (384 TMEM columns) when the column count allows it.
  w.group = boxes % 3 == 0 ? 3 : (boxes % 2 == 0 ? 2 : 1);
  if (g_override_group > 0 && boxes % g_override_group == 0) w.group = g_override_group;
  w.num_groups = boxes / w.group;
  w.num_tiles = static_cast<int>(m_rows / 128) * w.num_groups;
  w.k_blocks = static_cast<int>((pixels + 127) / 128);
  int s = split_k;
  if (s <= 0) {
    s = sm_count / w.num_tiles;
    if (s < 1) s = 1;
  }
  if (s > w.k_blocks) s = w.k_blocks;
  w.splits = s;
  return w;
}

// halo: mb is a halo map (make_map_conv_halo) and group == 3.
int launch_wgrad(const CUtensorMap& mdy, const CUtensorMap& mb, WGradParams p, int group, cudaStream_t stream,
                 bool halo = false) {
  CUtensorMap mp;
  if (int s = make_map_2d_store(&mp, p.acc, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, p.m_rows, p.n_cols, p.n_cols, 32,
                                32))
    return s;
  FP8_CUDA_TRY(cudaMemsetAsync(p.acc, 0, static_cast<size_t>(p.m_rows) * p.n_cols * sizeof(float), stream));
  if (halo) {
    FP8_REQUIRE(group == 3, FP8_ERR_UNSUPPORTED, "halo weight-gradient needs group 3, got %d", group);
    return launch_wgrad_cfg<3, true>(mdy, mb, mp, p, stream);
  }
  if (group == 1) return launch_wgrad_cfg<1>(mdy, mb, mp, p, stream);
  if (group == 2) return launch_wgrad_cfg<2>(mdy, mb, mp, p, stream);
  if (group == 3) return launch_wgrad_cfg<3>(mdy, mb, mp, p, stream);
  return set_error(FP8_ERR_UNSUPPORTED, "no weight-gradient instance for group=%d", group);
}

// Weight-gradient launch with the conversion folded in when the grid fits one CTA per SM
// (g_wgrad_fused); otherwise the split-K kernel and then wgrad_reduce_kernel.
int launch_wgrad_reduce(const float* partials, int splits, int64_t count, const float* sa, const float* sb,
                        void* out, int sm_count, cudaStream_t stream, bool f32_out);
int launch_wgrad_converted(const CUtensorMap& mdy, const CUtensorMap& mb, WGradParams p, int group, cudaStream_t stream,
                           bool halo, const float* sa, const float* sb, void* out, bool f32_out, DeviceState* st) {
  if (g_wgrad_fused && p.num_tiles * p.splits <= st->sm_count) {
    p.grid_arrive = fold_counter(st);
    p.grid_depart = fold_counter(st);
    p.scale_a = sa;
    p.scale_b = sb;
    p.out = out;
    p.out_f32 = f32_out ? 1 : 0;
    return launch_wgrad(mdy, mb, p, group, stream, halo);
  }
  if (int s = launch_wgrad(mdy, mb, p, group, stream, halo)) return s;
  return launch_wgrad_reduce(p.acc, 1, static_cast<int64_t>(p.m_rows) * p.n_cols, sa, sb, out, st->sm_count, stream,
                             f32_out);
}

int launch_wgrad_reduce(const float* partials, int splits, int64_t count, const float* sa, const float* sb,
                        void* out, int sm_count, cudaStream_t stream, bool f32_out) {
  const int64_t n4 = count / 4;
  int64_t blocks = (n4 + 255) / 256;
  if (blocks > 4 * sm_count) blocks = 4 * sm_count;
  if (blocks < 1) blocks = 1;
  if (f32_out)
    FP8_CUDA_TRY(launch_kernel(wgrad_reduce_kernel<float>, dim3(static_cast<unsigned>(blocks)), dim3(256), 0, stream,
                               1, kStreamingKernel, partials, splits, count, sa, sb, static_cast<float*>(out)));
  else
    FP8_CUDA_TRY(launch_kernel(wgrad_reduce_kernel<__nv_bfloat16>, dim3(static_cast<unsigned>(blocks)), dim3(256), 0,
                               stream, 1, kStreamingKernel, partials, splits, count, sa, sb,
                               static_cast<__nv_bfloat16*>(out)));
  count_launches(1);
  return FP8_OK;
}

// ------------------------------------------------------------------ group norm helpers
// CTAs per sample.  Each kernel gets as many as one wave of it holds (its
// occupancy x SMs, rounded down to whole CTAs per sample: a second, partial
// wave would cost a whole wave's time), with at least one row step of pixels
// each.  The partial sums of one kernel are merged by the next with the
// writer's count (GnShape::part_slices), so the two may differ.
int gn_slices_cap(int n, int hw, int c, int sm_count) {
  const int rows = kGnThreads / (c / 8);
  return std::max(1, std::min(8 * sm_count / std::max(n, 1), hw / rows));
}

template <typename K>
int gn_kernel_slices(K kern, size_t smem, int n, int hw, int c, int sm_count, int* slices) {
  int occ = 0;
  FP8_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, kGnThreads, smem));
  const int s = occ * sm_count / std::max(n, 1);
  *slices = std::max(1, std::min(s, gn_slices_cap(n, hw, c, sm_count)));
  return FP8_OK;
}

size_t gn_workspace(int n, int hw, int c, int sm_count) {
  return static_cast<size_t>(n) * gn_slices_cap(n, hw, c, sm_count) * 3 * c * sizeof(float);
}

template <typename TX, bool QUANT>
int launch_gn_fwd(const TX* x, GnShape sh, float* part, const GnActParams& q, float* stats, const GnOut& o,
                  size_t s1, size_t s2, int sm_count, cudaStream_t cs) {
  const bool drop = q.seed != nullptr && q.p > 0.0f;
  auto k1 = gn_stats_kernel<TX>;
  auto k2 = drop ? gn_act_fwd_kernel<TX, QUANT, true> : gn_act_fwd_kernel<TX, QUANT, false>;
  FP8_CUDA_TRY(cudaFuncSetAttribute(k1, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(s1)));
  FP8_CUDA_TRY(cudaFuncSetAttribute(k2, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(s2)));
  int sl1 = 1, sl2 = 1;
  if (int s = gn_kernel_slices(k1, s1, sh.n, sh.hw, sh.c, sm_count, &sl1)) return s;
  if (int s = gn_kernel_slices(k2, s2, sh.n, sh.hw, sh.c, sm_count, &sl2)) return s;
  const dim3 block(kGnThreads);
  sh.slices = sh.part_slices = sl1;
  FP8_CUDA_TRY(launch_kernel(k1, dim3(static_cast<unsigned>(sh.n * sl1)), block, s1, cs, 1, kStreamingKernel, x, sh,
                             part));
  sh.slices = sl2;
  FP8_CUDA_TRY(launch_kernel(k2, dim3(static_cast<unsigned>(sh.n * sl2)), block, s2, cs, 1, kStreamingKernel, x, sh,
                             static_cast<const float*>(part), q, stats, o));
  count_launches(2);
  return FP8_OK;
}

template <typename TX>
int launch_gn_bwd(const TX* x, const uint16_t* dy, GnShape sh, const float* stats, const GnActParams& q,
                  float* part, float* totals, TX* dx, size_t s1, size_t s2, int sm_count, cudaStream_t cs,
                  const GnOut* quant = nullptr, const TX* dx_add = nullptr) {
  const bool drop = q.seed != nullptr && q.p > 0.0f;
  auto k1 = drop ? gn_act_bwd_reduce_kernel<TX, true> : gn_act_bwd_reduce_kernel<TX, false>;
  auto k2 = drop ? gn_act_bwd_apply_kernel<TX, true, false> : gn_act_bwd_apply_kernel<TX, false, false>;
  if (quant != nullptr) {
    if constexpr (sizeof(TX) == 2)
      k2 = drop ? gn_act_bwd_apply_kernel<TX, true, true> : gn_act_bwd_apply_kernel<TX, false, true>;
    else
      return set_error(FP8_ERR_UNSUPPORTED, "the e4m3 group-norm gradient needs a bf16 x");
  }
  FP8_CUDA_TRY(cudaFuncSetAttribute(k1, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(s1)));
  FP8_CUDA_TRY(cudaFuncSetAttribute(k2, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(s2)));
  int sl1 = 1, sl2 = 1;
  if (int s = gn_kernel_slices(k1, s1, sh.n, sh.hw, sh.c, sm_count, &sl1)) return s;
  if (int s = gn_kernel_slices(k2, s2, sh.n, sh.hw, sh.c, sm_count, &sl2)) return s;
  const dim3 block(kGnThreads);
  sh.slices = sh.part_slices = sl1;
  FP8_CUDA_TRY(launch_kernel(k1, dim3(static_cast<unsigned>(sh.n * sl1)), block, s1, cs, 1, kStreamingKernel, x, dy,
                             sh, stats, q, part));
  sh.slices = sl2;
  FP8_CUDA_TRY(launch_kernel(k2, dim3(static_cast<unsigned>(sh.n * sl2)), block, s2, cs, 1, kStreamingKernel, x, dy,
                             sh, stats, q, static_cast<const float*>(part), totals, dx,
                             quant != nullptr ? *quant : GnOut{nullptr, nullptr, DelayedSource{}, nullptr, ScaleFold{}},
                             dx_add));
  count_launches(2);
  return FP8_OK;
}

int check_gn_args(const void* x, const void* out, const float* gamma, const float* beta, int n, int hw, int c,
                  int groups, int film_ld, const void* film, float p, float eps) {
  FP8_REQUIRE(n > 0 && hw > 0 && c > 0 && groups > 0, FP8_ERR_INVALID_ARGUMENT, "bad group-norm sizes");
  FP8_REQUIRE(c % 8 == 0 && c <= 512 && c % groups == 0, FP8_ERR_UNSUPPORTED,
              "group norm needs c %% 8 == 0, c <= 512, c %% groups == 0 (c=%d, groups=%d)", c, groups);
  FP8_REQUIRE(x && out && gamma && beta, FP8_ERR_INVALID_ARGUMENT, "NULL tensor");
  FP8_REQUIRE(aligned(x, 16) && aligned(out, 16), FP8_ERR_INVALID_ARGUMENT, "activations must be 16-byte aligned");
  FP8_REQUIRE(film == nullptr || film_ld >= 2 * c, FP8_ERR_INVALID_ARGUMENT, "film_ld must be >= 2c");
  FP8_REQUIRE(p >= 0.0f && p < 1.0f, FP8_ERR_INVALID_ARGUMENT, "dropout p must be in [0, 1)");
  FP8_REQUIRE(eps > 0.0f, FP8_ERR_INVALID_ARGUMENT, "eps must be > 0");
  return FP8_OK;
}

// ------------------------------------------------------------------ quantize launch helpers
// 16-byte aligned x with 8-byte aligned q takes the streaming kernels
// (quant_stream_kernel); anything else takes the grid-stride scalar kernels.
constexpr int kMaxQuantBlocksPerSm = 8;
constexpr int kMaxStreamBlocksPerSm = 3;  // 3 x kStreamSmemBytes fit in one SM's shared memory
int g_quant_amax_bps = 2;                 // CTAs per SM (grid cap) of the amax pass
int g_quant_cast_bps = 2;                 // CTAs per SM (grid cap) of the cast pass

int quant_grid(int64_t n, bool vec, int blocks_per_sm, int sm_count) {
  int64_t blocks;
  if (vec) {
    blocks = ((n & ~int64_t(7)) * 2 + kStreamChunkBytes - 1) / kStreamChunkBytes;
    if (blocks_per_sm > kMaxStreamBlocksPerSm) blocks_per_sm = kMaxStreamBlocksPerSm;
  } else {
    blocks = (n + kQuantThreads - 1) / kQuantThreads;
  }
  const int64_t cap = static_cast<int64_t>(sm_count) * blocks_per_sm;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  return static_cast<int>(blocks);
}

template <int KIND>
int launch_stream(int grid, const uint16_t* x, uint8_t* q, int64_t n, const float* partials_in, int n_partials,
                  DelayedSource prev_scale, float* scale_out, float* partials_out, int* err, cudaStream_t cs,
                  ScaleFold fold = ScaleFold{}) {
  FP8_CUDA_TRY(cudaFuncSetAttribute(quant_stream_kernel<KIND>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    static_cast<int>(kStreamSmemBytes)));
  FP8_CUDA_TRY(launch_kernel(quant_stream_kernel<KIND>, dim3(grid), dim3(kStreamThreads), kStreamSmemBytes, cs, 1,
                             kStreamingKernel, x, q, n, partials_in, n_partials, prev_scale, scale_out, partials_out,
                             err, fold));
  return FP8_OK;
}

// Current scaling: amax pass (parts CTAs, one partial each), then the cast pass.
// The shared-memory-resident current quantize (quant_resident_kernel) for the
// tensors of `m`, if it applies: every n a multiple of 8 (x 16-byte, q 8-byte
// aligned: the caller's vec path), at least 6 MB of bf16 in all (measured on one
// box: a 6.3 MB input + weight pair 8.0-11.3 us vs 12.8 us for the two passes, an
// 8.4 MB input 7.8-9.2 vs 10.1 us; a 4.2 MB input alone 7.0-9.9 vs 7.7 us, so
// smaller tensors keep the two passes) and each CTA's slices within its shared
// memory.  *launched = false otherwise.  It needs no workspace: the barrier and
// the maxima use words from the library's pool of self-resetting counters.
int launch_quant_resident(const MultiQuant& m, DeviceState* st, cudaStream_t cs, bool* launched) {
  *launched = false;
  const int G = st->sm_count;
  int64_t bytes = 0, smem = 0;
  for (int t = 0; t < m.count; ++t) {
    if (m.n[t] % 8 != 0) return FP8_OK;
    bytes += m.n[t] * 2;
    smem += ((m.n[t] / 8 + G - 1) / G) * 16;
  }
  if (bytes < (6 << 20) || smem > kResSmemCap) return FP8_OK;
  static std::once_flag once;
  static cudaError_t attr = cudaSuccess;
  std::call_once(once, [] {
    attr = cudaFuncSetAttribute(quant_resident_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kResSmemCap);
  });
  FP8_CUDA_TRY(attr);
  ResSlices sl{};
  ResSync sy{};
  sy.arrive = fold_counter(st);
  sy.depart = fold_counter(st);
  for (int t = 0; t < m.count; ++t) {
    sl.vq[t] = (m.n[t] / 8) / G;
    sl.vr[t] = static_cast<int>((m.n[t] / 8) % G);
    sy.amax[t] = fold_counter(st);
    sy.nan[t] = fold_counter(st);
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(G));
  cfg.blockDim = dim3(kResThreads);
  cfg.dynamicSmemBytes = static_cast<size_t>(smem);
  cfg.stream = cs;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeCooperative;  // all CTAs resident: they meet at a grid barrier
  at[0].val.cooperative = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  FP8_CUDA_TRY(cudaLaunchKernelEx(&cfg, quant_resident_kernel, m, sl, sy, st->err_ptr));
  count_launches(1);
  *launched = true;
  return FP8_OK;
}

int launch_quantize_current(const uint16_t* x, uint8_t* q, float* scale_out, float* partials, int parts, int64_t n,
                            bool vec, const DeviceState* st, cudaStream_t cs) {
  const int cast_blocks = quant_grid(n, vec, g_quant_cast_bps, st->sm_count);
  if (vec && g_quant_resident) {
    MultiQuant m{};
    m.count = 1;
    m.x[0] = x;
    m.q[0] = q;
    m.scale_out[0] = scale_out;
    m.n[0] = n;
    bool launched = false;
    if (int s = launch_quant_resident(m, const_cast<DeviceState*>(st), cs, &launched)) return s;
    if (launched) return FP8_OK;
  }
  if (vec) {
    if (int s = launch_stream<kStreamAmax>(parts, x, nullptr, n, nullptr, 0, DelayedSource{}, nullptr, partials,
                                           st->err_ptr, cs))
      return s;
    if (int s = launch_stream<kStreamCastCurrent>(cast_blocks, x, q, n, partials, parts, DelayedSource{}, scale_out,
                                                  nullptr, st->err_ptr, cs))
      return s;
  } else {
    FP8_CUDA_TRY(launch_kernel(amax_partials_kernel, dim3(parts), dim3(kQuantThreads), 0, cs, 1, kStreamingKernel, x, n,
                               partials));
    FP8_CUDA_TRY(launch_kernel(quantize_cast_kernel<kCurrent>, dim3(cast_blocks), dim3(kQuantThreads), 0, cs, 1,
                               kStreamingKernel, x, q, n, static_cast<const float*>(partials), parts, DelayedSource{},
                               scale_out, static_cast<float*>(nullptr), ScaleFold{}));
  }
  count_launches(2);
  FP8_CUDA_TRY(cudaGetLastError());
  return FP8_OK;
}

// Partials never exceed kMaxQuantBlocksPerSm per SM, whatever the tuning.
size_t quant_workspace_bytes(int sm_count) {
  return static_cast<size_t>(sm_count) * kMaxQuantBlocksPerSm * sizeof(float);
}

}  // namespace

// ======================================================================== C ABI
extern "C" {

int fp8_abi_version(void) { return 4; }

int fp8_last_error(char* buf, size_t len) {
  if (buf != nullptr && len > 0) {
    strncpy(buf, t_last_msg, len - 1);
    buf[len - 1] = 0;
  }
  return t_last_status;
}

}  // extern "C"

// One CTA waits, through the kernels' bounded mbarrier wait, on a barrier that
// nothing arrives on.  The wait gives up after limit_ns, records
// kErrTimeoutSelfTest and raises the CTA abort flag; every thread then returns.
// returned[0] = 1 when the waiting thread came back with "gave up".
__global__ void wait_selftest_kernel(int* err, uint64_t limit_ns, int* returned) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort_flag;
  pdl_wait();
  if (threadIdx.x == 0) {
    abort_flag = 0;
    mbar_init(&bar, 1);
    fence_barrier_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const bool done = mbar_wait_limit(&bar, 0, &abort_flag, err, kErrTimeoutSelfTest, limit_ns);
    returned[0] = done ? 2 : 1;
  }
  __syncthreads();
}

extern "C" {

int fp8_selftest_wait_timeout(uint64_t limit_ns, int* returned, fp8_stream_t stream) {
  FP8_REQUIRE(limit_ns > 0 && limit_ns <= 1000000000ull, FP8_ERR_INVALID_ARGUMENT,
              "limit_ns must be in (0, 1e9]");
  FP8_REQUIRE(returned != nullptr && aligned(returned, 4), FP8_ERR_INVALID_ARGUMENT, "bad returned pointer");
  DeviceState* st = nullptr;
  if (int s = device_state(&st)) return s;
  count_launches(1);
  FP8_CUDA_TRY(launch_kernel(wait_selftest_kernel, dim3(1), dim3(32), 0, reinterpret_cast<cudaStream_t>(stream), 1,
                             kStreamingKernel, st->err_ptr, limit_ns, returned));
  return ok();
}

int fp8_device_error(int* code_out, fp8_stream_t stream) {
  FP8_REQUIRE(code_out != nullptr, FP8_ERR_INVALID_ARGUMENT, "code_out is NULL");
  DeviceState* st = nullptr;
  if (int s = device_state(&st)) return s;
  FP8_CUDA_TRY(cudaStreamSynchronize(reinterpret_cast<cudaStream_t>(stream)));
  int code = 0;
  FP8_CUDA_TRY(cudaMemcpyFromSymbol(&code, g_fp8_device_error, sizeof(int)));
  if (code != 0) {
    const int zero = 0;
    FP8_CUDA_TRY(cudaMemcpyToSymbol(g_fp8_device_error, &zero, sizeof(int)));
  }
  *code_out = code;
  return ok();
}

int fp8_kernel_launch_count(unsigned long long* out) {
  FP8_REQUIRE(out != nullptr, FP8_ERR_INVALID_ARGUMENT, "out is NULL");
  *out = g_launches.load(std::memory_order_relaxed);
  return ok();
}

int fp8_sm_count(int* out) {
  FP8_REQUIRE(out != nullptr, FP8_ERR_INVALID_ARGUMENT, "out is NULL");
  DeviceState* st = nullptr;
  if (int s = device_state(&st)) return s;
  *out = st->sm_count;
  return ok();
}

size_t fp8_quantize_workspace_bytes(int64_t n) {
  int dev = 0;
  int sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (sms <= 0) sms = 148;
  (void)cudaGetLastError();
  (void)n;
  return quant_workspace_bytes(sms);
}

int fp8_quantize_current(const void* x_bf16, void* q_e4m3, float* scale_out, void* workspace,
                         size_t workspace_bytes, int64_t n, fp8_stream_t stream) {
  FP8_REQUIRE(n >= 0, FP8_ERR_INVALID_ARGUMENT, "n must be >= 0");
  FP8_REQUIRE(scale_out != nullptr && aligned(scale_out, 4), FP8_ERR_INVALID_ARGUMENT, "bad scale_out");
  FP8_REQUIRE(n == 0 || (x_bf16 != nullptr && q_e4m3 != nullptr), FP8_ERR_INVALID_ARGUMENT, "NULL tensor");
  FP8_REQUIRE(aligned(x_bf16, 2), FP8_ERR_INVALID_ARGUMENT, "x must be 2-byte aligned");
  DeviceState* st = nullptr;
  if (int s = device_state(&st)) return s;
  cudaStream_t cs = reinterpret_cast<cudaStream_t>(stream);
  const bool vec = aligned(x_bf16, 16) && aligned(q_e4m3, 8);
  const int parts = quant_grid(n, vec, g_quant_amax_bps, st->sm_count);
  FP8_REQUIRE(workspace != nullptr && workspace_bytes >= parts * sizeof(float) && aligned(workspace, 4),
              FP8_ERR_WORKSPACE, "quantize workspace too small: need %zu bytes", parts * sizeof(float));
  if (int s = launch_quantize_current(static_cast<const uint16_t*>(x_bf16), static_cast<uint8_t*>(q_e4m3), scale_out,
                                      static_cast<float*>(workspace), parts, n, vec, st, cs))
    return s;
  return ok();
}

}  // extern "C"

// ------------------------------------------------------------------ allocation-free quantize
// Scratch of fp8_quantize_current_noalloc: the per-CTA |x| maxima of the amax
// pass.  It is a fixed array in this library's own device memory, so callers
// that cannot allocate device memory (see include/fp8ops.h) still get the
// current-scaling quantize.  Every device that loads the library holds one copy
// (8 KB) until the process exits.
constexpr int kNoAllocPartials = 2048;
static __device__ __align__(256) float g_noalloc_partials[kNoAllocPartials];

namespace {
std::atomic<float*> g_noalloc_ptr[kMaxDevices] = {};
std::mutex g_noalloc_mu;

// Device address of g_noalloc_partials for the current device.  The host-side
// name of the array is only a stand-in; the address must come from the
// runtime, once per device, with that device current.
int noalloc_scratch(float** out) {
  int dev = 0;
  FP8_CUDA_TRY(cudaGetDevice(&dev));
  FP8_REQUIRE(dev >= 0 && dev < kMaxDevices, FP8_ERR_UNSUPPORTED, "device ordinal %d out of range", dev);
  float* ptr = g_noalloc_ptr[dev].load(std::memory_order_acquire);
  if (ptr == nullptr) {
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    ptr = g_noalloc_ptr[dev].load(std::memory_order_relaxed);
    if (ptr == nullptr) {
      void* p = nullptr;
      FP8_CUDA_TRY(cudaGetSymbolAddress(&p, g_noalloc_partials));
      ptr = static_cast<float*>(p);
      g_noalloc_ptr[dev].store(ptr, std::memory_order_release);
    }
  }
  *out = ptr;
  return FP8_OK;
}
}  // namespace

extern "C" {

int fp8_quantize_current_noalloc(const void* x_bf16, void* q_e4m3, float* scale_out, int64_t n,
                                 fp8_stream_t stream) {
  FP8_REQUIRE(n >= 0, FP8_ERR_INVALID_ARGUMENT, "n must be >= 0");
  FP8_REQUIRE(scale_out != nullptr && aligned(scale_out, 4), FP8_ERR_INVALID_ARGUMENT, "bad scale_out");
  FP8_REQUIRE(n == 0 || (x_bf16 != nullptr && q_e4m3 != nullptr), FP8_ERR_INVALID_ARGUMENT, "NULL tensor");
  FP8_REQUIRE(aligned(x_bf16, 2), FP8_ERR_INVALID_ARGUMENT, "x must be 2-byte aligned");
  DeviceState* st = nullptr;
  if (int s = device_state(&st)) return s;
  float* partials = nullptr;
  if (int s = noalloc_scratch(&partials)) return s;
  const bool vec = aligned(x_bf16, 16) && aligned(q_e4m3, 8);
  const int parts = quant_grid(n, vec, g_quant_amax_bps, st->sm_count);
  FP8_REQUIRE(parts <= kNoAllocPartials, FP8_ERR_UNSUPPORTED,
              "allocation-free quantize needs %d partial slots but its static scratch holds %d "
              "(device has too many SMs for it); use fp8_quantize_current with a workspace",
              parts, kNoAllocPartials);
  // Every CTA of the amax pass overwrites its own slot before the cast pass
  // reads slots [0, parts), so nothing has to be cleared between calls.
  if (int s = launch_quantize_current(static_cast<const uint16_t*>(x_bf16), static_cast<uint8_t*>(q_e4m3), scale_out,
                                      partials, parts, n, vec, st, reinterpret_cast<cudaStream_t>(stream)))
    return s;
  return ok();
}

namespace {
// One delayed cast: the scale comes from `src` (a previous scale or the max of a
// scale history), the tensor's own scale goes to *scale_curr_out and / or into
// the history (`wu`).
int quantize_delayed_impl(const void* x_bf16, void* q_e4m3, const DelayedSource& src, float* scale_curr_out,
                          const WindowUpdate& wu, void* workspace, size_t workspace_bytes, int64_t n,
                          fp8_stream_t stream) {
  FP8_REQUIRE(n >= 0, FP8_ERR_INVALID_ARGUMENT, "n must be >= 0");
  FP8_REQUIRE(n == 0 || (x_bf16 != nullptr && q_e4m3 != nullptr), FP8_ERR_INVALID_ARGUMENT, "NULL tensor");
  FP8_REQUIRE(aligned(x_bf16, 2), FP8_ERR_INVALID_ARGUMENT, "x must be 2-byte aligned");
  DeviceState* st = nullptr;
  if (int s = device_state(&st)) return s;
  cudaStream_t cs = reinterpret_cast<cudaStream_t>(stream);
  // The cast pass writes one partial per CTA, so its grid is the partial count.
  const bool vec = aligned(x_bf16, 16) && aligned(q_e4m3, 8);
  const int parts = quant_grid(n, vec, g_quant_cast_bps, st->sm_count);
  FP8_REQUIRE(workspace != nullptr && workspace_bytes >= parts * sizeof(float) && aligned(workspace, 4),
              FP8_ERR_WORKSPACE, "quantize workspace too small: need %zu bytes", parts * sizeof(float));
  float* partials = static_cast<float*>(workspace);
  const uint16_t* x = static_cast<const uint16_t*>(x_bf16);
  uint8_t* q = static_cast<uint8_t*>(q_e4m3);
  const ScaleFold fold{fold_counter(st), scale_curr_out, wu};
  if (vec) {
    if (int s = launch_stream<kStreamCastDelayed>(parts, x, q, n, nullptr, 0, src, nullptr, partials, st->err_ptr,
                                                  cs, fold))
      return s;
  } else {
    FP8_CUDA_TRY(launch_kernel(quantize_cast_kernel<kDelayed>, dim3(parts), dim3(kQuantThreads), 0, cs, 1,
                               kStreamingKernel, x, q, n, static_cast<const float*>(nullptr), 0, src,
                               static_cast<float*>(nullptr), partials, fold));
  }
  count_launches(1);
  FP8_CUDA_TRY(cudaGetLastError());
  return ok();
}

int check_window(const float* window, int window_len, const int64_t* window_pos, const float* used) {
  FP8_REQUIRE(window != nullptr && aligned(window, 4) && window_len > 0, FP8_ERR_INVALID_ARGUMENT,
              "bad scale history");
  FP8_REQUIRE(window_pos != nullptr && aligned(window_pos, 8), FP8_ERR_INVALID_ARGUMENT, "bad history position");
  FP8_REQUIRE(used != nullptr && aligned(used, 4), FP8_ERR_INVALID_ARGUMENT, "bad scale_used_out");
  return FP8_OK;
}
}  // namespace

int fp8_quantize_delayed(const void* x_bf16, void* q_e4m3, const float* prev_scale, float* scale_curr_out,
                         void* workspace, size_t workspace_bytes, int64_t n, fp8_stream_t stream) {
  FP8_REQUIRE(prev_scale != nullptr && aligned(prev_scale, 4), FP8_ERR_INVALID_ARGUMENT, "bad prev_scale");
  FP8_REQUIRE(scale_curr_out != nullptr && aligned(scale_curr_out, 4), FP8_ERR_INVALID_ARGUMENT,
              "bad scale_curr_out");
  return quantize_delayed_impl(x_bf16, q_e4m3, DelayedSource{prev_scale, nullptr, 0, nullptr}, scale_curr_out,
                               WindowUpdate{}, workspace, workspace_bytes, n, stream);
}

int fp8_quantize_delayed_window(const void* x_bf16, void* q_e4m3, float* window, int window_len,
                                int64_t* window_pos, int advance, float* scale_used_out, void* workspace,
                                size_t workspace_bytes, int64_t n, fp8_stream_t stream) {
  if (int s = check_window(window, window_len, window_pos, scale_used_out)) return s;
  return quantize_delayed_impl(x_bf16, q_e4m3, DelayedSource{nullptr, window, window_len, scale_used_out}, nullptr,
                               WindowUpdate{window, window_pos, window_len, advance ? 1 : 0, g_empty_zero}, workspace,
                               workspace_bytes, n, stream);
}

int fp8_transpose_2d(const void* src, void* dst, int64_t rows, int64_t cols, fp8_stream_t stream) {
  FP8_REQUIRE(rows >= 0 && cols >= 0, FP8_ERR_INVALID_ARGUMENT, "negative size");
  if (rows == 0 || cols == 0) return ok();
  FP8_REQUIRE(src != nullptr && dst != nullptr, FP8_ERR_INVALID_ARGUMENT, "NULL tensor");
  if (int s = launch_transpose(src, dst, rows, cols, cols, rows, 0, 0, 1, reinterpret_cast<cudaStream_t>(stream)))
    return s;
  return ok();
}

int fp8_conv_weight_transpose(const void* wq, void* wq_t, int cout, int cin, fp8_stream_t stream) {
  FP8_REQUIRE(cout > 0 && cin > 0, FP8_ERR_INVALID_ARGUMENT, "sizes must be positive");
  FP8_REQUIRE(wq != nullptr && wq_t != nullptr, FP8_ERR_INVALID_ARGUMENT, "NULL tensor");
  // src [Cout][9][Cin]: per tap a Cout x Cin matrix with leading dim 9*Cin, batch stride Cin.
  // dst [Cin][9][Cout]: per tap a Cin x Cout matrix with leading dim 9*Cout, batch stride Cout.
  if (int s = launch_transpose(wq, wq_t, cout, cin, 9ll * cin, 9ll * cout, cin, cout, 9,
                               reinterpret_cast<cudaStream_t>(stream)))
    return s;
  return ok();
}

int fp8_conv_weight_transpose_batch(int count, const void* const* wq, void* const* wq_t, const int* cout,
                                    const int* cin, fp8_stream_t stream) {
  FP8_REQUIRE(count > 0 && count <= kMaxTransTensors, FP8_ERR_UNSUPPORTED, "1..%d weights per call",
              kMaxTransTensors);
  FP8_REQUIRE(wq && wq_t && cout && cin, FP8_ERR_INVALID_ARGUMENT, "NULL argument");
  TransBatch b{};
  b.count = count;
  int64_t tiles = 0;
  for (int t = 0; t < count; ++t) {
    FP8_REQUIRE(cout[t] > 0 && cin[t] > 0 && cout[t] % kTransTile == 0 && cin[t] % kTransTile == 0,
                FP8_ERR_UNSUPPORTED, "weight %d: Cout and Cin must be positive multiples of %d", t, kTransTile);
    FP8_REQUIRE(wq[t] && wq_t[t] && aligned(wq[t], 16) && aligned(wq_t[t], 16), FP8_ERR_INVALID_ARGUMENT,
                "weight %d: pointers must be non-NULL and 16-byte aligned", t);
    b.src[t] = static_cast<const uint8_t*>(wq[t]);
    b.dst[t] = static_cast<uint8_t*>(wq_t[t]);
    b.cout[t] = cout[t];
    b.cin[t] = cin[t];
    b.tile_begin[t] = static_cast<int>(tiles);
    tiles += 9ll * (cout[t] / kTransTile) * (cin[t] / kTransTile);
    FP8_REQUIRE(tiles < (1ll << 31), FP8_ERR_UNSUPPORTED, "weights too large");
  }
  b.tile_begin[count] = static_cast<int>(tiles);
  FP8_CUDA_TRY(launch_kernel(transpose_conv_weights_kernel, dim3(static_cast<unsigned>(tiles)), dim3(256), 0,
                             reinterpret_cast<cudaStream_t>(stream), 1, kStreamingKernel, b));
  count_launches(1);
  return ok();
}

int fp8_conv3x3_fwd(const void* xq, const void* wq, void* y, const float* sx, const float* sw, const void* bias,
                    int epilogue, int batch, int height, int width, int cin, int cout, fp8_stream_t stream) {
  ConvTile t;
  if (int s = check_conv_args(batch, height, width, cin, cout, &t)) return s;
  if (int s = check_scale_ptrs(sx, sw)) return s;
  FP8_REQUIRE(xq && wq && y, FP8_ERR_INVALID_ARGUMENT, "NULL tensor");
  FP8_REQUIRE(aligned(xq, 16) && aligned(wq, 16) && aligned(y, 16), FP8_ERR_INVALID_ARGUMENT,
              "conv tensors must be 16-byte aligned");
  FP8_REQUIRE(epilogue >= FP8_EPILOGUE_NONE && epilogue <= FP8_EPILOGUE_BIAS_SILU, FP8_ERR_INVALID_ARGUMENT,
              "unknown epilogue %d", epilogue);
  FP8_REQUIRE(epilogue == FP8_EPILOGUE_NONE || (bias != nullptr && aligned(bias, 16)), FP8_ERR_INVALID_ARGUMENT,
              "bias epilogue needs a 16-byte aligned bias");
  DeviceState* st = nullptr;
  if (int s = device_state(&st)) return s;
  if (g_conv_algo != 1 && halo_applies(height, width)) {
    if (int s = launch_conv_halo(xq, wq, y, sx, sw, bias, epilogue, batch, height, width, cin, cout, true,
                                 st->err_ptr, st->sm_count, reinterpret_cast<cudaStream_t>(stream)))
      return s;
    return ok();
  }
  CUtensorMap ma, mb;
  if (int s = make_map_conv(&ma, xq, batch, height, width, cin, t)) return s;
  const int64_t M = static_cast<int64_t>(batch) * height * width;
  const int k_blocks = 9 * (cin / 128);
  int bm_sub, bn;
  choose_kgemm_tile({M, cout, k_blocks}, st->sm_count, &bm_sub, &bn);
  if (int s = make_map_2d(&mb, wq, cout, 9ll * cin, bn)) return s;
  CUtensorMap mo;
  if (int s = make_map_out_bf16(&mo, y, M, cout)) return s;
  KGemmParams p{};
  p.k_blocks = k_blocks;
  p.M = static_cast<int>(M);
  p.N = cout;
  p.a_conv = 1;
  p.HW = height * width;
  p.W = width;
  p.cchunks = cin / 128;
  p.tap_sign = 1;
  p.scale_a = sx;
  p.scale_b = sw;
  p.bias = static_cast<const __nv_bfloat16*>(bias);
  p.epilogue = epilogue;
  p.err = st->err_ptr;
  if (int s = launch_kgemm(ma, mb, mo, p, bm_sub, bn, st->sm_count, reinterpret_cast<cudaStream_t>(stream)))
    return s;
  return ok();
}

int fp8_conv3x3_dgrad(const void* dyq, const void* wq_t, void* dx, const float* sdy, const float* sw, int batch,
                      int height, int width, int cin, int cout, fp8_stream_t stream) {
  ConvTile t;
  if (int s = check_conv_args(batch, height, width, cin, cout, &t)) return s;
  if (int s = check_scale_ptrs(sdy, sw)) return s;
  FP8_REQUIRE(dyq && wq_t && dx, FP8_ERR_INVALID_ARGUMENT, "NULL tensor");
  FP8_REQUIRE(aligned(dyq, 16) && aligned(wq_t, 16) && aligned(dx, 16), FP8_ERR_INVALID_ARGUMENT,
              "conv tensors must be 16-byte aligned");
  DeviceState* st = nullptr;
  if (int s = device_state(&st)) return s;
  if (g_conv_algo != 1 && halo_applies(height, width)) {
    if (int s = launch_conv_halo(dyq, wq_t, dx, sdy, sw, nullptr, kEpiNone, batch, height, width, cout, cin, false,
                                 st->err_ptr, st->sm_count, reinterpret_cast<cudaStream_t>(stream)))
      return s;
    return ok();
  }
  CUtensorMap ma, mb;
  if (int s = make_map_conv(&ma, dyq, batch, height, width, cout, t)) return s;
  const int64_t M = static_cast<int64_t>(batch) * height * width;
  const int k_blocks = 9 * (cout / 128);
  int bm_sub, bn;
  choose_kgemm_tile({M, cin, k_blocks}, st->sm_count, &bm_sub, &bn);
  if (int s = make_map_2d(&mb, wq_t, cin, 9ll * cout, bn)) return s;
  CUtensorMap mo;
  if (int s = make_map_out_bf16(&mo, dx, M, cin)) return s;
  KGemmParams p{};
  p.k_blocks = k_blocks;
  p.M = static_cast<int>(M);
  p.N = cin;
  p.a_conv = 1;
  p.HW = height * width;
  p.W = width;
  p.cchunks = cout / 128;
  p.tap_sign = -1;
  p.scale_a = sdy;
  p.scale_b = sw;
  p.bias = nullptr;
  p.epilogue = kEpiNone;
  p.err = st->err_ptr;
  if (int s = launch_kgemm(ma, mb, mo, p, bm_sub, bn, st->sm_count, reinterpret_cast<cudaStream_t>(stream)))
    return s;
  return ok();
}

size_t fp8_conv3x3_wgrad_workspace_bytes(int batch, int height, int width, int cin, int cout, int split_k) {
  ConvTile t;
  if (batch <= 0 || cin % 128 != 0 || cout % 128 != 0 || cin <= 0 || cout <= 0 || !conv_tile(height, width, &t))
    return 0;
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (sms <= 0) sms = 148;
  (void)cudaGetLastError();
  (void)sms;
  (void)split_k;
  return static_cast<size_t>(cout) * 9 * cin * sizeof(float);
}

namespace {
int conv3x3_wgrad_impl(const void* xq, const void* dyq, void* dw, bool f32_out, const float* sx, const float* sdy,
                       int batch, int height, int width, int cin, int cout, int split_k, void* workspace,
                       size_t workspace_bytes, fp8_stream_t stream) {
  ConvTile t;
  if (int s = check_conv_args(batch, height, width, cin, cout, &t)) return s;
  if (int s = check_scale_ptrs(sx, sdy)) return s;
  FP8_REQUIRE(xq && dyq && dw, FP8_ERR_INVALID_ARGUMENT, "NULL tensor");
  FP8_REQUIRE(aligned(xq, 16) && aligned(dyq, 16) && aligned(dw, 16), FP8_ERR_INVALID_ARGUMENT,
              "conv tensors must be 16-byte aligned");
  DeviceState* st = nullptr;
  if (int s = device_state(&st)) return s;
  const int64_t pixels = static_cast<int64_t>(batch) * height * width;
  const WGradPlan w = plan_wgrad(cout, 9ll * cin, pixels, split_k, st->sm_count);
  const size_t need = static_cast<size_t>(cout) * 9 * cin * sizeof(float);
  FP8_REQUIRE(workspace != nullptr && workspace_bytes >= need && aligned(workspace, 16), FP8_ERR_WORKSPACE,
              "wgrad workspace too small: need %zu bytes", need);
  // Halo mode: 128-pixel K blocks of whole image rows of one image, 3-box groups.
  const bool halo = g_conv_algo != 1 && w.group == 3 && halo_applies(height, width);
  CUtensorMap mdy, mx;
  if (int s = make_map_2d(&mdy, dyq, pixels, cout, 128)) return s;
  if (halo) {
    if (int s = make_map_conv_halo(&mx, xq, batch, height, width, cin, 128 / width)) return s;
  } else {
    if (int s = make_map_conv(&mx, xq, batch, height, width, cin, t)) return s;
  }
  WGradParams p{};
  p.num_tiles = w.num_tiles;
  p.num_groups = w.num_groups;
  p.splits = w.splits;
  p.k_blocks = w.k_blocks;
  p.b_conv = 1;
  p.HW = height * width;
  p.W = width;
  p.cchunks = cin / 128;
  p.halo_box_bytes = (128 / width + 2) * width * 128;
  p.n_cols = 9 * cin;
  p.m_rows = cout;
  p.acc = static_cast<float*>(workspace);
  p.err = st->err_ptr;
  cudaStream_t cs = reinterpret_cast<cudaStream_t>(stream);
  if (int s = launch_wgrad_converted(mdy, mx, p, w.group, cs, halo, sx, sdy, dw, f32_out, st)) return s;
  return ok();
}
}  // namespace

int fp8_conv3x3_wgrad(const void* xq, const void* dyq, void* dw, const float* sx, const float* sdy, int batch,
                      int height, int width, int cin, int cout, int split_k, void* workspace,
                      size_t workspace_bytes, fp8_stream_t stream) {
  return conv3x3_wgrad_impl(xq, dyq, dw, false, sx, sdy, batch, height, width, cin, cout, split_k, workspace,
                            workspace_bytes, stream);
}

int fp8_conv3x3_wgrad_f32(const void* xq, const void* dyq, float* dw, const float* sx, const float* sdy, int batch,
                          int height, int width, int cin, int cout, int split_k, void* workspace,
                          size_t workspace_bytes, fp8_stream_t stream) {
  return conv3x3_wgrad_impl(xq, dyq, dw, true, sx, sdy, batch, height, width, cin, cout, split_k, workspace,
                            workspace_bytes, stream);
}

int fp8_gemm(const void* a, const void* b, void* out, const float* sa, const float* sb, const void* bias,
             int epilogue, int64_t m, int64_t n, int64_t k, fp8_stream_t stream) {
  FP8_REQUIRE(m > 0 && n > 0 && k > 0, FP8_ERR_INVALID_ARGUMENT, "GEMM sizes must be positive");
  FP8_REQUIRE(k % 16 == 0, FP8_ERR_UNSUPPORTED, "K must be a multiple of 16 (K=%lld)", (long long)k);
  FP8_REQUIRE(n % 32 == 0, FP8_ERR_UNSUPPORTED, "N must be a multiple of 32 (N=%lld)", (long long)n);
  FP8_REQUIRE(m < (1ll << 31) && n < (1ll << 31), FP8_ERR_UNSUPPORTED, "GEMM too large");
  if (int s = check_scale_ptrs(sa, sb)) return s;
  FP8_REQUIRE(a && b && out, FP8_ERR_INVALID_ARGUMENT, "NULL tensor");
  FP8_REQUIRE(aligned(a, 16) && aligned(b, 16) && aligned(out, 16), FP8_ERR_INVALID_ARGUMENT,
              "GEMM tensors must be 16-byte aligned");
  FP8_REQUIRE(epilogue >= FP8_EPILOGUE_NONE && epilogue <= FP8_EPILOGUE_BIAS_SILU, FP8_ERR_INVALID_ARGUMENT,
              "unknown epilogue %d", epilogue);
  FP8_REQUIRE(epilogue == FP8_EPILOGUE_NONE || (bias != nullptr && aligned(bias, 16)), FP8_ERR_INVALID_ARGUMENT,
              "bias epilogue needs a 16-byte aligned bias");
  DeviceState* st = nullptr;
  if (int s = device_state(&st)) return s;
  const int k_blocks = static_cast<int>((k + 127) / 128);
  int bm_sub, bn;
  choose_kgemm_tile({m, n, k_blocks, true}, st->sm_count, &bm_sub, &bn);
  CUtensorMap ma, mb;
  if (int s = make_map_2d(&ma, a, m, k, 128)) return s;
  if (int s = make_map_2d(&mb, b, n, k, bn)) return s;
  CUtensorMap mo;
  if (int s = make_map_out_bf16(&mo, out, m, n)) return s;
  KGemmParams p{};
  p.k_blocks = k_blocks;
  p.M = static_cast<int>(m);
  p.N = static_cast<int>(n);
  p.a_conv = 0;
  p.scale_a = sa;
  p.scale_b = sb;
  p.bias = static_cast<const __nv_bfloat16*>(bias);
  p.epilogue = epilogue;
  p.err = st->err_ptr;
  if (int s = launch_kgemm(ma, mb, mo, p, bm_sub, bn, st->sm_count, reinterpret_cast<cudaStream_t>(stream)))
    return s;
  return ok();
}

size_t fp8_gemm_wgrad_workspace_bytes(int64_t m, int64_t n, int64_t k, int split_k) {
  if (m <= 0 || n <= 0 || k <= 0 || n % 128 != 0 || k % 128 != 0) return 0;
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (sms <= 0) sms = 148;
  (void)cudaGetLastError();
  (void)sms;
  (void)split_k;
  return static_cast<size_t>(n) * k * sizeof(float);
}

int fp8_gemm_wgrad(const void* dy, const void* x, void* dw, const float* sdy, const float* sx, int64_t m,
                   int64_t n, int64_t k, int split_k, void* workspace, size_t workspace_bytes,
                   fp8_stream_t stream) {
  FP8_REQUIRE(m > 0 && n > 0 && k > 0, FP8_ERR_INVALID_ARGUMENT, "GEMM sizes must be positive");
  FP8_REQUIRE(n % 128 == 0 && k % 128 == 0, FP8_ERR_UNSUPPORTED,
              "weight-gradient N and K must be multiples of 128 (N=%lld K=%lld)", (long long)n, (long long)k);
  FP8_REQUIRE(m < (1ll << 31), FP8_ERR_UNSUPPORTED, "GEMM too large");
  if (int s = check_scale_ptrs(sdy, sx)) return s;
  FP8_REQUIRE(dy && x && dw, FP8_ERR_INVALID_ARGUMENT, "NULL tensor");
  FP8_REQUIRE(aligned(dy, 16) && aligned(x, 16) && aligned(dw, 16), FP8_ERR_INVALID_ARGUMENT,
              "GEMM tensors must be 16-byte aligned");
  DeviceState* st = nullptr;
  if (int s = device_state(&st)) return s;
  const WGradPlan w = plan_wgrad(n, k, m, split_k, st->sm_count);
  const size_t need = static_cast<size_t>(n) * k * sizeof(float);
  FP8_REQUIRE(workspace != nullptr && workspace_bytes >= need && aligned(workspace, 16), FP8_ERR_WORKSPACE,
              "wgrad workspace too small: need %zu bytes", need);
  CUtensorMap mdy, mx;
  if (int s = make_map_2d(&mdy, dy, m, n, 128)) return s;
  if (int s = make_map_2d(&mx, x, m, k, 128)) return s;
  WGradParams p{};
  p.num_tiles = w.num_tiles;
  p.num_groups = w.num_groups;
  p.splits = w.splits;
  p.k_blocks = w.k_blocks;
  p.b_conv = 0;
  p.n_cols = static_cast<int>(k);
  p.m_rows = static_cast<int>(n);
  p.acc = static_cast<float*>(workspace);
  p.err = st->err_ptr;
  cudaStream_t cs = reinterpret_cast<cudaStream_t>(stream);
  if (int s = launch_wgrad_converted(mdy, mx, p, w.group, cs, false, sdy, sx, dw, false, st)) return s;
  return ok();
}

int fp8_set_quantize_override(int amax_blocks_per_sm, int cast_blocks_per_sm) {
  FP8_REQUIRE(amax_blocks_per_sm >= 0 && amax_blocks_per_sm <= kMaxQuantBlocksPerSm && cast_blocks_per_sm >= 0 &&
                  cast_blocks_per_sm <= kMaxQuantBlocksPerSm,
              FP8_ERR_INVALID_ARGUMENT, "blocks per SM must be in 0..%d", kMaxQuantBlocksPerSm);
  g_quant_amax_bps = amax_blocks_per_sm > 0 ? amax_blocks_per_sm : 2;
  g_quant_cast_bps = cast_blocks_per_sm > 0 ? cast_blocks_per_sm : 2;
  return ok();
}

int fp8_set_pdl(int mode) {
  FP8_REQUIRE(mode >= 0 && mode <= 2, FP8_ERR_INVALID_ARGUMENT, "pdl mode must be 0, 1 or 2");
  g_pdl = mode;
  return ok();
}

int fp8_set_wgrad_fused(int enable) {
  FP8_REQUIRE(enable == 0 || enable == 1, FP8_ERR_INVALID_ARGUMENT, "enable must be 0 or 1");
  g_wgrad_fused = enable;
  return ok();
}

int fp8_set_quantize_resident(int enable) {
  FP8_REQUIRE(enable == 0 || enable == 1, FP8_ERR_INVALID_ARGUMENT, "enable must be 0 or 1");
  g_quant_resident = enable;
  return ok();
}

int fp8_set_empty_tensor_history(int mode) {
  FP8_REQUIRE(mode == 0 || mode == 1, FP8_ERR_INVALID_ARGUMENT, "empty-tensor history mode must be 0 or 1");
  g_empty_zero = mode;
  return ok();
}

int fp8_set_conv_algo(int algo) {
  FP8_REQUIRE(algo >= 0 && algo <= 4, FP8_ERR_INVALID_ARGUMENT, "conv algo must be 0 (auto), 1, 2, 3 or 4");
  g_conv_algo = algo;
  return ok();
}

int fp8_set_tile_override(int bm_sub, int bn, int wgrad_group) {
  FP8_REQUIRE(bm_sub == 0 || bm_sub == 1 || bm_sub == 2, FP8_ERR_INVALID_ARGUMENT, "bm_sub must be 0, 1 or 2");
  FP8_REQUIRE(bn == 0 || bn == 64 || bn == 128 || bn == 256, FP8_ERR_INVALID_ARGUMENT, "bn must be 0/64/128/256");
  FP8_REQUIRE(wgrad_group >= 0 && wgrad_group <= 3, FP8_ERR_INVALID_ARGUMENT, "group must be 0..3");
  g_override_bm_sub = bm_sub;
  g_override_bn = bn;
  g_override_group = wgrad_group;
  return ok();
}

}  // extern "C"

// ======================================================================== group norm + activation
extern "C" {

size_t fp8_gn_workspace_bytes(int n, int hw, int c) {
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  (void)cudaGetLastError();
  if (n <= 0 || hw <= 0 || c < 8) return 0;
  return gn_workspace(n, hw, c, sms > 0 ? sms : 148);
}

int fp8_gn_act_fwd(const void* x, int x_fp32, const float* gamma, const float* beta, const void* film,
                   int film_ld, const int64_t* seed, float p, float eps, float* stats, void* out, int n, int hw,
                   int c, int groups, void* workspace, size_t workspace_bytes, fp8_stream_t stream) {
  if (int s = check_gn_args(x, out, gamma, beta, n, hw, c, groups, film_ld, film, p, eps)) return s;
  FP8_REQUIRE(stats != nullptr, FP8_ERR_INVALID_ARGUMENT, "NULL stats");
  DeviceState* st = nullptr;
  if (int s = device_state(&st)) return s;
  const size_t need = gn_workspace(n, hw, c, st->sm_count);
  FP8_REQUIRE(workspace != nullptr && workspace_bytes >= need && aligned(workspace, 16), FP8_ERR_WORKSPACE,
              "group-norm workspace too small: need %zu bytes", need);
  const GnShape sh{n, hw, c, groups, 1, 1};
  GnActParams q{gamma, beta, static_cast<const uint16_t*>(film), film_ld, seed, p, eps};
  cudaStream_t cs = reinterpret_cast<cudaStream_t>(stream);
  float* part = static_cast<float*>(workspace);
  const size_t s1 = gn_stats_smem(c), s2 = gn_fwd_smem(c, groups);
  const GnOut o{static_cast<uint16_t*>(out), nullptr, DelayedSource{}, nullptr, ScaleFold{}};
  if (x_fp32) {
    if (int s = launch_gn_fwd<float, false>(static_cast<const float*>(x), sh, part, q, stats, o, s1, s2, st->sm_count,
                                               cs)) return s;
  } else {
    if (int s = launch_gn_fwd<uint16_t, false>(static_cast<const uint16_t*>(x), sh, part, q, stats, o, s1, s2,
                                                  st->sm_count, cs))
      return s;
  }
  FP8_CUDA_TRY(cudaGetLastError());
  return ok();
}

size_t fp8_gn_act_quant_workspace_bytes(int n, int hw, int c) {
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  (void)cudaGetLastError();
  if (n <= 0 || hw <= 0 || c < 8) return 0;
  if (sms <= 0) sms = 148;
  const int slices = gn_slices_cap(n, hw, c, sms);
  // group-norm partials, then one amax partial per apply CTA (16-byte aligned)
  return gn_workspace(n, hw, c, sms) + ((static_cast<size_t>(n) * slices * sizeof(float) + 15) & ~size_t(15));
}

namespace {
int gn_act_quant_impl(const void* x, int x_fp32, const float* gamma, const float* beta, const void* film,
                      int film_ld, const int64_t* seed, float p, float eps, const DelayedSource& src, float* stats,
                      void* q_e4m3, float* scale_curr_out, const WindowUpdate& wu, int n, int hw, int c, int groups,
                      void* workspace, size_t workspace_bytes, fp8_stream_t stream) {
  if (int s = check_gn_args(x, q_e4m3, gamma, beta, n, hw, c, groups, film_ld, film, p, eps)) return s;
  FP8_REQUIRE(stats != nullptr, FP8_ERR_INVALID_ARGUMENT, "NULL stats");
  DeviceState* st = nullptr;
  if (int s = device_state(&st)) return s;
  const GnShape sh{n, hw, c, groups, 1, 1};
  const size_t gn_bytes = gn_workspace(n, hw, c, st->sm_count);
  const size_t need =
      gn_bytes + ((static_cast<size_t>(n) * gn_slices_cap(n, hw, c, st->sm_count) * sizeof(float) + 15) & ~size_t(15));
  FP8_REQUIRE(workspace != nullptr && workspace_bytes >= need && aligned(workspace, 16), FP8_ERR_WORKSPACE,
              "group-norm workspace too small: need %zu bytes", need);
  GnActParams q{gamma, beta, static_cast<const uint16_t*>(film), film_ld, seed, p, eps};
  cudaStream_t cs = reinterpret_cast<cudaStream_t>(stream);
  float* part = static_cast<float*>(workspace);
  float* amax_part = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + gn_bytes);
  const GnOut o{nullptr, static_cast<uint8_t*>(q_e4m3), src, amax_part,
                ScaleFold{fold_counter(st), scale_curr_out, wu}};
  const size_t s1 = gn_stats_smem(c), s2 = gn_fwd_smem(c, groups);
  if (x_fp32) {
    if (int s = launch_gn_fwd<float, true>(static_cast<const float*>(x), sh, part, q, stats, o, s1, s2, st->sm_count,
                                           cs))
      return s;
  } else {
    if (int s = launch_gn_fwd<uint16_t, true>(static_cast<const uint16_t*>(x), sh, part, q, stats, o, s1, s2,
                                              st->sm_count, cs))
      return s;
  }
  FP8_CUDA_TRY(cudaGetLastError());
  return ok();
}
}  // namespace

int fp8_gn_act_quant_fwd(const void* x, int x_fp32, const float* gamma, const float* beta, const void* film,
                         int film_ld, const int64_t* seed, float p, float eps, const float* prev_scale,
                         float* stats, void* q_e4m3, float* scale_curr_out, int n, int hw, int c, int groups,
                         void* workspace, size_t workspace_bytes, fp8_stream_t stream) {
  FP8_REQUIRE(prev_scale != nullptr && scale_curr_out != nullptr, FP8_ERR_INVALID_ARGUMENT, "NULL scale");
  return gn_act_quant_impl(x, x_fp32, gamma, beta, film, film_ld, seed, p, eps,
                           DelayedSource{prev_scale, nullptr, 0, nullptr}, stats, q_e4m3, scale_curr_out,
                           WindowUpdate{}, n, hw, c, groups, workspace, workspace_bytes, stream);
}

int fp8_gn_act_quant_fwd_window(const void* x, int x_fp32, const float* gamma, const float* beta, const void* film,
                                int film_ld, const int64_t* seed, float p, float eps, float* window, int window_len,
                                int64_t* window_pos, int advance, float* scale_used_out, float* stats, void* q_e4m3,
                                int n, int hw, int c, int groups, void* workspace, size_t workspace_bytes,
                                fp8_stream_t stream) {
  if (int s = check_window(window, window_len, window_pos, scale_used_out)) return s;
  return gn_act_quant_impl(x, x_fp32, gamma, beta, film, film_ld, seed, p, eps,
                           DelayedSource{nullptr, window, window_len, scale_used_out}, stats, q_e4m3, nullptr,
                           WindowUpdate{window, window_pos, window_len, advance ? 1 : 0, g_empty_zero}, n, hw, c, groups, workspace,
                           workspace_bytes, stream);
}

}  // extern "C"

namespace {
int gn_act_bwd_impl(const void* x, int x_fp32, const void* dy, const float* gamma, const float* beta,
                    const void* film, int film_ld, const int64_t* seed, float p, float eps, const float* stats,
                    float* totals, const void* dx_add, void* dx, int n, int hw, int c, int groups, void* workspace,
                    size_t workspace_bytes, fp8_stream_t stream) {
  if (int s = check_gn_args(x, dx, gamma, beta, n, hw, c, groups, film_ld, film, p, eps)) return s;
  FP8_REQUIRE(dx_add == nullptr || aligned(dx_add, 16), FP8_ERR_INVALID_ARGUMENT, "dx_add must be 16-byte aligned");
  FP8_REQUIRE(dy != nullptr && aligned(dy, 16), FP8_ERR_INVALID_ARGUMENT, "dy must be 16-byte aligned");
  FP8_REQUIRE(stats != nullptr && totals != nullptr, FP8_ERR_INVALID_ARGUMENT, "NULL stats / totals");
  DeviceState* st = nullptr;
  if (int s = device_state(&st)) return s;
  const size_t need = gn_workspace(n, hw, c, st->sm_count);
  FP8_REQUIRE(workspace != nullptr && workspace_bytes >= need && aligned(workspace, 16), FP8_ERR_WORKSPACE,
              "group-norm workspace too small: need %zu bytes", need);
  const GnShape sh{n, hw, c, groups, 1, 1};
  GnActParams q{gamma, beta, static_cast<const uint16_t*>(film), film_ld, seed, p, eps};
  cudaStream_t cs = reinterpret_cast<cudaStream_t>(stream);
  float* part = static_cast<float*>(workspace);
  const size_t s1 = gn_bwd_reduce_smem(c, groups), s2 = gn_bwd_apply_smem(c, groups);
  const uint16_t* ds = static_cast<const uint16_t*>(dy);
  if (x_fp32) {
    if (int s = launch_gn_bwd(static_cast<const float*>(x), ds, sh, stats, q, part, totals, static_cast<float*>(dx),
                              s1, s2, st->sm_count, cs, nullptr, static_cast<const float*>(dx_add)))
      return s;
  } else {
    if (int s = launch_gn_bwd(static_cast<const uint16_t*>(x), ds, sh, stats, q, part, totals,
                              static_cast<uint16_t*>(dx), s1, s2, st->sm_count, cs, nullptr,
                              static_cast<const uint16_t*>(dx_add)))
      return s;
  }
  FP8_CUDA_TRY(cudaGetLastError());
  return ok();
}
}  // namespace

extern "C" {

int fp8_gn_act_bwd(const void* x, int x_fp32, const void* dy, const float* gamma, const float* beta,
                   const void* film, int film_ld, const int64_t* seed, float p, float eps, const float* stats,
                   float* totals, void* dx, int n, int hw, int c, int groups, void* workspace,
                   size_t workspace_bytes, fp8_stream_t stream) {
  return gn_act_bwd_impl(x, x_fp32, dy, gamma, beta, film, film_ld, seed, p, eps, stats, totals, nullptr, dx, n, hw,
                         c, groups, workspace, workspace_bytes, stream);
}

int fp8_gn_act_bwd_accumulate(const void* x, int x_fp32, const void* dy, const float* gamma, const float* beta,
                              const void* film, int film_ld, const int64_t* seed, float p, float eps,
                              const float* stats, float* totals, const void* dx_add, void* dx, int n, int hw, int c,
                              int groups, void* workspace, size_t workspace_bytes, fp8_stream_t stream) {
  FP8_REQUIRE(dx_add != nullptr, FP8_ERR_INVALID_ARGUMENT, "NULL dx_add");
  return gn_act_bwd_impl(x, x_fp32, dy, gamma, beta, film, film_ld, seed, p, eps, stats, totals, dx_add, dx, n, hw,
                         c, groups, workspace, workspace_bytes, stream);
}

size_t fp8_gn_act_bwd_quant_workspace_bytes(int n, int hw, int c) { return fp8_gn_act_quant_workspace_bytes(n, hw, c); }

int fp8_gn_act_bwd_quant(const void* x, const void* dy, const float* gamma, const float* beta, const void* film,
                         int film_ld, const int64_t* seed, float p, float eps, const float* stats, float* totals,
                         void* dx, void* dxq, float* window, int window_len, int64_t* window_pos,
                         float* scale_used_out, int n, int hw, int c, int groups, void* workspace,
                         size_t workspace_bytes, fp8_stream_t stream) {
  if (int s = check_gn_args(x, dx, gamma, beta, n, hw, c, groups, film_ld, film, p, eps)) return s;
  FP8_REQUIRE(dy != nullptr && aligned(dy, 16), FP8_ERR_INVALID_ARGUMENT, "dy must be 16-byte aligned");
  FP8_REQUIRE(dxq != nullptr && aligned(dxq, 16), FP8_ERR_INVALID_ARGUMENT, "dxq must be 16-byte aligned");
  FP8_REQUIRE(stats != nullptr && totals != nullptr, FP8_ERR_INVALID_ARGUMENT, "NULL stats / totals");
  if (int s = check_window(window, window_len, window_pos, scale_used_out)) return s;
  DeviceState* st = nullptr;
  if (int s = device_state(&st)) return s;
  const size_t gn_bytes = gn_workspace(n, hw, c, st->sm_count);
  const size_t need =
      gn_bytes + ((static_cast<size_t>(n) * gn_slices_cap(n, hw, c, st->sm_count) * sizeof(float) + 15) & ~size_t(15));
  FP8_REQUIRE(workspace != nullptr && workspace_bytes >= need && aligned(workspace, 16), FP8_ERR_WORKSPACE,
              "group-norm workspace too small: need %zu bytes", need);
  const GnShape sh{n, hw, c, groups, 1, 1};
  GnActParams q{gamma, beta, static_cast<const uint16_t*>(film), film_ld, seed, p, eps};
  float* part = static_cast<float*>(workspace);
  float* amax_part = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + gn_bytes);
  const GnOut o{nullptr, static_cast<uint8_t*>(dxq), DelayedSource{nullptr, window, window_len, scale_used_out},
                amax_part, ScaleFold{fold_counter(st), nullptr, WindowUpdate{window, window_pos, window_len, 0, g_empty_zero}}};
  if (int s = launch_gn_bwd(static_cast<const uint16_t*>(x), static_cast<const uint16_t*>(dy), sh, stats, q, part,
                            totals, static_cast<uint16_t*>(dx), gn_bwd_reduce_smem(c, groups),
                            gn_bwd_apply_smem(c, groups), st->sm_count, reinterpret_cast<cudaStream_t>(stream), &o))
    return s;
  FP8_CUDA_TRY(cudaGetLastError());
  return ok();
}

}  // extern "C"

// ======================================================================== multi-tensor quantize
extern "C" {

size_t fp8_quantize_multi_workspace_bytes(int count) {
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  (void)cudaGetLastError();
  if (count < 1 || count > kMaxMultiTensors) return 0;
  return static_cast<size_t>(count) * quant_workspace_bytes(sms > 0 ? sms : 148);
}

int fp8_quantize_current_multi(int count, const void* const* x_bf16, void* const* q_e4m3, float* const* scale_out,
                               const int64_t* n, void* workspace, size_t workspace_bytes, fp8_stream_t stream) {
  FP8_REQUIRE(count >= 1 && count <= kMaxMultiTensors, FP8_ERR_INVALID_ARGUMENT, "count must be 1..%d",
              kMaxMultiTensors);
  FP8_REQUIRE(x_bf16 && q_e4m3 && scale_out && n, FP8_ERR_INVALID_ARGUMENT, "NULL argument array");
  bool vec = true;
  for (int t = 0; t < count; ++t) {
    FP8_REQUIRE(n[t] >= 0, FP8_ERR_INVALID_ARGUMENT, "n[%d] must be >= 0", t);
    FP8_REQUIRE(scale_out[t] != nullptr && aligned(scale_out[t], 4), FP8_ERR_INVALID_ARGUMENT, "bad scale_out[%d]",
                t);
    FP8_REQUIRE(n[t] == 0 || (x_bf16[t] != nullptr && q_e4m3[t] != nullptr), FP8_ERR_INVALID_ARGUMENT,
                "NULL tensor %d", t);
    FP8_REQUIRE(aligned(x_bf16[t], 2), FP8_ERR_INVALID_ARGUMENT, "x[%d] must be 2-byte aligned", t);
    vec = vec && aligned(x_bf16[t], 16) && aligned(q_e4m3[t], 8);
  }
  if (!vec) {  // odd views: one call per tensor (each uses the first slots of the workspace)
    for (int t = 0; t < count; ++t)
      if (int s = fp8_quantize_current(x_bf16[t], q_e4m3[t], scale_out[t], workspace, workspace_bytes, n[t], stream))
        return s;
    return ok();
  }
  DeviceState* st = nullptr;
  if (int s = device_state(&st)) return s;
  MultiQuant m{};
  m.count = count;
  m.chunk_begin[0] = 0;
  for (int t = 0; t < count; ++t) {
    m.x[t] = static_cast<const uint16_t*>(x_bf16[t]);
    m.q[t] = static_cast<uint8_t*>(q_e4m3[t]);
    m.scale_out[t] = scale_out[t];
    m.n[t] = n[t];
    m.main_bytes[t] = (n[t] & ~int64_t(7)) * 2;
    m.chunk_begin[t + 1] = m.chunk_begin[t] + (m.main_bytes[t] + kStreamChunkBytes - 1) / kStreamChunkBytes;
  }
  auto grid_for = [&](int bps) {
    int64_t g = m.chunk_begin[count];
    const int64_t cap = static_cast<int64_t>(st->sm_count) * std::min(bps, kMaxStreamBlocksPerSm);
    if (g > cap) g = cap;
    return static_cast<int>(g < 1 ? 1 : g);
  };
  const int parts = grid_for(g_quant_amax_bps);
  const int cast_blocks = grid_for(g_quant_cast_bps);
  FP8_REQUIRE(workspace != nullptr && aligned(workspace, 4) &&
                  workspace_bytes >= static_cast<size_t>(count) * parts * sizeof(float),
              FP8_ERR_WORKSPACE, "quantize workspace too small: need %zu bytes",
              static_cast<size_t>(count) * parts * sizeof(float));
  float* partials = static_cast<float*>(workspace);
  cudaStream_t cs = reinterpret_cast<cudaStream_t>(stream);
  if (g_quant_resident) {
    bool launched = false;
    if (int s = launch_quant_resident(m, st, cs, &launched)) return s;
    if (launched) return ok();
  }
  FP8_CUDA_TRY(cudaFuncSetAttribute(quant_multi_amax_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    static_cast<int>(kStreamSmemBytes)));
  FP8_CUDA_TRY(cudaFuncSetAttribute(quant_multi_cast_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    static_cast<int>(kStreamSmemBytes)));
  FP8_CUDA_TRY(launch_kernel(quant_multi_amax_kernel, dim3(parts), dim3(kStreamThreads), kStreamSmemBytes, cs, 1,
                             kStreamingKernel, m, partials, st->err_ptr));
  FP8_CUDA_TRY(launch_kernel(quant_multi_cast_kernel, dim3(cast_blocks), dim3(kStreamThreads), kStreamSmemBytes, cs, 1,
                             kStreamingKernel, m, static_cast<const float*>(partials), parts, st->err_ptr));
  count_launches(2);
  FP8_CUDA_TRY(cudaGetLastError());
  return ok();
}

}  // extern "C"

// ======================================================================== data-grad on the forward's weights
namespace {
// Whether fp8_conv3x3_dgrad_w reads wq in place (the transposed halo kernel);
// dx is 16-byte aligned by the entry point's own check.
bool dgrad_reads_w_in_place(int height, int width, int cin, int cout) {
  return (g_conv_algo == 0 || g_conv_algo == 4) && halo_applies(height, width) &&
         (width == 32 || width == 16) && cout == 128 && cin % 128 == 0 && (height * width) % 256 == 0;
}
}  // namespace

extern "C" {

size_t fp8_conv3x3_dgrad_w_workspace_bytes(int batch, int height, int width, int cin, int cout) {
  (void)batch;
  if (cin <= 0 || cout <= 0 || dgrad_reads_w_in_place(height, width, cin, cout)) return 0;
  return static_cast<size_t>(9) * cin * cout;
}

int fp8_conv3x3_dgrad_w(const void* dyq, const void* wq, void* dx, const float* sdy, const float* sw, int batch,
                        int height, int width, int cin, int cout, void* workspace, size_t workspace_bytes,
                        fp8_stream_t stream) {
  ConvTile t;
  if (int s = check_conv_args(batch, height, width, cin, cout, &t)) return s;
  if (int s = check_scale_ptrs(sdy, sw)) return s;
  FP8_REQUIRE(dyq && wq && dx, FP8_ERR_INVALID_ARGUMENT, "NULL tensor");
  FP8_REQUIRE(aligned(dyq, 16) && aligned(wq, 16) && aligned(dx, 16), FP8_ERR_INVALID_ARGUMENT,
              "conv tensors must be 16-byte aligned");
  const bool in_place = dgrad_reads_w_in_place(height, width, cin, cout);
  const size_t need = in_place ? 0 : static_cast<size_t>(9) * cin * cout;
  FP8_REQUIRE(in_place || (workspace != nullptr && workspace_bytes >= need && aligned(workspace, 16)),
              FP8_ERR_WORKSPACE, "data-grad workspace too small: need %zu bytes for the re-laid-out weights", need);
  cudaStream_t cs = reinterpret_cast<cudaStream_t>(stream);
  if (in_place) {
    DeviceState* st = nullptr;
    if (int s = device_state(&st)) return s;
    if (int s = launch_conv_halo(dyq, wq, dx, sdy, sw, nullptr, kEpiNone, batch, height, width, cout, cin, false,
                                 st->err_ptr, st->sm_count, cs, true))
      return s;
    return ok();
  }
  if (int s = fp8_conv_weight_transpose(wq, workspace, cout, cin, stream)) return s;
  return fp8_conv3x3_dgrad(dyq, workspace, dx, sdy, sw, batch, height, width, cin, cout, stream);
}

}  // extern "C"

// ======================================================================== layer norm (attention tokens)
namespace {

int ln_vpl(int c) { return c <= 256 ? 1 : (c <= 512 ? 2 : 4); }

int check_ln_args(const void* x, const void* out, const float* gamma, int64_t tokens, int c) {
  FP8_REQUIRE(tokens >= 0 && c > 0, FP8_ERR_INVALID_ARGUMENT, "bad layer-norm sizes");
  FP8_REQUIRE(c % 8 == 0 && c <= 1024, FP8_ERR_UNSUPPORTED, "layer norm needs c %% 8 == 0 and c <= 1024 (c=%d)", c);
  FP8_REQUIRE(tokens == 0 || (x && out && gamma), FP8_ERR_INVALID_ARGUMENT, "NULL tensor");
  FP8_REQUIRE(aligned(x, 16) && aligned(out, 16), FP8_ERR_INVALID_ARGUMENT, "tokens must be 16-byte aligned");
  return FP8_OK;
}

int ln_bwd_ctas(int64_t tokens, int sm_count) {
  const int64_t need = (tokens + kLnWarps - 1) / kLnWarps;
  return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(need, 4ll * sm_count)));
}

template <typename TX, int VPL>
int launch_ln_fwd(const TX* x, const float* gamma, const float* beta, float eps, void* y, float* mr,
                  int64_t tokens, int c, int sm_count, cudaStream_t cs) {
  const int64_t need = (tokens + kLnWarps - 1) / kLnWarps;
  const unsigned grid = static_cast<unsigned>(std::max<int64_t>(1, std::min<int64_t>(need, 8ll * sm_count)));
  FP8_CUDA_TRY(launch_kernel(ln_fwd_kernel<TX, VPL>, dim3(grid), dim3(kLnThreads), 0, cs, 1, kStreamingKernel, x,
                             gamma, beta, tokens, c, eps, static_cast<uint16_t*>(y), reinterpret_cast<float2*>(mr)));
  count_launches(1);
  return FP8_OK;
}

template <typename TX, int VPL>
int launch_ln_bwd(const TX* x, const uint16_t* dy, const float* gamma, const float* mr, TX* dx, float* dgamma,
                  float* dbeta, float* part, int64_t tokens, int c, int sm_count, cudaStream_t cs) {
  const int parts = ln_bwd_ctas(tokens, sm_count);
  const size_t smem = static_cast<size_t>(kLnWarps) * 2 * c * sizeof(float);
  FP8_CUDA_TRY(cudaFuncSetAttribute(ln_bwd_kernel<TX, VPL>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    static_cast<int>(smem)));
  FP8_CUDA_TRY(launch_kernel(ln_bwd_kernel<TX, VPL>, dim3(parts), dim3(kLnThreads), smem, cs, 1, kStreamingKernel, x,
                             dy, gamma, reinterpret_cast<const float2*>(mr), tokens, c, dx, part));
  FP8_CUDA_TRY(launch_kernel(ln_param_reduce_kernel, dim3((2 * c + kLnWarps - 1) / kLnWarps), dim3(kLnThreads), 0, cs,
                             1, kStreamingKernel, static_cast<const float*>(part), parts, c, dgamma, dbeta));
  count_launches(2);
  return FP8_OK;
}

}  // namespace

extern "C" {

size_t fp8_layer_norm_workspace_bytes(int64_t tokens, int c) {
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  (void)cudaGetLastError();
  if (tokens <= 0 || c <= 0) return 0;
  if (sms <= 0) sms = 148;
  return static_cast<size_t>(ln_bwd_ctas(tokens, sms)) * 2 * c * sizeof(float);
}

int fp8_layer_norm_fwd(const void* x, int x_fp32, const float* gamma, const float* beta, float eps, void* y_bf16,
                       float* mean_rstd, int64_t tokens, int c, fp8_stream_t stream) {
  if (int s = check_ln_args(x, y_bf16, gamma, tokens, c)) return s;
  FP8_REQUIRE(tokens == 0 || (beta && mean_rstd), FP8_ERR_INVALID_ARGUMENT, "NULL beta / statistics");
  FP8_REQUIRE(eps > 0.0f, FP8_ERR_INVALID_ARGUMENT, "eps must be > 0");
  if (tokens == 0) return ok();
  DeviceState* st = nullptr;
  if (int s = device_state(&st)) return s;
  cudaStream_t cs = reinterpret_cast<cudaStream_t>(stream);
  const int vpl = ln_vpl(c);
  int s = FP8_OK;
  if (x_fp32) {
    const float* xf = static_cast<const float*>(x);
    s = vpl == 1 ? launch_ln_fwd<float, 1>(xf, gamma, beta, eps, y_bf16, mean_rstd, tokens, c, st->sm_count, cs)
        : vpl == 2 ? launch_ln_fwd<float, 2>(xf, gamma, beta, eps, y_bf16, mean_rstd, tokens, c, st->sm_count, cs)
                   : launch_ln_fwd<float, 4>(xf, gamma, beta, eps, y_bf16, mean_rstd, tokens, c, st->sm_count, cs);
  } else {
    const uint16_t* xb = static_cast<const uint16_t*>(x);
    s = vpl == 1 ? launch_ln_fwd<uint16_t, 1>(xb, gamma, beta, eps, y_bf16, mean_rstd, tokens, c, st->sm_count, cs)
        : vpl == 2 ? launch_ln_fwd<uint16_t, 2>(xb, gamma, beta, eps, y_bf16, mean_rstd, tokens, c, st->sm_count, cs)
                   : launch_ln_fwd<uint16_t, 4>(xb, gamma, beta, eps, y_bf16, mean_rstd, tokens, c, st->sm_count, cs);
  }
  if (s) return s;
  FP8_CUDA_TRY(cudaGetLastError());
  return ok();
}

int fp8_layer_norm_bwd(const void* x, int x_fp32, const void* dy_bf16, const float* gamma, const float* mean_rstd,
                       void* dx, float* dgamma, float* dbeta, int64_t tokens, int c, void* workspace,
                       size_t workspace_bytes, fp8_stream_t stream) {
  if (int s = check_ln_args(x, dx, gamma, tokens, c)) return s;
  FP8_REQUIRE(tokens == 0 || (dy_bf16 && aligned(dy_bf16, 16) && mean_rstd && dgamma && dbeta),
              FP8_ERR_INVALID_ARGUMENT, "NULL or unaligned dy / statistics / parameter gradients");
  if (tokens == 0) return ok();
  DeviceState* st = nullptr;
  if (int s = device_state(&st)) return s;
  const size_t need = static_cast<size_t>(ln_bwd_ctas(tokens, st->sm_count)) * 2 * c * sizeof(float);
  FP8_REQUIRE(workspace != nullptr && workspace_bytes >= need && aligned(workspace, 16), FP8_ERR_WORKSPACE,
              "layer-norm workspace too small: need %zu bytes", need);
  cudaStream_t cs = reinterpret_cast<cudaStream_t>(stream);
  float* part = static_cast<float*>(workspace);
  const uint16_t* dy = static_cast<const uint16_t*>(dy_bf16);
  const int vpl = ln_vpl(c);
  const int sms = st->sm_count;
  int s = FP8_OK;
  if (x_fp32) {
    const float* xf = static_cast<const float*>(x);
    float* d = static_cast<float*>(dx);
    s = vpl == 1 ? launch_ln_bwd<float, 1>(xf, dy, gamma, mean_rstd, d, dgamma, dbeta, part, tokens, c, sms, cs)
        : vpl == 2 ? launch_ln_bwd<float, 2>(xf, dy, gamma, mean_rstd, d, dgamma, dbeta, part, tokens, c, sms, cs)
                   : launch_ln_bwd<float, 4>(xf, dy, gamma, mean_rstd, d, dgamma, dbeta, part, tokens, c, sms, cs);
  } else {
    const uint16_t* xb = static_cast<const uint16_t*>(x);
    uint16_t* d = static_cast<uint16_t*>(dx);
    s = vpl == 1 ? launch_ln_bwd<uint16_t, 1>(xb, dy, gamma, mean_rstd, d, dgamma, dbeta, part, tokens, c, sms, cs)
        : vpl == 2 ? launch_ln_bwd<uint16_t, 2>(xb, dy, gamma, mean_rstd, d, dgamma, dbeta, part, tokens, c, sms, cs)
                   : launch_ln_bwd<uint16_t, 4>(xb, dy, gamma, mean_rstd, d, dgamma, dbeta, part, tokens, c, sms, cs);
  }
  if (s) return s;
  FP8_CUDA_TRY(cudaGetLastError());
  return ok();
}

}  // extern "C"

extern "C" int fp8_gn_param_grads(const float* totals, const void* film, int film_ld, int n, int c, float* dgamma,
                                  float* dbeta, void* dfilm, int dfilm_ld, fp8_stream_t stream) {
  FP8_REQUIRE(n > 0 && c > 0, FP8_ERR_INVALID_ARGUMENT, "bad sizes");
  FP8_REQUIRE(totals && dgamma && dbeta, FP8_ERR_INVALID_ARGUMENT, "NULL tensor");
  FP8_REQUIRE(film == nullptr || (film_ld >= 2 * c && dfilm != nullptr && dfilm_ld >= 2 * c),
              FP8_ERR_INVALID_ARGUMENT, "FiLM gradients need film_ld, dfilm_ld >= 2c and a dfilm buffer");
  DeviceState* st = nullptr;
  if (int s = device_state(&st)) return s;
  (void)st;
  FP8_CUDA_TRY(launch_kernel(gn_param_grads_kernel, dim3((c + 31) / 32), dim3(32 * kGnParamLanes), 0,
                             reinterpret_cast<cudaStream_t>(stream), 1, kStreamingKernel, totals,
                             static_cast<const uint16_t*>(film), film_ld, n, c, dgamma, dbeta,
                             static_cast<uint16_t*>(dfilm), dfilm_ld));
  count_launches(1);
  return ok();
}

// ======================================================================== resampling + concatenation
namespace {

unsigned resample_grid(int64_t vectors, int sm_count) {
  const int64_t blocks = (vectors + kResampleThreads - 1) / kResampleThreads;
  return static_cast<unsigned>(std::max<int64_t>(1, std::min<int64_t>(blocks, 16ll * sm_count)));
}

int check_resample(const void* p, int dtype, const char* what) {
  FP8_REQUIRE(dtype == 0 || dtype == 1, FP8_ERR_INVALID_ARGUMENT, "%s dtype must be 0 (bf16) or 1 (fp32)", what);
  FP8_REQUIRE(p != nullptr && aligned(p, 16), FP8_ERR_INVALID_ARGUMENT, "%s must be non-NULL and 16-byte aligned",
              what);
  return FP8_OK;
}

template <typename TA, typename TS, typename TO>
int launch_up_cat(const void* a, const void* s, void* y, void* y16, int n, int h, int w, int c1, int c2, int f,
                  bool bwd, int sm_count, cudaStream_t cs) {
  const int64_t vecs = static_cast<int64_t>(n) * h * w * (c1 + c2) / 8;
  if (!bwd) {
    FP8_CUDA_TRY(launch_kernel(up_cat_kernel<TA, TS, TO>, dim3(resample_grid(vecs, sm_count)), dim3(kResampleThreads),
                               0, cs, 1, kStreamingKernel, static_cast<const TA*>(a), static_cast<const TS*>(s), n, h,
                               w, c1, c2, f, static_cast<TO*>(y), static_cast<uint16_t*>(y16)));
  } else {  // a, s are the gradients (outputs); y (and y16) the incoming gradients
    FP8_CUDA_TRY(launch_kernel(up_cat_bwd_kernel<TA, TS, TO>, dim3(resample_grid(vecs, sm_count)),
                               dim3(kResampleThreads), 0, cs, 1, kStreamingKernel, static_cast<const TO*>(y),
                               static_cast<const uint16_t*>(y16), n, h, w, c1, c2, f,
                               static_cast<TA*>(const_cast<void*>(a)), static_cast<TS*>(const_cast<void*>(s))));
  }
  count_launches(1);
  return FP8_OK;
}

template <typename TA, typename TS>
int up_cat_out(int y_dtype, const void* a, const void* s, void* y, void* y16, int n, int h, int w, int c1, int c2,
               int f, bool bwd, int sms, cudaStream_t cs) {
  return y_dtype ? launch_up_cat<TA, TS, float>(a, s, y, y16, n, h, w, c1, c2, f, bwd, sms, cs)
                 : launch_up_cat<TA, TS, uint16_t>(a, s, y, y16, n, h, w, c1, c2, f, bwd, sms, cs);
}

int up_cat_dispatch(int a_dtype, int s_dtype, int y_dtype, const void* a, const void* s, void* y, void* y16, int n,
                    int h, int w, int c1, int c2, int f, bool bwd, int sms, cudaStream_t cs) {
  if (a_dtype)
    return s_dtype ? up_cat_out<float, float>(y_dtype, a, s, y, y16, n, h, w, c1, c2, f, bwd, sms, cs)
                   : up_cat_out<float, uint16_t>(y_dtype, a, s, y, y16, n, h, w, c1, c2, f, bwd, sms, cs);
  return s_dtype ? up_cat_out<uint16_t, float>(y_dtype, a, s, y, y16, n, h, w, c1, c2, f, bwd, sms, cs)
                 : up_cat_out<uint16_t, uint16_t>(y_dtype, a, s, y, y16, n, h, w, c1, c2, f, bwd, sms, cs);
}

int check_up_cat(int n, int h, int w, int c1, int c2, int factor) {
  FP8_REQUIRE(n > 0 && h > 0 && w > 0 && c1 > 0 && c2 > 0, FP8_ERR_INVALID_ARGUMENT, "bad sizes");
  FP8_REQUIRE(c1 % 8 == 0 && c2 % 8 == 0, FP8_ERR_UNSUPPORTED, "channel counts must be multiples of 8");
  FP8_REQUIRE((factor == 1 || factor == 2) && h % factor == 0 && w % factor == 0, FP8_ERR_UNSUPPORTED,
              "factor must be 1 or 2 and divide the output size");
  return FP8_OK;
}

}  // namespace

extern "C" {

int fp8_resample_down2(const void* x, int x_dtype, float* y, int n, int h, int w, int c, fp8_stream_t stream) {
  FP8_REQUIRE(n > 0 && h > 0 && w > 0 && c > 0, FP8_ERR_INVALID_ARGUMENT, "bad sizes");
  FP8_REQUIRE(c % 8 == 0 && h % 2 == 0 && w % 2 == 0, FP8_ERR_UNSUPPORTED, "needs c %% 8 == 0 and even h, w");
  if (int s = check_resample(x, x_dtype, "x")) return s;
  if (int s = check_resample(y, 1, "y")) return s;
  DeviceState* st = nullptr;
  if (int s = device_state(&st)) return s;
  cudaStream_t cs = reinterpret_cast<cudaStream_t>(stream);
  const dim3 grid(resample_grid(static_cast<int64_t>(n) * (h / 2) * (w / 2) * c / 8, st->sm_count));
  if (x_dtype)
    FP8_CUDA_TRY(launch_kernel(down2_kernel<float>, grid, dim3(kResampleThreads), 0, cs, 1, kStreamingKernel,
                               static_cast<const float*>(x), n, h, w, c, y));
  else
    FP8_CUDA_TRY(launch_kernel(down2_kernel<uint16_t>, grid, dim3(kResampleThreads), 0, cs, 1, kStreamingKernel,
                               static_cast<const uint16_t*>(x), n, h, w, c, y));
  count_launches(1);
  return ok();
}

int fp8_resample_down2_bwd(const float* dy, void* dx, int dx_dtype, int n, int h, int w, int c,
                           fp8_stream_t stream) {
  FP8_REQUIRE(n > 0 && h > 0 && w > 0 && c > 0, FP8_ERR_INVALID_ARGUMENT, "bad sizes");
  FP8_REQUIRE(c % 8 == 0 && h % 2 == 0 && w % 2 == 0, FP8_ERR_UNSUPPORTED, "needs c %% 8 == 0 and even h, w");
  if (int s = check_resample(dy, 1, "dy")) return s;
  if (int s = check_resample(dx, dx_dtype, "dx")) return s;
  DeviceState* st = nullptr;
  if (int s = device_state(&st)) return s;
  cudaStream_t cs = reinterpret_cast<cudaStream_t>(stream);
  const dim3 grid(resample_grid(static_cast<int64_t>(n) * h * w * c / 8, st->sm_count));
  if (dx_dtype)
    FP8_CUDA_TRY(launch_kernel(down2_bwd_kernel<float>, grid, dim3(kResampleThreads), 0, cs, 1, kStreamingKernel, dy,
                               n, h, w, c, static_cast<float*>(dx)));
  else
    FP8_CUDA_TRY(launch_kernel(down2_bwd_kernel<uint16_t>, grid, dim3(kResampleThreads), 0, cs, 1, kStreamingKernel,
                               dy, n, h, w, c, static_cast<uint16_t*>(dx)));
  count_launches(1);
  return ok();
}

int fp8_up_cat(const void* a, int a_dtype, const void* s, int s_dtype, void* y, int y_dtype, int n, int h, int w,
               int c1, int c2, int factor, fp8_stream_t stream) {
  if (int r = check_up_cat(n, h, w, c1, c2, factor)) return r;
  if (int r = check_resample(a, a_dtype, "a")) return r;
  if (int r = check_resample(s, s_dtype, "s")) return r;
  if (int r = check_resample(y, y_dtype, "y")) return r;
  DeviceState* st = nullptr;
  if (int r = device_state(&st)) return r;
  if (int r = up_cat_dispatch(a_dtype, s_dtype, y_dtype, a, s, y, nullptr, n, h, w, c1, c2, factor, false,
                              st->sm_count, reinterpret_cast<cudaStream_t>(stream)))
    return r;
  return ok();
}

int fp8_up_cat_bwd(const void* dy, int y_dtype, void* da, int a_dtype, void* ds, int s_dtype, int n, int h, int w,
                   int c1, int c2, int factor, fp8_stream_t stream) {
  if (int r = check_up_cat(n, h, w, c1, c2, factor)) return r;
  if (int r = check_resample(dy, y_dtype, "dy")) return r;
  if (int r = check_resample(da, a_dtype, "da")) return r;
  if (int r = check_resample(ds, s_dtype, "ds")) return r;
  DeviceState* st = nullptr;
  if (int r = device_state(&st)) return r;
  if (int r = up_cat_dispatch(a_dtype, s_dtype, y_dtype, da, ds, const_cast<void*>(dy), nullptr, n, h, w, c1, c2,
                              factor, true, st->sm_count, reinterpret_cast<cudaStream_t>(stream)))
    return r;
  return ok();
}

int fp8_up_cat_pair(const void* a, int a_dtype, const void* s, int s_dtype, float* y, void* y_bf16, int n, int h,
                    int w, int c1, int c2, int factor, fp8_stream_t stream) {
  if (int r = check_up_cat(n, h, w, c1, c2, factor)) return r;
  if (int r = check_resample(a, a_dtype, "a")) return r;
  if (int r = check_resample(s, s_dtype, "s")) return r;
  if (int r = check_resample(y, 1, "y")) return r;
  if (int r = check_resample(y_bf16, 0, "y_bf16")) return r;
  DeviceState* st = nullptr;
  if (int r = device_state(&st)) return r;
  if (int r = up_cat_dispatch(a_dtype, s_dtype, 1, a, s, y, y_bf16, n, h, w, c1, c2, factor, false, st->sm_count,
                              reinterpret_cast<cudaStream_t>(stream)))
    return r;
  return ok();
}

int fp8_up_cat_pair_bwd(const float* dy, const void* dy_bf16, void* da, int a_dtype, void* ds, int s_dtype, int n,
                        int h, int w, int c1, int c2, int factor, fp8_stream_t stream) {
  if (int r = check_up_cat(n, h, w, c1, c2, factor)) return r;
  if (int r = check_resample(dy, 1, "dy")) return r;
  if (int r = check_resample(dy_bf16, 0, "dy_bf16")) return r;
  if (int r = check_resample(da, a_dtype, "da")) return r;
  if (int r = check_resample(ds, s_dtype, "ds")) return r;
  DeviceState* st = nullptr;
  if (int r = device_state(&st)) return r;
  if (int r = up_cat_dispatch(a_dtype, s_dtype, 1, da, ds, const_cast<float*>(dy), const_cast<void*>(dy_bf16), n, h,
                              w, c1, c2, factor, true, st->sm_count, reinterpret_cast<cudaStream_t>(stream)))
    return r;
  return ok();
}

}  // extern "C"

// ======================================================================== batched weight quantize
namespace {
int weight_chunks(int64_t n) { return static_cast<int>((n + kWeightChunk - 1) / kWeightChunk); }
}  // namespace

extern "C" {

size_t fp8_quantize_weights_delayed_workspace_bytes(int count, const int64_t* n) {
  if (count <= 0 || n == nullptr) return 0;
  size_t chunks = 0;
  for (int t = 0; t < count; ++t) chunks += n[t] > 0 ? static_cast<size_t>(weight_chunks(n[t])) : 0;
  return chunks * sizeof(float);
}

int fp8_quantize_weights_delayed(int count, const float* const* w, void* const* q, const int64_t* n,
                                 float* const* windows, int window_len, const int64_t* const* pos,
                                 float* const* scale_used, void* workspace, size_t workspace_bytes,
                                 fp8_stream_t stream) {
  FP8_REQUIRE(count > 0 && count <= kMaxBatchWeights, FP8_ERR_UNSUPPORTED, "1..%d weights per call",
              kMaxBatchWeights);
  FP8_REQUIRE(w && q && n && windows && pos && scale_used && window_len > 0, FP8_ERR_INVALID_ARGUMENT,
              "NULL argument");
  WeightBatch b{};
  b.count = count;
  b.window_len = window_len;
  b.empty_zero = g_empty_zero;
  int chunks = 0;
  for (int t = 0; t < count; ++t) {
    FP8_REQUIRE(n[t] > 0 && n[t] < (1ll << 31), FP8_ERR_INVALID_ARGUMENT, "weight %d: bad size", t);
    FP8_REQUIRE(w[t] && aligned(w[t], 4) && q[t] && aligned(q[t], 2) && windows[t] && aligned(windows[t], 4) &&
                    pos[t] && aligned(pos[t], 8) && scale_used[t] && aligned(scale_used[t], 4),
                FP8_ERR_INVALID_ARGUMENT, "weight %d: NULL or unaligned pointer", t);
    b.w[t] = w[t];
    b.q[t] = static_cast<uint8_t*>(q[t]);
    b.window[t] = windows[t];
    b.pos[t] = pos[t];
    b.used[t] = scale_used[t];
    b.n[t] = n[t];
    b.chunk_begin[t] = chunks;
    chunks += weight_chunks(n[t]);
  }
  b.chunk_begin[count] = chunks;
  FP8_REQUIRE(workspace != nullptr && aligned(workspace, 4) && workspace_bytes >= chunks * sizeof(float),
              FP8_ERR_WORKSPACE, "workspace too small: need %zu bytes", chunks * sizeof(float));
  DeviceState* st = nullptr;
  if (int s = device_state(&st)) return s;
  (void)st;
  cudaStream_t cs = reinterpret_cast<cudaStream_t>(stream);
  float* partials = static_cast<float*>(workspace);
  FP8_CUDA_TRY(launch_kernel(weight_window_max_kernel, dim3(count), dim3(kQuantThreads), 0, cs, 1, kStreamingKernel,
                             b));
  FP8_CUDA_TRY(launch_kernel(weight_cast_kernel, dim3(chunks), dim3(kQuantThreads), 0, cs, 1, kStreamingKernel, b,
                             partials));
  FP8_CUDA_TRY(launch_kernel(weight_finalize_kernel, dim3(count), dim3(kQuantThreads), 0, cs, 1, kStreamingKernel,
                             b, static_cast<const float*>(partials)));
  count_launches(3);
  return ok();
}

}  // extern "C"

// ======================================================================== clip + AdamW + EMA
namespace {
int opt_chunks(int64_t n) { return static_cast<int>((n + kOptChunk - 1) / kOptChunk); }

// Groups of at most kOptTensors tensors: [first, last) ranges into the caller's arrays.
template <typename F>
int for_each_group(int count, F&& f) {
  for (int first = 0; first < count; first += kOptTensors)
    if (int s = f(first, std::min(count, first + kOptTensors))) return s;
  return FP8_OK;
}
}  // namespace

extern "C" {

size_t fp8_adamw_ema_workspace_bytes(int count, const int64_t* n) {
  if (count <= 0 || n == nullptr) return 0;
  size_t chunks = 0;
  for (int t = 0; t < count; ++t) chunks += n[t] > 0 ? static_cast<size_t>(opt_chunks(n[t])) : 0;
  return 16 + chunks * sizeof(float);
}

int fp8_adamw_ema_step(int count, float* const* params, const float* const* grads, float* const* exp_avg,
                       float* const* exp_avg_sq, float* const* ema, const int64_t* n, float* step, float lr,
                       float beta1, float beta2, float eps, float weight_decay, float ema_beta, float max_grad_norm,
                       void* workspace, size_t workspace_bytes, fp8_stream_t stream) {
  FP8_REQUIRE(count > 0, FP8_ERR_INVALID_ARGUMENT, "no parameters");
  FP8_REQUIRE(params && grads && exp_avg && exp_avg_sq && n && step, FP8_ERR_INVALID_ARGUMENT, "NULL argument");
  FP8_REQUIRE(aligned(step, 4), FP8_ERR_INVALID_ARGUMENT, "step must be a 4-byte aligned float");
  int64_t chunks = 0;
  for (int t = 0; t < count; ++t) {
    FP8_REQUIRE(n[t] > 0 && n[t] < (1ll << 31), FP8_ERR_INVALID_ARGUMENT, "tensor %d: bad size", t);
    FP8_REQUIRE(params[t] && grads[t] && exp_avg[t] && exp_avg_sq[t], FP8_ERR_INVALID_ARGUMENT,
                "tensor %d: NULL pointer", t);
    chunks += opt_chunks(n[t]);
  }
  FP8_REQUIRE(workspace != nullptr && aligned(workspace, 16) &&
                  workspace_bytes >= 16 + static_cast<size_t>(chunks) * sizeof(float),
              FP8_ERR_WORKSPACE, "workspace too small: need %zu bytes", 16 + static_cast<size_t>(chunks) * 4);
  DeviceState* st = nullptr;
  if (int s = device_state(&st)) return s;
  (void)st;
  cudaStream_t cs = reinterpret_cast<cudaStream_t>(stream);
  float* coef = static_cast<float*>(workspace);
  float* partials = coef + 4;
  auto group = [&](int first, int last, OptGroup* g) {
    *g = OptGroup{};
    g->count = last - first;
    int c = 0;
    for (int t = first; t < last; ++t) {
      const int i = t - first;
      g->p[i] = params[t];
      g->g[i] = grads[t];
      g->m[i] = exp_avg[t];
      g->v[i] = exp_avg_sq[t];
      g->ema[i] = ema != nullptr ? ema[t] : nullptr;
      g->n[i] = n[t];
      g->chunk_begin[i] = c;
      c += opt_chunks(n[t]);
    }
    g->chunk_begin[g->count] = c;
    return c;
  };
  int part0 = 0;
  if (max_grad_norm > 0.0f) {
    if (int s = for_each_group(count, [&](int first, int last) {
          OptGroup g;
          const int c = group(first, last, &g);
          FP8_CUDA_TRY(launch_kernel(opt_sumsq_kernel, dim3(c), dim3(kOptThreads), 0, cs, 1, kStreamingKernel, g,
                                     partials, part0));
          part0 += c;
          count_launches(1);
          return FP8_OK;
        }))
      return s;
  }
  FP8_CUDA_TRY(launch_kernel(opt_norm_kernel, dim3(1), dim3(kOptThreads), 0, cs, 1, kStreamingKernel,
                             static_cast<const float*>(partials), part0, max_grad_norm, coef, step));
  count_launches(1);
  const OptHyper h{lr, beta1, beta2, eps, weight_decay, ema_beta, max_grad_norm, coef, step};
  if (int s = for_each_group(count, [&](int first, int last) {
        OptGroup g;
        const int c = group(first, last, &g);
        FP8_CUDA_TRY(launch_kernel(opt_update_kernel, dim3(c), dim3(kOptThreads), 0, cs, 1, kStreamingKernel, g, h));
        count_launches(1);
        return FP8_OK;
      }))
    return s;
  return ok();
}

}  // extern "C"

// ======================================================================== residual joins
namespace {
template <typename TA, typename TB, typename TO>
int launch_add_scale(const void* a, const void* b, void* y, int64_t vecs, float inv, bool bwd, int sms,
                     cudaStream_t cs) {
  const dim3 grid(resample_grid(vecs, sms)), block(kResampleThreads);
  if (!bwd)
    FP8_CUDA_TRY(launch_kernel(add_scale_kernel<TA, TB, TO>, grid, block, 0, cs, 1, kStreamingKernel,
                               static_cast<const TA*>(a), static_cast<const TB*>(b), vecs, inv, static_cast<TO*>(y)));
  else  // a, b: the two gradients; y: the incoming gradient
    FP8_CUDA_TRY(launch_kernel(add_scale_bwd_kernel<TA, TB, TO>, grid, block, 0, cs, 1, kStreamingKernel,
                               static_cast<const TO*>(y), vecs, inv, static_cast<TA*>(const_cast<void*>(a)),
                               static_cast<TB*>(const_cast<void*>(b))));
  count_launches(1);
  return FP8_OK;
}

template <typename TA, typename TB>
int add_scale_out(int y_dtype, const void* a, const void* b, void* y, int64_t vecs, float inv, bool bwd, int sms,
                  cudaStream_t cs) {
  return y_dtype ? launch_add_scale<TA, TB, float>(a, b, y, vecs, inv, bwd, sms, cs)
                 : launch_add_scale<TA, TB, uint16_t>(a, b, y, vecs, inv, bwd, sms, cs);
}

int add_scale_dispatch(int a_dtype, int b_dtype, int y_dtype, const void* a, const void* b, void* y, int64_t n,
                       float inv, bool bwd, int sms, cudaStream_t cs) {
  const int64_t vecs = n / 8;
  if (a_dtype)
    return b_dtype ? add_scale_out<float, float>(y_dtype, a, b, y, vecs, inv, bwd, sms, cs)
                   : add_scale_out<float, uint16_t>(y_dtype, a, b, y, vecs, inv, bwd, sms, cs);
  return b_dtype ? add_scale_out<uint16_t, float>(y_dtype, a, b, y, vecs, inv, bwd, sms, cs)
                 : add_scale_out<uint16_t, uint16_t>(y_dtype, a, b, y, vecs, inv, bwd, sms, cs);
}
}  // namespace

extern "C" {

int fp8_add_scale(const void* a, int a_dtype, const void* b, int b_dtype, void* y, int y_dtype, int64_t n,
                  float inv_divisor, fp8_stream_t stream) {
  FP8_REQUIRE(n > 0 && n % 8 == 0, FP8_ERR_UNSUPPORTED, "n must be a positive multiple of 8");
  if (int r = check_resample(a, a_dtype, "a")) return r;
  if (int r = check_resample(b, b_dtype, "b")) return r;
  if (int r = check_resample(y, y_dtype, "y")) return r;
  DeviceState* st = nullptr;
  if (int r = device_state(&st)) return r;
  if (int r = add_scale_dispatch(a_dtype, b_dtype, y_dtype, a, b, y, n, inv_divisor, false, st->sm_count,
                                 reinterpret_cast<cudaStream_t>(stream)))
    return r;
  return ok();
}

int fp8_add_scale_bwd(const void* dy, int y_dtype, void* da, int a_dtype, void* db, int b_dtype, int64_t n,
                      float inv_divisor, fp8_stream_t stream) {
  FP8_REQUIRE(n > 0 && n % 8 == 0, FP8_ERR_UNSUPPORTED, "n must be a positive multiple of 8");
  if (int r = check_resample(dy, y_dtype, "dy")) return r;
  if (int r = check_resample(da, a_dtype, "da")) return r;
  if (int r = check_resample(db, b_dtype, "db")) return r;
  DeviceState* st = nullptr;
  if (int r = device_state(&st)) return r;
  if (int r = add_scale_dispatch(a_dtype, b_dtype, y_dtype, da, db, const_cast<void*>(dy), n, inv_divisor, true,
                                 st->sm_count, reinterpret_cast<cudaStream_t>(stream)))
    return r;
  return ok();
}

// ======================================================================== batched casts
int fp8_cast_batch(int count, const void* const* src, void* const* dst, const int64_t* n, int to_bf16,
                   fp8_stream_t stream) {
  FP8_REQUIRE(count > 0 && count <= kCastTensors, FP8_ERR_UNSUPPORTED, "1..%d tensors per call", kCastTensors);
  FP8_REQUIRE(src && dst && n, FP8_ERR_INVALID_ARGUMENT, "NULL argument");
  CastBatch b{};
  b.count = count;
  int64_t chunks = 0;
  for (int t = 0; t < count; ++t) {
    FP8_REQUIRE(n[t] >= 0, FP8_ERR_INVALID_ARGUMENT, "tensor %d: negative size", t);
    FP8_REQUIRE(n[t] == 0 || (src[t] != nullptr && dst[t] != nullptr), FP8_ERR_INVALID_ARGUMENT,
                "tensor %d: NULL pointer", t);
    FP8_REQUIRE(aligned(src[t], to_bf16 ? 4 : 2) && aligned(dst[t], to_bf16 ? 2 : 4), FP8_ERR_INVALID_ARGUMENT,
                "tensor %d: misaligned for its dtype", t);
    b.src[t] = src[t];
    b.dst[t] = dst[t];
    b.n[t] = n[t];
    b.chunk_begin[t] = static_cast<int>(chunks);
    chunks += (n[t] + kCastChunk - 1) / kCastChunk;
    FP8_REQUIRE(chunks < (1ll << 30), FP8_ERR_UNSUPPORTED, "tensors too large");
  }
  b.chunk_begin[count] = static_cast<int>(chunks);
  if (chunks == 0) return ok();
  DeviceState* st = nullptr;
  if (int r = device_state(&st)) return r;
  (void)st;
  cudaStream_t cs = reinterpret_cast<cudaStream_t>(stream);
  if (to_bf16)
    FP8_CUDA_TRY(launch_kernel(cast_batch_kernel<true>, dim3(static_cast<unsigned>(chunks)), dim3(kCastThreads), 0, cs,
                               1, kStreamingKernel, b));
  else
    FP8_CUDA_TRY(launch_kernel(cast_batch_kernel<false>, dim3(static_cast<unsigned>(chunks)), dim3(kCastThreads), 0,
                               cs, 1, kStreamingKernel, b));
  count_launches(1);
  return ok();
}

}  // extern "C"

// ======================================================================== join backward + dY quantize
namespace {
int add_scale_quant_grid(int64_t n, int sm_count) {
  const int64_t per_cta = static_cast<int64_t>(kResampleThreads) * kJoinUnroll;
  return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>((n / 8 + per_cta - 1) / per_cta, 4ll * sm_count)));
}

template <typename TA, typename TO>
int launch_add_scale_bwd_quant(const void* dy, void* da, void* db, void* dbq, const DelayedSource& src,
                               float* partials, const ScaleFold& fold, int64_t n, float inv, int grid,
                               cudaStream_t cs) {
  FP8_CUDA_TRY(launch_kernel(add_scale_bwd_quant_kernel<TA, TO>, dim3(static_cast<unsigned>(grid)),
                             dim3(kResampleThreads), 0, cs, 1, kStreamingKernel, static_cast<const TO*>(dy), n / 8,
                             inv, static_cast<TA*>(da), static_cast<uint16_t*>(db), static_cast<uint8_t*>(dbq), src,
                             partials, fold));
  count_launches(1);
  return FP8_OK;
}
}  // namespace

extern "C" {

size_t fp8_add_scale_bwd_quant_workspace_bytes(int64_t n) {
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  (void)cudaGetLastError();
  if (n <= 0 || n % 8 != 0) return 0;
  if (sms <= 0) sms = 148;
  return static_cast<size_t>(add_scale_quant_grid(n, sms)) * sizeof(float);
}

int fp8_add_scale_bwd_quant(const void* dy, int y_dtype, void* da, int a_dtype, void* db_bf16, void* dbq_e4m3,
                            float* window, int window_len, int64_t* window_pos, float* scale_used_out, int64_t n,
                            float inv_divisor, void* workspace, size_t workspace_bytes, fp8_stream_t stream) {
  FP8_REQUIRE(n > 0 && n % 8 == 0, FP8_ERR_UNSUPPORTED, "n must be a positive multiple of 8");
  if (int r = check_resample(dy, y_dtype, "dy")) return r;
  if (int r = check_resample(da, a_dtype, "da")) return r;
  if (int r = check_resample(db_bf16, 0, "db")) return r;
  FP8_REQUIRE(dbq_e4m3 != nullptr && aligned(dbq_e4m3, 16), FP8_ERR_INVALID_ARGUMENT,
              "dbq must be non-NULL and 16-byte aligned");
  if (int r = check_window(window, window_len, window_pos, scale_used_out)) return r;
  DeviceState* st = nullptr;
  if (int r = device_state(&st)) return r;
  const int grid = add_scale_quant_grid(n, st->sm_count);
  FP8_REQUIRE(workspace != nullptr && workspace_bytes >= grid * sizeof(float) && aligned(workspace, 4),
              FP8_ERR_WORKSPACE, "join workspace too small: need %zu bytes", grid * sizeof(float));
  const DelayedSource src{nullptr, window, window_len, scale_used_out};
  const ScaleFold fold{fold_counter(st), nullptr, WindowUpdate{window, window_pos, window_len, 0, g_empty_zero}};
  float* partials = static_cast<float*>(workspace);
  cudaStream_t cs = reinterpret_cast<cudaStream_t>(stream);
  int r;
  if (a_dtype)
    r = y_dtype ? launch_add_scale_bwd_quant<float, float>(dy, da, db_bf16, dbq_e4m3, src, partials, fold, n,
                                                            inv_divisor, grid, cs)
                : launch_add_scale_bwd_quant<float, uint16_t>(dy, da, db_bf16, dbq_e4m3, src, partials, fold, n,
                                                               inv_divisor, grid, cs);
  else
    r = y_dtype ? launch_add_scale_bwd_quant<uint16_t, float>(dy, da, db_bf16, dbq_e4m3, src, partials, fold, n,
                                                               inv_divisor, grid, cs)
                : launch_add_scale_bwd_quant<uint16_t, uint16_t>(dy, da, db_bf16, dbq_e4m3, src, partials, fold, n,
                                                                  inv_divisor, grid, cs);
  if (r) return r;
  return ok();
}

}  // extern "C"

// ------------------------------------------------------------------ FP8 attention
namespace {
int attn_check(const void* qkv, int batch, int seq, int heads, int head_dim, int ld_qkv, int ld_o) {
  FP8_REQUIRE(head_dim == kAttnHeadDim, FP8_ERR_UNSUPPORTED, "attention head_dim must be %d", kAttnHeadDim);
  FP8_REQUIRE(seq >= 16 && seq <= kAttnMaxSeq && seq % 16 == 0, FP8_ERR_UNSUPPORTED,
              "attention sequence length must be a multiple of 16 in [16, %d]", kAttnMaxSeq);
  FP8_REQUIRE(batch > 0 && heads > 0 && static_cast<int64_t>(batch) * heads <= (1 << 30), FP8_ERR_INVALID_ARGUMENT,
              "bad batch / heads");
  FP8_REQUIRE(ld_qkv >= 3 * heads * head_dim && ld_qkv % 8 == 0 && ld_o >= heads * head_dim && ld_o % 8 == 0,
              FP8_ERR_INVALID_ARGUMENT, "row strides must cover the heads and be multiples of 8 elements");
  FP8_REQUIRE(qkv != nullptr && aligned(qkv, 16), FP8_ERR_INVALID_ARGUMENT, "qkv must be 16-byte aligned");
  return FP8_OK;
}
}  // namespace

extern "C" {

int fp8_attention_fwd(const void* qkv, void* o, float* lse, float* scales, int batch, int seq, int heads,
                      int head_dim, int ld_qkv, int ld_o, fp8_stream_t stream) {
  if (int s = attn_check(qkv, batch, seq, heads, head_dim, ld_qkv, ld_o)) return s;
  FP8_REQUIRE(o && aligned(o, 16) && lse && aligned(lse, 4) && scales && aligned(scales, 16), FP8_ERR_INVALID_ARGUMENT,
              "o must be 16-byte aligned, lse 4-byte and scales 16-byte");
  DeviceState* st = nullptr;
  if (int s = device_state(&st)) return s;
  AttnParams p{};
  p.qkv = static_cast<const uint16_t*>(qkv);
  p.o = static_cast<uint16_t*>(o);
  p.lse = lse;
  p.scales = scales;
  p.seq = seq;
  p.heads = heads;
  p.ld_qkv = ld_qkv;
  p.ld_o = ld_o;
  p.err = st->err_ptr;
  constexpr int smem = AttnFwdLayout::kSmemBytes;
  FP8_CUDA_TRY(cudaFuncSetAttribute(attn_fwd_fp8_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  count_launches(1);
  const int nqt = (seq + 127) / 128;
  FP8_CUDA_TRY(launch_kernel(attn_fwd_fp8_kernel, dim3(static_cast<unsigned>(batch * heads * nqt)), dim3(kAttnThreads), smem,
                             reinterpret_cast<cudaStream_t>(stream), 1, kTensorKernel, p));
  return ok();
}

int fp8_attention_bwd(const void* qkv, const void* o, const void* dout, const float* lse, const float* scales,
                      void* dqkv, int batch, int seq, int heads, int head_dim, int ld_qkv, int ld_o,
                      fp8_stream_t stream) {
  if (int s = attn_check(qkv, batch, seq, heads, head_dim, ld_qkv, ld_o)) return s;
  FP8_REQUIRE(o && aligned(o, 16) && dout && aligned(dout, 16) && dqkv && aligned(dqkv, 16) && lse &&
                  aligned(lse, 4) && scales && aligned(scales, 16),
              FP8_ERR_INVALID_ARGUMENT, "o, dout and dqkv must be 16-byte aligned, lse 4-byte and scales 16-byte");
  DeviceState* st = nullptr;
  if (int s = device_state(&st)) return s;
  AttnParams p{};
  p.qkv = static_cast<const uint16_t*>(qkv);
  p.o_in = static_cast<const uint16_t*>(o);
  p.dout = static_cast<const uint16_t*>(dout);
  p.dqkv = static_cast<uint16_t*>(dqkv);
  p.lse = const_cast<float*>(lse);
  p.scales = const_cast<float*>(scales);
  p.seq = seq;
  p.heads = heads;
  p.ld_qkv = ld_qkv;
  p.ld_o = ld_o;
  p.err = st->err_ptr;
  constexpr int smem = AttnBwdLayout::kSmemBytes;
  FP8_CUDA_TRY(cudaFuncSetAttribute(attn_bwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  count_launches(1);
  FP8_CUDA_TRY(launch_kernel(attn_bwd_kernel, dim3(static_cast<unsigned>(batch * heads)), dim3(kAttnThreads), smem,
                             reinterpret_cast<cudaStream_t>(stream), 1, kTensorKernel, p));
  return ok();
}

}  // extern "C"
