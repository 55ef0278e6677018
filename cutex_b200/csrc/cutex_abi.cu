// Host side of libcutex_mxfp8.so: argument validation, configuration
// resolution, TMA descriptor encoding and kernel launch for the C ABI in
// include/cutex_mxfp8.h. Nothing here allocates device memory or
// synchronises a stream (except cutex_last_device_status, by contract).
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstddef>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "../../include/cutex_mxfp8.h"
#include "mxfp8_gemm.cuh"
#include "mxfp8_quant.cuh"
#include "mxfp8_quant_columnwise.cuh"
#include "mxfp8_skinny.cuh"

namespace cutex {
namespace {

constexpr int kMaxDevices = 64;
constexpr int64_t kMaxDim = (int64_t{1} << 31) - 1;
constexpr int kMaxGatherPeers = 7;  // peers of the fused all-gather (8 GPUs per node)
static_assert(sizeof(cutex_epilogue) == 80 && offsetof(cutex_epilogue, out_dtype) == 32 &&
                  offsetof(cutex_epilogue, d_scales) == 40,
              "cutex_epilogue layout (mirrored by the Python binding)");
static_assert(sizeof(cutex_gemm_config) == 64 && sizeof(cutex_gemm_info) == 64, "config / info layouts");

struct DeviceState {
  bool ready = false;
  int status = CUTEX_OK;
  int sm_count = 0;
  int cc_major = 0, cc_minor = 0;
};

std::mutex g_mutex;
DeviceState g_devices[kMaxDevices];

// Per-device caches (kernel attributes, occupancy, the no-allocation scratch
// address, the host pipeline's streams) are only valid inside the CUDA context
// they were filled in. Each device has an epoch that changes whenever the
// current context of that device is a different one (a device reset destroys
// the primary context; its successor gets a new, never reused, context ID), and
// every cache records the epoch it was filled in. g_epoch is guarded by g_mutex.
unsigned long long g_ctx_id[kMaxDevices];
unsigned g_epoch[kMaxDevices];

unsigned long long current_context_id() {
  static PFN_cuCtxGetCurrent_v4000 get_ctx = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      p = nullptr;
    return reinterpret_cast<PFN_cuCtxGetCurrent_v4000>(p);
  }();
  static PFN_cuCtxGetId_v12000 get_id = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      p = nullptr;
    return reinterpret_cast<PFN_cuCtxGetId_v12000>(p);
  }();
  CUcontext ctx = nullptr;
  unsigned long long id = 0;
  if (get_ctx == nullptr || get_id == nullptr || get_ctx(&ctx) != CUDA_SUCCESS || ctx == nullptr ||
      get_id(ctx, &id) != CUDA_SUCCESS)
    return 0;
  return id;
}

// With g_mutex held: the device's epoch, advanced if its current context changed.
// Before the runtime has created a context there is none to ask about (ID 0):
// the first real ID seen then advances the epoch once. Only driver queries are
// made here, nothing that a stream capture forbids.
unsigned device_epoch_locked(int dev) {
  const unsigned long long id = current_context_id();
  if (g_epoch[dev] == 0 || (id != 0 && id != g_ctx_id[dev])) {
    g_ctx_id[dev] = id;
    ++g_epoch[dev];
    g_devices[dev].ready = false;
  }
  return g_epoch[dev];
}

unsigned device_epoch(int dev) {
  std::lock_guard<std::mutex> lock(g_mutex);
  return device_epoch_locked(dev);
}

int current_device_state(DeviceState** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return CUTEX_ERR_CUDA;
  std::lock_guard<std::mutex> lock(g_mutex);
  device_epoch_locked(dev);
  DeviceState& st = g_devices[dev];
  if (!st.ready) {
    if (cudaDeviceGetAttribute(&st.sm_count, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&st.cc_major, cudaDevAttrComputeCapabilityMajor, dev) !=
            cudaSuccess ||
        cudaDeviceGetAttribute(&st.cc_minor, cudaDevAttrComputeCapabilityMinor, dev) !=
            cudaSuccess) {
      return CUTEX_ERR_CUDA;
    }
    st.status = (st.cc_major == 10 && st.cc_minor == 0) ? CUTEX_OK : CUTEX_ERR_UNSUPPORTED_DEVICE;
    st.ready = true;
  }
  *out = &st;
  return st.status;
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) !=
            cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      p = nullptr;
    return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }();
  return fn;
}

bool encode(CUtensorMap* map, CUtensorMapDataType dtype, uint32_t rank, const void* ptr,
            const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box,
            CUtensorMapSwizzle swizzle, CUtensorMapL2promotion promo) {
  auto fn = encode_fn();
  if (fn == nullptr) return false;
  cuuint64_t d[5];
  cuuint64_t s[4];
  cuuint32_t b[5];
  cuuint32_t e[5];
  for (uint32_t i = 0; i < rank; ++i) {
    d[i] = dims[i];
    b[i] = box[i];
    e[i] = 1;
    if (i + 1 < rank) s[i] = strides_bytes[i];
  }
  return fn(map, dtype, rank, const_cast<void*>(ptr), d, s, b, e, CU_TENSOR_MAP_INTERLEAVE_NONE,
            swizzle, promo, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// K-major e4m3 operand [rows, K] read in (box_rows x 128) tiles, 128-byte swizzle.
bool encode_operand(CUtensorMap* map, const void* p, int64_t rows, int64_t K, uint32_t box_rows) {
  const uint64_t dims[2] = {static_cast<uint64_t>(K), static_cast<uint64_t>(rows)};
  const uint64_t strides[1] = {static_cast<uint64_t>(K)};
  const uint32_t box[2] = {128u, box_rows};
  return encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, p, dims, strides, box,
                CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B);
}

// Swizzled scales viewed as [row blocks][K/128][128 x u32]: one 512-byte chunk
// per (128-row block, 128-K stage); `blocks` consecutive row blocks per load.
bool encode_scales(CUtensorMap* map, const void* p, int64_t rows, int64_t K, uint32_t blocks) {
  const int64_t row_blocks = (rows + 127) / 128;
  const uint64_t dims[3] = {128u, static_cast<uint64_t>(K / 128), static_cast<uint64_t>(row_blocks)};
  const uint64_t strides[2] = {512u, static_cast<uint64_t>(K / 128) * 512u};
  const uint32_t box[3] = {128u, 1u, blocks};
  return encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT32, 3, p, dims, strides, box,
                CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE);
}

// bf16 output [M, N] with row stride ldd, written in 32 x 64 boxes.
bool encode_output(CUtensorMap* map, void* p, int64_t M, int64_t N, int64_t ldd) {
  const uint64_t dims[2] = {static_cast<uint64_t>(N), static_cast<uint64_t>(M)};
  const uint64_t strides[1] = {static_cast<uint64_t>(ldd) * 2u};
  const uint32_t box[2] = {64u, 32u};
  return encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, p, dims, strides, box,
                CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE);
}

// bf16 output [M, N] of the skinny kernel: 32 x 32 boxes (one epilogue warp's
// 32 columns), no swizzle.
bool encode_output_skinny(CUtensorMap* map, void* p, int64_t M, int64_t N, int64_t ldd) {
  const uint64_t dims[2] = {static_cast<uint64_t>(N), static_cast<uint64_t>(M)};
  const uint64_t strides[1] = {static_cast<uint64_t>(ldd) * 2u};
  const uint32_t box[2] = {32u, 32u};
  return encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, p, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_NONE,
                CU_TENSOR_MAP_L2_PROMOTION_NONE);
}

// e4m3 output [M, N] with row stride ldd bytes, 32 x 64 boxes, 64-byte swizzle.
bool encode_output_fp8(CUtensorMap* map, void* p, int64_t M, int64_t N, int64_t ldd) {
  const uint64_t dims[2] = {static_cast<uint64_t>(N), static_cast<uint64_t>(M)};
  const uint64_t strides[1] = {static_cast<uint64_t>(ldd)};
  const uint32_t box[2] = {64u, 32u};
  return encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, p, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_64B,
                CU_TENSOR_MAP_L2_PROMOTION_NONE);
}

// Columnwise quantiser input x [rows, cols] (fp32 or bf16, row stride ldx
// elements) read in 128-row x tile_cols-column boxes; columns past `cols` read as 0.
bool encode_columnwise_input(CUtensorMap* map, const void* x, int dtype, int64_t rows, int64_t cols, int64_t ldx,
                             int tile_cols) {
  const uint64_t elem = dtype == 0 ? 4u : 2u;
  const uint64_t dims[2] = {static_cast<uint64_t>(cols), static_cast<uint64_t>(rows)};
  const uint64_t strides[1] = {static_cast<uint64_t>(ldx) * elem};
  const uint32_t box[2] = {static_cast<uint32_t>(tile_cols), static_cast<uint32_t>(kColTileRows)};
  return encode(map, dtype == 0 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, x, dims,
                strides, box, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B);
}

// Columnwise quantiser output qt [cols, rows] e4m3 written in tile_cols-row x
// 128-byte boxes with a 128-byte swizzle; rows past `cols` are clipped.
bool encode_columnwise_output(CUtensorMap* map, void* qt, int64_t rows, int64_t cols, int tile_cols) {
  const uint64_t dims[2] = {static_cast<uint64_t>(rows), static_cast<uint64_t>(cols)};
  const uint64_t strides[1] = {static_cast<uint64_t>(rows)};
  const uint32_t box[2] = {static_cast<uint32_t>(kColTileRows), static_cast<uint32_t>(tile_cols)};
  return encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, qt, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B,
                CU_TENSOR_MAP_L2_PROMOTION_NONE);
}

template <int kDtype>
int launch_quantize_columnwise_t(const CUtensorMap& tmap, const CUtensorMap& tmap_qt, int64_t rows, int64_t cols,
                                 void* sft, int sm_count, cudaStream_t stream) {
  using C = ColCfg<kDtype>;
  const void* fn = reinterpret_cast<const void*>(&mxfp8_quantize_columnwise_kernel<kDtype>);
  // Per device (the shared-memory attribute is set in each device's context):
  // resident CTAs per SM, for one wave of persistent CTAs.
  static int per_sm[kMaxDevices] = {};
  static unsigned per_sm_epoch[kMaxDevices] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return CUTEX_ERR_CUDA;
  int resident = 0;
  {
    std::lock_guard<std::mutex> lock(g_mutex);
    const unsigned epoch = device_epoch_locked(dev);
    if (per_sm_epoch[dev] != epoch) {
      if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmemBytes) != cudaSuccess)
        return CUTEX_ERR_CUDA;
      per_sm[dev] = resident_ctas(fn, C::kThreads, C::kSmemBytes);
      per_sm_epoch[dev] = epoch;
    }
    resident = per_sm[dev];
  }
  const int64_t cols_pad = (cols + 127) & ~int64_t{127};
  const int64_t num_tiles = (cols_pad / C::kCols) * (rows / kColTileRows);
  const int64_t wave = int64_t{sm_count} * resident;
  const unsigned blocks = static_cast<unsigned>(std::max<int64_t>(1, std::min(num_tiles, wave)));
  mxfp8_quantize_columnwise_kernel<kDtype><<<blocks, C::kThreads, C::kSmemBytes, stream>>>(
      tmap, tmap_qt, rows, cols, static_cast<uint8_t*>(sft));
  return cudaGetLastError() == cudaSuccess ? CUTEX_OK : CUTEX_ERR_CUDA;
}

// ------------------------------------------------------------ kernel registry

using KernelFn = void (*)(CUtensorMap, CUtensorMap, CUtensorMap, CUtensorMap, CUtensorMap,
                          GemmArgs);

struct Variant {
  int cta_group, tile_n, stages, epi_bufs, sf_bufs, dynamic, smem_bytes;
  const void* fn;
  const void* fn_trace;   // instrumented twin (cutex_mxfp8_gemm_trace), or null
  const void* fn_epi[4];  // fused-epilogue twins: [1] BF16 out, [2] E4M3 + scales out, [3] all-gather
  const void* fn_fault;   // error-path self-test twin (cutex_mxfp8_selftest_wait_timeout), or null
  // Epoch (device_epoch) in which each build's shared-memory attribute was set.
  unsigned attr_set_trace[kMaxDevices];
  unsigned attr_set_fault[kMaxDevices];
  unsigned attr_set[kMaxDevices];
  unsigned attr_set_epi[4][kMaxDevices];
  int max_clusters[kMaxDevices];
  unsigned max_clusters_epoch[kMaxDevices];
};

template <int CG, int BN, int S, int E, int F, bool D, bool T = false, bool X = false, bool Q = false>
Variant make_variant() {
  Variant v{};
  v.cta_group = CG;
  v.tile_n = BN;
  v.stages = S;
  v.epi_bufs = E;
  v.sf_bufs = F;
  v.dynamic = D ? 1 : 0;
  v.smem_bytes = GemmCfg<CG, BN, S, E, F>::kSmemBytes;
  v.fn = reinterpret_cast<const void*>(&mxfp8_gemm_kernel<CG, BN, S, E, F, D>);
  v.fn_trace = T ? reinterpret_cast<const void*>(&mxfp8_gemm_kernel<CG, BN, S, E, F, D, true>) : nullptr;
  v.fn_epi[0] = nullptr;
  v.fn_epi[1] = X ? reinterpret_cast<const void*>(&mxfp8_gemm_kernel<CG, BN, S, E, F, D, false, 1>) : nullptr;
  v.fn_epi[2] = X ? reinterpret_cast<const void*>(&mxfp8_gemm_kernel<CG, BN, S, E, F, D, false, 2>) : nullptr;
  v.fn_epi[3] = X ? reinterpret_cast<const void*>(&mxfp8_gemm_kernel<CG, BN, S, E, F, D, false, 3>) : nullptr;
  if constexpr (Q) v.fn_fault = reinterpret_cast<const void*>(&mxfp8_gemm_kernel<CG, BN, S, E, F, D, false, 0, true>);
  return v;
}

// Instantiated kernels: (cta group, tile_n, stages, epilogue buffers, SF buffers,
// dynamic CLC scheduler, [instrumented twin]).
Variant g_variants[] = {
    // dynamic (cluster launch control) scheduling: the default
    make_variant<2, 256, 6, 1, 1, true, true, true>(), make_variant<2, 256, 5, 2, 1, true, false, true>(),
    make_variant<2, 256, 6, 1, 2, true>(), make_variant<2, 256, 4, 2, 1, true>(),
    make_variant<2, 128, 6, 2, 1, true>(), make_variant<2, 128, 8, 1, 1, true>(),
    make_variant<1, 256, 4, 1, 1, true, true, true>(), make_variant<1, 256, 3, 2, 1, true>(),
    make_variant<1, 128, 6, 1, 1, true, false, true>(), make_variant<1, 128, 5, 2, 1, true>(),
    // static persistent scheduling
    make_variant<1, 128, 4, 2, 2, false>(), make_variant<1, 128, 5, 2, 2, false>(),
    make_variant<1, 128, 6, 1, 2, false>(), make_variant<1, 128, 6, 1, 1, false, false, false, true>(),
    make_variant<1, 256, 3, 2, 2, false>(), make_variant<1, 256, 4, 1, 2, false>(),
    make_variant<1, 256, 4, 1, 1, false, true>(), make_variant<2, 256, 4, 2, 2, false>(),
    make_variant<2, 256, 5, 2, 2, false>(), make_variant<2, 256, 6, 1, 2, false>(),
    make_variant<2, 256, 6, 1, 1, false, true>(), make_variant<2, 256, 6, 1, 4, false>(),
    make_variant<2, 256, 5, 2, 1, false, true>(), make_variant<2, 256, 5, 2, 4, false>(),
};

Variant* find_variant(int cg, int bn, int stages, int epi, int sfb, int dynamic) {
  Variant* best = nullptr;
  for (auto& v : g_variants) {
    if (v.cta_group != cg || v.tile_n != bn || v.dynamic != dynamic) continue;
    if (stages != 0 && v.stages != stages) continue;
    if (epi != 0 && v.epi_bufs != epi) continue;
    if (sfb != 0 && v.sf_bufs != sfb) continue;
    // Default (measured, burst, 2-CTA 256x256 at 8192^3 and 16384^3): the deepest
    // ring with one SF buffer and, at equal depth, the fewest epilogue buffers.
    auto rank = [](const Variant& x) { return x.stages * 100 + (x.sf_bufs == 1 ? 10 : 0) - x.epi_bufs; };
    if (best == nullptr || rank(v) > rank(*best)) best = &v;
  }
  return best;
}

// Skinny (M <= 128) kernels: (padded M, stages, 128-row B tiles per CTA tile).
struct SkinnyVariant {
  int npad, stages, tiles, smem_bytes;
  const void* fn;
  unsigned attr_set[kMaxDevices];  // epoch in which the shared-memory attribute was set
};

template <int NP, int S, int T = 1>
SkinnyVariant make_skinny() {
  SkinnyVariant v{};
  v.npad = NP;
  v.stages = S;
  v.tiles = T;
  v.smem_bytes = SkinnyCfg<NP, S, T>::kSmemBytes;
  v.fn = reinterpret_cast<const void*>(&mxfp8_skinny_kernel<NP, S, T>);
  return v;
}

SkinnyVariant g_skinny[] = {
    make_skinny<16, 10>(),    make_skinny<32, 10>(),    make_skinny<64, 8>(), make_skinny<128, 6>(),
    make_skinny<64, 5, 2>(), make_skinny<128, 4, 2>(),
};

SkinnyVariant* find_skinny(int64_t M, int tiles) {
  for (auto& v : g_skinny)
    if (M <= v.npad && v.tiles == tiles) return &v;
  return nullptr;
}

struct Plan {
  Variant* variant;
  SkinnyVariant* skinny;
  int kernel;
  int tile_n;
  int raster_group;
  int raster_along_n;
  int grid_ctas;
  int num_m_tiles, num_n_tiles, num_tiles;
  int streamk;                // skinny: stream-K split over the grid (needs workspace)
  int dp_tiles;               // skinny stream-K: tiles taken whole before the split range
  int64_t workspace_bytes;    // skinny stream-K: partial slots + tile counters
  int64_t ws_partials_bytes;  // offset of the counters inside the workspace
};

// Skinny stream-K workspace layout, fixed per device and B-tiles-per-CTA-tile
// count so that one workspace can serve calls of any shape: a partial-sum
// region sized for the largest grid and padded M (2 slots x sm_count CTAs x
// tiles x 128 x 128 fp32), then one uint32 arrival counter per CTA tile of B.
// Counters never alias partial slots, and every completed call leaves the
// counters it used at zero.
void skinny_workspace(int sm_count, int n_tiles, int tiles, int64_t* partial_bytes, int64_t* total) {
  *partial_bytes = static_cast<int64_t>(2) * sm_count * tiles * 128 * 128 * 4;
  *total = *partial_bytes + ((static_cast<int64_t>(n_tiles) * 4 + 255) / 256) * 256;
}

bool cfg_reserved_zero(const cutex_gemm_config* cfg) {
  for (int r : cfg->reserved)
    if (r != 0) return false;
  return true;
}

int validate_shape(int64_t M, int64_t N, int64_t K) {
  if (M < 1 || N < 1 || K < 1) return CUTEX_ERR_SHAPE;
  if (M > kMaxDim || N > kMaxDim || K > kMaxDim) return CUTEX_ERR_SHAPE;
  if (K % 128 != 0 || N % 16 != 0) return CUTEX_ERR_ALIGN;
  return CUTEX_OK;
}

// plain: a launch of the plain kernel builds (not the traced or fused-epilogue
// twins, which exist for the dynamic-scheduler variants only).
int resolve_plan(const cutex_gemm_config* cfg_in, int64_t M, int64_t N, int64_t K, int sm_count,
                 Plan* plan, bool plain = true) {
  cutex_gemm_config cfg{};
  if (cfg_in != nullptr) {
    cfg = *cfg_in;
    if (!cfg_reserved_zero(&cfg)) return CUTEX_ERR_INVALID_ARGUMENT;
  }
  if (cfg.kernel < 0 || cfg.kernel > CUTEX_KERNEL_SKINNY || cfg.stages < 0 || cfg.raster_group < 0 ||
      cfg.max_ctas < 0 || cfg.split_k < 0 || cfg.epi_buffers < 0 || cfg.epi_buffers > 2 ||
      cfg.sf_buffers < 0 || cfg.sf_buffers > 4 || cfg.scheduler < 0 || cfg.scheduler > 1 ||
      (cfg.raster_along_n != 0 && cfg.raster_along_n != 1))
    return CUTEX_ERR_INVALID_ARGUMENT;
  if (cfg.tile_n != 0 && cfg.tile_n != 128 && cfg.tile_n != 256) return CUTEX_ERR_INVALID_ARGUMENT;
  int kernel = cfg.kernel;
  const bool auto_kernel = kernel == CUTEX_KERNEL_AUTO;
  if (auto_kernel) {
    // The largest tile whose first wave keeps at least half of the SMs busy:
    // CTA-pair 256x256, else single-CTA 128x256, else single-CTA 128x128
    // (measured: 2048^3 pairs 9.9 us vs 10.8 us 128x256; 1024^3 128x128 5.2 us
    // vs 6.7 us 128x256).
    const int64_t pair_tiles = ((M + 255) / 256) * ((N + 255) / 256);
    const int64_t wide_tiles = ((M + 127) / 128) * ((N + 255) / 256);
    if (M <= 128) {
      kernel = CUTEX_KERNEL_SKINNY;
    } else if (N % 256 == 0 && 2 * pair_tiles >= sm_count / 2) {
      kernel = CUTEX_KERNEL_2CTA;
    } else {
      kernel = CUTEX_KERNEL_1CTA;
      if (cfg.tile_n == 0 && plain && (N % 256 != 0 || wide_tiles < sm_count / 2)) cfg.tile_n = 128;
    }
  }
  plan->skinny = nullptr;
  plan->variant = nullptr;
  plan->streamk = 0;
  plan->dp_tiles = 0;
  plan->workspace_bytes = 0;
  plan->ws_partials_bytes = 0;
  if (kernel == CUTEX_KERNEL_SKINNY) {
    // 0 = stream-K (library choice of full data-parallel waves), 1 = no split,
    // 2 = pure stream-K, 3 = full data-parallel waves + stream-K remainder.
    if (cfg.split_k > 3) return CUTEX_ERR_INVALID_ARGUMENT;
    if (cfg.tile_n != 0 && cfg.tile_n != 128 && cfg.tile_n != 256) return CUTEX_ERR_INVALID_ARGUMENT;
    SkinnyVariant* sv1 = find_skinny(M, 1);
    if (sv1 == nullptr) return CUTEX_ERR_SHAPE;  // the skinny kernel covers M <= 128
    int grid = sm_count;
    if (cfg.max_ctas != 0) grid = std::min(grid, cfg.max_ctas);
    const int64_t tiles128 = (N + 127) / 128;
    // AUTO is stream-K for every padded M: each SM streams the same share of B,
    // where whole tiles leave a second wave on 76 of 148 SMs (N = 28672).
    // Measured at N = 28672, K = 8192: M = 128 44.7 us vs 46.9 us whole,
    // M = 64 39.4 vs 41.8, M = 16 39.9 vs 40.5.
    // Two 128-row B tiles per CTA tile (tile_n 256): one A stage serves both
    // tiles, stream-K or whole tiles as for single tiles.
    const int tiles = cfg.tile_n == 256 ? 2 : 1;
    SkinnyVariant* sv = find_skinny(M, tiles);
    if (sv == nullptr) return CUTEX_ERR_INVALID_ARGUMENT;  // no double-tile build for this padded M
    if (cfg.stages != 0 && cfg.stages != sv->stages) return CUTEX_ERR_INVALID_ARGUMENT;
    plan->skinny = sv;
    plan->kernel = kernel;
    plan->tile_n = 128 * tiles;
    plan->num_m_tiles = 1;
    plan->num_n_tiles = static_cast<int>((tiles128 + tiles - 1) / tiles);
    plan->num_tiles = plan->num_n_tiles;
    plan->raster_group = 1;
    plan->raster_along_n = 0;
    const int64_t units = static_cast<int64_t>(plan->num_n_tiles) * (K / 128);
    plan->streamk = cfg.split_k == 1 ? 0 : 1;
    grid = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(grid, plan->streamk ? units : plan->num_n_tiles)));
    plan->grid_ctas = grid;
    plan->dp_tiles = 0;
    if (plan->streamk && cfg.split_k == 3) plan->dp_tiles = plan->num_n_tiles / grid * grid;
    if (plan->streamk)
      skinny_workspace(sm_count, plan->num_n_tiles, tiles, &plan->ws_partials_bytes, &plan->workspace_bytes);
    return CUTEX_OK;
  }
  int tile_n = cfg.tile_n;
  if (kernel == CUTEX_KERNEL_2CTA) {
    // 256x256 pair tiles. The 256x128 pair tile exists as an explicit option only:
    // measured, it halves the B bytes per tile but starves the per-SM operand feed
    // and runs at ~60 % of the 256x256 rate at 4096^3..16384^3.
    if (tile_n == 0) tile_n = 256;
  } else if (tile_n == 0) {
    tile_n = (N % 256 == 0 && M > 128) ? 256 : 128;
  }
  const int cg = kernel == CUTEX_KERNEL_2CTA ? 2 : 1;
  int dynamic = cfg.scheduler == 1 ? 0 : 1;
  if (auto_kernel && plain && cfg.scheduler == 0 && cfg.max_ctas == 0) {
    // All tiles fit in one wave of resident CTAs (pairs): nothing to balance,
    // and the static grid skips the scheduler's round trip per tile
    // (measured 2048^3: 9.9 us static vs 10.8 us dynamic).
    const int64_t n_tiles = ((M + 128 * cg - 1) / (128 * cg)) * ((N + tile_n - 1) / tile_n);
    if (n_tiles <= sm_count / cg) dynamic = 0;
  }
  int stages = cfg.stages, epi_buffers = cfg.epi_buffers;
  if (plain && cg == 2 && tile_n == 256 && stages == 0 && epi_buffers == 0 && cfg.sf_buffers == 0 && K >= 16384) {
    // Long K: a 5-stage ring with two epilogue buffers per warp. Measured on two
    // boxes (graphs of back-to-back launches, alternating): +0.5-0.9 % at K = 16384
    // (16384^3, 8192^2 x 16384, 8192 x 28672 x 16384, 16384 x 2048 x 16384) and
    // +3 % at 16384^2 x 32768; at K = 8192 and below the 6-stage ring with one
    // buffer is 0.2-1.3 % faster.
    stages = 5;
    epi_buffers = 2;
  }
  Variant* v = find_variant(cg, tile_n, stages, epi_buffers, cfg.sf_buffers, dynamic);
  if (v == nullptr) return CUTEX_ERR_INVALID_ARGUMENT;
  plan->variant = v;
  plan->kernel = kernel;
  plan->tile_n = tile_n;
  plan->num_m_tiles = static_cast<int>((M + 128 * cg - 1) / (128 * cg));
  plan->num_n_tiles = static_cast<int>((N + tile_n - 1) / tile_n);
  const int64_t tiles = static_cast<int64_t>(plan->num_m_tiles) * plan->num_n_tiles;
  if (tiles > kMaxDim) return CUTEX_ERR_SHAPE;
  plan->num_tiles = static_cast<int>(tiles);
  plan->raster_group = cfg.raster_group != 0 ? cfg.raster_group : 8;
  plan->raster_along_n = cfg.raster_along_n;
  if (cfg.raster_group == 0 && cg == 2 && tile_n == 256) {
    // Library choice of both: the group spans the dimension with fewer tiles
    // and walks the longer one, so the short side's panels (kept evict-last)
    // serve the whole walk and the long side's stream through once; 16 tiles
    // wide at K <= 8192, 8 above (about the same panel bytes). Measured
    // (TFLOP/s, graphs of back-to-back launches, against 8 tiles walking M):
    // 16384 x 2048 x 16384 2977 vs 2736, 16384 x 4096 x 16384 2954 vs 2844,
    // 16384 x 8192 x 16384 2949 vs 2916, 2048 x 16384 x 16384 2968 vs 2965
    // (walking N: 2729), 8192 x 28672 x 8192 3002 vs 2903, 8192^3 2921 vs 2841;
    // 16384^3 unchanged (2965), 4096^3 insensitive.
    plan->raster_along_n = plan->num_n_tiles < plan->num_m_tiles ? 1 : 0;
    plan->raster_group = K <= 8192 ? 16 : 8;
  }
  if (v->dynamic) {
    // One cluster per tile; resident clusters cancel and take over pending ones.
    plan->grid_ctas = plan->num_tiles * cg;
    return CUTEX_OK;
  }
  int units = sm_count / cg;  // persistent CTAs (pairs) that fit, one per SM
  if (cfg.max_ctas != 0) units = std::min(units, std::max(1, cfg.max_ctas / cg));
  units = std::max(1, std::min(units, plan->num_tiles));
  plan->grid_ctas = units * cg;
  return CUTEX_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int launch_gemm(const Plan& plan, int dev, const void* a, const void* b, const void* sfa,
                const void* sfb, void* d, int64_t M, int64_t N, int64_t K, int64_t ldd,
                cudaStream_t stream, unsigned long long* trace = nullptr, int trace_cap = 0,
                const cutex_epilogue* epi = nullptr, const CUtensorMap* peer_maps = nullptr, int num_peers = 0,
                int fault_kit = -1) {
  Variant* v = plan.variant;
  const bool traced = trace != nullptr;
  const bool fault = fault_kit >= 0;
  if (traced && v->fn_trace == nullptr) return CUTEX_ERR_INVALID_ARGUMENT;
  const int epi_kind = peer_maps != nullptr ? 3 : (epi == nullptr ? 0 : (epi->out_dtype == 1 ? 2 : 1));
  if (epi_kind != 0 && (traced || v->fn_epi[epi_kind] == nullptr)) return CUTEX_ERR_INVALID_ARGUMENT;
  if (fault && (traced || epi_kind != 0 || v->fn_fault == nullptr)) return CUTEX_ERR_INVALID_ARGUMENT;
  const void* fn = fault ? v->fn_fault : traced ? v->fn_trace : (epi_kind != 0 ? v->fn_epi[epi_kind] : v->fn);
  const int cg = v->cta_group;
  CUtensorMap ta, tb, tsa, tsb, td;
  const bool out_ok = epi_kind == 2 ? encode_output_fp8(&td, d, M, N, ldd) : encode_output(&td, d, M, N, ldd);
  if (!encode_operand(&ta, a, M, K, 128) || !encode_operand(&tb, b, N, K, v->tile_n / cg) ||
      !encode_scales(&tsa, sfa, M, K, 1) || !encode_scales(&tsb, sfb, N, K, v->tile_n / 128) || !out_ok)
    return CUTEX_ERR_CUDA;
  unsigned epoch = 0;
  {
    std::lock_guard<std::mutex> lock(g_mutex);
    epoch = device_epoch_locked(dev);
    unsigned& set = fault ? v->attr_set_fault[dev]
                    : traced ? v->attr_set_trace[dev]
                             : (epi_kind != 0 ? v->attr_set_epi[epi_kind][dev] : v->attr_set[dev]);
    if (set != epoch) {
      if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, v->smem_bytes) !=
          cudaSuccess)
        return CUTEX_ERR_CUDA;
      set = epoch;
    }
  }
  GemmArgs args{};
  args.num_m_tiles = plan.num_m_tiles;
  args.num_n_tiles = plan.num_n_tiles;
  args.num_tiles = plan.num_tiles;
  args.num_k_blocks = static_cast<int>(K / 128);
  args.raster_group = plan.raster_group;
  args.raster_along_n = plan.raster_along_n;
  args.trace = trace;
  args.trace_cap = trace_cap;
  args.alpha = 1.0f;
  args.beta = 0.0f;
  args.M = static_cast<int>(M);
  args.N = static_cast<int>(N);
  args.peer_maps = peer_maps;
  args.num_peers = num_peers;
  args.fault_withhold_kit = fault_kit;
  if (epi != nullptr) {
    args.alpha = epi->alpha;
    args.beta = epi->beta;
    args.c = static_cast<const __nv_bfloat16*>(epi->c);
    args.ldc = epi->ldc;
    args.bias = static_cast<const __nv_bfloat16*>(epi->bias);
    args.d_scales = static_cast<uint8_t*>(epi->d_scales);
  }

  cudaLaunchConfig_t lc{};
  lc.gridDim = dim3(static_cast<unsigned>(plan.grid_ctas), 1, 1);
  lc.blockDim = dim3(v->dynamic ? 224 : 192, 1, 1);
  lc.dynamicSmemBytes = static_cast<size_t>(v->smem_bytes);
  lc.stream = stream;
  cudaLaunchAttribute attr[2];
  if (cg == 2) {
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    lc.attrs = attr;
    lc.numAttrs = 1;
    // A persistent grid must be co-resident: cap it at the number of CTA pairs
    // the GPCs can hold at once (queried once per device and variant).
    int max_clusters = 0;
    {
      std::lock_guard<std::mutex> lock(g_mutex);
      if (v->max_clusters_epoch[dev] == epoch) max_clusters = v->max_clusters[dev];
    }
    if (max_clusters == 0) {
      if (cudaOccupancyMaxActiveClusters(&max_clusters, fn, &lc) != cudaSuccess ||
          max_clusters < 1)
        return CUTEX_ERR_CUDA;
      std::lock_guard<std::mutex> lock(g_mutex);
      v->max_clusters[dev] = max_clusters;
      v->max_clusters_epoch[dev] = epoch;
    }
    if (!v->dynamic && plan.grid_ctas > 2 * max_clusters)
      lc.gridDim.x = static_cast<unsigned>(2 * max_clusters);
  }
  // Programmatic dependent launch (the kernel waits with griddepcontrol.wait
  // before its first global access).
  attr[lc.numAttrs].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[lc.numAttrs].val.programmaticStreamSerializationAllowed = 1;
  lc.attrs = attr;
  lc.numAttrs += 1;
  void* params[] = {&ta, &tb, &tsa, &tsb, &td, &args};
  if (cudaLaunchKernelExC(&lc, fn, params) != cudaSuccess) return CUTEX_ERR_CUDA;
  return CUTEX_OK;
}

int launch_skinny(const Plan& plan, int dev, const void* a, const void* b, const void* sfa,
                  const void* sfb, void* d, int64_t M, int64_t N, int64_t K, int64_t ldd,
                  void* workspace, cudaStream_t stream) {
  SkinnyVariant* v = plan.skinny;
  CUtensorMap tb, ta, tsb, tsa, td;
  if (!encode_operand(&tb, b, N, K, static_cast<uint32_t>(128 * v->tiles)) ||
      !encode_operand(&ta, a, M, K, static_cast<uint32_t>(v->npad)) ||
      !encode_scales(&tsb, sfb, N, K, static_cast<uint32_t>(v->tiles)) || !encode_scales(&tsa, sfa, M, K, 1) ||
      !encode_output_skinny(&td, d, M, N, ldd))
    return CUTEX_ERR_CUDA;
  {
    std::lock_guard<std::mutex> lock(g_mutex);
    const unsigned epoch = device_epoch_locked(dev);
    if (v->attr_set[dev] != epoch) {
      if (cudaFuncSetAttribute(v->fn, cudaFuncAttributeMaxDynamicSharedMemorySize, v->smem_bytes) !=
          cudaSuccess)
        return CUTEX_ERR_CUDA;
      v->attr_set[dev] = epoch;
    }
  }
  SkinnyArgs args{};
  args.M = static_cast<int>(M);
  args.N = static_cast<int>(N);
  args.num_n_tiles = plan.num_n_tiles;
  args.num_k_blocks = static_cast<int>(K / 128);
  args.dp_tiles = plan.streamk ? plan.dp_tiles : 0;
  args.units = static_cast<long long>(plan.num_n_tiles - args.dp_tiles) * args.num_k_blocks;
  args.streamk = plan.streamk;
  args.ldd = ldd;
  args.d = static_cast<__nv_bfloat16*>(d);
  args.partials = plan.streamk ? static_cast<float*>(workspace) : nullptr;
  args.counters = plan.streamk
                      ? reinterpret_cast<unsigned int*>(static_cast<char*>(workspace) + plan.ws_partials_bytes)
                      : nullptr;
  cudaLaunchConfig_t lc{};
  lc.gridDim = dim3(static_cast<unsigned>(plan.grid_ctas), 1, 1);
  lc.blockDim = dim3(192, 1, 1);
  lc.dynamicSmemBytes = static_cast<size_t>(v->smem_bytes);
  lc.stream = stream;
  // Programmatic dependent launch: the kernel waits (griddepcontrol.wait) for
  // the previous kernel of the stream before touching global memory, so its
  // launch and set-up overlap that kernel's last CTAs.
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  lc.attrs = attr;
  lc.numAttrs = 1;
  void* params[] = {&tb, &ta, &tsb, &tsa, &td, &args};
  if (cudaLaunchKernelExC(&lc, v->fn, params) != cudaSuccess) return CUTEX_ERR_CUDA;
  return CUTEX_OK;
}

}  // namespace
}  // namespace cutex

using namespace cutex;

extern "C" int cutex_mxfp8_query(const cutex_gemm_config* cfg, int64_t M, int64_t N, int64_t K,
                                 cutex_gemm_info* info) {
  if (info == nullptr) return CUTEX_ERR_INVALID_ARGUMENT;
  const int st = validate_shape(M, N, K);
  if (st != CUTEX_OK) return st;
  int sm_count = 148;
  DeviceState* ds = nullptr;
  if (current_device_state(&ds) == CUTEX_OK) sm_count = ds->sm_count;
  Plan plan{};
  const int rc = resolve_plan(cfg, M, N, K, sm_count, &plan);
  if (rc != CUTEX_OK) return rc;
  std::memset(info, 0, sizeof(*info));
  info->kernel = plan.kernel;
  info->tile_k = 128;
  info->grid_ctas = plan.grid_ctas;
  info->num_tiles = plan.num_tiles;
  info->raster_group = plan.raster_group;
  if (plan.skinny != nullptr) {
    info->tile_m = plan.skinny->npad;  // padded M: the MMA's N side
    info->tile_n = plan.tile_n;
    info->stages = plan.skinny->stages;
    info->cluster_size = 1;
    info->smem_bytes = plan.skinny->smem_bytes;
    info->split_k = plan.streamk ? 0 : 1;  // 0: stream-K over the grid
    info->epi_buffers = 0;
    info->sf_buffers = 2;
    info->workspace_bytes = plan.workspace_bytes;
    return CUTEX_OK;
  }
  info->tile_m = 128 * plan.variant->cta_group;
  info->tile_n = plan.tile_n;
  info->stages = plan.variant->stages;
  info->cluster_size = plan.variant->cta_group;
  info->smem_bytes = plan.variant->smem_bytes;
  info->split_k = 1;
  info->epi_buffers = plan.variant->epi_bufs;
  info->sf_buffers = plan.variant->sf_bufs;
  info->scheduler = plan.variant->dynamic ? 0 : 1;
  info->workspace_bytes = 0;
  return CUTEX_OK;
}

extern "C" int cutex_mxfp8_gemm(const void* a, const void* b, const void* sfa, const void* sfb,
                                void* d, int64_t M, int64_t N, int64_t K, int64_t ldd,
                                const cutex_gemm_config* cfg, void* workspace,
                                int64_t workspace_bytes, cutex_stream_t stream) {
  (void)workspace;
  if (a == nullptr || b == nullptr || sfa == nullptr || sfb == nullptr || d == nullptr)
    return CUTEX_ERR_INVALID_ARGUMENT;
  if (workspace_bytes < 0) return CUTEX_ERR_INVALID_ARGUMENT;
  int st = validate_shape(M, N, K);
  if (st != CUTEX_OK) return st;
  if (ldd < N || ldd % 8 != 0 || ldd > kMaxDim) return CUTEX_ERR_ALIGN;
  if (!aligned16(a) || !aligned16(b) || !aligned16(sfa) || !aligned16(sfb) || !aligned16(d))
    return CUTEX_ERR_ALIGN;
  DeviceState* ds = nullptr;
  st = current_device_state(&ds);
  if (st != CUTEX_OK) return st;
  Plan plan{};
  st = resolve_plan(cfg, M, N, K, ds->sm_count, &plan);
  if (st != CUTEX_OK) return st;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return CUTEX_ERR_CUDA;
  if (plan.skinny != nullptr) {
    if (plan.streamk && (workspace == nullptr || workspace_bytes < plan.workspace_bytes)) {
      // Explicit stream-K needs the workspace; AUTO without one takes whole tiles instead.
      if (cfg != nullptr && cfg->kernel == CUTEX_KERNEL_SKINNY) return CUTEX_ERR_WORKSPACE;
      cutex_gemm_config whole = cfg != nullptr ? *cfg : cutex_gemm_config{};
      whole.kernel = CUTEX_KERNEL_SKINNY;
      whole.split_k = 1;
      st = resolve_plan(&whole, M, N, K, ds->sm_count, &plan);
      if (st != CUTEX_OK) return st;
    }
    if (plan.streamk && (reinterpret_cast<uintptr_t>(workspace) & 255u) != 0) return CUTEX_ERR_ALIGN;
    return launch_skinny(plan, dev, a, b, sfa, sfb, d, M, N, K, ldd, workspace,
                         reinterpret_cast<cudaStream_t>(stream));
  }
  return launch_gemm(plan, dev, a, b, sfa, sfb, d, M, N, K, ldd,
                     reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int cutex_mxfp8_gemm_ex(const void* a, const void* b, const void* sfa, const void* sfb, void* d,
                                   int64_t M, int64_t N, int64_t K, int64_t ldd, const cutex_gemm_config* cfg,
                                   const cutex_epilogue* epi, void* workspace, int64_t workspace_bytes,
                                   cutex_stream_t stream) {
  if (epi == nullptr) return cutex_mxfp8_gemm(a, b, sfa, sfb, d, M, N, K, ldd, cfg, workspace, workspace_bytes, stream);
  if (a == nullptr || b == nullptr || sfa == nullptr || sfb == nullptr || d == nullptr)
    return CUTEX_ERR_INVALID_ARGUMENT;
  if (epi->out_dtype != 0 && epi->out_dtype != 1) return CUTEX_ERR_INVALID_ARGUMENT;
  if (epi->reserved0 != 0) return CUTEX_ERR_INVALID_ARGUMENT;
  for (int64_t r : epi->reserved)
    if (r != 0) return CUTEX_ERR_INVALID_ARGUMENT;
  int st = validate_shape(M, N, K);
  if (st != CUTEX_OK) return st;
  if (M > 0x7FFFFFFF - 256) return CUTEX_ERR_SHAPE;  // the kernel indexes rows as int
  if (!aligned16(a) || !aligned16(b) || !aligned16(sfa) || !aligned16(sfb) || !aligned16(d))
    return CUTEX_ERR_ALIGN;
  if (epi->out_dtype == 0) {
    if (ldd < N || ldd % 8 != 0 || ldd > kMaxDim) return CUTEX_ERR_ALIGN;
  } else {
    // e4m3 D (ldd in bytes) and its scales: whole 128-column scale atoms along N.
    if (epi->d_scales == nullptr) return CUTEX_ERR_INVALID_ARGUMENT;
    if (N % 128 != 0 || ldd < N || ldd % 16 != 0 || ldd > kMaxDim || !aligned16(epi->d_scales))
      return CUTEX_ERR_ALIGN;
  }
  if (epi->bias != nullptr && !aligned16(epi->bias)) return CUTEX_ERR_ALIGN;
  if (epi->c != nullptr && epi->beta != 0.0f &&
      (!aligned16(epi->c) || epi->ldc < N || epi->ldc % 8 != 0 || epi->ldc > kMaxDim))
    return CUTEX_ERR_ALIGN;
  DeviceState* ds = nullptr;
  st = current_device_state(&ds);
  if (st != CUTEX_OK) return st;
  // The fused builds are large-tile kernels only: route AUTO away from the
  // skinny kernel, reject an explicit skinny request.
  cutex_gemm_config c2 = cfg != nullptr ? *cfg : cutex_gemm_config{};
  if (c2.kernel == CUTEX_KERNEL_SKINNY) return CUTEX_ERR_INVALID_ARGUMENT;
  if (c2.kernel == CUTEX_KERNEL_AUTO) c2.kernel = (N % 256 == 0 && M > 128) ? CUTEX_KERNEL_2CTA : CUTEX_KERNEL_1CTA;
  Plan plan{};
  st = resolve_plan(&c2, M, N, K, ds->sm_count, &plan, /*plain=*/false);
  if (st != CUTEX_OK) return st;
  if (plan.variant == nullptr || plan.variant->fn_epi[epi->out_dtype == 1 ? 2 : 1] == nullptr)
    return CUTEX_ERR_INVALID_ARGUMENT;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return CUTEX_ERR_CUDA;
  return launch_gemm(plan, dev, a, b, sfa, sfb, d, M, N, K, ldd, reinterpret_cast<cudaStream_t>(stream), nullptr, 0,
                     epi);
}

namespace {

PFN_cuMemGetAddressRange_v3020 address_range_fn() {
  static PFN_cuMemGetAddressRange_v3020 fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      p = nullptr;
    return reinterpret_cast<PFN_cuMemGetAddressRange_v3020>(p);
  }();
  return fn;
}

}  // namespace

extern "C" int cutex_ipc_export(const void* dev_ptr, void* handle, int64_t* offset) {
  if (dev_ptr == nullptr || handle == nullptr || offset == nullptr) return CUTEX_ERR_INVALID_ARGUMENT;
  auto range = address_range_fn();
  if (range == nullptr) return CUTEX_ERR_CUDA;
  CUdeviceptr base = 0;
  size_t size = 0;
  if (range(&base, &size, reinterpret_cast<CUdeviceptr>(dev_ptr)) != CUDA_SUCCESS) return CUTEX_ERR_CUDA;
  cudaIpcMemHandle_t h{};
  if (cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base)) != cudaSuccess) return CUTEX_ERR_CUDA;
  static_assert(sizeof(h) == 64, "IPC handle size");
  std::memcpy(handle, &h, sizeof(h));
  *offset = static_cast<int64_t>(reinterpret_cast<CUdeviceptr>(dev_ptr) - base);
  return CUTEX_OK;
}

extern "C" int cutex_ipc_import(const void* handle, int64_t offset, void** dev_ptr, void** mapping) {
  if (handle == nullptr || dev_ptr == nullptr || mapping == nullptr || offset < 0) return CUTEX_ERR_INVALID_ARGUMENT;
  cudaIpcMemHandle_t h{};
  std::memcpy(&h, handle, sizeof(h));
  void* base = nullptr;
  if (cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) return CUTEX_ERR_CUDA;
  *mapping = base;
  *dev_ptr = static_cast<char*>(base) + offset;
  return CUTEX_OK;
}

extern "C" int cutex_ipc_close(void* mapping) {
  if (mapping == nullptr) return CUTEX_ERR_INVALID_ARGUMENT;
  return cudaIpcCloseMemHandle(mapping) == cudaSuccess ? CUTEX_OK : CUTEX_ERR_CUDA;
}

extern "C" int cutex_mxfp8_allgather_maps(const void* const* peer_d, int32_t num_peers, int64_t M, int64_t N,
                                          int64_t ldd, void* map_buffer, int64_t map_buffer_bytes,
                                          cutex_stream_t stream) {
  if (peer_d == nullptr || map_buffer == nullptr) return CUTEX_ERR_INVALID_ARGUMENT;
  if (num_peers < 1 || num_peers > kMaxGatherPeers) return CUTEX_ERR_INVALID_ARGUMENT;
  if (map_buffer_bytes < static_cast<int64_t>(num_peers) * static_cast<int64_t>(sizeof(CUtensorMap)))
    return CUTEX_ERR_WORKSPACE;
  if ((reinterpret_cast<uintptr_t>(map_buffer) & 63u) != 0) return CUTEX_ERR_ALIGN;  // CUtensorMap alignment
  if (M < 1 || N < 1 || M > kMaxDim || N > kMaxDim) return CUTEX_ERR_SHAPE;
  if (N % 16 != 0 || ldd < N || ldd % 8 != 0 || ldd > kMaxDim) return CUTEX_ERR_ALIGN;
  for (int p = 0; p < num_peers; ++p)
    if (peer_d[p] == nullptr || !aligned16(peer_d[p])) return CUTEX_ERR_ALIGN;
  CUtensorMap maps[kMaxGatherPeers];
  for (int p = 0; p < num_peers; ++p)
    if (!encode_output(&maps[p], const_cast<void*>(peer_d[p]), M, N, ldd)) return CUTEX_ERR_CUDA;
  // From host memory: the call returns once the array has been staged.
  return cudaMemcpyAsync(map_buffer, maps, sizeof(CUtensorMap) * num_peers, cudaMemcpyHostToDevice,
                         reinterpret_cast<cudaStream_t>(stream)) == cudaSuccess
             ? CUTEX_OK
             : CUTEX_ERR_CUDA;
}

extern "C" int cutex_mxfp8_gemm_allgather(const void* a, const void* b, const void* sfa, const void* sfb, void* d,
                                          int64_t M, int64_t N, int64_t K, int64_t ldd, const void* map_buffer,
                                          int32_t num_peers, const cutex_gemm_config* cfg, cutex_stream_t stream) {
  if (a == nullptr || b == nullptr || sfa == nullptr || sfb == nullptr || d == nullptr || map_buffer == nullptr)
    return CUTEX_ERR_INVALID_ARGUMENT;
  if (num_peers < 1 || num_peers > kMaxGatherPeers) return CUTEX_ERR_INVALID_ARGUMENT;
  if ((reinterpret_cast<uintptr_t>(map_buffer) & 63u) != 0) return CUTEX_ERR_ALIGN;
  int st = validate_shape(M, N, K);
  if (st != CUTEX_OK) return st;
  if (ldd < N || ldd % 8 != 0 || ldd > kMaxDim) return CUTEX_ERR_ALIGN;
  if (!aligned16(a) || !aligned16(b) || !aligned16(sfa) || !aligned16(sfb) || !aligned16(d)) return CUTEX_ERR_ALIGN;
  DeviceState* ds = nullptr;
  st = current_device_state(&ds);
  if (st != CUTEX_OK) return st;
  cutex_gemm_config c2 = cfg != nullptr ? *cfg : cutex_gemm_config{};
  if (c2.kernel == CUTEX_KERNEL_SKINNY) return CUTEX_ERR_INVALID_ARGUMENT;
  if (c2.kernel == CUTEX_KERNEL_AUTO) c2.kernel = (N % 256 == 0 && M > 128) ? CUTEX_KERNEL_2CTA : CUTEX_KERNEL_1CTA;
  Plan plan{};
  st = resolve_plan(&c2, M, N, K, ds->sm_count, &plan, /*plain=*/false);
  if (st != CUTEX_OK) return st;
  if (plan.variant == nullptr || plan.variant->fn_epi[3] == nullptr) return CUTEX_ERR_INVALID_ARGUMENT;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return CUTEX_ERR_CUDA;
  return launch_gemm(plan, dev, a, b, sfa, sfb, d, M, N, K, ldd, reinterpret_cast<cudaStream_t>(stream), nullptr, 0,
                     nullptr, static_cast<const CUtensorMap*>(map_buffer), num_peers);
}

extern "C" int cutex_mxfp8_gemm_trace(const void* a, const void* b, const void* sfa,
                                      const void* sfb, void* d, int64_t M, int64_t N, int64_t K,
                                      int64_t ldd, const cutex_gemm_config* cfg,
                                      unsigned long long* trace, int32_t trace_cap,
                                      cutex_stream_t stream) {
  if (a == nullptr || b == nullptr || sfa == nullptr || sfb == nullptr || d == nullptr ||
      trace == nullptr || trace_cap < 1)
    return CUTEX_ERR_INVALID_ARGUMENT;
  int st = validate_shape(M, N, K);
  if (st != CUTEX_OK) return st;
  if (ldd < N || ldd % 8 != 0 || ldd > kMaxDim) return CUTEX_ERR_ALIGN;
  if (!aligned16(a) || !aligned16(b) || !aligned16(sfa) || !aligned16(sfb) || !aligned16(d) ||
      (reinterpret_cast<uintptr_t>(trace) & 7u) != 0)
    return CUTEX_ERR_ALIGN;
  DeviceState* ds = nullptr;
  st = current_device_state(&ds);
  if (st != CUTEX_OK) return st;
  Plan plan{};
  st = resolve_plan(cfg, M, N, K, ds->sm_count, &plan, /*plain=*/false);
  if (st != CUTEX_OK) return st;
  if (plan.variant == nullptr) return CUTEX_ERR_INVALID_ARGUMENT;  // no traced skinny build
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return CUTEX_ERR_CUDA;
  return launch_gemm(plan, dev, a, b, sfa, sfb, d, M, N, K, ldd,
                     reinterpret_cast<cudaStream_t>(stream), trace, trace_cap);
}

extern "C" int cutex_mxfp8_selftest_wait_timeout(const void* a, const void* b, const void* sfa, const void* sfb,
                                                void* d, int64_t M, int64_t N, int64_t K, int32_t withhold_stage,
                                                cutex_stream_t stream) {
  if (a == nullptr || b == nullptr || sfa == nullptr || sfb == nullptr || d == nullptr) return CUTEX_ERR_INVALID_ARGUMENT;
  int st = validate_shape(M, N, K);
  if (st != CUTEX_OK) return st;
  // The withheld stage must be one every CTA reaches: inside its first tile.
  if (withhold_stage < 0 || withhold_stage >= K / 128) return CUTEX_ERR_INVALID_ARGUMENT;
  if (!aligned16(a) || !aligned16(b) || !aligned16(sfa) || !aligned16(sfb) || !aligned16(d)) return CUTEX_ERR_ALIGN;
  DeviceState* ds = nullptr;
  st = current_device_state(&ds);
  if (st != CUTEX_OK) return st;
  cutex_gemm_config cfg{};
  cfg.kernel = CUTEX_KERNEL_1CTA;
  cfg.tile_n = 128;
  cfg.stages = 6;
  cfg.epi_buffers = 1;
  cfg.sf_buffers = 1;
  cfg.scheduler = 1;
  Plan plan{};
  st = resolve_plan(&cfg, M, N, K, ds->sm_count, &plan, /*plain=*/false);
  if (st != CUTEX_OK) return st;
  if (plan.variant == nullptr || plan.variant->fn_fault == nullptr) return CUTEX_ERR_INVALID_ARGUMENT;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return CUTEX_ERR_CUDA;
  return launch_gemm(plan, dev, a, b, sfa, sfb, d, M, N, K, N, reinterpret_cast<cudaStream_t>(stream), nullptr, 0,
                     nullptr, nullptr, 0, withhold_stage);
}

extern "C" int cutex_dense_gemm_v13(const void* a, const void* b, const void* sfa, const void* sfb,
                                    void* c, int32_t max_active_clusters, cutex_stream_t stream) {
  cutex_gemm_config cfg{};
  cfg.kernel = CUTEX_KERNEL_2CTA;
  cfg.tile_n = 256;
  cfg.max_ctas = max_active_clusters > 0 ? 2 * max_active_clusters : 0;
  const int64_t n = 16384;
  return cutex_mxfp8_gemm(a, b, sfa, sfb, c, n, n, n, n, &cfg, nullptr, 0, stream);
}

extern "C" int cutex_mxfp8_quantize(const void* x, int32_t x_dtype, int64_t rows, int64_t K,
                                    int64_t ldx, void* q, void* sf, cutex_stream_t stream) {
  if (x == nullptr || q == nullptr || sf == nullptr) return CUTEX_ERR_INVALID_ARGUMENT;
  if (x_dtype != 0 && x_dtype != 1) return CUTEX_ERR_INVALID_ARGUMENT;
  if (rows < 1 || K < 1 || rows > kMaxDim || K > kMaxDim) return CUTEX_ERR_SHAPE;
  if (K % 128 != 0 || ldx < K || ldx % 8 != 0) return CUTEX_ERR_ALIGN;
  if (!aligned16(x) || !aligned16(q) || !aligned16(sf)) return CUTEX_ERR_ALIGN;
  DeviceState* ds = nullptr;
  const int st = current_device_state(&ds);
  if (st != CUTEX_OK) return st;
  return launch_quantize(x, x_dtype, rows, K, ldx, q, sf, ds->sm_count,
                         reinterpret_cast<cudaStream_t>(stream))
             ? CUTEX_OK
             : CUTEX_ERR_CUDA;
}

extern "C" int cutex_mxfp8_quantize_columnwise(const void* x, int32_t x_dtype, int64_t rows, int64_t cols,
                                               int64_t ldx, void* qt, void* sft, cutex_stream_t stream) {
  if (x == nullptr || qt == nullptr || sft == nullptr) return CUTEX_ERR_INVALID_ARGUMENT;
  if (x_dtype != 0 && x_dtype != 1) return CUTEX_ERR_INVALID_ARGUMENT;
  if (rows < 1 || cols < 1 || rows > kMaxDim || cols > kMaxDim) return CUTEX_ERR_SHAPE;
  if (rows % 128 != 0 || ldx < cols || ldx % 8 != 0) return CUTEX_ERR_ALIGN;
  if (!aligned16(x) || !aligned16(qt) || !aligned16(sft)) return CUTEX_ERR_ALIGN;
  DeviceState* ds = nullptr;
  const int st = current_device_state(&ds);
  if (st != CUTEX_OK) return st;
  CUtensorMap tmap, tmap_qt;
  const int tile_cols = x_dtype == 0 ? ColCfg<0>::kCols : ColCfg<1>::kCols;
  if (!encode_columnwise_input(&tmap, x, x_dtype, rows, cols, ldx, tile_cols) ||
      !encode_columnwise_output(&tmap_qt, qt, rows, cols, tile_cols))
    return CUTEX_ERR_CUDA;
  const cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  return x_dtype == 0 ? launch_quantize_columnwise_t<0>(tmap, tmap_qt, rows, cols, sft, ds->sm_count, s)
                      : launch_quantize_columnwise_t<1>(tmap, tmap_qt, rows, cols, sft, ds->sm_count, s);
}

extern "C" const char* cutex_status_string(int status) {
  switch (status) {
    case CUTEX_OK: return "CUTEX_OK";
    case CUTEX_ERR_INVALID_ARGUMENT: return "CUTEX_ERR_INVALID_ARGUMENT: invalid argument or configuration";
    case CUTEX_ERR_SHAPE: return "CUTEX_ERR_SHAPE: unsupported problem shape";
    case CUTEX_ERR_ALIGN: return "CUTEX_ERR_ALIGN: pointer, stride or K alignment rule violated";
    case CUTEX_ERR_UNSUPPORTED_DEVICE: return "CUTEX_ERR_UNSUPPORTED_DEVICE: requires compute capability 10.0 (B200)";
    case CUTEX_ERR_CUDA: return "CUTEX_ERR_CUDA: CUDA runtime or driver call failed";
    case CUTEX_ERR_TIMEOUT: return "CUTEX_ERR_TIMEOUT: device-side wait exceeded its limit";
    case CUTEX_ERR_WORKSPACE: return "CUTEX_ERR_WORKSPACE: workspace missing or too small";
    case CUTEX_ERR_DEVICE_CHECK: return "CUTEX_ERR_DEVICE_CHECK: a device-side consistency check failed";
    default: return "CUTEX_ERR_UNKNOWN";
  }
}

extern "C" int cutex_last_device_status(cutex_stream_t stream) {
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  int value = 0;
  if (cudaStreamSynchronize(s) != cudaSuccess) return CUTEX_ERR_CUDA;
  if (cudaMemcpyFromSymbol(&value, g_cutex_device_status, sizeof(int)) != cudaSuccess)
    return CUTEX_ERR_CUDA;
  if (value != 0) {
    const int zero = 0;
    if (cudaMemcpyToSymbol(g_cutex_device_status, &zero, sizeof(int)) != cudaSuccess)
      return CUTEX_ERR_CUDA;
    return value >= 0x200 ? CUTEX_ERR_DEVICE_CHECK : CUTEX_ERR_TIMEOUT;
  }
  return CUTEX_OK;
}

namespace cutex {
// One warp; lane 7 fails a check with a known value (no memory is accessed
// apart from the status word and the check record).
__global__ void device_check_selftest_kernel() {
  dev_check(threadIdx.x != 7, kChkSelfTest, 0x5EED00 + static_cast<long long>(threadIdx.x));
}
}  // namespace cutex

extern "C" int cutex_build_checked(void) { return kCheckedBuild ? 1 : 0; }

extern "C" int cutex_device_check_record(cutex_stream_t stream, int32_t* site, int64_t* value) {
  if (site == nullptr || value == nullptr) return CUTEX_ERR_INVALID_ARGUMENT;
  if (cudaStreamSynchronize(reinterpret_cast<cudaStream_t>(stream)) != cudaSuccess) return CUTEX_ERR_CUDA;
  long long rec[2] = {0, 0};
  if (cudaMemcpyFromSymbol(rec, g_cutex_check_record, sizeof(rec)) != cudaSuccess) return CUTEX_ERR_CUDA;
  if (rec[0] != 0) {
    const long long zero[2] = {0, 0};
    if (cudaMemcpyToSymbol(g_cutex_check_record, zero, sizeof(zero)) != cudaSuccess) return CUTEX_ERR_CUDA;
  }
  *site = static_cast<int32_t>(rec[0]);
  *value = static_cast<int64_t>(rec[1]);
  return CUTEX_OK;
}

extern "C" int cutex_selftest_device_check(cutex_stream_t stream) {
  if (!kCheckedBuild) return CUTEX_ERR_INVALID_ARGUMENT;
  DeviceState* ds = nullptr;
  const int st = current_device_state(&ds);
  if (st != CUTEX_OK) return st;
  device_check_selftest_kernel<<<1, 32, 0, reinterpret_cast<cudaStream_t>(stream)>>>();
  return cudaGetLastError() == cudaSuccess ? CUTEX_OK : CUTEX_ERR_CUDA;
}

extern "C" int cutex_device_sm_count(int32_t* sm_count) {
  if (sm_count == nullptr) return CUTEX_ERR_INVALID_ARGUMENT;
  DeviceState* ds = nullptr;
  const int st = current_device_state(&ds);
  if (ds == nullptr) return st;
  *sm_count = ds->sm_count;
  return st;
}

extern "C" const char* cutex_version(void) {
  return kCheckedBuild ? "cutex-b200 0.1.0 sm_100a checked" : "cutex-b200 0.1.0 sm_100a";
}

// ---------------------------------------------------------------------------
// No-allocation entry point for the split-K skinny GEMM.
//
// Some callers cannot allocate device memory at the point where they launch a
// GEMM: code running inside a memory-capped pool or a custom allocator that
// forbids out-of-band cudaMalloc, real-time loops that must not hit the driver
// allocator, and plugins that are handed only the operand and output buffers.
// For them the skinny kernel's split-K workspace lives in a file-scope device
// array that the library owns. The array exists once per device for as long as
// the library is loaded: every GPU on which this library's module is loaded
// holds these 20.06 MiB until the process exits.
//
// Layout (same as the caller-provided workspace): partial sums for up to 160
// SMs x 2 slots x 128 x 128 fp32 (20 MiB), then 64 KiB of arrival counters,
// one uint32 per 128 rows of N (N <= 2,097,152).
namespace cutex {
namespace {

constexpr int64_t kStaticScratchPartialBytes = int64_t{2} * 160 * 128 * 128 * 4;
constexpr int64_t kStaticScratchCounterBytes = int64_t{64} * 1024;

}  // namespace
}  // namespace cutex

static __device__ __align__(256) unsigned char
    g_skinny_static_scratch[cutex::kStaticScratchPartialBytes + cutex::kStaticScratchCounterBytes];

namespace cutex {
namespace {

void* g_static_scratch_ptr[kMaxDevices];
unsigned g_static_scratch_epoch[kMaxDevices];  // device_epoch in which the address was fetched

}  // namespace
}  // namespace cutex

extern "C" int cutex_mxfp8_gemm_skinny_static(const void* a, const void* b, const void* sfa,
                                              const void* sfb, void* d, int64_t M, int64_t N,
                                              int64_t K, int64_t ldd, cutex_stream_t stream) {
  if (a == nullptr || b == nullptr || sfa == nullptr || sfb == nullptr || d == nullptr)
    return CUTEX_ERR_INVALID_ARGUMENT;
  int st = validate_shape(M, N, K);
  if (st != CUTEX_OK) return st;
  if (M > 128) return CUTEX_ERR_SHAPE;  // only the skinny kernel uses scratch memory
  if (ldd < N || ldd % 8 != 0 || ldd > kMaxDim) return CUTEX_ERR_ALIGN;
  if (!aligned16(a) || !aligned16(b) || !aligned16(sfa) || !aligned16(sfb) || !aligned16(d))
    return CUTEX_ERR_ALIGN;
  DeviceState* ds = nullptr;
  st = current_device_state(&ds);
  if (st != CUTEX_OK) return st;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return CUTEX_ERR_CUDA;

  // Set-up, once per device and with that device current: in host code the
  // array's name is only a host-side stand-in, so fetch its device address. The
  // address is fetched again if the device's context changed since (after a
  // device reset the module, and the array, are loaded anew).
  void* scratch = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_mutex);
    const unsigned epoch = device_epoch_locked(dev);
    if (g_static_scratch_ptr[dev] == nullptr || g_static_scratch_epoch[dev] != epoch) {
      void* p = nullptr;
      if (cudaGetSymbolAddress(&p, g_skinny_static_scratch) != cudaSuccess || p == nullptr)
        return CUTEX_ERR_CUDA;
      g_static_scratch_ptr[dev] = p;
      g_static_scratch_epoch[dev] = epoch;
    }
    scratch = g_static_scratch_ptr[dev];
  }

  cutex_gemm_config cfg{};
  cfg.kernel = CUTEX_KERNEL_SKINNY;  // split_k = 0: stream-K over all SMs
  cfg.tile_n = 128;                  // one 128-row B tile per CTA tile: the array holds one-tile slots
  Plan plan{};
  st = resolve_plan(&cfg, M, N, K, ds->sm_count, &plan);
  if (st != CUTEX_OK) return st;
  // Limits of the fixed array, checked separately: at most 160 SMs of partial
  // slots and 16384 counters (N <= 2,097,152).
  const int64_t counter_bytes = plan.workspace_bytes - plan.ws_partials_bytes;
  if (plan.ws_partials_bytes > kStaticScratchPartialBytes ||
      static_cast<int64_t>(plan.num_n_tiles) * 4 > kStaticScratchCounterBytes ||
      counter_bytes > kStaticScratchCounterBytes)
    return CUTEX_ERR_WORKSPACE;

  // The array keeps the previous call's contents; the arrival counters must
  // start at zero, so clear the ones this call uses (the partial sums need no
  // clearing). This is a memset on stream order, not an allocation.
  if (cudaMemsetAsync(static_cast<char*>(scratch) + plan.ws_partials_bytes, 0,
                      static_cast<size_t>(counter_bytes),
                      reinterpret_cast<cudaStream_t>(stream)) != cudaSuccess)
    return CUTEX_ERR_CUDA;
  return launch_skinny(plan, dev, a, b, sfa, sfb, d, M, N, K, ldd, scratch,
                       reinterpret_cast<cudaStream_t>(stream));
}

// ---------------------------------------------------------------- host-buffer pipeline
//
// cutex_mxfp8_gemm_host: copies in, block GEMMs and copies out on three
// library-owned streams per device, ordered by events. Streams and events are
// created once per device (no device memory is allocated).

namespace {

constexpr int kMaxHostBlocks = 16;

struct HostPipe {
  bool ready = false;
  cudaStream_t h2d = nullptr, comp = nullptr, d2h = nullptr;
  cudaEvent_t start = nullptr, end_h2d = nullptr, end_comp = nullptr, end_d2h = nullptr;
  cudaEvent_t a_in[kMaxHostBlocks] = {}, b_in[kMaxHostBlocks] = {};
  cudaEvent_t done[kMaxHostBlocks * kMaxHostBlocks] = {};
  unsigned epoch = 0;  // device_epoch the streams and events were created in
};

HostPipe g_pipes[kMaxDevices];
std::mutex g_pipe_mutex;

int host_pipe(int dev, HostPipe** out) {
  HostPipe& p = g_pipes[dev];
  const unsigned epoch = device_epoch(dev);
  if (p.epoch != epoch) {
    // Created in a context that no longer exists: those handles are gone with it.
    p = HostPipe{};
    p.epoch = epoch;
  }
  if (!p.ready) {
    const unsigned ev_flags = cudaEventDisableTiming;
    bool ok = cudaStreamCreateWithFlags(&p.h2d, cudaStreamNonBlocking) == cudaSuccess &&
              cudaStreamCreateWithFlags(&p.comp, cudaStreamNonBlocking) == cudaSuccess &&
              cudaStreamCreateWithFlags(&p.d2h, cudaStreamNonBlocking) == cudaSuccess &&
              cudaEventCreateWithFlags(&p.start, ev_flags) == cudaSuccess &&
              cudaEventCreateWithFlags(&p.end_h2d, ev_flags) == cudaSuccess &&
              cudaEventCreateWithFlags(&p.end_comp, ev_flags) == cudaSuccess &&
              cudaEventCreateWithFlags(&p.end_d2h, ev_flags) == cudaSuccess;
    for (int i = 0; ok && i < kMaxHostBlocks; ++i)
      ok = cudaEventCreateWithFlags(&p.a_in[i], ev_flags) == cudaSuccess &&
           cudaEventCreateWithFlags(&p.b_in[i], ev_flags) == cudaSuccess;
    for (int i = 0; ok && i < kMaxHostBlocks * kMaxHostBlocks; ++i)
      ok = cudaEventCreateWithFlags(&p.done[i], ev_flags) == cudaSuccess;
    if (!ok) return CUTEX_ERR_CUDA;  // a later call retries the missing objects' creation
    p.ready = true;
  }
  *out = &p;
  return CUTEX_OK;
}

int64_t ceil_div64(int64_t a, int64_t b) { return (a + b - 1) / b; }

}  // namespace

extern "C" int cutex_mxfp8_gemm_host(const void* a_host, const void* b_host, const void* sfa_host,
                                     const void* sfb_host, void* d_host, void* a_dev, void* b_dev,
                                     void* sfa_dev, void* sfb_dev, void* d_dev, int64_t M, int64_t N,
                                     int64_t K, const cutex_gemm_config* cfg, int32_t blocks,
                                     void* workspace, int64_t workspace_bytes, cutex_stream_t stream) {
  if (a_host == nullptr || b_host == nullptr || sfa_host == nullptr || sfb_host == nullptr ||
      d_host == nullptr || a_dev == nullptr || b_dev == nullptr || sfa_dev == nullptr ||
      sfb_dev == nullptr || d_dev == nullptr || workspace_bytes < 0)
    return CUTEX_ERR_INVALID_ARGUMENT;
  if (blocks < 1 || blocks > kMaxHostBlocks) return CUTEX_ERR_INVALID_ARGUMENT;
  int st = validate_shape(M, N, K);
  if (st != CUTEX_OK) return st;
  if (!aligned16(a_dev) || !aligned16(b_dev) || !aligned16(sfa_dev) || !aligned16(sfb_dev) ||
      !aligned16(d_dev))
    return CUTEX_ERR_ALIGN;
  DeviceState* ds = nullptr;
  st = current_device_state(&ds);
  if (st != CUTEX_OK) return st;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return CUTEX_ERR_CUDA;
  // Validate the configuration once on the whole shape.
  Plan whole_plan{};
  st = resolve_plan(cfg, M, N, K, ds->sm_count, &whole_plan);
  if (st != CUTEX_OK) return st;

  // Block sizes: multiples of 256 rows / columns (whole 128-row scale blocks,
  // whole CTA-pair tiles); the last block of each dimension may be shorter.
  const int64_t bm = std::max<int64_t>(256, ceil_div64(ceil_div64(M, blocks), 256) * 256);
  const int64_t bn = std::max<int64_t>(256, ceil_div64(ceil_div64(N, blocks), 256) * 256);
  const int gm = static_cast<int>(ceil_div64(M, bm));
  const int gn = static_cast<int>(ceil_div64(N, bn));
  const int64_t sf_row = K / 32;  // scale bytes per operand row
  auto sf_bytes = [&](int64_t rows) { return ceil_div64(rows, 128) * 128 * sf_row; };
  const char* ah = static_cast<const char*>(a_host);
  const char* bh = static_cast<const char*>(b_host);
  const char* sah = static_cast<const char*>(sfa_host);
  const char* sbh = static_cast<const char*>(sfb_host);
  char* dh = static_cast<char*>(d_host);
  char* ad = static_cast<char*>(a_dev);
  char* bd = static_cast<char*>(b_dev);
  char* sad = static_cast<char*>(sfa_dev);
  char* sbd = static_cast<char*>(sfb_dev);
  char* dd = static_cast<char*>(d_dev);
  const cudaStream_t user = reinterpret_cast<cudaStream_t>(stream);

  std::lock_guard<std::mutex> lock(g_pipe_mutex);
  HostPipe* p = nullptr;
  st = host_pipe(dev, &p);
  if (st != CUTEX_OK) return st;
  bool ok = cudaEventRecord(p->start, user) == cudaSuccess &&
            cudaStreamWaitEvent(p->h2d, p->start, 0) == cudaSuccess &&
            cudaStreamWaitEvent(p->comp, p->start, 0) == cudaSuccess &&
            cudaStreamWaitEvent(p->d2h, p->start, 0) == cudaSuccess;
  int gemm_status = CUTEX_OK;
  // One block GEMM and its D2H copy, after A panel i and B panel j have landed.
  auto run_block = [&](int i, int j) {
    const int64_t m0 = i * bm, n0 = j * bn;
    const int64_t rows = std::min(bm, M - m0), cols = std::min(bn, N - n0);
    const int64_t d_off = (m0 * N + n0) * 2;
    ok = ok && cudaStreamWaitEvent(p->comp, p->a_in[i], 0) == cudaSuccess &&
         cudaStreamWaitEvent(p->comp, p->b_in[j], 0) == cudaSuccess;
    if (!ok || gemm_status != CUTEX_OK) return;
    gemm_status = cutex_mxfp8_gemm(ad + m0 * K, bd + n0 * K, sad + m0 * sf_row, sbd + n0 * sf_row, dd + d_off,
                                   rows, cols, K, N, cfg, workspace, workspace_bytes, p->comp);
    cudaEvent_t e = p->done[i * gn + j];
    ok = ok && cudaEventRecord(e, p->comp) == cudaSuccess &&
         cudaStreamWaitEvent(p->d2h, e, 0) == cudaSuccess &&
         cudaMemcpy2DAsync(dh + d_off, static_cast<size_t>(N) * 2, dd + d_off, static_cast<size_t>(N) * 2,
                           static_cast<size_t>(cols) * 2, static_cast<size_t>(rows), cudaMemcpyDeviceToHost,
                           p->d2h) == cudaSuccess;
  };
  // All copies in first (so the copy engine never waits for the host to
  // enqueue block GEMMs), then the blocks in growing-square order.
  const int steps = std::max(gm, gn);
  for (int s = 0; ok && s < steps; ++s) {
    if (s < gm) {
      const int64_t m0 = s * bm, rows = std::min(bm, M - m0);
      ok = cudaMemcpyAsync(ad + m0 * K, ah + m0 * K, static_cast<size_t>(rows * K), cudaMemcpyHostToDevice,
                           p->h2d) == cudaSuccess &&
           cudaMemcpyAsync(sad + m0 * sf_row, sah + m0 * sf_row, static_cast<size_t>(sf_bytes(rows)),
                           cudaMemcpyHostToDevice, p->h2d) == cudaSuccess &&
           cudaEventRecord(p->a_in[s], p->h2d) == cudaSuccess;
    }
    if (ok && s < gn) {
      const int64_t n0 = s * bn, rows = std::min(bn, N - n0);
      ok = cudaMemcpyAsync(bd + n0 * K, bh + n0 * K, static_cast<size_t>(rows * K), cudaMemcpyHostToDevice,
                           p->h2d) == cudaSuccess &&
           cudaMemcpyAsync(sbd + n0 * sf_row, sbh + n0 * sf_row, static_cast<size_t>(sf_bytes(rows)),
                           cudaMemcpyHostToDevice, p->h2d) == cudaSuccess &&
           cudaEventRecord(p->b_in[s], p->h2d) == cudaSuccess;
    }
  }
  for (int s = 0; ok && gemm_status == CUTEX_OK && s < steps; ++s) {
    // Every block whose larger index is s: row s against columns 0..s, then
    // rows 0..s-1 against column s.
    if (s < gm)
      for (int j = 0; j <= std::min(s, gn - 1); ++j) run_block(s, j);
    if (s < gn)
      for (int i = 0; i < std::min(s, gm); ++i) run_block(i, s);
  }
  // Join: the caller's stream waits for all three streams, even after an error.
  const bool joined = cudaEventRecord(p->end_h2d, p->h2d) == cudaSuccess &&
                      cudaEventRecord(p->end_comp, p->comp) == cudaSuccess &&
                      cudaEventRecord(p->end_d2h, p->d2h) == cudaSuccess &&
                      cudaStreamWaitEvent(user, p->end_h2d, 0) == cudaSuccess &&
                      cudaStreamWaitEvent(user, p->end_comp, 0) == cudaSuccess &&
                      cudaStreamWaitEvent(user, p->end_d2h, 0) == cudaSuccess;
  if (gemm_status != CUTEX_OK) return gemm_status;
  return ok && joined ? CUTEX_OK : CUTEX_ERR_CUDA;
}
