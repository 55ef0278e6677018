// Persistent, warp-specialised MXFP8 block-scaled GEMM for sm_100a.
//
//   D[M,N] bf16 = (A[M,K] e4m3 * SFA) . (B[N,K] e4m3 * SFB)^T, FP32 accumulate.
//
// One CTA (kCtaGroup = 1) or one CTA pair (kCtaGroup = 2, cluster of 2) owns a
// (128*kCtaGroup) x kTileN output tile at a time and walks a static,
// grouped-raster sequence of tiles (persistent grid sized to the SM count).
//
// Warp roles (192 threads, 224 with the dynamic scheduler):
//   warps 0-3  epilogue: TMEM -> registers -> BF16 -> swizzled SMEM -> TMA store.
//              Warp w owns TMEM lanes [32w, 32w+32), i.e. output rows 32w..32w+31.
//   warp 4     MMA issuer (the pair leader's warp when kCtaGroup = 2): the warp
//              waits converged and one elected lane per K-stage copies the
//              SFA/SFB chunks SMEM->TMEM (tcgen05.cp), issues four K=32
//              block-scaled MMAs and commits the stage back.
//   warp 5     TMA producer (every CTA; one elected lane issues): A, B, SFA, SFB
//              tiles into a kStages-deep ring guarded by full/empty mbarriers.
//   warp 6     tile scheduler (dynamic builds, pair leader): cluster launch control.
//
// TMEM plan (512 columns, 32-bit): two accumulator buffers alternate by tile.
// When two full buffers plus the scale-factor columns do not fit (tile_n =
// 256), buffer 1 starts at column 512 - 256 - 16*kSFBufs and overlaps the end of
// buffer 0; the epilogue reads the overlapping 64-column chunk first and then
// releases the accumulator, so the next tile's MMAs start while the rest of
// the tile is still being stored. Scale factors: SFA 4 columns (128 rows),
// SFB 4 columns per 128 rows of N, byte k of a column = K-block k of a stage,
// in kSFBufs rotating 16-column buffers at the top of TMEM.
//
// K-stage: 128 K values. A stage holds the A tile (128 x 128 B), this CTA's B
// rows (kTileN/kCtaGroup x 128 B), the 512-byte SFA chunk and the full SFB
// chunk(s) of the MMA's N (each CTA of a pair loads its own copy; no load is
// broadcast to several CTAs).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp8.h>

#include "device_status.cuh"  // status word, DeviceError, dev_check
#include "mxfp8_quant.cuh"    // sf_offset: the 128x4 scale layout
#include "ptx.cuh"

namespace cutex {

struct GemmArgs {
  int num_m_tiles;  // output tiles along M (tile rows = 128 * kCtaGroup)
  int num_n_tiles;  // output tiles along N
  int num_tiles;
  int num_k_blocks;  // K / 128
  int raster_group;
  int raster_along_n;
  unsigned long long* trace;  // traced builds only: event buffer (see Tracer)
  int trace_cap;              // events per (CTA, role) region
  // Fused-epilogue builds (kEpi > 0): D = alpha * acc + beta * C + bias[col],
  // then BF16 (kEpi = 1) or E4M3 with E8M0 scales per 1x32 block along N
  // (kEpi = 2; scales in the 128x4 swizzled layout of an [M, K = N] operand).
  float alpha, beta;
  const __nv_bfloat16* c;  // [M, N] bf16, row stride ldc (elements), or null
  long long ldc;
  const __nv_bfloat16* bias;  // [N] bf16 or null
  uint8_t* d_scales;          // kEpi = 2
  int M, N;
  // kEpi = 3 (fused all-gather): every D chunk is also stored, by TMA from the
  // same staging buffer, through each of num_peers tensor maps (global memory)
  // that describe the peers' copies of D (NVLink peer memory).
  const CUtensorMap* peer_maps;
  int num_peers;
  // Error-path self-test builds (kFaultTest) only: the producer issues no copies
  // for this CTA's K-stage with linear index fault_withhold_kit.
  int fault_withhold_kit;
};

// Wait limit of the error-path self-test builds: short enough for a test, far
// above the time any stage of a small GEMM takes to arrive.
constexpr uint64_t kFaultTestWaitNs = 1000000ull;  // 1 ms

// In-kernel event trace of the first CTA (pair): each role's recording thread
// appends (globaltimer ns, event << 56 | tile << 24 | k_block) records to its own
// region [rank * 3 + role] of `trace`; record 0 of a region holds the count.
// Compiled only into the kTrace instantiations, never into benchmarked kernels.
enum TraceEvent : uint32_t {
  kEvStart = 1,
  kEvEnd = 2,
  kEvProdWait = 3,    // producer: wait for an empty stage
  kEvProdGo = 4,      // producer: stage free, TMA issued next
  kEvMmaAccWait = 5,  // MMA: wait for the accumulator (epilogue release)
  kEvMmaAccGo = 6,
  kEvMmaFullWait = 7,  // MMA: wait for a loaded stage
  kEvMmaFullGo = 8,
  kEvMmaIssued = 9,    // MMA: stage's MMAs issued and committed
  kEvMmaTileDone = 10,
  kEvEpiWait = 11,  // epilogue: wait for a finished accumulator
  kEvEpiGo = 12,
  kEvEpiRelease = 13,
  kEvEpiTileDone = 14,
  kEvEpiLoaded = 15,  // epilogue: first (overlapping) chunk read from TMEM
};

template <bool kOn>
struct Tracer {
  unsigned long long* region = nullptr;
  int cap = 0;
  int n = 0;
  __device__ __forceinline__ void open(const GemmArgs& a, bool traced_cta, int region_idx) {
    if constexpr (kOn) {
      if (traced_cta && a.trace != nullptr) {
        region = a.trace + static_cast<size_t>(region_idx) * (a.trace_cap + 1) * 2;
        cap = a.trace_cap;
      }
    }
  }
  __device__ __forceinline__ void rec(uint32_t ev, int tile, int kb) {
    if constexpr (kOn) {
      if (region != nullptr && n < cap) {
        region[2 * (n + 1)] = ptx::globaltimer();
        region[2 * (n + 1) + 1] = (static_cast<unsigned long long>(ev) << 56) |
                                  (static_cast<unsigned long long>(tile & 0xFFFFFFF) << 24) |
                                  static_cast<unsigned long long>(kb & 0xFFFFFF);
        ++n;
      }
    }
  }
  // Timestamp now, record later (rec_at): keeps trace stores out of a stretch that
  // ends in a release (a release would wait for the stores to become visible).
  __device__ __forceinline__ unsigned long long stamp() const {
    if constexpr (kOn) return region != nullptr ? ptx::globaltimer() : 0ull;
    return 0ull;
  }
  __device__ __forceinline__ void rec_at(uint32_t ev, unsigned long long t_ns, int tile, int kb) {
    if constexpr (kOn) {
      if (region != nullptr && n < cap) {
        region[2 * (n + 1)] = t_ns;
        region[2 * (n + 1) + 1] = (static_cast<unsigned long long>(ev) << 56) |
                                  (static_cast<unsigned long long>(tile & 0xFFFFFFF) << 24) |
                                  static_cast<unsigned long long>(kb & 0xFFFFFF);
        ++n;
      }
    }
  }
  __device__ __forceinline__ void close() {
    if constexpr (kOn) {
      if (region != nullptr) region[0] = static_cast<unsigned long long>(n);
    }
  }
};

// Traced builds also record every CTA's [start, end] globaltimer after the six
// role regions, trace[6 * (trace_cap + 1) * 2 + 2 * blockIdx.x + {0, 1}], and the
// SM cycle counter at the same two points after those, at + 2 * gridDim.x
// (cycles over nanoseconds = the SM clock the CTA actually ran at).
template <bool kOn>
__device__ __forceinline__ void trace_cta_time(const GemmArgs& a, int which) {
  if constexpr (kOn) {
    if (a.trace != nullptr) {
      unsigned long long* base = a.trace + static_cast<size_t>(6) * (a.trace_cap + 1) * 2;
      const unsigned long long clk = ptx::clock64();
      base[2 * blockIdx.x + which] = ptx::globaltimer();
      base[2 * gridDim.x + 2 * blockIdx.x + which] = clk;
    }
  }
}

constexpr int kSmemLimit = 232448;  // max dynamic shared memory per block on sm_100

constexpr int align_up(int x, int a) { return (x + a - 1) / a * a; }

template <int kCtaGroup, int kTileN, int kStages, int kEpiBufs, int kSFBufs>
struct GemmCfg {
  static constexpr int kThreads = 192;
  static constexpr int kTileM = 128;  // rows per CTA
  static constexpr int kTileK = 128;  // K values (bytes) per stage
  static constexpr int kLoadN = kTileN / kCtaGroup;  // B rows each CTA loads
  static constexpr int kABytes = kTileM * kTileK;
  static constexpr int kBBytes = kLoadN * kTileK;
  static constexpr int kSFABytes = 512;
  static constexpr int kSFBBytes = (kTileN / 128) * 512;
  static constexpr int kStageBytes = kABytes + kBBytes + kSFABytes + kSFBBytes;
  static constexpr uint32_t kTxBytes = kStageBytes * kCtaGroup;

  static constexpr int kOffA = 0;
  static constexpr int kOffB = kOffA + kStages * kABytes;
  static constexpr int kOffSFA = kOffB + kStages * kBBytes;
  static constexpr int kOffSFB = kOffSFA + kStages * kSFABytes;
  static constexpr int kOffC = align_up(kOffSFB + kStages * kSFBBytes, 1024);
  static constexpr int kCBufBytes = 32 * 64 * 2;  // 32 rows x 64 bf16, 128B-swizzled
  static constexpr int kOffBar = kOffC + 4 * kEpiBufs * kCBufBytes;
  // full[S], empty[S], acc_full[2], acc_empty[2], work_full[2], work_empty[2], clc
  static constexpr int kNumBars = 2 * kStages + 9;
  static constexpr int kOffMisc = align_up(kOffBar + kNumBars * 8, 16);
  static constexpr int kOffTmemSlot = kOffMisc;       // TMEM base address from tcgen05.alloc
  static constexpr int kOffWorkSlot = kOffMisc + 16;  // two tile ids of the work ring
  static constexpr int kOffClcResp = kOffMisc + 32;   // 16-byte try_cancel response
  static constexpr int kSmemBytes = kOffMisc + 48 + 1024;  // + base alignment slack

  static constexpr int kTmemCols = 512;
  static constexpr int kSFACols = 4;
  static constexpr int kSFBCols = (kTileN / 128) * 4;
  // Scale factors rotate through kSFBufs 16-column buffers (one per K-stage in
  // flight), so the SMEM->TMEM copy of stage k+1 never waits for the MMAs of
  // stage k to finish reading the previous scales.
  static constexpr int kSFBufCols = 16;
  static constexpr int kSFReserved = kSFBufCols * kSFBufs;
  static constexpr bool kOverlap = 2 * kTileN + kSFReserved > kTmemCols;
  static constexpr int kAcc1Col = kOverlap ? (kTmemCols - kSFReserved - kTileN) : kTileN;
  static constexpr int kSFACol = kOverlap ? (kTmemCols - kSFReserved) : 2 * kTileN;
  static constexpr int kSFBCol = kSFACol + kSFACols;
  static constexpr int kChunks = kTileN / 64;
  // First 64-column chunk the epilogue reads from buffer 0 / buffer 1.
  static constexpr int kFirstChunk0 = kOverlap ? kAcc1Col / 64 : 0;
  static constexpr uint32_t kIdesc = ptx::mxf8_idesc(kTileM * kCtaGroup, kTileN);

  static_assert(kCtaGroup == 1 || kCtaGroup == 2, "cta group");
  static_assert(kTileN == 128 || kTileN == 256, "tile_n");
  static_assert(kSFACols + kSFBCols <= kSFBufCols, "scale-factor columns");
  static_assert(kSFBufs == 1 || kSFBufs == 2 || kSFBufs == 4, "scale-factor buffers");
  static_assert(kSFACol + kSFReserved <= kTmemCols, "TMEM plan");
  static_assert(!kOverlap || (kTileN - kAcc1Col) <= 64 - (kAcc1Col % 64),
                "overlap must sit inside one epilogue chunk");
  static_assert(kSmemBytes <= kSmemLimit, "shared memory budget");
  static_assert(kEpiBufs == 1 || kEpiBufs == 2, "epilogue buffers");
};

__device__ __forceinline__ void tile_coords(int t, const GemmArgs& a, int& mt, int& nt) {
  const int g_size = a.raster_group;
  if (!a.raster_along_n) {
    const int per_group = g_size * a.num_n_tiles;
    const int g = t / per_group;
    const int r = t - g * per_group;
    const int m0 = g * g_size;
    const int gm = min(g_size, a.num_m_tiles - m0);
    mt = m0 + r % gm;
    nt = r / gm;
  } else {
    const int per_group = g_size * a.num_m_tiles;
    const int g = t / per_group;
    const int r = t - g * per_group;
    const int n0 = g * g_size;
    const int gn = min(g_size, a.num_n_tiles - n0);
    nt = n0 + r % gn;
    mt = r / gn;
  }
}

__device__ __forceinline__ uint32_t pack_bf16x2(uint32_t lo, uint32_t hi) {
  __nv_bfloat162 h = __floats2bfloat162_rn(__uint_as_float(lo), __uint_as_float(hi));
  return *reinterpret_cast<uint32_t*>(&h);
}

// alpha * acc + beta * C[row, n0 + j] + bias[n0 + j] on one row's 64
// accumulator columns (fp32 bits, columns 0-31 in v0, 32-63 in v1). N is a
// multiple of 16, so each 8-column group is wholly inside or outside D.
__device__ __forceinline__ void epilogue_affine(uint32_t (&v0)[32], uint32_t (&v1)[32], const GemmArgs& a, int row,
                                                int n0) {
  const float alpha = a.alpha;
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    v0[j] = __float_as_uint(__uint_as_float(v0[j]) * alpha);
    v1[j] = __float_as_uint(__uint_as_float(v1[j]) * alpha);
  }
  const bool use_c = a.c != nullptr && a.beta != 0.f && row < a.M;
#pragma unroll
  for (int g = 0; g < 8; ++g) {
    if (n0 + 8 * g >= a.N) break;
    uint32_t* v = g < 4 ? &v0[8 * g] : &v1[8 * (g - 4)];
    if (use_c) {
      const uint4 cv = __ldcs(reinterpret_cast<const uint4*>(a.c + static_cast<long long>(row) * a.ldc + n0 + 8 * g));
      const uint32_t w[4] = {cv.x, cv.y, cv.z, cv.w};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        v[2 * q] = __float_as_uint(fmaf(a.beta, __uint_as_float(w[q] << 16), __uint_as_float(v[2 * q])));
        v[2 * q + 1] = __float_as_uint(fmaf(a.beta, __uint_as_float(w[q] & 0xFFFF0000u), __uint_as_float(v[2 * q + 1])));
      }
    }
    if (a.bias != nullptr) {
      const uint4 bv = __ldg(reinterpret_cast<const uint4*>(a.bias + n0 + 8 * g));
      const uint32_t w[4] = {bv.x, bv.y, bv.z, bv.w};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        v[2 * q] = __float_as_uint(__uint_as_float(v[2 * q]) + __uint_as_float(w[q] << 16));
        v[2 * q + 1] = __float_as_uint(__uint_as_float(v[2 * q + 1]) + __uint_as_float(w[q] & 0xFFFF0000u));
      }
    }
  }
}

// One 1x32 block (fp32 bits) -> 8 words of E4M3 codes + the E8M0 scale byte,
// with the quantiser's rule (scale exponent floor(log2 amax) - 8, 0x00 for an
// all-zero block, 0xFF and zero codes for a block holding a non-finite value).
__device__ __forceinline__ uint32_t quantize_block32(const uint32_t (&v)[32], uint32_t (&w)[8]) {
  float amax = 0.f;
  uint32_t nonfinite = 0;
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    const uint32_t bits = v[j] & 0x7FFFFFFFu;
    nonfinite |= bits >= 0x7F800000u ? 1u : 0u;
    amax = fmaxf(amax, __uint_as_float(bits));
  }
  const uint32_t exp_field = __float_as_uint(amax) >> 23;
  const uint32_t sbyte = nonfinite ? 0xFFu : (exp_field >= 8u ? exp_field - 8u : 0u);
  const float mult = __uint_as_float((254u - (nonfinite ? 127u : sbyte)) << 23);  // 2^(127 - sbyte), exact
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    const uint32_t lo = static_cast<uint32_t>(__nv_cvt_float2_to_fp8x2(
        make_float2(__uint_as_float(v[4 * q]) * mult, __uint_as_float(v[4 * q + 1]) * mult), __NV_SATFINITE, __NV_E4M3));
    const uint32_t hi = static_cast<uint32_t>(__nv_cvt_float2_to_fp8x2(
        make_float2(__uint_as_float(v[4 * q + 2]) * mult, __uint_as_float(v[4 * q + 3]) * mult), __NV_SATFINITE,
        __NV_E4M3));
    w[q] = nonfinite ? 0u : (lo | (hi << 16));
  }
  return sbyte;
}

__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c,
                                             uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c),
               "r"(d)
               : "memory");
}

// Where each role gets its next output tile.
//  static (kDynamic = false): tiles cluster_id, cluster_id + num_clusters, ...
//  dynamic: a two-slot ring in shared memory filled by the pair leader's
//  scheduler warp (the cluster's own tile first, then tiles of clusters it
//  cancelled through cluster launch control); a negative id ends the walk.
//  Every consumer reads the slot and then releases it on the leader's
//  work_empty barrier (peer CTAs arrive remotely), so the scheduler never
//  overwrites an id before all eleven (pair) or six (single CTA) consumers have
//  read it.
template <bool kDynamic, bool kPair>
struct TileSource {
  int t = 0, step = 1, num_tiles = 0;
  uint32_t w = 0, full0 = 0, empty0 = 0, slot0 = 0;
  bool peer = false;

  __device__ __forceinline__ void init(int first, int stride, int tiles, uint32_t full_bar0,
                                      uint32_t empty_bar0, uint32_t slot_addr0, bool is_peer) {
    t = first;
    step = stride;
    num_tiles = tiles;
    full0 = full_bar0;
    empty0 = empty_bar0;
    slot0 = slot_addr0;
    peer = is_peer;
  }

  // Called by the consuming threads of a role: one thread (producer, MMA issuer)
  // or all lanes of a warp (epilogue, whole_warp = true, which syncs the warp
  // so every lane has read the slot before `releaser` frees it).
  __device__ __forceinline__ bool next(int& tile, bool releaser, bool whole_warp, int* status) {
    if constexpr (!kDynamic) {
      if (t >= num_tiles) return false;
      tile = t;
      t += step;
      return true;
    } else {
      const uint32_t s = w & 1u;
      bool ok = ptx::mbar_wait<true>(full0 + 8u * s, (w >> 1) & 1u, status, kDevTimeoutScheduler);
      if (whole_warp) ok = __all_sync(0xffffffffu, ok) != 0;
      if (!ok) return false;
      tile = static_cast<int>(ptx::ld_shared_u32(slot0 + 4u * s));
      if (tile >= num_tiles) {  // never act on an id outside the grid's tiles
        atomicCAS(status, 0, kDevBadTile);
        tile = -1;
      }
      if (whole_warp) __syncwarp();
      if (releaser) {
        if (kPair && peer) ptx::mbar_arrive_cluster(ptx::mapa(empty0 + 8u * s, 0));
        else ptx::mbar_arrive(empty0 + 8u * s);
      }
      ++w;
      return tile >= 0;
    }
  }
};

// Wait ~50 us so that TMA loads already in flight land before the CTA exits on
// an error path (loads of valid addresses complete on their own).
__device__ __forceinline__ void settle_inflight_copies() {
  const uint64_t t0 = ptx::globaltimer();
  while (ptx::globaltimer() - t0 < 50000ull) __nanosleep(1000);
}

// kFaultTest: the error-path self-test twin (static scheduler only). Every
// bounded wait gives up after kFaultTestWaitNs, and the producer skips the
// copies of K-stage args.fault_withhold_kit (and its expect-tx), so the MMA
// issuer waits for data that never arrives while nothing is in flight for that
// stage; the roles then time out in turn and the CTA settles, frees TMEM and
// exits with the error recorded in g_cutex_device_status.
template <int kCtaGroup, int kTileN, int kStages, int kEpiBufs, int kSFBufs, bool kDynamic,
          bool kTrace = false, int kEpi = 0, bool kFaultTest = false>
__global__ void __launch_bounds__(kDynamic ? 224 : 192, 1)
    mxfp8_gemm_kernel(const __grid_constant__ CUtensorMap tmap_a,
                      const __grid_constant__ CUtensorMap tmap_b,
                      const __grid_constant__ CUtensorMap tmap_sfa,
                      const __grid_constant__ CUtensorMap tmap_sfb,
                      const __grid_constant__ CUtensorMap tmap_d, const GemmArgs args) {
  using C = GemmCfg<kCtaGroup, kTileN, kStages, kEpiBufs, kSFBufs>;
  constexpr bool kPair = kCtaGroup == 2;
  static_assert(!(kFaultTest && (kDynamic || kTrace || kEpi != 0)), "self-test twin: static, plain epilogue");
  constexpr uint64_t kLimit = kFaultTest ? kFaultTestWaitNs : ptx::kWaitLimitNs;

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_base = ptx::smem_u32(smem_raw);
  const uint32_t smem = (raw_base + 1023u) & ~1023u;
  uint8_t* smem_ptr = smem_raw + (smem - raw_base);

  const int warp = threadIdx.x >> 5;
  const uint32_t lane = ptx::lane_id();
  const uint32_t rank = kPair ? ptx::cluster_ctarank() : 0u;
  const bool leader = rank == 0;
  const int cluster_id = blockIdx.x / kCtaGroup;
  const int num_clusters = gridDim.x / kCtaGroup;
  int* status = &g_cutex_device_status;

  const uint32_t bar0 = smem + C::kOffBar;
  auto full_bar = [&](int s) { return bar0 + 8u * s; };
  auto empty_bar = [&](int s) { return bar0 + 8u * (kStages + s); };
  auto acc_full_bar = [&](int b) { return bar0 + 8u * (2 * kStages + b); };
  auto acc_empty_bar = [&](int b) { return bar0 + 8u * (2 * kStages + 2 + b); };
  const uint32_t work_full0 = bar0 + 8u * (2 * kStages + 4);
  const uint32_t work_empty0 = bar0 + 8u * (2 * kStages + 6);
  const uint32_t clc_bar = bar0 + 8u * (2 * kStages + 8);
  const uint32_t work_slot0 = smem + C::kOffWorkSlot;
  volatile uint32_t* tmem_slot = reinterpret_cast<volatile uint32_t*>(smem_ptr + C::kOffTmemSlot);

  if (warp == 5 && lane == 0) {
    ptx::prefetch_tmap(&tmap_a);
    ptx::prefetch_tmap(&tmap_b);
    ptx::prefetch_tmap(&tmap_sfa);
    ptx::prefetch_tmap(&tmap_sfb);
    ptx::prefetch_tmap(&tmap_d);
    for (int s = 0; s < kStages; ++s) {
      ptx::mbar_init(full_bar(s), 1);
      ptx::mbar_init(empty_bar(s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      ptx::mbar_init(acc_full_bar(b), 1);
      ptx::mbar_init(acc_empty_bar(b), 4 * kCtaGroup);
      ptx::mbar_init(work_full0 + 8u * b, 1);
      // producer + epilogue warps of every CTA, + the leader's MMA issuer
      ptx::mbar_init(work_empty0 + 8u * b, 5 * kCtaGroup + 1);
    }
    ptx::mbar_init(clc_bar, 1);
    ptx::fence_mbar_init();
  }
  if (warp == 4) {
    ptx::tmem_alloc<kCtaGroup>(ptx::smem_u32(const_cast<uint32_t*>(tmem_slot)), C::kTmemCols);
    ptx::tmem_relinquish<kCtaGroup>();
  }
  ptx::tc_fence_before();
  if constexpr (kPair) ptx::cluster_sync(); else __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // Launched with programmatic stream serialization: the set-up above may
  // overlap the end of the previous kernel in the stream; no global memory is
  // touched before that kernel has completed. The next launch may be
  // scheduled from here on (its CTAs take SMs as these CTAs exit).
  ptx::grid_dependency_wait();
  ptx::launch_dependents();
  Tracer<kTrace> tr;
  if (threadIdx.x == 0) trace_cta_time<kTrace>(args, 0);
  TileSource<kDynamic, kPair> src;
  src.init(cluster_id, num_clusters, args.num_tiles, work_full0, work_empty0, work_slot0, !leader);
  int t = 0;

  if constexpr (kDynamic) {
    if (warp == 6) {
      // -------------------------------------------------------- tile scheduler
      if (leader && lane == 0) {
        int tile = cluster_id;
        uint32_t clc_phase = 0;
        const uint32_t resp = smem + C::kOffClcResp;
        for (uint32_t w = 0;; ++w) {
          const uint32_t s = w & 1u;
          if (!ptx::mbar_wait<kPair>(work_empty0 + 8u * s, ((w >> 1) & 1u) ^ 1u, status,
                                     kDevTimeoutScheduler))
            break;
          ptx::st_shared_u32(work_slot0 + 4u * s, static_cast<uint32_t>(tile));
          ptx::mbar_arrive(work_full0 + 8u * s);
          if constexpr (kPair) {
            ptx::st_shared_cluster_u32(ptx::mapa(work_slot0 + 4u * s, 1), static_cast<uint32_t>(tile));
            ptx::mbar_arrive_cluster(ptx::mapa(work_full0 + 8u * s, 1));
          }
          if (tile < 0) break;
          // Steal the next not-yet-started cluster's tile (or learn there is none).
          ptx::mbar_arrive_expect_tx(clc_bar, 16);
          ptx::clc_try_cancel(resp, clc_bar);
          if (!ptx::mbar_wait(clc_bar, clc_phase, status, kDevTimeoutScheduler)) {
            tile = -1;  // publish the end marker so every role leaves its loop
            continue;
          }
          clc_phase ^= 1u;
          uint32_t first_x = 0;
          tile = ptx::clc_query(resp, first_x) ? static_cast<int>(first_x / kCtaGroup) : -1;
          if (tile >= 0 && (first_x >= gridDim.x || first_x % kCtaGroup != 0 || tile >= args.num_tiles)) {
            atomicCAS(status, 0, kDevBadTile);  // inconsistent response: stop scheduling
            tile = -1;
          }
          ptx::fence_proxy_async_smem();  // the response buffer is rewritten by the next request
        }
      }
      __syncwarp();
    }
  }

  if (warp == 5) {
    // ------------------------------------------------------------ TMA producer
    // The whole warp walks the tiles and waits (converged); one elected lane
    // issues the copies.
    if (lane == 0) tr.open(args, cluster_id == 0, static_cast<int>(rank) * 3 + 0);
    tr.rec(kEvStart, 0, 0);
    uint32_t kit = 0;
    bool ok = true;
    while (ok && src.next(t, lane == 0, true, status)) {
      int mt, nt;
      tile_coords(t, args, mt, nt);
      if (!dev_check(mt >= 0 && mt < args.num_m_tiles && nt >= 0 && nt < args.num_n_tiles, kChkTile, t)) {
        ok = false;
        break;
      }
      const int a_row = mt * (128 * kCtaGroup) + static_cast<int>(rank) * 128;
      const int b_row = nt * kTileN + static_cast<int>(rank) * C::kLoadN;
      const int sfa_blk = a_row / 128;
      const int sfb_blk = (nt * kTileN) / 128;
      for (int kb = 0; kb < args.num_k_blocks; ++kb, ++kit) {
        const int s = static_cast<int>(kit % kStages);
        const uint32_t round = kit / kStages;
        tr.rec(kEvProdWait, t, kb);
        if (!ptx::mbar_wait_warp<false, kLimit>(empty_bar(s), (round & 1u) ^ 1u, status, kDevTimeoutProducer)) {
          ok = false;
          break;
        }
        tr.rec(kEvProdGo, t, kb);
        const bool withheld = kFaultTest && kit == static_cast<uint32_t>(args.fault_withhold_kit);
        if (!withheld && ptx::elect_one()) {
          const uint64_t pol = ptx::policy_evict_normal();
          // L2 policy by reuse: inside a raster group the operand panels along the
          // group's short side are read by every wave of the group, those along the
          // walk by one wave only. Keeping the first and streaming the second
          // measured 4 % faster and 3.5 % less energy per GEMM at 16384^3 (1 % at
          // 8192 x 28672 x 8192) than one policy for both.
          const uint64_t pol_a = args.raster_along_n ? ptx::policy_evict_first() : ptx::policy_evict_last();
          const uint64_t pol_b = args.raster_along_n ? ptx::policy_evict_last() : ptx::policy_evict_first();
          if (leader) ptx::mbar_arrive_expect_tx(full_bar(s), C::kTxBytes);
          const uint32_t sa = smem + C::kOffA + s * C::kABytes;
          const uint32_t sb = smem + C::kOffB + s * C::kBBytes;
          const uint32_t ssfa = smem + C::kOffSFA + s * C::kSFABytes;
          const uint32_t ssfb = smem + C::kOffSFB + s * C::kSFBBytes;
          const int kx = kb * 128;
          if constexpr (kPair) {
            const uint32_t fb = ptx::mapa(full_bar(s), 0);
            ptx::tma_load_2d_pair(sa, &tmap_a, fb, kx, a_row, pol_a);
            ptx::tma_load_2d_pair(sb, &tmap_b, fb, kx, b_row, pol_b);
            ptx::tma_load_3d_pair(ssfa, &tmap_sfa, fb, 0, kb, sfa_blk, pol);
            ptx::tma_load_3d_pair(ssfb, &tmap_sfb, fb, 0, kb, sfb_blk, pol);
          } else {
            const uint32_t fb = full_bar(s);
            ptx::tma_load_2d(sa, &tmap_a, fb, kx, a_row, pol_a);
            ptx::tma_load_2d(sb, &tmap_b, fb, kx, b_row, pol_b);
            ptx::tma_load_3d(ssfa, &tmap_sfa, fb, 0, kb, sfa_blk, pol);
            ptx::tma_load_3d(ssfb, &tmap_sfb, fb, 0, kb, sfb_blk, pol);
          }
        }
        __syncwarp();
      }
    }
    // Drain: every stage this CTA filled has been consumed by the MMAs.
    for (int i = 0; ok && i < kStages; ++i) {
      const uint32_t k2 = kit + i;
      ok = ptx::mbar_wait_warp<false, kLimit>(empty_bar(static_cast<int>(k2 % kStages)), ((k2 / kStages) & 1u) ^ 1u,
                                              status, kDevTimeoutProducer);
    }
    if (!ok) settle_inflight_copies();
    tr.rec(kEvEnd, 0, 0);
    tr.close();
  } else if (warp == 4) {
    // ------------------------------------------------------------ MMA issuer
    // The whole warp walks the tiles and waits (converged); one elected lane
    // issues the tcgen05 operations. Issued from a lone-lane branch instead,
    // the SMEM->TMEM scale copies and the MMAs stop overlapping once the tensor
    // pipe has run empty (a wait at a tile boundary or for data), which cost
    // ~15 % of the tensor pipe.
    if (leader) {
      if (lane == 0) tr.open(args, cluster_id == 0, 1);
      tr.rec(kEvStart, 0, 0);
      uint32_t kit = 0;
      bool ok = true;
      int it = 0;
      for (; ok && src.next(t, lane == 0, true, status); ++it) {
        const int buf = it & 1;
        tr.rec(kEvMmaAccWait, t, 0);
        if constexpr (C::kOverlap) {
          if (it >= 1)
            ok = ptx::mbar_wait_warp<kPair, kLimit>(acc_empty_bar((it - 1) & 1), ((it - 1) >> 1) & 1, status,
                                                    kDevTimeoutAccEmpty);
        } else {
          if (it >= 2)
            ok = ptx::mbar_wait_warp<kPair, kLimit>(acc_empty_bar(buf), ((it - 2) >> 1) & 1, status,
                                                    kDevTimeoutAccEmpty);
        }
        if (!ok) break;
        tr.rec(kEvMmaAccGo, t, 0);
        ptx::tc_fence_after();
        const uint32_t d_t = tmem_base + (buf ? C::kAcc1Col : 0);
        if (!dev_check((buf ? C::kAcc1Col : 0) + kTileN <= C::kTmemCols, kChkTmemCols, buf ? C::kAcc1Col : 0)) {
          ok = false;
          break;
        }
        for (int kb = 0; kb < args.num_k_blocks; ++kb, ++kit) {
          const int s = static_cast<int>(kit % kStages);
          tr.rec(kEvMmaFullWait, t, kb);
          if (!ptx::mbar_wait_warp<false, kLimit>(full_bar(s), (kit / kStages) & 1u, status, kDevTimeoutMma)) {
            ok = false;
            break;
          }
          tr.rec(kEvMmaFullGo, t, kb);
          ptx::tc_fence_after();
          const uint32_t sf_off = static_cast<uint32_t>(kit % kSFBufs) * C::kSFBufCols;
          if (!dev_check(C::kSFBCol + sf_off + C::kSFBCols <= C::kTmemCols, kChkTmemCols, C::kSFBCol + sf_off)) {
            ok = false;
            break;
          }
          if (ptx::elect_one()) {
            const uint32_t sa = smem + C::kOffA + s * C::kABytes;
            const uint32_t sb = smem + C::kOffB + s * C::kBBytes;
            const uint32_t ssfa = smem + C::kOffSFA + s * C::kSFABytes;
            const uint32_t ssfb = smem + C::kOffSFB + s * C::kSFBBytes;
            const uint32_t sfa_t = tmem_base + C::kSFACol + sf_off;
            const uint32_t sfb_t = tmem_base + C::kSFBCol + sf_off;
            ptx::tmem_cp_32x128b_x4<kCtaGroup>(sfa_t, ptx::sf_chunk_desc(ssfa));
#pragma unroll
            for (int h = 0; h < kTileN / 128; ++h)
              ptx::tmem_cp_32x128b_x4<kCtaGroup>(sfb_t + 4 * h, ptx::sf_chunk_desc(ssfb + 512 * h));
            const uint64_t a_desc = ptx::kmajor_sw128_desc(sa);
            const uint64_t b_desc = ptx::kmajor_sw128_desc(sb);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              // Advance 32 bytes (one K=32 slice) inside the 128-byte swizzled rows.
              ptx::mma_mxf8f6f4<kCtaGroup>(d_t, a_desc + 2 * j, b_desc + 2 * j,
                                           ptx::with_scale_id(C::kIdesc, j),
                                           sfa_t | (static_cast<uint32_t>(j) << 30),
                                           sfb_t | (static_cast<uint32_t>(j) << 30),
                                           (kb | j) != 0 ? 1u : 0u);
            }
            ptx::tc_commit<kCtaGroup>(empty_bar(s));
            if constexpr (kPair) ptx::tc_commit<kCtaGroup>(ptx::mapa(empty_bar(s), 1));
          }
          __syncwarp();
          tr.rec(kEvMmaIssued, t, kb);
        }
        if (!ok) break;
        if (ptx::elect_one()) {
          ptx::tc_commit<kCtaGroup>(acc_full_bar(buf));
          if constexpr (kPair) ptx::tc_commit<kCtaGroup>(ptx::mapa(acc_full_bar(buf), 1));
        }
        __syncwarp();
        tr.rec(kEvMmaTileDone, t, 0);
      }
      tr.rec(kEvEnd, 0, 0);
      tr.close();
    }
    __syncwarp();
  } else if (warp < 4) {
    // ------------------------------------------------------------ epilogue (warps 0-3 only;
    // warp 6, the scheduler of the dynamic build, has no TMEM lane quarter)
    const uint32_t cbuf = smem + C::kOffC + warp * kEpiBufs * C::kCBufBytes;
    uint32_t chunk_ctr = 0;
    int it = 0;
    if (warp == 0 && lane == 0) tr.open(args, cluster_id == 0, static_cast<int>(rank) * 3 + 2);
    tr.rec(kEvStart, 0, 0);
    for (; src.next(t, lane == 0, true, status); ++it) {
      int mt, nt;
      tile_coords(t, args, mt, nt);
      if (!dev_check(mt >= 0 && mt < args.num_m_tiles && nt >= 0 && nt < args.num_n_tiles, kChkTile, t)) break;
      const int m_row = mt * (128 * kCtaGroup) + static_cast<int>(rank) * 128 + warp * 32;
      const int n_col = nt * kTileN;
      const int buf = it & 1;
      tr.rec(kEvEpiWait, t, 0);
      if (!ptx::mbar_wait<false, kLimit>(acc_full_bar(buf), (it >> 1) & 1, status, kDevTimeoutEpilogue)) break;
      const unsigned long long t_go = tr.stamp();
      unsigned long long t_loaded = 0;
      ptx::tc_fence_after();
      const uint32_t acc = tmem_base + (static_cast<uint32_t>(warp * 32) << 16) +
                           static_cast<uint32_t>(buf ? C::kAcc1Col : 0);
      const int first = buf == 0 ? C::kFirstChunk0 : 0;
      bool chunks_ok = true;
#pragma unroll 1
      for (int i = 0; i < C::kChunks; ++i) {
        const int c = (first + i) % C::kChunks;
        // Checked builds: the chunk's TMEM columns, and the store's origin inside
        // D's padded extent (a TMA store may not start at a negative coordinate).
        if (!dev_check((buf ? C::kAcc1Col : 0) + c * 64 + 64 <= C::kTmemCols, kChkTmemCols,
                       (buf ? C::kAcc1Col : 0) + c * 64) ||
            !dev_check(m_row >= 0 && m_row < args.num_m_tiles * 128 * kCtaGroup && n_col + c * 64 >= 0 &&
                           n_col + c * 64 < args.num_n_tiles * kTileN,
                       kChkStore, (static_cast<long long>(m_row) << 32) | static_cast<uint32_t>(n_col + c * 64))) {
          chunks_ok = false;
          break;
        }
        uint32_t v0[32], v1[32];
        ptx::tmem_ld_32x32b_x32(acc + c * 64, v0);
        ptx::tmem_ld_32x32b_x32(acc + c * 64 + 32, v1);
        ptx::tmem_wait_ld();
        const bool release = C::kOverlap ? (i == 0) : (i == C::kChunks - 1);
        if (i == 0) t_loaded = tr.stamp();
        if (release) {
          ptx::tc_fence_before();
          __syncwarp();
          if (lane == 0) {
            // The accumulator columns were read (wait::ld) and fenced; the
            // barrier publishes no memory data, so a CTA-scope release suffices.
            if constexpr (kPair) ptx::mbar_arrive_cluster_cta_release(ptx::mapa(acc_empty_bar(buf), 0));
            else ptx::mbar_arrive(acc_empty_bar(buf));
          }
          const unsigned long long t_rel = tr.stamp();
          tr.rec_at(kEvEpiGo, t_go, t, 0);
          tr.rec_at(kEvEpiLoaded, t_loaded, t, 0);
          tr.rec_at(kEvEpiRelease, t_rel, t, 0);
        }
        const uint32_t slot = chunk_ctr % kEpiBufs;
        if constexpr (kEpi == 1 || kEpi == 2)
          epilogue_affine(v0, v1, args, m_row + static_cast<int>(lane), n_col + c * 64);
        if (chunk_ctr >= static_cast<uint32_t>(kEpiBufs)) {
          if (lane == 0) ptx::bulk_wait_group_read<kEpiBufs - 1>();
          __syncwarp();
        }
        if constexpr (kEpi == 2) {
          // E4M3 row of 64 bytes, 64-byte swizzle (16-byte chunk ^ (row >> 1) & 3),
          // and the two scale bytes of its 1x32 blocks (one 16-bit store).
          uint32_t w0[8], w1[8];
          const uint32_t s0 = quantize_block32(v0, w0);
          const uint32_t s1 = quantize_block32(v1, w1);
          const uint32_t row_addr = cbuf + slot * C::kCBufBytes + lane * 64u;
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const uint32_t* w = q < 2 ? &w0[4 * q] : &w1[4 * (q - 2)];
            st_shared_v4(row_addr + ((static_cast<uint32_t>(q) ^ ((lane >> 1) & 3u)) << 4), w[0], w[1], w[2], w[3]);
          }
          const int row = m_row + static_cast<int>(lane);
          const int n0 = n_col + c * 64;
          if (row < ((args.M + 127) & ~127) && n0 < args.N) {
            const bool real = row < args.M;  // padding rows of the scale layout: 0x00
            const int64_t off = sf_offset(row, n0 >> 5, args.N);
            if (dev_check(off >= 0 && off + 2 <= static_cast<int64_t>((args.M + 127) & ~127) * (args.N >> 5),
                          kChkScaleOffset, off))
              *reinterpret_cast<uint16_t*>(args.d_scales + off) = static_cast<uint16_t>(real ? (s0 | (s1 << 8)) : 0u);
          }
        } else {
          const uint32_t row_addr = cbuf + slot * C::kCBufBytes + lane * 128u;
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const uint32_t* src = j < 4 ? &v0[j * 8] : &v1[(j - 4) * 8];
            st_shared_v4(row_addr + ((static_cast<uint32_t>(j) ^ (lane & 7u)) << 4),
                         pack_bf16x2(src[0], src[1]), pack_bf16x2(src[2], src[3]),
                         pack_bf16x2(src[4], src[5]), pack_bf16x2(src[6], src[7]));
          }
        }
        ptx::fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          // D is written once and not read by this kernel: evict-first keeps the
          // operand panels the raster group reuses in L2 (measured 1-3 % faster and
          // 1-4 % less energy per GEMM at 16384^3 and 8192 x 28672 x 8192).
          ptx::tma_store_2d_hint(&tmap_d, cbuf + slot * C::kCBufBytes, n_col + c * 64, m_row,
                                 ptx::policy_evict_first());
          if constexpr (kEpi == 3) {
            for (int p = 0; p < args.num_peers; ++p)
              ptx::tma_store_2d(args.peer_maps + p, cbuf + slot * C::kCBufBytes, n_col + c * 64, m_row);
          }
          ptx::bulk_commit_group();
        }
        ++chunk_ctr;
      }
      if (!chunks_ok) break;
      tr.rec(kEvEpiTileDone, t, 0);
    }
    if (lane == 0) ptx::bulk_wait_group_all();
    __syncwarp();
    tr.rec(kEvEnd, 0, 0);
    tr.close();
  }

  // ------------------------------------------------------------ teardown
  ptx::tc_fence_before();
  if constexpr (kPair) ptx::cluster_sync(); else __syncthreads();
  if (threadIdx.x == 0) trace_cta_time<kTrace>(args, 1);
  if (warp == 4) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc<kCtaGroup>(tmem_base, C::kTmemCols);
  }
}

}  // namespace cutex
