// Skinny MXFP8 GEMM (M <= 128): HBM-bound streaming of B with swapped operands.
//
//   D[M,N] = A[M,K] . B[N,K]^T  is computed as  D^T[N,M] = B . A^T :
//   the MMA's 128-row side walks 128-row tiles of B (N), its N side is the
//   padded M (kNPad = 16..128). B is read once from HBM (evict-first), A and its
//   scales stay L2-resident (evict-last) and are re-read per K-stage.
//
// Work split: the first dp_tiles tiles go whole, round-robin over the grid
// (data-parallel waves); the (N-tile, K-stage) units of the remaining tiles are
// cut into gridDim.x equal contiguous ranges, one per CTA (stream-K), so every
// SM streams the same number of bytes. dp_tiles = 0 is pure stream-K,
// dp_tiles = all tiles is pure data-parallel. A CTA that covers a whole tile
// writes BF16 D directly. A tile cut between CTAs is finished through a
// workspace: each contributor stores its FP32 partial in its own slot, then
// increments the tile's arrival counter; the contributor that arrives last sums
// all partials in contributor order (deterministic), writes D, and resets the
// counter to zero for the next call. Nobody waits for another CTA.
//
// A CTA tile is kTiles x 128 rows of B (kTiles = 2: two MMAs per K-step share
// the A stage, which halves A's L2 traffic and leaves more of the stage ring to
// B). A partial slot holds all kTiles 128-row tiles of a CTA tile.
//
// Warp roles (192 threads) as in the large kernel: warps 0-3 epilogue (TMEM lane
// quarter w = rows 32w..32w+31 of each 128-row B tile), warp 4 MMA issuer,
// warp 5 TMA. TMEM: one or two accumulators of kTiles x kNPad columns (two when
// they fit beside the scales, alternating by segment) + scale columns (MMA-A
// scales = B's chunks, MMA-B scales = A's chunk) in two buffers.
#pragma once

#include <cuda_bf16.h>

#include "mxfp8_gemm.cuh"
#include "ptx.cuh"

namespace cutex {

struct SkinnyArgs {
  int M;              // rows of A (<= kNPad)
  int N;              // rows of B
  int num_n_tiles;    // ceil(N / 128)
  int num_k_blocks;   // K / 128
  long long units;    // stream-K units: (num_n_tiles - dp_tiles) * num_k_blocks
  int streamk;        // 1: stream-K over the tiles from dp_tiles on; 0: whole tiles round-robin
  int dp_tiles;       // tiles [0, dp_tiles) whole, round-robin (stream-K mode)
  long long ldd;      // row stride of D (elements)
  __nv_bfloat16* d;
  float* partials;    // [2 * gridDim.x][kTiles][kNPad][128] fp32 slots (stream-K only)
  unsigned int* counters;  // [num_n_tiles] arrival counters, zero between calls
};

template <int kNPad, int kStages, int kTiles = 1>
struct SkinnyCfg {
  static constexpr int kBBytes = kTiles * 128 * 128;  // kTiles 128-row x 128-K tiles of B
  static constexpr int kABytes = kNPad * 128;          // kNPad rows of A
  static constexpr int kSFBBytes = kTiles * 512;
  static constexpr int kStageBytes = kBBytes + kABytes + kSFBBytes + 512;
  static constexpr int kOffB = 0;
  static constexpr int kOffA = kOffB + kStages * kBBytes;
  static constexpr int kOffSFB = kOffA + kStages * kABytes;  // B's scale chunks (MMA A side)
  static constexpr int kOffSFA = kOffSFB + kStages * kSFBBytes;  // A's scale chunk (MMA B side)
  // D staging: per epilogue warp kEpiBufs boxes of [32 rows m][32 columns n] bf16.
  static constexpr int kEpiBufs = kNPad > 32 ? 2 : 1;
  static constexpr int kDBoxBytes = 32 * 32 * 2;
  static constexpr int kOffD = kOffSFA + kStages * 512;
  static constexpr int kOffBar = align_up(kOffD + 4 * kEpiBufs * kDBoxBytes, 8);
  static constexpr int kNumBars = 2 * kStages + 4;
  static constexpr int kOffSlot = kOffBar + kNumBars * 8;  // TMEM address + last-arrival flag
  static constexpr int kSmemBytes = kOffSlot + 16 + 1024;
  static constexpr int kTmemCols = 512;
  static constexpr int kAccCols = kTiles * kNPad;
  static constexpr int kSFBufCols = 16;  // [B chunks 4 * kTiles | A chunk 4]
  static constexpr int kAccBufs = 2 * kAccCols + 2 * kSFBufCols <= kTmemCols ? 2 : 1;
  static constexpr int kAcc1Col = kAccCols;
  static constexpr int kSFCol = kAccBufs * kAccCols;  // two buffers of kSFBufCols columns
  static constexpr uint32_t kTxBytes = kStageBytes;
  static constexpr uint32_t kIdesc = ptx::mxf8_idesc(128, kNPad);
  static_assert(kNPad % 16 == 0 && kNPad >= 16 && kNPad <= 128, "padded M");
  static_assert(kTiles == 1 || kTiles == 2, "B tiles per CTA tile");
  static_assert(4 * kTiles + 4 <= kSFBufCols, "scale columns");
  static_assert(kSFCol + 2 * kSFBufCols <= kTmemCols, "TMEM plan");
  static_assert(kSmemBytes <= kSmemLimit, "shared memory budget");
};

// Converts kCnt values of this thread's D column n (rows m0 .. m0 + kCnt - 1) to
// bf16 in the warp's next [32 m][32 n] staging box, then lane 0 stores the box
// at (n0 of the warp, m0) with TMA; rows and columns outside D are clipped by
// the tensor map. The box is reused once its previous store has read it.
template <int kCnt, int kEpiBufs>
__device__ __forceinline__ void skinny_emit(const float (&v)[kCnt], __nv_bfloat16* stage, uint32_t stage_addr,
                                            int& buf, uint32_t lane, const CUtensorMap* tmap_d, int n0, int m0) {
  static_assert(kCnt == 16 || kCnt == 32, "rows per box");
  if (lane == 0) ptx::bulk_wait_group_read<kEpiBufs - 1>();
  __syncwarp();
  __nv_bfloat16* box = stage + buf * 32 * 32;
#pragma unroll
  for (int j = 0; j < kCnt; ++j) box[j * 32 + lane] = __float2bfloat16_rn(v[j]);
  ptx::fence_proxy_async_smem();
  __syncwarp();
  if (lane == 0) {
    ptx::tma_store_2d(tmap_d, stage_addr + static_cast<uint32_t>(buf) * 2048u, n0, m0);
    ptx::bulk_commit_group();
  }
  buf = (buf + 1) % kEpiBufs;
}

// Units [start(c), start(c+1)) of CTA c.
__device__ __forceinline__ long long sk_start(long long c, long long P, long long U) {
  return c * U / P;
}

// CTA whose range holds unit u: the largest c with start(c) <= u.
__device__ __forceinline__ long long sk_owner(long long u, long long P, long long U) {
  return ((u + 1) * P - 1) / U;
}

// Walks a CTA's segments: (tile, first K-stage, end K-stage) in order; whole
// round-robin tiles first, then the CTA's stream-K range.
struct SegmentWalker {
  long long u, u_end;  // stream-K units (relative to tile dp_tiles)
  int tile_rr;         // next round-robin tile
  int rr_end;          // round-robin tiles end here
  __device__ __forceinline__ void init(const SkinnyArgs& a) {
    tile_rr = blockIdx.x;
    if (a.streamk) {
      rr_end = a.dp_tiles;
      u = sk_start(blockIdx.x, gridDim.x, a.units);
      u_end = sk_start(blockIdx.x + 1, gridDim.x, a.units);
    } else {
      rr_end = a.num_n_tiles;
      u = 0;
      u_end = 0;
    }
  }
  __device__ __forceinline__ bool next(const SkinnyArgs& a, int& tile, int& kb0, int& kb1) {
    if (tile_rr < rr_end) {
      tile = tile_rr;
      tile_rr += gridDim.x;
      kb0 = 0;
      kb1 = a.num_k_blocks;
      return true;
    }
    if (u >= u_end) return false;
    const int rel = static_cast<int>(u / a.num_k_blocks);
    tile = a.dp_tiles + rel;
    kb0 = static_cast<int>(u - static_cast<long long>(rel) * a.num_k_blocks);
    const long long left = u_end - u;
    kb1 = static_cast<int>(min(static_cast<long long>(a.num_k_blocks), kb0 + left));
    u += kb1 - kb0;
    return true;
  }
};

template <int kNPad, int kStages, int kTiles = 1>
__global__ void __launch_bounds__(192, 1)
    mxfp8_skinny_kernel(const __grid_constant__ CUtensorMap tmap_b,
                        const __grid_constant__ CUtensorMap tmap_a,
                        const __grid_constant__ CUtensorMap tmap_sfb,
                        const __grid_constant__ CUtensorMap tmap_sfa,
                        const __grid_constant__ CUtensorMap tmap_d, const SkinnyArgs args) {
  using C = SkinnyCfg<kNPad, kStages, kTiles>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_base = ptx::smem_u32(smem_raw);
  const uint32_t smem = (raw_base + 1023u) & ~1023u;
  uint8_t* smem_ptr = smem_raw + (smem - raw_base);
  const int warp = threadIdx.x >> 5;
  const uint32_t lane = ptx::lane_id();
  int* status = &g_cutex_device_status;

  const uint32_t bar0 = smem + C::kOffBar;
  auto full_bar = [&](int s) { return bar0 + 8u * s; };
  auto empty_bar = [&](int s) { return bar0 + 8u * (kStages + s); };
  auto acc_full_bar = [&](int b) { return bar0 + 8u * (2 * kStages + b); };
  auto acc_empty_bar = [&](int b) { return bar0 + 8u * (2 * kStages + 2 + b); };
  volatile uint32_t* slot = reinterpret_cast<volatile uint32_t*>(smem_ptr + C::kOffSlot);

  if (warp == 5 && lane == 0) {
    ptx::prefetch_tmap(&tmap_b);
    ptx::prefetch_tmap(&tmap_a);
    ptx::prefetch_tmap(&tmap_sfb);
    ptx::prefetch_tmap(&tmap_sfa);
    for (int s = 0; s < kStages; ++s) {
      ptx::mbar_init(full_bar(s), 1);
      ptx::mbar_init(empty_bar(s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      ptx::mbar_init(acc_full_bar(b), 1);
      ptx::mbar_init(acc_empty_bar(b), 4);
    }
    ptx::fence_mbar_init();
  }
  if (warp == 4) {
    ptx::tmem_alloc<1>(ptx::smem_u32(const_cast<uint32_t*>(slot)), C::kTmemCols);
    ptx::tmem_relinquish<1>();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem_base = slot[0];
  // Launched with programmatic stream serialization: the set-up above may
  // overlap the end of the previous kernel in the stream; no global memory is
  // touched before that kernel has completed. The next launch of this kernel
  // may be scheduled from here on (its CTAs take SMs as these CTAs exit).
  ptx::grid_dependency_wait();
  ptx::launch_dependents();

  SegmentWalker walk;
  walk.init(args);
  int tile, kb0, kb1;

  if (warp == 5) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      const uint64_t stream_pol = ptx::policy_evict_first();
      const uint64_t keep_pol = ptx::policy_evict_last();
      uint32_t kit = 0;
      bool ok = true;
      while (ok && walk.next(args, tile, kb0, kb1)) {
        if (!dev_check(tile >= 0 && tile < args.num_n_tiles && kb0 >= 0 && kb0 < kb1 && kb1 <= args.num_k_blocks,
                       kChkSkinnySegment, (static_cast<long long>(tile) << 32) | static_cast<uint32_t>(kb0))) {
          ok = false;
          break;
        }
        for (int kb = kb0; kb < kb1; ++kb, ++kit) {
          const int s = static_cast<int>(kit % kStages);
          if (!ptx::mbar_wait(empty_bar(s), ((kit / kStages) & 1u) ^ 1u, status, kDevTimeoutProducer)) {
            ok = false;
            break;
          }
          const uint32_t fb = full_bar(s);
          ptx::mbar_arrive_expect_tx(fb, C::kTxBytes);
          ptx::tma_load_2d(smem + C::kOffB + s * C::kBBytes, &tmap_b, fb, kb * 128, tile * 128 * kTiles,
                           stream_pol);
          ptx::tma_load_2d(smem + C::kOffA + s * C::kABytes, &tmap_a, fb, kb * 128, 0, keep_pol);
          ptx::tma_load_3d(smem + C::kOffSFB + s * C::kSFBBytes, &tmap_sfb, fb, 0, kb, tile * kTiles, stream_pol);
          ptx::tma_load_3d(smem + C::kOffSFA + s * 512, &tmap_sfa, fb, 0, kb, 0, keep_pol);
        }
      }
      for (int i = 0; ok && i < kStages; ++i) {
        const uint32_t k2 = kit + i;
        ok = ptx::mbar_wait(empty_bar(static_cast<int>(k2 % kStages)), ((k2 / kStages) & 1u) ^ 1u, status,
                            kDevTimeoutProducer);
      }
      if (!ok) settle_inflight_copies();
    }
    __syncwarp();
  } else if (warp == 4) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      uint32_t kit = 0;
      int seg = 0;
      bool ok = true;
      while (ok && walk.next(args, tile, kb0, kb1)) {
        // Accumulator buffer `buf` is used for the use-th time by this segment.
        const int buf = seg % C::kAccBufs, use = seg / C::kAccBufs;
        if (use >= 1 &&
            !ptx::mbar_wait(acc_empty_bar(buf), (use - 1) & 1, status, kDevTimeoutAccEmpty))
          break;
        ptx::tc_fence_after();
        const uint32_t d_t = tmem_base + (buf ? C::kAcc1Col : 0);
        if (!dev_check((buf ? C::kAcc1Col : 0) + C::kAccCols <= C::kSFCol, kChkTmemCols, buf ? C::kAcc1Col : 0)) break;
        for (int kb = kb0; kb < kb1; ++kb, ++kit) {
          const int s = static_cast<int>(kit % kStages);
          if (!ptx::mbar_wait(full_bar(s), (kit / kStages) & 1u, status, kDevTimeoutMma)) {
            ok = false;
            break;
          }
          ptx::tc_fence_after();
          // Scale buffer: [B tile chunks 4 * kTiles columns | A chunk 4 columns].
          if (!dev_check(C::kSFCol + (kit & 1u) * C::kSFBufCols + C::kSFBufCols <= C::kTmemCols, kChkTmemCols,
                         C::kSFCol + (kit & 1u) * C::kSFBufCols)) {
            ok = false;
            break;
          }
          const uint32_t sf_t = tmem_base + C::kSFCol + (kit & 1u) * C::kSFBufCols;
          const uint32_t sfa_t = sf_t + 4 * kTiles;
#pragma unroll
          for (int t = 0; t < kTiles; ++t)
            ptx::tmem_cp_32x128b_x4<1>(sf_t + 4 * t, ptx::sf_chunk_desc(smem + C::kOffSFB + s * C::kSFBBytes + 512 * t));
          ptx::tmem_cp_32x128b_x4<1>(sfa_t, ptx::sf_chunk_desc(smem + C::kOffSFA + s * 512));
          const uint64_t b_desc = ptx::kmajor_sw128_desc(smem + C::kOffA + s * C::kABytes);
#pragma unroll
          for (int t = 0; t < kTiles; ++t) {
            const uint64_t a_desc = ptx::kmajor_sw128_desc(smem + C::kOffB + s * C::kBBytes + t * 128 * 128);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              ptx::mma_mxf8f6f4<1>(d_t + t * kNPad, a_desc + 2 * j, b_desc + 2 * j, ptx::with_scale_id(C::kIdesc, j),
                                   (sf_t + 4 * t) | (static_cast<uint32_t>(j) << 30),
                                   sfa_t | (static_cast<uint32_t>(j) << 30), (kb != kb0 || j != 0) ? 1u : 0u);
            }
          }
          ptx::tc_commit<1>(empty_bar(s));
        }
        if (!ok) break;
        ptx::tc_commit<1>(acc_full_bar(buf));
        ++seg;
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue
    const int P = gridDim.x;
    const long long U = args.units;
    const int first_tile =
        args.streamk ? args.dp_tiles + static_cast<int>(sk_start(blockIdx.x, P, U) / args.num_k_blocks) : -1;
    const uint32_t tid = threadIdx.x;  // 0..127: row of the B tile = column of D
    const uint32_t dstage_addr = smem + C::kOffD + static_cast<uint32_t>(warp) * C::kEpiBufs * C::kDBoxBytes;
    __nv_bfloat16* dstage = reinterpret_cast<__nv_bfloat16*>(smem_ptr + C::kOffD + warp * C::kEpiBufs * C::kDBoxBytes);
    int dbuf = 0;
    int seg = 0;
    while (walk.next(args, tile, kb0, kb1)) {
      const int buf = seg % C::kAccBufs, use = seg / C::kAccBufs;
      if (!ptx::mbar_wait(acc_full_bar(buf), use & 1, status, kDevTimeoutEpilogue)) break;
      ptx::tc_fence_after();
      const uint32_t acc = tmem_base + (static_cast<uint32_t>(warp * 32) << 16) +
                           static_cast<uint32_t>(buf ? C::kAcc1Col : 0);
      const bool whole = kb0 == 0 && kb1 == args.num_k_blocks;
      const int n0w = tile * kTiles * 128 + warp * 32;  // first D column of this warp's boxes
      // A tile cut between CTAs: the contributors of its K-range and whether all
      // the others have already published their slots. If so this CTA is the
      // last: it sums their slots with its own accumulator read straight from
      // TMEM (no slot of its own, no second pass over global memory), writes D
      // and resets the counter. The sum runs in contributor order either way,
      // so the result does not depend on which contributor finishes last.
      int c0 = 0, c1 = 0;
      bool early_last = false;
      if (!whole) {
        const long long t_u0 = static_cast<long long>(tile - args.dp_tiles) * args.num_k_blocks;
        c0 = static_cast<int>(sk_owner(t_u0, P, U));
        c1 = static_cast<int>(sk_owner(t_u0 + args.num_k_blocks - 1, P, U));
        // Checked builds: the counter and every contributor's slot (2 c or 2 c + 1,
        // c in [c0, c1]) inside the workspace. The same values in all 128
        // threads, so the epilogue warps leave together, before any named barrier.
        if (!dev_check(tile >= args.dp_tiles && tile < args.num_n_tiles && c0 >= 0 && c0 <= c1 && c1 < P &&
                           c0 <= static_cast<int>(blockIdx.x) && static_cast<int>(blockIdx.x) <= c1,
                       kChkWorkspace, (static_cast<long long>(c0) << 32) | static_cast<uint32_t>(c1)))
          break;
        if (tid == 0) {
          unsigned int done;
          asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(done) : "l"(args.counters + tile) : "memory");
          slot[1] = done == static_cast<unsigned int>(c1 - c0) ? 1u : 0u;
        }
        ptx::named_barrier(1, 128);
        early_last = slot[1] != 0u;
      }
      // Contributor cc's slot, 128-row tile t of it: [kNPad / 4][128 rows][4 columns] fp32.
      auto slot_of = [&](int cc, int t) {
        const int ft = args.dp_tiles + static_cast<int>(sk_start(cc, P, U) / args.num_k_blocks);
        const int s = (ft == tile) ? 2 * cc : 2 * cc + 1;
        return reinterpret_cast<const float4*>(args.partials + (static_cast<size_t>(s) * kTiles + t) * kNPad * 128);
      };
      constexpr int kPass = kNPad < 64 ? kNPad : 64;  // columns per reduction pass
      constexpr int kQ = kPass / 4;                    // float4 per thread per pass
      auto store_row = [&](const float4 (&sum)[kQ], int c, int t) {
        if constexpr (kPass == 16) {
          float f[16];
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            f[4 * q] = sum[q].x; f[4 * q + 1] = sum[q].y; f[4 * q + 2] = sum[q].z; f[4 * q + 3] = sum[q].w;
          }
          skinny_emit<16, C::kEpiBufs>(f, dstage, dstage_addr, dbuf, lane, &tmap_d, n0w + t * 128, c);
        } else {
#pragma unroll
          for (int h = 0; h < kPass / 32; ++h) {
            float f[32];
#pragma unroll
            for (int q = 0; q < 8; ++q) {
              const float4 x = sum[8 * h + q];
              f[4 * q] = x.x; f[4 * q + 1] = x.y; f[4 * q + 2] = x.z; f[4 * q + 3] = x.w;
            }
            skinny_emit<32, C::kEpiBufs>(f, dstage, dstage_addr, dbuf, lane, &tmap_d, n0w + t * 128, c + 32 * h);
          }
        }
      };
      if (early_last) {
        __threadfence();
        const int nc = c1 - c0 + 1;
#pragma unroll 1
        for (int t = 0; t < kTiles; ++t) {
#pragma unroll 1
          for (int c = 0; c < kNPad; c += kPass) {
            float4 sum[kQ];
#pragma unroll
            for (int q = 0; q < kQ; ++q) sum[q] = make_float4(0.f, 0.f, 0.f, 0.f);
            for (int i = 0; i < nc; ++i) {
              float4 x[kQ];
              if (c0 + i == static_cast<int>(blockIdx.x)) {
#pragma unroll
                for (int h = 0; h < kPass / 16; ++h) {
                  uint32_t v[16];
                  ptx::tmem_ld_32x32b_x16(acc + t * kNPad + c + 16 * h, v);
                  ptx::tmem_wait_ld();
#pragma unroll
                  for (int q = 0; q < 4; ++q)
                    x[4 * h + q] = make_float4(__uint_as_float(v[4 * q]), __uint_as_float(v[4 * q + 1]),
                                               __uint_as_float(v[4 * q + 2]), __uint_as_float(v[4 * q + 3]));
                }
              } else {
                const float4* sx = slot_of(c0 + i, t);
#pragma unroll
                for (int q = 0; q < kQ; ++q) x[q] = __ldcg(sx + (c / 4 + q) * 128 + tid);
              }
#pragma unroll
              for (int q = 0; q < kQ; ++q) {
                sum[q].x += x[q].x; sum[q].y += x[q].y; sum[q].z += x[q].z; sum[q].w += x[q].w;
              }
            }
            store_row(sum, c, t);
          }
        }
        ptx::tc_fence_before();
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive(acc_empty_bar(buf));
        if (tid == 0) args.counters[tile] = 0u;
        ptx::named_barrier(1, 128);
        ++seg;
        continue;
      }
      float* part = nullptr;
      if (!whole) {
        const int s = (tile == first_tile) ? 2 * blockIdx.x : 2 * blockIdx.x + 1;
        part = args.partials + static_cast<size_t>(s) * kTiles * kNPad * 128;
      }
#pragma unroll 1
      for (int t = 0; t < kTiles; ++t) {
        if (whole) {
          if constexpr (kNPad == 16) {
            uint32_t v[16];
            ptx::tmem_ld_32x32b_x16(acc + t * kNPad, v);
            ptx::tmem_wait_ld();
            float f[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) f[j] = __uint_as_float(v[j]);
            skinny_emit<16, C::kEpiBufs>(f, dstage, dstage_addr, dbuf, lane, &tmap_d, n0w + t * 128, 0);
          } else {
#pragma unroll 1
            for (int c = 0; c < kNPad; c += 32) {
              uint32_t v[32];
              ptx::tmem_ld_32x32b_x32(acc + t * kNPad + c, v);
              ptx::tmem_wait_ld();
              float f[32];
#pragma unroll
              for (int j = 0; j < 32; ++j) f[j] = __uint_as_float(v[j]);
              skinny_emit<32, C::kEpiBufs>(f, dstage, dstage_addr, dbuf, lane, &tmap_d, n0w + t * 128, c);
            }
          }
          continue;
        }
#pragma unroll 1
        for (int c = 0; c < kNPad; c += 16) {
          uint32_t v[16];
          ptx::tmem_ld_32x32b_x16(acc + t * kNPad + c, v);
          ptx::tmem_wait_ld();
          // Slot layout per 128-row tile [kNPad / 4][128 rows][4 columns]: one 16-byte
          // store per thread and column group, 512 contiguous bytes per warp.
          float4* part4 = reinterpret_cast<float4*>(part + static_cast<size_t>(t) * kNPad * 128);
#pragma unroll
          for (int q = 0; q < 4; ++q)
            part4[(c / 4 + q) * 128 + tid] =
                make_float4(__uint_as_float(v[4 * q]), __uint_as_float(v[4 * q + 1]), __uint_as_float(v[4 * q + 2]),
                            __uint_as_float(v[4 * q + 3]));
        }
      }
      ptx::tc_fence_before();
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(acc_empty_bar(buf));
      if (!whole) {
        // Publish the slot, count arrivals; the contributor that arrives last sums.
        __threadfence();
        ptx::named_barrier(1, 128);
        if (tid == 0) {
          const unsigned int prev = atomicAdd(&args.counters[tile], 1u);
          slot[1] = (prev == static_cast<unsigned int>(c1 - c0)) ? 1u : 0u;
        }
        ptx::named_barrier(1, 128);
        if (slot[1] != 0u) {
          __threadfence();
          // Contributor order, two contributors' loads (2 x 16 float4 per thread)
          // in flight per step: the loop is latency-bound.
          const int nc = c1 - c0 + 1;
#pragma unroll 1
          for (int tc = 0; tc < kTiles * kNPad; tc += kPass) {
            const int t = tc / kNPad, c = tc % kNPad;  // kPass divides kNPad
            float4 sum[kQ];
#pragma unroll
            for (int q = 0; q < kQ; ++q) sum[q] = make_float4(0.f, 0.f, 0.f, 0.f);
            int i = 0;
            for (; i + 1 < nc; i += 2) {
              const float4* sx = slot_of(c0 + i, t);
              const float4* sy = slot_of(c0 + i + 1, t);
              float4 x[kQ], y[kQ];
#pragma unroll
              for (int q = 0; q < kQ; ++q) x[q] = __ldcg(sx + (c / 4 + q) * 128 + tid);
#pragma unroll
              for (int q = 0; q < kQ; ++q) y[q] = __ldcg(sy + (c / 4 + q) * 128 + tid);
#pragma unroll
              for (int q = 0; q < kQ; ++q) {
                sum[q].x += x[q].x; sum[q].y += x[q].y; sum[q].z += x[q].z; sum[q].w += x[q].w;
                sum[q].x += y[q].x; sum[q].y += y[q].y; sum[q].z += y[q].z; sum[q].w += y[q].w;
              }
            }
            if (i < nc) {
              const float4* sx = slot_of(c0 + i, t);
              float4 x[kQ];
#pragma unroll
              for (int q = 0; q < kQ; ++q) x[q] = __ldcg(sx + (c / 4 + q) * 128 + tid);
#pragma unroll
              for (int q = 0; q < kQ; ++q) {
                sum[q].x += x[q].x; sum[q].y += x[q].y; sum[q].z += x[q].z; sum[q].w += x[q].w;
              }
            }
            store_row(sum, c, t);
          }
          if (tid == 0) args.counters[tile] = 0u;
        }
        ptx::named_barrier(1, 128);
      }
      ++seg;
    }
    if (lane == 0) ptx::bulk_wait_group_all();  // D stores complete before the CTA exits
  }

  ptx::tc_fence_before();
  __syncthreads();
  if (warp == 4) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc<1>(tmem_base, C::kTmemCols);
  }
}

}  // namespace cutex
