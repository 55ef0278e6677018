// Columnwise MXFP8 quantiser: the operand layout a GEMM needs when the
// reduction runs over the rows of x (weight gradients reduce over tokens; input
// gradients read W along its columns). For x[rows, cols] it writes
// qt[cols, rows] = quantise(x^T): the 1x32 blocks run down the columns of x, and
// the scales land in the 128x4 swizzled layout of a [cols, K = rows] operand.
// Same per-block rule as the rowwise kernel (mxfp8_quant.cuh).
//
// Persistent CTAs (one wave) walk 128-row x kCols-column tiles of x (in
// groups of kGroupRows row tiles, row tile fastest inside a group; kCols = 64
// for fp32, 128 for bf16, so both read 256-byte row segments and 32 KB tiles). TMA brings each tile into a kStages-deep ring in
// shared memory (dense rows; columns past `cols` read as zero), so kStages - 1
// tiles are in flight while one is quantised and no registers hold loads. The
// CTA has 4 kCols threads; warp w takes 32-row block w % 4 of tile columns
// 32 (w / 4) .. + 31: one lane per column (consecutive lanes read consecutive
// elements of a row: no bank conflicts), and each lane holds a whole
// 32-element block (no shuffles). The codes go to a [kCols qt rows][128 bytes]
// staging tile (128-byte swizzle) that one TMA store writes out, and the four
// scale bytes of a column leave as one 32-bit store.
// Columns from `cols` to the next multiple of 128 (the scale layout's padding
// rows) get scale 0x00 and no element writes.
#pragma once

#include <cuda_bf16.h>

#include "mxfp8_gemm.cuh"  // device status word, settle_inflight_copies
#include "mxfp8_quant.cuh"
#include "ptx.cuh"

namespace cutex {

constexpr int kColTileRows = 128;
// Ring depth per CTA: 2 tiles of 32 KB. The kernel stalls mostly at its
// per-tile CTA barriers, so more CTAs per SM with shallower rings beat fewer
// CTAs with deeper ones (fp32 at 16384^2: 3 stages 234 us, 2 stages 230 us).
constexpr int kColStages = 2;

template <int kDtype>  // 0: float32, 1: bfloat16
struct ColCfg {
  static constexpr int kElemBytes = kDtype == 0 ? 4 : 2;
  static constexpr int kCols = kDtype == 0 ? 64 : 128;  // tile columns: 256-byte row segments
  static constexpr int kThreads = 4 * kCols;             // one thread per (column, 32-row block)
  static constexpr int kMinBlocks = kDtype == 0 ? 1 : 2;
  // Row tiles per group in the tile order (tile_origin). Measured at 16384^2,
  // in us for groups of 1 / 4 / 8 / 16 / 32 row tiles: fp32 234.6 / 231.5 /
  // 234.3 / 241.4 / 247.0, bf16 153.4 / 150.1 / 149.0 / 147.1 / 149.3.
  static constexpr int kGroupRows = kDtype == 0 ? 4 : 16;
  static constexpr int kTileBytes = kColTileRows * kCols * kElemBytes;
  static constexpr int kStages = kColStages;
  static constexpr int kOutBytes = kCols * kColTileRows;  // E4M3 codes [kCols qt rows][128]
  static constexpr int kOffOut = 0;                        // 1024-aligned (128-byte swizzle)
  static constexpr int kOffStages = kOffOut + kOutBytes;
  static constexpr int kOffScales = kOffStages + kStages * kTileBytes;  // [kCols columns][4 blocks]
  static constexpr int kOffBar = kOffScales + kCols * 4;
  static constexpr int kSmemBytes = kOffBar + 8 * kStages + 1024;  // + base alignment slack
};

template <int kDtype>
__global__ void __launch_bounds__(ColCfg<kDtype>::kThreads, ColCfg<kDtype>::kMinBlocks)
    mxfp8_quantize_columnwise_kernel(const __grid_constant__ CUtensorMap tmap_x,
                                     const __grid_constant__ CUtensorMap tmap_qt, int64_t rows, int64_t cols,
                                     uint8_t* __restrict__ sft) {
  using C = ColCfg<kDtype>;
  constexpr int kCols = C::kCols;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_base = ptx::smem_u32(smem_raw);
  const uint32_t smem = (raw_base + 1023u) & ~1023u;
  uint8_t* smem_ptr = smem_raw + (smem - raw_base);
  auto full_bar = [&](int s) { return smem + C::kOffBar + 8u * s; };
  int* status = &g_cutex_device_status;

  const int64_t cols_pad = (cols + 127) & ~int64_t{127};
  const int64_t col_tiles = cols_pad / kCols;
  const int64_t row_tiles = rows / kColTileRows;
  const int64_t num_tiles = col_tiles * row_tiles;
  const int t = threadIdx.x;
  const int warp = t >> 5, lane = t & 31;
  const int blk = warp & 3;                  // 32-row block of the tile
  const int lcol = (warp >> 2) * 32 + lane;  // column within the tile

  // Tile u -> (first row, first column) of x. Tiles come in groups of
  // kGroupRows row tiles; inside a group the row tile runs fastest, so the
  // CTAs in flight together read a band of kGroupRows x 128 rows of x in runs
  // of several KB and write runs of kGroupRows x 128 bytes of each qt row
  // (with the column tile fastest, each qt row got 128-byte runs).
  auto tile_origin = [&](int64_t u, int64_t& r0, int64_t& c0) {
    const int64_t per_group = int64_t{C::kGroupRows} * col_tiles;
    const int64_t g = u / per_group, w = u - g * per_group;
    const int64_t rows_in_group = min(int64_t{C::kGroupRows}, row_tiles - g * C::kGroupRows);
    r0 = (g * C::kGroupRows + w % rows_in_group) * kColTileRows;
    c0 = (w / rows_in_group) * kCols;
  };
  auto issue = [&](int64_t u, int s) {  // one thread: TMA of tile u into stage s
    int64_t r0, c0;
    tile_origin(u, r0, c0);
    ptx::mbar_arrive_expect_tx(full_bar(s), C::kTileBytes);
    ptx::tma_load_2d(smem + C::kOffStages + s * C::kTileBytes, &tmap_x, full_bar(s), static_cast<int32_t>(c0),
                     static_cast<int32_t>(r0), ptx::policy_evict_first());
  };
  if (t == 0) {
    ptx::prefetch_tmap(&tmap_x);
    ptx::prefetch_tmap(&tmap_qt);
    for (int s = 0; s < C::kStages; ++s) ptx::mbar_init(full_bar(s), 1);
    ptx::fence_mbar_init();
  }
  __syncthreads();
  if (t == 0) {
    for (int s = 0; s < C::kStages; ++s) {
      const int64_t u = blockIdx.x + static_cast<int64_t>(s) * gridDim.x;
      if (u < num_tiles) issue(u, s);
    }
  }
  bool ok = true;
  int i = 0;
  for (int64_t u = blockIdx.x; u < num_tiles; u += gridDim.x, ++i) {
    const int s = i % C::kStages;
    // Every thread waits (bounded); the CTA leaves together if any wait gave up.
    ok = ptx::mbar_wait(full_bar(s), static_cast<uint32_t>(i / C::kStages) & 1u, status, kDevTimeoutQuantize);
    ok = __syncthreads_and(ok) != 0;
    if (!ok) break;
    int64_t r0, c0;
    tile_origin(u, r0, c0);
    // Checked builds: the tile inside x (rows) and the padded columns; the CTA
    // leaves together (every thread computes the same origin).
    if (!dev_check(r0 >= 0 && r0 + kColTileRows <= rows && c0 >= 0 && c0 + kCols <= cols_pad, kChkQuantTile, u)) {
      ok = false;
      break;
    }
    const int64_t c = c0 + lcol;  // output row of qt
    const uint8_t* stage = smem_ptr + C::kOffStages + s * C::kTileBytes;
    float v[32];
    uint32_t amax = 0u;  // magnitude bits: integer order is value order, NaN/inf the maximum
#pragma unroll
    for (int k = 0; k < 32; ++k) {
      const int idx = (blk * 32 + k) * kCols + lcol;
      if constexpr (kDtype == 0)
        v[k] = reinterpret_cast<const float*>(stage)[idx];
      else
        v[k] = __uint_as_float(static_cast<uint32_t>(reinterpret_cast<const uint16_t*>(stage)[idx]) << 16);
      amax = max(amax, __float_as_uint(v[k]) & 0x7FFFFFFFu);
    }
    if (t == 0) ptx::bulk_wait_group_read<0>();  // the previous tile's store has read the staging tile
    __syncthreads();  // stage s is read and the staging tile is free
    if (t == 0) {
      const int64_t un = u + static_cast<int64_t>(C::kStages) * gridDim.x;
      if (un < num_tiles) issue(un, s);  // refill stage s with the tile kStages ahead
    }
    const bool nonfinite = amax >= 0x7F800000u;
    const uint32_t exp_field = amax >> 23;
    const uint32_t sbyte = nonfinite ? 0xFFu : (exp_field >= 8u ? exp_field - 8u : 0u);
    uint32_t w[8];
    if (!nonfinite) {
      const float mult = __uint_as_float((254u - sbyte) << 23);  // 2^(127 - sbyte), exact
#pragma unroll
      for (int j = 0; j < 8; ++j)
        w[j] = fp8x2(v[4 * j] * mult, v[4 * j + 1] * mult) | (fp8x2(v[4 * j + 2] * mult, v[4 * j + 3] * mult) << 16);
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) w[j] = 0u;
    }
    // qt row lcol of the staging tile, bytes 32 blk .. + 31: 16-byte chunks
    // 2 blk and 2 blk + 1, placed at chunk ^ (row % 8) (the 128-byte swizzle).
    const uint32_t row_addr = smem + C::kOffOut + static_cast<uint32_t>(lcol) * 128u;
#pragma unroll
    for (int h = 0; h < 2; ++h)
      st_shared_v4(row_addr + ((static_cast<uint32_t>(2 * blk + h) ^ (static_cast<uint32_t>(lcol) & 7u)) << 4),
                   w[4 * h], w[4 * h + 1], w[4 * h + 2], w[4 * h + 3]);
    smem_ptr[C::kOffScales + lcol * 4 + blk] = static_cast<uint8_t>(c < cols ? sbyte : 0u);
    ptx::fence_proxy_async_smem();
    __syncthreads();
    if (t == 0) {  // rows of qt past `cols` are clipped by the tensor map
      ptx::tma_store_2d(&tmap_qt, smem + C::kOffOut, static_cast<int32_t>(r0), static_cast<int32_t>(c0));
      ptx::bulk_commit_group();
    }
    if (t < kCols) {
      // Column c0 + t: its four blocks' scale bytes are 4 consecutive bytes of
      // the 128x4 layout (r0 / 32 is a multiple of 4).
      const int64_t cc = c0 + t;
      const int64_t off = sf_offset(cc, r0 >> 5, rows);
      if (cc < cols_pad && dev_check(off >= 0 && off + 4 <= cols_pad * (rows >> 5), kChkScaleOffset, off))
        *reinterpret_cast<uint32_t*>(sft + off) = *reinterpret_cast<const uint32_t*>(smem_ptr + C::kOffScales + t * 4);
    }
  }
  if (t == 0) ptx::bulk_wait_group_all();  // code stores complete before the CTA exits
  if (!ok) settle_inflight_copies();       // loads already issued land before the CTA exits
}

}  // namespace cutex
