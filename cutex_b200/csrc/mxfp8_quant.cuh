// MXFP8 quantiser (OCP MX v1.0, E4M3 elements, E8M0 scales) writing the
// SM100 128x4 swizzled scale layout the GEMM consumes.
//
// Per 1x32 block of a row: amax = max|x|; if the block holds a non-finite
// value the scale byte is 0xFF (NaN) and the elements are written as 0.
// Otherwise the scale byte is max(exponent_field(amax) - 8, 0), i.e. the
// scale exponent floor(log2(amax)) - 8 clamped below at -127 (an all-zero
// block gets 0x00), and each element is x * 2^-(byte-127) converted to E4M3
// with round-to-nearest-even and saturation to +-448.
//
// HBM-bound: four threads share one 32-element block (8 elements each, 16 or
// 32 bytes per thread per load), a warp covers 256 contiguous elements of a
// row, and the grid strides over [rows_padded x K/8]. Padding rows of the last
// 128-row scale block get scale 0x00 and no element writes.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp8.h>

#include <cstdint>

namespace cutex {

__host__ __device__ inline int64_t sf_offset(int64_t r, int64_t c, int64_t K) {
  return ((r >> 7) * (K >> 7) + (c >> 2)) * 512 + (r & 31) * 16 + ((r & 127) >> 5) * 4 + (c & 3);
}

__device__ __forceinline__ uint32_t fp8x2(float lo, float hi) {
  return static_cast<uint32_t>(__nv_cvt_float2_to_fp8x2(make_float2(lo, hi), __NV_SATFINITE, __NV_E4M3));
}

template <int kDtype>  // 0: float32, 1: bfloat16
__global__ void __launch_bounds__(256) mxfp8_quantize_kernel(const void* __restrict__ x, int64_t rows,
                                                             int64_t K, int64_t ldx,
                                                             uint8_t* __restrict__ q,
                                                             uint8_t* __restrict__ sf) {
  const int64_t k8 = K >> 3;  // 8-element groups per row
  const int64_t rows_pad = (rows + 127) & ~int64_t{127};
  const int64_t total = rows_pad * k8;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  // Trip count is uniform across each group of 4 lanes (total % 4 == 0 and the
  // start index is a multiple of 4 apart within a quad), so the shuffles below
  // always see their partner lanes.
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total; i += stride) {
    const int64_t r = i / k8;
    const int64_t g = i - r * k8;  // 8-element group within the row
    float v[8];
    if (r < rows) {
      if constexpr (kDtype == 0) {
        const float4* p = reinterpret_cast<const float4*>(static_cast<const float*>(x) + r * ldx + g * 8);
        const float4 a = __ldcs(p);
        const float4 b = __ldcs(p + 1);
        v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
        v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
      } else {
        const uint4 a = __ldcs(reinterpret_cast<const uint4*>(
            static_cast<const __nv_bfloat16*>(x) + r * ldx + g * 8));
        const uint32_t w[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          v[2 * j] = __uint_as_float(w[j] << 16);
          v[2 * j + 1] = __uint_as_float(w[j] & 0xFFFF0000u);
        }
      }
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = 0.f;
    }
    float amax = 0.f;
    uint32_t nonfinite = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const uint32_t bits = __float_as_uint(v[j]) & 0x7FFFFFFFu;
      nonfinite |= bits >= 0x7F800000u ? 1u : 0u;
      amax = fmaxf(amax, __uint_as_float(bits));
    }
    amax = fmaxf(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, 1));
    amax = fmaxf(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, 2));
    nonfinite |= __shfl_xor_sync(0xFFFFFFFFu, nonfinite, 1);
    nonfinite |= __shfl_xor_sync(0xFFFFFFFFu, nonfinite, 2);
    const uint32_t exp_field = __float_as_uint(amax) >> 23;
    const uint32_t sbyte = nonfinite ? 0xFFu : (exp_field >= 8u ? exp_field - 8u : 0u);
    if (r < rows) {
      uint2 out = make_uint2(0u, 0u);
      if (!nonfinite) {
        const float mult = __uint_as_float((254u - sbyte) << 23);  // 2^(127 - sbyte), exact
        out.x = fp8x2(v[0] * mult, v[1] * mult) | (fp8x2(v[2] * mult, v[3] * mult) << 16);
        out.y = fp8x2(v[4] * mult, v[5] * mult) | (fp8x2(v[6] * mult, v[7] * mult) << 16);
      }
      *reinterpret_cast<uint2*>(q + r * K + g * 8) = out;
    }
    if ((g & 3) == 0) sf[sf_offset(r, g >> 2, K)] = static_cast<uint8_t>(sbyte);
  }
}

inline bool launch_quantize(const void* x, int dtype, int64_t rows, int64_t K, int64_t ldx, void* q,
                            void* sf, int sm_count, cudaStream_t stream) {
  const int64_t rows_pad = (rows + 127) & ~int64_t{127};
  const int64_t total = rows_pad * (K >> 3);
  const int threads = 256;
  int64_t blocks = (total + threads - 1) / threads;
  blocks = blocks < int64_t{sm_count} * 8 ? blocks : int64_t{sm_count} * 8;
  if (blocks < 1) blocks = 1;
  if (dtype == 0)
    mxfp8_quantize_kernel<0><<<static_cast<unsigned>(blocks), threads, 0, stream>>>(
        x, rows, K, ldx, static_cast<uint8_t*>(q), static_cast<uint8_t*>(sf));
  else
    mxfp8_quantize_kernel<1><<<static_cast<unsigned>(blocks), threads, 0, stream>>>(
        x, rows, K, ldx, static_cast<uint8_t*>(q), static_cast<uint8_t*>(sf));
  return cudaGetLastError() == cudaSuccess;
}

// Columnwise quantiser: the operand layout a GEMM needs when the reduction
// runs over the rows of x (weight gradients reduce over tokens; input
// gradients read W along its columns). For x[rows, cols] it writes
// qt[cols, rows] = quantise(x^T): 1x32 blocks run down the columns of x, and
// the scales land in the 128x4 swizzled layout of a [cols, K = rows] operand.
// Same per-block rule as the rowwise kernel.
//
// A CTA stages a 128-row x 64-column tile of x in shared memory (coalesced
// 16/32-byte loads along the rows), then warp w quantises block w % 4 (rows
// 32b..32b+31) of columns 32 (w / 4) .. + 31: one lane per column, so each
// lane holds a whole 32-element block (no shuffles) and writes 32 contiguous
// bytes of qt and one scale byte. Columns from cols up to the next multiple of
// 128 (the scale layout's padding rows) get scale 0x00 and no element writes.
constexpr int kColTileRows = 128;
constexpr int kColTileCols = 64;

template <int kDtype>  // 0: float32, 1: bfloat16
__global__ void __launch_bounds__(256) mxfp8_quantize_columnwise_kernel(const void* __restrict__ x, int64_t rows,
                                                                        int64_t cols, int64_t ldx,
                                                                        uint8_t* __restrict__ qt,
                                                                        uint8_t* __restrict__ sft) {
  __shared__ float tile[kColTileRows][kColTileCols + 1];
  const int64_t c0 = static_cast<int64_t>(blockIdx.x) * kColTileCols;
  const int64_t r0 = static_cast<int64_t>(blockIdx.y) * kColTileRows;
  const int t = threadIdx.x;
  // Load: 8 consecutive columns per thread, 8 threads per row, 32 rows per pass.
  const int lc = (t & 7) * 8;
#pragma unroll
  for (int pass = 0; pass < 4; ++pass) {
    const int lr = pass * 32 + (t >> 3);
    const int64_t c = c0 + lc;
    float v[8];
    if (c + 8 <= cols) {
      if constexpr (kDtype == 0) {
        const float4* p = reinterpret_cast<const float4*>(static_cast<const float*>(x) + (r0 + lr) * ldx + c);
        const float4 a = __ldcs(p);
        const float4 b = __ldcs(p + 1);
        v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
        v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
      } else {
        const uint4 a = __ldcs(reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(x) +
                                                             (r0 + lr) * ldx + c));
        const uint32_t w[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          v[2 * j] = __uint_as_float(w[j] << 16);
          v[2 * j + 1] = __uint_as_float(w[j] & 0xFFFF0000u);
        }
      }
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        float e = 0.f;
        if (c + j < cols) {
          if constexpr (kDtype == 0) {
            e = static_cast<const float*>(x)[(r0 + lr) * ldx + c + j];
          } else {
            const uint16_t h = reinterpret_cast<const uint16_t*>(x)[(r0 + lr) * ldx + c + j];
            e = __uint_as_float(static_cast<uint32_t>(h) << 16);
          }
        }
        v[j] = e;
      }
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) tile[lr][lc + j] = v[j];
  }
  __syncthreads();
  const int warp = t >> 5, lane = t & 31;
  const int blk = warp & 3;                          // 32-row block of the tile
  const int lcol = (warp >> 2) * 32 + lane;          // column within the tile
  const int64_t c = c0 + lcol;                       // output row of qt
  float v[32];
  float amax = 0.f;
  uint32_t nonfinite = 0;
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    v[i] = tile[blk * 32 + i][lcol];
    const uint32_t bits = __float_as_uint(v[i]) & 0x7FFFFFFFu;
    nonfinite |= bits >= 0x7F800000u ? 1u : 0u;
    amax = fmaxf(amax, __uint_as_float(bits));
  }
  const uint32_t exp_field = __float_as_uint(amax) >> 23;
  const uint32_t sbyte = nonfinite ? 0xFFu : (exp_field >= 8u ? exp_field - 8u : 0u);
  const int64_t cols_pad = (cols + 127) & ~int64_t{127};
  if (c < cols) {
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
    uint4* dst = reinterpret_cast<uint4*>(qt + c * rows + r0 + blk * 32);
    dst[0] = make_uint4(w[0], w[1], w[2], w[3]);
    dst[1] = make_uint4(w[4], w[5], w[6], w[7]);
  }
  if (c < cols_pad) sft[sf_offset(c, (r0 >> 5) + blk, rows)] = static_cast<uint8_t>(c < cols ? sbyte : 0u);
}

inline bool launch_quantize_columnwise(const void* x, int dtype, int64_t rows, int64_t cols, int64_t ldx, void* qt,
                                       void* sft, cudaStream_t stream) {
  const int64_t cols_pad = (cols + 127) & ~int64_t{127};
  const dim3 grid(static_cast<unsigned>(cols_pad / kColTileCols), static_cast<unsigned>(rows / kColTileRows));
  if (dtype == 0)
    mxfp8_quantize_columnwise_kernel<0><<<grid, 256, 0, stream>>>(x, rows, cols, ldx, static_cast<uint8_t*>(qt),
                                                                  static_cast<uint8_t*>(sft));
  else
    mxfp8_quantize_columnwise_kernel<1><<<grid, 256, 0, stream>>>(x, rows, cols, ldx, static_cast<uint8_t*>(qt),
                                                                  static_cast<uint8_t*>(sft));
  return cudaGetLastError() == cudaSuccess;
}

}  // namespace cutex
