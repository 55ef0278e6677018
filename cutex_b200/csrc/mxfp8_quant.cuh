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
// row. A CTA walks whole rows (grid-stride over the padded rows) and its
// threads stride along the row, so no index needs a division; each thread
// loads 128 bytes of a row before quantising them, so enough loads are in
// flight per SM. Inputs are loaded and codes stored with the streaming cache
// operators (each byte is touched once; measured 4-6 % faster than default
// stores at 16384 x 16384). Padding rows of the last 128-row scale block get
// scale 0x00 and no element writes.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp8.h>

#include <cstdint>

#include "device_status.cuh"

namespace cutex {

__host__ __device__ inline int64_t sf_offset(int64_t r, int64_t c, int64_t K) {
  return ((r >> 7) * (K >> 7) + (c >> 2)) * 512 + (r & 31) * 16 + ((r & 127) >> 5) * 4 + (c & 3);
}

__device__ __forceinline__ uint32_t fp8x2(float lo, float hi) {
  return static_cast<uint32_t>(__nv_cvt_float2_to_fp8x2(make_float2(lo, hi), __NV_SATFINITE, __NV_E4M3));
}

// Raw words of one 8-element group: 8 fp32 or 4 bf16x2.
template <int kDtype>
struct GroupRaw {
  uint32_t w[kDtype == 0 ? 8 : 4];
};

// Loads group g of row r (zeros for a padding row r >= rows).
template <int kDtype>
__device__ __forceinline__ void load_group(const void* __restrict__ x, int64_t rows, int64_t ldx, int64_t r,
                                           int64_t g, GroupRaw<kDtype>& raw) {
  if (r < rows) {
    if constexpr (kDtype == 0) {
      const uint4* p = reinterpret_cast<const uint4*>(static_cast<const float*>(x) + r * ldx + g * 8);
      const uint4 a = __ldcs(p);
      const uint4 b = __ldcs(p + 1);
      raw.w[0] = a.x; raw.w[1] = a.y; raw.w[2] = a.z; raw.w[3] = a.w;
      raw.w[4] = b.x; raw.w[5] = b.y; raw.w[6] = b.z; raw.w[7] = b.w;
    } else {
      const uint4 a =
          __ldcs(reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(x) + r * ldx + g * 8));
      raw.w[0] = a.x; raw.w[1] = a.y; raw.w[2] = a.z; raw.w[3] = a.w;
    }
  } else {
#pragma unroll
    for (int j = 0; j < (kDtype == 0 ? 8 : 4); ++j) raw.w[j] = 0u;
  }
}

// The 8 fp32 values of a loaded group.
template <int kDtype>
__device__ __forceinline__ void unpack_group(const GroupRaw<kDtype>& raw, float (&v)[8]) {
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    if constexpr (kDtype == 0)
      v[j] = __uint_as_float(raw.w[j]);
    else
      v[j] = __uint_as_float(j % 2 == 0 ? raw.w[j / 2] << 16 : raw.w[j / 2] & 0xFFFF0000u);
  }
}

// Quantises group g of row r (values v) and stores its codes and, from the
// quad's first lane, the block's scale byte. The four lanes of a quad hold one
// 1x32 block; `quad` is their lane mask.
__device__ __forceinline__ void finish_group(const float (&v)[8], int64_t rows, int64_t K, uint8_t* __restrict__ q,
                                             uint8_t* __restrict__ sf, int64_t r, int64_t g, unsigned quad) {
  // amax on the magnitude bit patterns: for non-negative floats integer order is
  // value order, and a NaN or infinity (bits >= 0x7F800000) is the maximum.
  uint32_t amax = 0u;
#pragma unroll
  for (int j = 0; j < 8; ++j) amax = max(amax, __float_as_uint(v[j]) & 0x7FFFFFFFu);
  amax = max(amax, __shfl_xor_sync(quad, amax, 1));
  amax = max(amax, __shfl_xor_sync(quad, amax, 2));
  const bool nonfinite = amax >= 0x7F800000u;
  const uint32_t exp_field = amax >> 23;
  const uint32_t sbyte = nonfinite ? 0xFFu : (exp_field >= 8u ? exp_field - 8u : 0u);
  if (r < rows) {
    uint2 out = make_uint2(0u, 0u);
    if (!nonfinite) {
      const float mult = __uint_as_float((254u - sbyte) << 23);  // 2^(127 - sbyte), exact
      out.x = fp8x2(v[0] * mult, v[1] * mult) | (fp8x2(v[2] * mult, v[3] * mult) << 16);
      out.y = fp8x2(v[4] * mult, v[5] * mult) | (fp8x2(v[6] * mult, v[7] * mult) << 16);
    }
    if (dev_check(r >= 0 && g >= 0 && g * 8 + 8 <= K, kChkCodeOffset, r * K + g * 8))
      __stcs(reinterpret_cast<uint2*>(q + r * K + g * 8), out);  // streaming: written once, not read here
  }
  if ((g & 3) == 0) {
    // sf_offset(r, c = g / 4, K) with the row's part hoisted: 512-byte chunk
    // (r / 128, c / 4), byte (r % 32) * 16 + (r % 128 / 32) * 4 + c % 4.
    const int64_t row_part = ((r >> 7) * (K >> 7)) * 512 + (r & 31) * 16 + ((r & 127) >> 5) * 4;
    const uint32_t c = static_cast<uint32_t>(g) >> 2;
    const int64_t off = row_part + ((c >> 2) << 9) + (c & 3u);
    if (dev_check(off >= 0 && off < ((rows + 127) & ~int64_t{127}) * (K >> 5), kChkScaleOffset, off))
      sf[off] = static_cast<uint8_t>(sbyte);
  }
}

// 16 bf16 elements (two 8-element groups, 8 packed words) of a 1x32 block held
// by a lane pair: the block amax on packed 16-bit magnitudes (a bf16
// magnitude's bit pattern orders like its value, and its exponent field is the
// fp32 one), the scale byte, and the 16 E4M3 codes. Same rule and bits as
// finish_group, with fewer instructions per element: the bf16 form of the
// quantiser is issue-bound, not HBM-bound, with 8 elements per lane.
__device__ __forceinline__ uint32_t bf16x2_e4m3x2(uint32_t w, float mult) {
  return fp8x2(__uint_as_float(w << 16) * mult, __uint_as_float(w & 0xFFFF0000u) * mult);
}

__device__ __forceinline__ uint4 quantize_bf16_half_block(const uint4 a, const uint4 b, unsigned pair,
                                                          uint32_t& sbyte) {
  const uint32_t m = __vmaxu2(__vmaxu2(__vmaxu2(a.x & 0x7FFF7FFFu, a.y & 0x7FFF7FFFu),
                                       __vmaxu2(a.z & 0x7FFF7FFFu, a.w & 0x7FFF7FFFu)),
                              __vmaxu2(__vmaxu2(b.x & 0x7FFF7FFFu, b.y & 0x7FFF7FFFu),
                                       __vmaxu2(b.z & 0x7FFF7FFFu, b.w & 0x7FFF7FFFu)));
  uint32_t amax = max(m & 0xFFFFu, m >> 16);
  amax = max(amax, __shfl_xor_sync(pair, amax, 1));
  const bool nonfinite = amax >= 0x7F80u;  // an infinity or NaN in the block
  const uint32_t exp_field = amax >> 7;
  sbyte = nonfinite ? 0xFFu : (exp_field >= 8u ? exp_field - 8u : 0u);
  const float mult = __uint_as_float((254u - (nonfinite ? 127u : sbyte)) << 23);  // 2^(127 - sbyte), exact
  const uint4 out = make_uint4(bf16x2_e4m3x2(a.x, mult) | (bf16x2_e4m3x2(a.y, mult) << 16),
                               bf16x2_e4m3x2(a.z, mult) | (bf16x2_e4m3x2(a.w, mult) << 16),
                               bf16x2_e4m3x2(b.x, mult) | (bf16x2_e4m3x2(b.y, mult) << 16),
                               bf16x2_e4m3x2(b.z, mult) | (bf16x2_e4m3x2(b.w, mult) << 16));
  return nonfinite ? make_uint4(0u, 0u, 0u, 0u) : out;
}

// bf16 input: rows walked as in the fp32 form (whole rows per CTA, threads along
// the row), each lane taking 16 consecutive elements (a lane pair holds one
// 1x32 block) and 2 such units (64 bytes of loads) per step before any is
// quantised; the row's bounds, addresses and scale-row offset are computed once
// per row. (At 16384^2: 2 units per step, 47 registers, 138.5-139.3 us; 4 units,
// 64 registers and fewer resident CTAs, 141.1-141.5 us; 8 units, 110 registers,
// 157 us; 1 unit 139.0-139.5 us.) The two 16-byte loads of a unit are adjacent, so a warp's pair of
// load instructions covers 1 KB of the row exactly once.
__device__ __forceinline__ void quantize_rows_bf16(const __nv_bfloat16* __restrict__ x, int64_t rows, int64_t K,
                                                   int64_t ldx, uint8_t* __restrict__ q, uint8_t* __restrict__ sf) {
  constexpr int kU = 2;
  const int k16 = static_cast<int>(K >> 4);  // 16-element units per row (K < 2^31, a multiple of 8 units)
  const int64_t rows_pad = (rows + 127) & ~int64_t{127};
  const unsigned pair = 0x3u << (threadIdx.x & 30u);
  const int bd = static_cast<int>(blockDim.x);
  for (int64_t r = blockIdx.x; r < rows_pad; r += gridDim.x) {
    uint8_t* sf_row = sf + ((r >> 7) * (K >> 7)) * 512 + (r & 31) * 16 + ((r & 127) >> 5) * 4;
    // Checked builds: every scale byte of the row inside the scale array.
    const int64_t sf_row_off = sf_row - sf;
    const int64_t sf_bytes = rows_pad * (K >> 5);
    if (r >= rows) {  // padding row of the last 128-row scale block: scale 0x00, no codes
      for (int c = threadIdx.x; c < (k16 >> 1); c += bd) {
        const int64_t off = ((c >> 2) << 9) + (c & 3);
        if (dev_check(sf_row_off + off < sf_bytes, kChkScaleOffset, sf_row_off + off)) sf_row[off] = 0;
      }
      continue;
    }
    const uint4* xr = reinterpret_cast<const uint4*>(x + r * ldx);
    uint4* qr = reinterpret_cast<uint4*>(q + r * K);
    auto emit = [&](const uint4 lo, const uint4 hi, int j) {
      uint32_t sbyte;
      const uint4 codes = quantize_bf16_half_block(lo, hi, pair, sbyte);
      if (dev_check(j >= 0 && j < k16, kChkCodeOffset, r * K + 16 * static_cast<int64_t>(j)))
        __stcs(qr + j, codes);  // streaming: written once, not read here
      if ((j & 1) == 0) {
        const int c = j >> 1;  // the 1x32 block
        const int64_t off = ((c >> 2) << 9) + (c & 3);
        if (dev_check(sf_row_off + off < sf_bytes, kChkScaleOffset, sf_row_off + off))
          sf_row[off] = static_cast<uint8_t>(sbyte);
      }
    };
    int j0 = threadIdx.x;
    // Whole steps: every unit of the step is inside the row (all of them when K
    // is a multiple of 16 * blockDim * kU, e.g. K = 16384), no bounds checks.
    const int full_end = k16 - (kU - 1) * bd;
    for (; j0 < full_end; j0 += bd * kU) {
      uint4 raw[2 * kU];
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        raw[2 * u] = __ldcs(xr + 2 * (j0 + u * bd));
        raw[2 * u + 1] = __ldcs(xr + 2 * (j0 + u * bd) + 1);
      }
#pragma unroll
      for (int u = 0; u < kU; ++u) emit(raw[2 * u], raw[2 * u + 1], j0 + u * bd);
    }
    // The rest of the row (k16 and bd are even: a lane pair takes each branch together).
    for (; j0 < k16; j0 += bd * kU) {
      uint4 raw[2 * kU];
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        const int j = j0 + u * bd;
        raw[2 * u] = j < k16 ? __ldcs(xr + 2 * j) : make_uint4(0u, 0u, 0u, 0u);
        raw[2 * u + 1] = j < k16 ? __ldcs(xr + 2 * j + 1) : make_uint4(0u, 0u, 0u, 0u);
      }
#pragma unroll
      for (int u = 0; u < kU; ++u)
        if (j0 + u * bd < k16) emit(raw[2 * u], raw[2 * u + 1], j0 + u * bd);
    }
  }
}

template <int kDtype>  // 0: float32, 1: bfloat16
__global__ void __launch_bounds__(256) mxfp8_quantize_kernel(const void* __restrict__ x, int64_t rows,
                                                             int64_t K, int64_t ldx,
                                                             uint8_t* __restrict__ q,
                                                             uint8_t* __restrict__ sf) {
  const int64_t k8 = K >> 3;  // 8-element groups per row (a multiple of 16)
  const int64_t rows_pad = (rows + 127) & ~int64_t{127};
  // blockDim.x and k8 are multiples of 4, so the four lanes of a quad always
  // take the same trip through the row loop.
  if constexpr (kDtype == 1) {
    quantize_rows_bf16(static_cast<const __nv_bfloat16*>(x), rows, K, ldx, q, sf);
    return;
  }
  const unsigned quad = 0xFu << (threadIdx.x & 28u);
  // kU groups per thread and step, all loaded (as raw words, 32 registers)
  // before any is quantised: 128 bytes of loads in flight per thread, which is
  // what the HBM latency needs at the occupancy this register count allows.
  constexpr int kU = 4;
  const int64_t step = static_cast<int64_t>(blockDim.x) * kU;
  for (int64_t r = blockIdx.x; r < rows_pad; r += gridDim.x) {
    for (int64_t g0 = threadIdx.x; g0 < k8; g0 += step) {
      GroupRaw<kDtype> raw[kU];
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        const int64_t g = g0 + u * static_cast<int64_t>(blockDim.x);
        if (g < k8) load_group<kDtype>(x, rows, ldx, r, g, raw[u]);
      }
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        const int64_t g = g0 + u * static_cast<int64_t>(blockDim.x);
        if (g < k8) {
          float v[8];
          unpack_group<kDtype>(raw[u], v);
          finish_group(v, rows, K, q, sf, r, g, quad);
        }
      }
    }
  }
}

// CTAs of `kernel` resident per SM at `threads` threads and `smem` bytes
// (queried once per kernel; 1 if the query fails).
inline int resident_ctas(const void* kernel, int threads, size_t smem) {
  int n = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kernel, threads, smem) != cudaSuccess || n < 1) n = 1;
  return n;
}

inline bool launch_quantize(const void* x, int dtype, int64_t rows, int64_t K, int64_t ldx, void* q,
                            void* sf, int sm_count, cudaStream_t stream) {
  const int64_t rows_pad = (rows + 127) & ~int64_t{127};
  const int64_t k8 = K >> 3;
  // Whole rows per CTA; threads along the row (a multiple of 32, at most 256).
  // One wave of resident CTAs, each walking a strided set of rows.
  // bf16 lanes take 16 elements each, fp32 lanes 8 per group.
  const int64_t units = dtype == 0 ? k8 : k8 / 2;
  const int threads = static_cast<int>(units >= 256 ? 256 : ((units + 31) / 32) * 32);
  static const int per_sm[2] = {resident_ctas(reinterpret_cast<const void*>(&mxfp8_quantize_kernel<0>), 256, 0),
                                resident_ctas(reinterpret_cast<const void*>(&mxfp8_quantize_kernel<1>), 256, 0)};
  const int64_t wave = int64_t{sm_count} * per_sm[dtype == 0 ? 0 : 1];
  int64_t blocks = rows_pad < wave ? rows_pad : wave;
  if (blocks < 1) blocks = 1;
  if (dtype == 0)
    mxfp8_quantize_kernel<0><<<static_cast<unsigned>(blocks), threads, 0, stream>>>(
        x, rows, K, ldx, static_cast<uint8_t*>(q), static_cast<uint8_t*>(sf));
  else
    mxfp8_quantize_kernel<1><<<static_cast<unsigned>(blocks), threads, 0, stream>>>(
        x, rows, K, ldx, static_cast<uint8_t*>(q), static_cast<uint8_t*>(sf));
  return cudaGetLastError() == cudaSuccess;
}

}  // namespace cutex
