// Shared device helpers of the B200 low-precision library: status reporting, element
// loads of bf16 / fp16 / fp32 rows, the number formats (e4m3fn, e8m0, e2m1) with the
// reference's rounding rules, and warp / block reductions.
//
// Arithmetic that must match the reference bit for bit (kernel-agent's
// src/kernel_agent/kernels/quant.py) is written with explicit round-to-nearest intrinsics
// (__fmul_rn, __fadd_rn, __fdiv_rn): the compiler never contracts those into an FMA.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <stdint.h>

#include "../../include/kab.h"

namespace kab {

// ------------------------------------------------------------------ status

// Error bits a kernel raises on the device (a wait that gave up, an index that would have
// left its buffer) into its translation unit's status word; the host reads them with
// kab_device_status().
enum DeviceError : unsigned {
  kDevTimeout = 1u,
  kDevBounds = 2u,
};

// ------------------------------------------------------------------ element loads

enum InType : int { kF32 = KAB_F32, kBF16 = KAB_BF16, kF16 = KAB_F16 };

template <int T> struct InTraits;
template <> struct InTraits<kF32> { using type = float; static constexpr int bytes = 4; };
template <> struct InTraits<kBF16> { using type = __nv_bfloat16; static constexpr int bytes = 2; };
template <> struct InTraits<kF16> { using type = __half; static constexpr int bytes = 2; };

template <int T>
__device__ __forceinline__ float load_elem(const void* base, int64_t i) {
  if constexpr (T == kF32) return __ldg(reinterpret_cast<const float*>(base) + i);
  else if constexpr (T == kBF16)
    return __bfloat162float(__ldg(reinterpret_cast<const __nv_bfloat16*>(base) + i));
  else return __half2float(__ldg(reinterpret_cast<const __half*>(base) + i));
}

// Eight consecutive elements starting at an index that is a multiple of 8 (16-byte
// aligned for 2-byte types, two 16-byte loads for fp32).
template <int T>
__device__ __forceinline__ void load8(const void* base, int64_t i, float (&v)[8]) {
  if constexpr (T == kF32) {
    const float4* p = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(base) + i);
    float4 a = __ldg(p), b = __ldg(p + 1);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  } else {
    uint4 raw = __ldg(reinterpret_cast<const uint4*>(
        reinterpret_cast<const char*>(base) + i * 2));
    const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      if constexpr (T == kBF16) {
        v[2 * j] = __uint_as_float(w[j] << 16);
        v[2 * j + 1] = __uint_as_float(w[j] & 0xFFFF0000u);
      } else {
        __half2 h = *reinterpret_cast<const __half2*>(&w[j]);
        float2 f = __half22float2(h);
        v[2 * j] = f.x;
        v[2 * j + 1] = f.y;
      }
    }
  }
}

// The 8 floats of 16 bytes of 2-byte elements (bf16 or fp16), element 0 in the low half.
template <int T>
__device__ __forceinline__ void unpack8(const uint4& raw, float (&v)[8]) {
  const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    if constexpr (T == kBF16) {
      v[2 * j] = __uint_as_float(w[j] << 16);
      v[2 * j + 1] = __uint_as_float(w[j] & 0xFFFF0000u);
    } else {
      const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[j]));
      v[2 * j] = f.x;
      v[2 * j + 1] = f.y;
    }
  }
}

// fp32 -> bf16 bits, round to nearest even; NaN -> 0x7FC0 (torch's conversion).
__device__ __forceinline__ uint16_t f32_to_bf16_bits(float f) {
  uint32_t u = __float_as_uint(f);
  if ((u & 0x7FFFFFFFu) > 0x7F800000u) return 0x7FC0;
  u += 0x7FFFu + ((u >> 16) & 1u);
  return static_cast<uint16_t>(u >> 16);
}
__device__ __forceinline__ float round_bf16(float f) {
  return __uint_as_float(static_cast<uint32_t>(f32_to_bf16_bits(f)) << 16);
}
__device__ __forceinline__ uint16_t f32_to_f16_bits(float f) {
  __half h = __float2half_rn(f);
  return *reinterpret_cast<uint16_t*>(&h);
}

// ------------------------------------------------------------------ comparisons that keep NaN

// torch's clamp / amax propagate NaN; fminf / fmaxf would drop it.
__device__ __forceinline__ float clamp_keep_nan(float v, float lo, float hi) {
  return v < lo ? lo : (v > hi ? hi : v);
}
__device__ __forceinline__ float min_keep_nan(float v, float hi) { return v > hi ? hi : v; }
// max of |values| where a NaN wins (amax of a block holding a NaN is NaN).
__device__ __forceinline__ float amax_step(float acc, float v) {
  float a = fabsf(v);
  return (a > acc || a != a) ? a : acc;
}
__device__ __forceinline__ float amax_merge(float x, float y) {
  return (y > x || y != y) ? y : x;
}

template <int WIDTH = 32>
__device__ __forceinline__ float warp_amax(float v) {
#pragma unroll
  for (int o = WIDTH / 2; o > 0; o >>= 1) v = amax_merge(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Block-wide NaN-keeping amax; every thread gets the result. `red` holds >= 32 floats.
__device__ __forceinline__ float block_amax(float v, float* red) {
  v = warp_amax(v);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nwarps = (blockDim.x + 31) >> 5;
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float r = lane < nwarps ? red[lane] : 0.0f;
  r = warp_amax(r);
  return r;
}

// ------------------------------------------------------------------ e4m3fn / e8m0 / e2m1

// e4m3fn byte of v (|v| <= 448 or NaN), round to nearest even: cvt.rn.satfinite.
__device__ __forceinline__ uint8_t e4m3_byte(float v) {
  return static_cast<uint8_t>(__nv_cvt_float_to_fp8(v, __NV_SATFINITE, __NV_E4M3));
}
// two e4m3fn bytes (x in the low byte).
__device__ __forceinline__ uint16_t e4m3_pair(float x, float y) {
  return static_cast<uint16_t>(
      __nv_cvt_float2_to_fp8x2(make_float2(x, y), __NV_SATFINITE, __NV_E4M3));
}
// the exact fp32 value of an e4m3fn byte (0x7F / 0xFF: NaN).
__device__ __forceinline__ float e4m3_value(uint8_t b) {
  const uint32_t e = (b >> 3) & 0xF, m = b & 7;
  float mag;
  if ((b & 0x7F) == 0x7F) mag = __uint_as_float(0x7FC00000u);
  else if (e == 0) mag = static_cast<float>(m) * 0.001953125f;  // m * 2^-9, exact
  else mag = __uint_as_float(((e + 120u) << 23) | (m << 20));
  return (b & 0x80) ? -mag : mag;
}
// The same value by the hardware conversion (e4m3 -> f16 is exact, f16 -> f32 too).
__device__ __forceinline__ float e4m3_value_hw(uint8_t b) {
  const __half_raw h = __nv_cvt_fp8_to_halfraw(static_cast<__nv_fp8_storage_t>(b), __NV_E4M3);
  return __half2float(__half(h));
}
// 2^(b - 127) for an e8m0 byte b (b == 0: 2^-127, an fp32 subnormal; 255: NaN).
__device__ __forceinline__ float e8m0_value(uint8_t b) {
  if (b == 255) return __uint_as_float(0x7FC00000u);
  if (b == 0) return __uint_as_float(0x00400000u);
  return __uint_as_float(static_cast<uint32_t>(b) << 23);
}
// 2^-e as fp32 for an unbiased exponent -127 <= e <= 127 (2^127 down to 2^-127).
__device__ __forceinline__ float pow2_neg(int e) {
  const int be = 127 - e;  // biased exponent of 2^-e
  if (be >= 1) return __uint_as_float(static_cast<uint32_t>(be) << 23);
  return __uint_as_float(0x00400000u);  // e == 127: 2^-127
}

// e2m1 code (0..15, sign in bit 3) of an fp32 value already clamped to [-6, 6], by the
// reference's midpoint comparisons: ties at 0.75 / 1.75 / 3.5 up, at 0.25 / 1.25 / 2.5 / 5
// down (round to nearest even); no negative zero; NaN -> 0.
__device__ __forceinline__ uint32_t e2m1_code(float v) {
  const float m = fabsf(v);
  uint32_t idx = (m > 0.25f) + (m >= 0.75f) + (m > 1.25f) + (m >= 1.75f) + (m > 2.5f) +
                 (m >= 3.5f) + (m > 5.0f);
  return idx | ((v < 0.0f && idx) ? 8u : 0u);
}

// ------------------------------------------------------------------ the swizzled scale layout

// Byte offset of scale [row, col] of a [rows, cols] scale matrix in cuBLASLt's 128 x 4
// blocked layout (quant.py:540-547 mx_scale_offset).
__host__ __device__ __forceinline__ int64_t scale_offset_swizzled(int64_t row, int64_t col,
                                                                  int64_t cols) {
  const int64_t blocks_per_row = (cols + 3) / 4;
  const int64_t block = (row / 128) * blocks_per_row + col / 4;
  return block * 512 + (row % 32) * 16 + ((row % 128) / 32) * 4 + col % 4;
}

}  // namespace kab
