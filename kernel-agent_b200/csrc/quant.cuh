// Activation / weight quantise producers: HBM-bound, one pass over the input.
//
//  * per-row INT8 / FP8 (per token or per output channel), optionally fused with
//    SiLU(gate) * up (FP8) or a SmoothQuant divisor / multiplier (INT8);
//  * 1 x G groups and B x B blocks of FP8 (the blockwise recipe);
//  * MXFP8 (e4m3 + e8m0 per 32), optionally fused with SiLU(gate) * up;
//  * NVFP4 (e2m1 + e4m3 per 16 + fp32 outer / tensor scale) and MXFP4 (e2m1 + e8m0 per 32),
//    activations and weights, optionally fused with SiLU(gate) * up;
//  * the global amax of a matrix (NVFP4 tensor scales).
//
// Rows are read with 16-byte vector loads (8 elements per thread per chunk) and kept in
// registers between the reduction and the conversion, so HBM sees one read of the input
// and one write of the codes. Every rounding follows kernel-agent's
// src/kernel_agent/kernels/quant.py (line numbers at each function).
#pragma once

#include "codes.cuh"

namespace kab {

constexpr float kInt8Step = 0.007874015718698502f;     // fp32(1 / 127), quant.py:764
constexpr float kNvfp4OuterStep = 0.00037202381645329297f;  // fp32(1 / 2688), quant.py:1033

// ------------------------------------------------------------------ SiLU(gate) * up

// F.silu(g) * u with the rounding points of eager (triton_fp8_producers.py:136-147): the
// SiLU rounded to the input dtype, the product rounded to it again. `expf` is CUDA's.
// (An intermediate value: the hardware conversion rounds to nearest even like the stored
// outputs' f32_to_bf16_bits; only a NaN's payload can differ, and a NaN stays a NaN.)
template <int T>
__device__ __forceinline__ float round_to_input(float f) {
  if constexpr (T == kBF16) return __bfloat162float(__float2bfloat16_rn(f));
  else if constexpr (T == kF16) return __half2float(__float2half_rn(f));
  else return f;
}
// RN(g / d) rounded to the input dtype: the rounding to bf16 / fp16 is a step function with
// steps at floats of at most 9 / 12 significant bits, so g * rcp(d) decides it unless the
// product lies next to such a float (then the IEEE division does).
template <int T>
__device__ __forceinline__ float div_to_input(float g, float d) {
  if constexpr (T == kF32) {
    return __fdiv_rn(g, d);
  } else {
    constexpr int LOW = T == kBF16 ? 15 : 12;
    const float a = fabsf(d);
    float q = __fmul_rn(g, rcp_approx(d));
    if (!(a >= 2.350988701644575e-38f && a <= 4.253529586511731e+37f) || near_short<LOW>(q)) q = __fdiv_rn(g, d);
    return round_to_input<T>(q);
  }
}
template <int T>
__device__ __forceinline__ float silu_mul(float g, float u) {
  const float a = div_to_input<T>(g, __fadd_rn(1.0f, expf(-g)));
  return round_to_input<T>(__fmul_rn(a, u));
}

// Optional write of the producer's own output h (the input dtype), for checking.
template <int T>
__device__ __forceinline__ void store_h8(void* h, int64_t i, const float (&v)[8]) {
  if constexpr (T == kF32) {
    float4* p = reinterpret_cast<float4*>(reinterpret_cast<float*>(h) + i);
    p[0] = make_float4(v[0], v[1], v[2], v[3]);
    p[1] = make_float4(v[4], v[5], v[6], v[7]);
  } else {
    uint32_t w[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      uint16_t lo, hi;
      if constexpr (T == kBF16) { lo = f32_to_bf16_bits(v[2 * j]); hi = f32_to_bf16_bits(v[2 * j + 1]); }
      else { lo = f32_to_f16_bits(v[2 * j]); hi = f32_to_f16_bits(v[2 * j + 1]); }
      w[j] = static_cast<uint32_t>(lo) | (static_cast<uint32_t>(hi) << 16);
    }
    *reinterpret_cast<uint4*>(reinterpret_cast<char*>(h) + i * 2) = make_uint4(w[0], w[1], w[2], w[3]);
  }
}

// Loads a chunk of 8 producer values: x itself, or silu(x) * up.
template <int T, bool SILU>
__device__ __forceinline__ void load_producer8(const void* x, const void* up, int64_t ix,
                                               int64_t iu, float (&v)[8]) {
  load8<T>(x, ix, v);
  if constexpr (SILU) {
    float u[8];
    load8<T>(up, iu, u);
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = silu_mul<T>(v[j], u[j]);
  }
}

// ------------------------------------------------------------------ MX exponent rules

// frexp of an fp32 value as (ex, mantissa == 0.5): q = m * 2^ex, m in [0.5, 1); 0, inf and
// NaN give ex = 0 with m != 0.5 (glibc's and torch's frexp).
__device__ __forceinline__ void frexp_parts(float q, int& ex, bool& half) {
  const uint32_t u = __float_as_uint(q) & 0x7FFFFFFFu;
  const uint32_t E = u >> 23, f = u & 0x7FFFFFu;
  if (u == 0 || E == 0xFF) { ex = 0; half = false; return; }
  if (E == 0) {  // subnormal: q = f * 2^-149
    const int p = 31 - __clz(f);
    ex = p - 148;
    half = (f & (f - 1)) == 0;
    return;
  }
  ex = static_cast<int>(E) - 126;
  half = f == 0;
}
// 2^e as fp32 (0 below 2^-149, inf from 2^128 on): torch.pow(2.0, e.double()).float().
__device__ __forceinline__ float pow2f(int e) {
  if (e >= 128) return __uint_as_float(0x7F800000u);
  if (e >= -126) return __uint_as_float(static_cast<uint32_t>(e + 127) << 23);
  if (e >= -149) return __uint_as_float(1u << (e + 149));
  return 0.0f;
}
// quant.py:479-495 mx_scale_exponents for one block maximum (rule 0: ceil, 1: floor).
__device__ __forceinline__ int mx_exponent(float a, int rule) {
  int e;
  if (rule == 1) {
    int ex; bool half;
    frexp_parts(a, ex, half);
    e = ex - 1 - 8;
  } else {
    int ex; bool half;
    frexp_parts(__fdiv_rn(a, kFp8Max), ex, half);
    e = ex - (half ? 1 : 0);
    e += (a > __fmul_rn(kFp8Max, pow2f(e))) ? 1 : 0;
  }
  if (!(a > 0.0f)) e = -127;
  return e < -127 ? -127 : (e > 127 ? 127 : e);
}
// quant.py:1092-1099 (activations, MXFP4): e = ex - 3 + (m > 0.75) from frexp(bmax).
__device__ __forceinline__ int mxfp4_act_exponent(float bmax) {
  const uint32_t u = __float_as_uint(bmax) & 0x7FFFFFFFu;
  int ex; bool half;
  frexp_parts(bmax, ex, half);
  // m > 0.75 <=> the normalised mantissa 1.f > 1.5 <=> the top fraction bit set with more
  // bits below it, on the normalised significand
  bool over;
  const uint32_t E = u >> 23, f = u & 0x7FFFFFu;
  if (u == 0 || E == 0xFF) over = false;                      // m is 0 / inf / NaN
  else if (E != 0) over = f > 0x400000u;                      // 1.f > 1.5
  else { const int p = 31 - __clz(f); const uint32_t g = f << (23 - p); over = (g & 0x7FFFFFu) > 0x400000u; }
  int e = ex - 3 + (over ? 1 : 0);
  if (!(bmax > 0.0f)) e = -127;
  return e < -127 ? -127 : (e > 127 ? 127 : e);
}
// quant.py:258-261 (weights, MXFP4): ceil(log2(bmax / 6)) from frexp(bmax / 6).
__device__ __forceinline__ int mxfp4_weight_exponent(float bmax) {
  int ex; bool half;
  frexp_parts(__fdiv_rn(bmax, 6.0f), ex, half);
  int e = ex - (half ? 1 : 0);
  if (!(bmax > 0.0f)) e = -127;
  return e < -127 ? -127 : (e > 127 ? 127 : e);
}

// ------------------------------------------------------------------ per-row INT8 / FP8

// MAXC: chunks of 8 elements each thread keeps in registers (0: reread the row).
// OUT 0: INT8 (SMOOTH 0 none, 1 divide: activations, 2 multiply: weights); 1: FP8.
template <int T, int MAXC, int OUT, int SMOOTH, bool SILU>
__global__ void __launch_bounds__(256)
quant_rows_kernel(const void* __restrict__ x, int64_t ldx, const void* __restrict__ up,
                  int64_t ldu, int64_t k, const float* __restrict__ smooth,
                  void* __restrict__ q, float* __restrict__ scale, void* __restrict__ h) {
  __shared__ float red[32];
  const int64_t row = blockIdx.x;
  const int64_t nchunks = k >> 3;
  const int64_t xo = row * ldx, uo = row * ldu;
  auto value8 = [&](int64_t c, float (&v)[8]) {
    load_producer8<T, SILU>(x, up, xo + c * 8, uo + c * 8, v);
    if constexpr (SMOOTH != 0) {
      const float4* sp = reinterpret_cast<const float4*>(smooth + c * 8);
      const float4 s0 = __ldg(sp), s1 = __ldg(sp + 1);
      const float s[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = SMOOTH == 1 ? __fdiv_rn(v[j], s[j]) : __fmul_rn(v[j], s[j]);
    }
  };
  float cache[MAXC > 0 ? MAXC : 1][8];
  uint32_t abits = 0;
  if constexpr (MAXC > 0) {
#pragma unroll
    for (int c = 0; c < MAXC; ++c) {
      const int64_t ci = threadIdx.x + static_cast<int64_t>(c) * blockDim.x;
      if (ci < nchunks) {
        value8(ci, cache[c]);
        abits = abs_bits_max8(cache[c], abits);
      }
    }
  } else {
    for (int64_t ci = threadIdx.x; ci < nchunks; ci += blockDim.x) {
      float v[8];
      value8(ci, v);
      abits = abs_bits_max8(v, abits);
    }
  }
  const float amax = block_amax(__uint_as_float(abits), red);
  float sc;
  if constexpr (OUT == 0) sc = amax > 0.0f ? __fmul_rn(amax, kInt8Step) : 1.0f;   // quant.py:777-780
  else sc = amax > 0.0f ? __fdiv_rn(amax, kFp8Max) : 1.0f;                        // quant.py:374-375
  if (threadIdx.x == 0) scale[row] = sc;
  const Divisor div(sc);
  auto emit = [&](int64_t ci, float (&v)[8]) {
    if (h != nullptr) store_h8<T>(h, row * k + ci * 8, v);
    float qv[8];
    if constexpr (OUT == 0) {  // quant.py:770-774: round(v / scale) to nearest even, ±127
      quotients<kLowInt8>(v, div, qv);
      *reinterpret_cast<uint2*>(reinterpret_cast<int8_t*>(q) + row * k + ci * 8) = int8x8(qv);
    } else {  // quant.py:376: (v / scale).clamp(±448) to e4m3
      *reinterpret_cast<uint2*>(reinterpret_cast<uint8_t*>(q) + row * k + ci * 8) = e4m3x8_quotients(v, div);
    }
  };
  if constexpr (MAXC > 0) {
#pragma unroll
    for (int c = 0; c < MAXC; ++c) {
      const int64_t ci = threadIdx.x + static_cast<int64_t>(c) * blockDim.x;
      if (ci < nchunks) emit(ci, cache[c]);
    }
  } else {
    for (int64_t ci = threadIdx.x; ci < nchunks; ci += blockDim.x) {
      float v[8];
      value8(ci, v);
      emit(ci, v);
    }
  }
}

// ------------------------------------------------------------------ FP8 1 x G groups

// fp8lib.py:22-27 fq_groups: scale = amax / 448 per group (0 -> 1), codes e4m3(v / scale).
// LANES = G / 8 threads share a group (G = 32, 64 or 128).
template <int T, int LANES>
__global__ void __launch_bounds__(256)
quant_groups_kernel(const void* __restrict__ x, int64_t ldx, int64_t k, uint8_t* __restrict__ q,
                    float* __restrict__ scales) {
  const int64_t row = blockIdx.x;
  const int64_t j = static_cast<int64_t>(blockIdx.y) * blockDim.x + threadIdx.x;  // chunk of 8
  const bool live = j < (k >> 3);
  float v[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  if (live) load8<T>(x, row * ldx + j * 8, v);
  uint32_t abits = abs_bits_max8(v, 0u);
#pragma unroll
  for (int o = LANES / 2; o > 0; o >>= 1) abits = max(abits, __shfl_xor_sync(0xffffffffu, abits, o));
  if (!live) return;
  float s = __fdiv_rn(__uint_as_float(abits), kFp8Max);
  s = s > 0.0f ? s : 1.0f;  // fp8lib.py:17-18 _safe
  *reinterpret_cast<uint2*>(q + row * k + j * 8) = e4m3x8_quotients(v, Divisor(s));
  if ((j % LANES) == 0) scales[row * (k / (LANES * 8)) + j / LANES] = s;
}

// ------------------------------------------------------------------ FP8 B x B blocks

// fp8lib.py:35-39 fq_block: one scale per 128 x 128 tile of a weight [N, K]; one CTA of
// 256 threads per tile, 64 elements per thread in registers.
template <int T>
__global__ void __launch_bounds__(256)
quant_blocks128_kernel(const void* __restrict__ w, int64_t ldw, int64_t k,
                       uint8_t* __restrict__ q, float* __restrict__ scales) {
  __shared__ float red[32];
  const int64_t nb = blockIdx.y, kb = blockIdx.x;
  float v[8][8];
  uint32_t abits = 0;
#pragma unroll
  for (int c = 0; c < 8; ++c) {  // 2048 chunks of 8: row = idx / 16, column chunk = idx % 16
    const int idx = threadIdx.x + c * 256;
    const int64_t r = nb * 128 + (idx >> 4), col = kb * 128 + (idx & 15) * 8;
    load8<T>(w, r * ldw + col, v[c]);
    abits = abs_bits_max8(v[c], abits);
  }
  const float amax = block_amax(__uint_as_float(abits), red);
  float s = __fdiv_rn(amax, kFp8Max);
  s = s > 0.0f ? s : 1.0f;
  if (threadIdx.x == 0) scales[nb * (k / 128) + kb] = s;
  const Divisor div(s);
#pragma unroll
  for (int c = 0; c < 8; ++c) {
    const int idx = threadIdx.x + c * 256;
    const int64_t r = nb * 128 + (idx >> 4), col = kb * 128 + (idx & 15) * 8;
    *reinterpret_cast<uint2*>(q + r * k + col) = e4m3x8_quotients(v[c], div);
  }
}

// ------------------------------------------------------------------ MXFP8

// quant.py:506-526 quantize_mxfp8 (and the fused SiLU * up producer): 4 lanes hold one
// block of 32; scale byte e + 127 row-major [rows, K / 32] or in the swizzled layout.
template <int T, bool SILU>
__global__ void __launch_bounds__(256)
quant_mxfp8_kernel(const void* __restrict__ x, int64_t ldx, const void* __restrict__ up,
                   int64_t ldu, int64_t k, int rule, int swizzle, uint8_t* __restrict__ q,
                   uint8_t* __restrict__ scales, void* __restrict__ h) {
  const int64_t row = blockIdx.x;
  const int64_t j = static_cast<int64_t>(blockIdx.y) * blockDim.x + threadIdx.x;  // chunk of 8
  const bool live = j < (k >> 3);
  float v[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  if (live) load_producer8<T, SILU>(x, up, row * ldx + j * 8, row * ldu + j * 8, v);
  uint32_t abits = abs_bits_max8(v, 0u);
  abits = max(abits, __shfl_xor_sync(0xffffffffu, abits, 1));
  abits = max(abits, __shfl_xor_sync(0xffffffffu, abits, 2));
  if (!live) return;
  const int e = mx_exponent(__uint_as_float(abits), rule);
  const float inv = pow2_neg(e);  // x / 2^e == x * 2^-e exactly (one rounding of the same value)
  if (SILU && h != nullptr) store_h8<T>(h, row * k + j * 8, v);
  float qv[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) qv[i] = __fmul_rn(v[i], inv);
  *reinterpret_cast<uint2*>(q + row * k + j * 8) = e4m3x8(qv);
  if ((j & 3) == 0) {
    const int64_t cols = k >> 5, col = j >> 2;
    const int64_t off = swizzle ? scale_offset_swizzled(row, col, cols) : row * cols + col;
    scales[off] = static_cast<uint8_t>(e + 127);
  }
}

// ------------------------------------------------------------------ NVFP4 / MXFP4

// FMT 0: NVFP4 (16 per e4m3 scale), 1: MXFP4 (32 per e8m0 scale).
// MODE 0: activations per token (outer from the row's amax), 1: activations with one amax
// per call (*amax_in), 2: weights (tensor scale *ts_in; quant.py:217-272).
// One CTA per row; each thread owns NB whole scale blocks of the row (block bi = thread +
// j * blockDim), kept in registers between the row reduction and the conversion: the block
// scale is computed once per block and the codes of a block leave in one 8- or 16-byte store.
template <int T, int NB, int FMT, int MODE, bool SILU>
__global__ void __launch_bounds__(512)
quant_fp4_kernel(const void* __restrict__ x, int64_t ldx, const void* __restrict__ up,
                 int64_t ldu, int64_t rows, int64_t k, const float* __restrict__ amax_in,
                 const float* __restrict__ ts_in, int swizzle, uint8_t* __restrict__ q,
                 uint8_t* __restrict__ scales, float* __restrict__ outer_out,
                 void* __restrict__ h) {
  __shared__ float red[32];
  constexpr int BLOCK = FMT == 0 ? 16 : 32;
  constexpr int CH = BLOCK / 8;  // chunks of 8 per block
  const int64_t row = blockIdx.x;
  const int nblk = static_cast<int>(k / BLOCK);
  float v[NB][BLOCK];
  uint32_t bbits[NB];  // max |v| of each block, as bits (NaN-keeping)
  uint32_t abits = 0;
#pragma unroll
  for (int b = 0; b < NB; ++b) {
    const int bi = threadIdx.x + b * blockDim.x;
#pragma unroll
    for (int j = 0; j < BLOCK; ++j) v[b][j] = 0.0f;
    if (bi < nblk) {
#pragma unroll
      for (int c = 0; c < CH; ++c) {
        float chunk[8];
        const int64_t col = static_cast<int64_t>(bi) * BLOCK + c * 8;
        load_producer8<T, SILU>(x, up, row * ldx + col, row * ldu + col, chunk);
        if (SILU && h != nullptr) store_h8<T>(h, row * k + col, chunk);
#pragma unroll
        for (int j = 0; j < 8; ++j) v[b][c * 8 + j] = chunk[j];
      }
    }
    uint32_t m = 0;
#pragma unroll
    for (int j = 0; j < BLOCK; ++j) m = max(m, __float_as_uint(v[b][j]) & 0x7FFFFFFFu);
    bbits[b] = m;
    abits = max(abits, m);
  }
  float s_outer = 1.0f;  // outer (activations) or tensor scale (weights)
  if constexpr (FMT == 0) {
    if constexpr (MODE == 0) {
      const float amax = block_amax(__uint_as_float(abits), red);
      s_outer = amax > 0.0f ? __fmul_rn(amax, kNvfp4OuterStep) : 1.0f;  // quant.py:1104
    } else if constexpr (MODE == 1) {
      const float a = *amax_in;
      s_outer = a > 0.0f ? __fmul_rn(a, kNvfp4OuterStep) : 1.0f;
    } else {
      s_outer = *ts_in;
    }
  }
  if (threadIdx.x == 0 && outer_out != nullptr) outer_out[row] = s_outer;
  const float div6 = __fmul_rn(s_outer, 6.0f);  // fp32(outer * 6), fp32(6 * tensor_scale)
  const Divisor by6(div6);
  const int64_t cols = nblk;
#pragma unroll
  for (int b = 0; b < NB; ++b) {
    const int bi = threadIdx.x + b * blockDim.x;
    if (bi >= nblk) continue;
    const float bmax = __uint_as_float(bbits[b]);
    uint32_t sbyte;
    float step;
    if constexpr (FMT == 0) {
      // e4m3(min(bmax / (outer * 6), 448)): satfinite saturates like the clamp, keeps NaN
      const float bm[1] = {bmax};
      float ratio[1];
      quotients<kLowE4m3>(bm, by6, ratio);
      sbyte = e4m3_byte(ratio[0]);
      step = __fmul_rn(e4m3_value_hw(static_cast<uint8_t>(sbyte)), s_outer);
    } else {
      const int e = MODE == 2 ? mxfp4_weight_exponent(bmax) : mxfp4_act_exponent(bmax);
      sbyte = static_cast<uint32_t>(e + 127);
      step = e8m0_value(static_cast<uint8_t>(sbyte));
    }
    // weights divide by step.clamp_min(1e-38) (quant.py:265); a zero (or NaN) step gives 0 codes
    const float div = (MODE == 2 && step < 1e-38f) ? 1e-38f : step;
    uint32_t packed[CH];
#pragma unroll
    for (int c = 0; c < CH; ++c) packed[c] = 0;
    if (step > 0.0f) {
      quotients<kLowE2m1>(v[b], Divisor(div), v[b]);  // in place: the values are not needed again
      if (bbits[b] > 0x7F800000u) {  // a NaN in the block: its codes are 0
#pragma unroll
        for (int j = 0; j < BLOCK; ++j) v[b][j] = v[b][j] == v[b][j] ? v[b][j] : 0.0f;
      }
#pragma unroll
      for (int c = 0; c < CH; ++c) {
        float e8[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) e8[j] = v[b][c * 8 + j];
        packed[c] = e2m1x8(e8);
      }
    }
    uint8_t* dst = q + row * (k >> 1) + static_cast<int64_t>(bi) * (BLOCK / 2);
    if constexpr (CH == 2) *reinterpret_cast<uint2*>(dst) = make_uint2(packed[0], packed[1]);
    else *reinterpret_cast<uint4*>(dst) = make_uint4(packed[0], packed[1], packed[2], packed[3]);
    const int64_t off = swizzle ? scale_offset_swizzled(row, bi, cols) : row * cols + bi;
    scales[off] = static_cast<uint8_t>(sbyte);
  }
}

constexpr int kFp4MaxRowBlocks = 32768 / 16;  // scale blocks of the longest row (k <= 32768)

// Lean NVFP4 / MXFP4 producer for bf16 / fp16 inputs without the SiLU gate: the codes and
// scales of quant_fp4_kernel (the same block scale, the same quotient RN(v * y) with the same
// exactness window and IEEE-division fallback, the same e2m1 conversion), in fewer
// instructions per element:
//  * the row is kept as packed 16-bit pairs; block maxima come from __vmaxu2 on |pairs|
//    (non-negative bf16 / fp16 values order like their bit patterns, NaN above inf);
//  * two quotients per mul.rn.f32x2;
//  * instead of the exactness window (which trips on any quotient near a float with three
//    significant bits: 6.7 % of the blocks of config 4's activations, ratios of bf16 values
//    often being exact), each block's codes are taken twice, from the products with the
//    reciprocal nudged up and down by 2^-19; agreeing codes are the quotient's codes (only a
//    quotient within about 2^-19 of an actual e2m1 midpoint makes them differ);
//  * a block whose codes differ goes on a shared-memory list and is recomputed with the IEEE
//    division after the row by the whole CTA, instead of one lane dividing while its warp
//    waits.
template <int T>
__device__ __forceinline__ float half_bits_to_float(uint32_t h) {
  if constexpr (T == kBF16) return __uint_as_float(h << 16);
  else return __half2float(__ushort_as_half(static_cast<unsigned short>(h)));
}
// (the pairs are register pairs: mov.b64 {lo, hi} costs no instruction)
__device__ __forceinline__ float2 mul2_rn(float2 a, float b) {
  float2 r;
  asm("{\n .reg .b64 x, y, z;\n mov.b64 x, {%2, %3};\n mov.b64 y, {%4, %4};\n mul.rn.f32x2 z, x, y;\n"
      " mov.b64 {%0, %1}, z;\n}"
      : "=f"(r.x), "=f"(r.y)
      : "f"(a.x), "f"(a.y), "f"(b));
  return r;
}
__device__ __forceinline__ float2 mul2_rn(float2 a, float2 b) {
  float2 r;
  asm("{\n .reg .b64 x, y, z;\n mov.b64 x, {%2, %3};\n mov.b64 y, {%4, %5};\n mul.rn.f32x2 z, x, y;\n"
      " mov.b64 {%0, %1}, z;\n}"
      : "=f"(r.x), "=f"(r.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return r;
}
template <int T>
__device__ __forceinline__ float2 unpack2(uint32_t w) {
  if constexpr (T == kBF16) return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xFFFF0000u));
  else return __half22float2(*reinterpret_cast<const __half2*>(&w));
}

// The scale byte and step of one block from its |max| (16-bit pattern): quant.py:1067-1107
// (NVFP4: e4m3(min(bmax / (outer * 6), 448)), step = value * outer; MXFP4: the e8m0 exponent
// rule of activations or weights).
template <int T, int FMT, int MODE>
__device__ __forceinline__ void fp4_block_scale(uint32_t bm, float s_outer, const Divisor& by6, uint32_t& sbyte,
                                                float& step) {
  const float bmax = half_bits_to_float<T>(bm);
  if constexpr (FMT == 0) {
    const float bmv[1] = {bmax};
    float ratio[1];
    quotients<kLowE4m3>(bmv, by6, ratio);
    sbyte = e4m3_byte(ratio[0]);
    step = __fmul_rn(e4m3_value_hw(static_cast<uint8_t>(sbyte)), s_outer);
  } else {
    const int e = MODE == 2 ? mxfp4_weight_exponent(bmax) : mxfp4_act_exponent(bmax);
    sbyte = static_cast<uint32_t>(e + 127);
    step = e8m0_value(static_cast<uint8_t>(sbyte));
  }
}

// e2m1 codes of one block's quotients t (NaN quotients of a block holding a NaN become 0).
template <int T, int BLOCK>
__device__ __forceinline__ void fp4_block_pack(float (&t)[BLOCK], uint32_t bm, uint32_t (&packed)[BLOCK / 8]) {
  constexpr uint32_t kHalfInf = T == kBF16 ? 0x7F80u : 0x7C00u;
  if (bm > kHalfInf) {
#pragma unroll
    for (int j = 0; j < BLOCK; ++j) t[j] = t[j] == t[j] ? t[j] : 0.0f;
  }
#pragma unroll
  for (int c = 0; c < BLOCK / 8; ++c) {
    float e8[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) e8[j] = t[c * 8 + j];
    packed[c] = e2m1x8(e8);
  }
}

// Two floats rounded to nearest even into one packed T word (low half: a): the hardware
// conversion of round_to_input, two at a time. A NaN comes out as the hardware's NaN.
template <int T>
__device__ __forceinline__ uint32_t pack2_rn(float a, float b) {
  uint32_t r;
  if constexpr (T == kBF16) {
    const __nv_bfloat162 p = __floats2bfloat162_rn(a, b);
    r = *reinterpret_cast<const uint32_t*>(&p);
  } else {
    const __half2 p = __floats2half2_rn(a, b);
    r = *reinterpret_cast<const uint32_t*>(&p);
  }
  return r;
}

// h = T(T(x * r) * w) of W packed words of x (two T values each) in place; wr: the weight's
// matching 16-byte chunks. The products are fp32 (two per mul.rn.f32x2), each rounded to T
// as round_to_input does (a NaN as the hardware's: block_absmax<NORM> then re-patterns it).
template <int T, int W>
__device__ __forceinline__ void norm_words(uint32_t (&v)[W], const uint4* __restrict__ wr, float r) {
#pragma unroll
  for (int c = 0; c < W / 4; ++c) {
    const uint4 wq = __ldg(wr + c);
    const uint32_t ww[4] = {wq.x, wq.y, wq.z, wq.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 a = mul2_rn(unpack2<T>(v[4 * c + i]), r);
      const uint32_t xr = pack2_rn<T>(a.x, a.y);
      const float2 p = mul2_rn(unpack2<T>(xr), unpack2<T>(ww[i]));
      v[4 * c + i] = pack2_rn<T>(p.x, p.y);
    }
  }
}

// |max| (16-bit pattern) of W packed words; with NORM, a block holding a NaN first gets the
// stored outputs' NaN pattern (f32_to_bf16_bits / f32_to_f16_bits of a NaN) in place, so its
// words equal those kab_rmsnorm writes.
template <int T, int W, bool NORM>
__device__ __forceinline__ uint32_t block_absmax(uint32_t (&v)[W]) {
  uint32_t m = 0;
#pragma unroll
  for (int j = 0; j < W; ++j) m = __vmaxu2(m, v[j] & 0x7FFF7FFFu);
  uint32_t bm = max(m & 0xFFFFu, m >> 16);
  const uint32_t inf = T == kBF16 ? 0x7F80u : 0x7C00u;
  if (NORM && bm > inf) {
#pragma unroll
    for (int j = 0; j < W; ++j) {
      uint32_t lo = v[j] & 0xFFFFu, hi = v[j] >> 16;
      if constexpr (T == kBF16) {
        if ((lo & 0x7FFFu) > inf) lo = f32_to_bf16_bits(__uint_as_float(0x7FC00000u));
        if ((hi & 0x7FFFu) > inf) hi = f32_to_bf16_bits(__uint_as_float(0x7FC00000u));
      } else {
        if ((lo & 0x7FFFu) > inf) lo = f32_to_f16_bits(__uint_as_float(0x7FC00000u));
        if ((hi & 0x7FFFu) > inf) hi = f32_to_f16_bits(__uint_as_float(0x7FC00000u));
      }
      v[j] = lo | (hi << 16);
    }
    m = 0;
#pragma unroll
    for (int j = 0; j < W; ++j) m = __vmaxu2(m, v[j] & 0x7FFF7FFFu);
    bm = max(m & 0xFFFFu, m >> 16);
  }
  return bm;
}

// (NVFP4 with up to two blocks per thread: at most 42 registers, six 256-thread CTAs per SM)
// NORM: the row is first RMSNorm'd (triton_fp4_producers.py:261-294). The blocks are loaded
// into registers and staged in shared memory, whence the sum of squares is taken in
// rmsnorm_rows_kernel's order (its 256 threads, emulated by any multiple of 32), so r and
// h = T(T(x * r) * w) are bit for bit the two-pass ones; h is quantised from registers (and
// written to hout [rows, k] when given); blocks redone with the IEEE division recompute
// their h from the staged x. Launched with k * 2 + (k / block) * 4 bytes of dynamic shared
// memory.
template <int T, int NB, int FMT, int MODE, bool NORM = false>
// (NVFP4 runs at 128 threads per row for most widths: capped at 64 registers with four blocks
// per thread and at 40 with one or two, more CTAs (rows) fit an SM, which keeps more rows'
// loads in flight: 46.4 vs 50.1 us on x [8192, 8192] bf16, and the fused RMSNorm producer 77.5
// vs 79.3 us on x [16384, 4096] bf16, one B200)
__global__ void __launch_bounds__(512, FMT == 0 ? (NB <= 2 ? 3 : 2) : 1)
quant_fp4_fast_kernel(const void* __restrict__ x, int64_t ldx, int64_t k, const float* __restrict__ amax_in,
                      const float* __restrict__ ts_in, int swizzle, uint8_t* __restrict__ q,
                      uint8_t* __restrict__ scales, float* __restrict__ outer_out,
                      const void* __restrict__ nw = nullptr, float eps = 0.0f, void* __restrict__ hout = nullptr) {
  __shared__ float red[32];
  // blocks whose quotients need the IEEE division, redone by the whole CTA after the row
  __shared__ int fix[kFp4MaxRowBlocks];
  __shared__ int nfix;
  extern __shared__ uint4 fp4_row_smem[];  // NORM: the row of x (k * 2 bytes), then its fix list
  constexpr int BLOCK = FMT == 0 ? 16 : 32;
  int* const fixp = NORM ? reinterpret_cast<int*>(fp4_row_smem + (k >> 3)) : fix;
  if (threadIdx.x == 0) nfix = 0;
  __syncthreads();
  constexpr int W = BLOCK / 2;  // packed words per block
  const int64_t row = blockIdx.x;
  const int nblk = static_cast<int>(k / BLOCK);
  const uint4* xr = reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(x) + row * ldx);
  uint32_t w[NB][W];
  uint32_t bm[NB];  // |max| of each block as a 16-bit pattern
  uint32_t am = 0;
#pragma unroll
  for (int b = 0; b < NB; ++b) {
    const int bi = threadIdx.x + b * blockDim.x;
    if (bi < nblk) {
#pragma unroll
      for (int c = 0; c < W / 4; ++c) {
        const uint4 r = __ldg(xr + static_cast<int64_t>(bi) * (W / 4) + c);
        w[b][4 * c] = r.x;
        w[b][4 * c + 1] = r.y;
        w[b][4 * c + 2] = r.z;
        w[b][4 * c + 3] = r.w;
        if constexpr (NORM) fp4_row_smem[bi * (W / 4) + c] = r;
      }
    } else {
#pragma unroll
      for (int j = 0; j < W; ++j) w[b][j] = 0;
    }
  }
  float r_norm = 1.0f;
  if constexpr (NORM) {
    // the sum of squares of rmsnorm_rows_kernel's 256 threads, from the staged row: virtual
    // thread v = tid + blockDim * u sums chunks v, v + 256, ... in turn; each warp's butterfly
    // per u is that of virtual warp v / 32 (blockDim is a multiple of 32)
    __syncthreads();
    const int lane = threadIdx.x & 31;
    const int chunks = static_cast<int>(k >> 3);
    for (int v0 = threadIdx.x - lane; v0 < 256; v0 += blockDim.x) {
      float ss = 0.0f;
      for (int c = v0 + lane; c < chunks; c += 256) {
        const uint4 q4 = fp4_row_smem[c];
        const uint32_t qw[4] = {q4.x, q4.y, q4.z, q4.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 f = unpack2<T>(qw[i]);
          ss = __fadd_rn(ss, __fmul_rn(f.x, f.x));
          ss = __fadd_rn(ss, __fmul_rn(f.y, f.y));
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, o));
      if (lane == 0) red[v0 >> 5] = ss;
    }
    __syncthreads();
    float tot = lane < 8 ? red[lane] : 0.0f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) tot = __fadd_rn(tot, __shfl_xor_sync(0xffffffffu, tot, o));
    r_norm = rsqrtf(__fadd_rn(__fdiv_rn(tot, static_cast<float>(k)), eps));
    __syncthreads();  // red is reused for the row's amax
#pragma unroll
    for (int b = 0; b < NB; ++b) {  // h = T(T(x * r) * w) in place, and into hout when given
      const int bi = threadIdx.x + b * blockDim.x;
      if (bi >= nblk) continue;
      norm_words<T, W>(w[b], reinterpret_cast<const uint4*>(nw) + static_cast<int64_t>(bi) * (W / 4), r_norm);
      bm[b] = block_absmax<T, W, true>(w[b]);
      if (hout != nullptr) {
        uint4* hr = reinterpret_cast<uint4*>(reinterpret_cast<uint16_t*>(hout) + row * k) +
                    static_cast<int64_t>(bi) * (W / 4);
#pragma unroll
        for (int c = 0; c < W / 4; ++c) hr[c] = make_uint4(w[b][4 * c], w[b][4 * c + 1], w[b][4 * c + 2], w[b][4 * c + 3]);
      }
    }
  }
#pragma unroll
  for (int b = 0; b < NB; ++b) {
    if constexpr (NORM) {
      if (threadIdx.x + b * blockDim.x >= nblk) bm[b] = 0;  // zero words
    } else {
      bm[b] = block_absmax<T, W, false>(w[b]);
    }
    am = max(am, bm[b]);
  }
  float s_outer = 1.0f;
  if constexpr (FMT == 0) {
    if constexpr (MODE == 0) {
      const float amax = block_amax(half_bits_to_float<T>(am), red);
      s_outer = amax > 0.0f ? __fmul_rn(amax, kNvfp4OuterStep) : 1.0f;  // quant.py:1104
    } else if constexpr (MODE == 1) {
      const float a = *amax_in;
      s_outer = a > 0.0f ? __fmul_rn(a, kNvfp4OuterStep) : 1.0f;
    } else {
      s_outer = *ts_in;
    }
  }
  if (threadIdx.x == 0 && outer_out != nullptr) outer_out[row] = s_outer;
  const Divisor by6(__fmul_rn(s_outer, 6.0f));
#pragma unroll
  for (int b = 0; b < NB; ++b) {
    const int bi = threadIdx.x + b * blockDim.x;
    if (bi >= nblk) continue;
    uint32_t sbyte;
    float step;
    fp4_block_scale<T, FMT, MODE>(bm[b], s_outer, by6, sbyte, step);
    const float div = (MODE == 2 && step < 1e-38f) ? 1e-38f : step;
    uint32_t packed[BLOCK / 8];
#pragma unroll
    for (int c = 0; c < BLOCK / 8; ++c) packed[c] = 0;
    if (step > 0.0f) {
      // The codes of v * y(1 + 2^-19) and of v * y(1 - 2^-19) bracket those of the IEEE
      // quotient RN(v / step): y, the hardware reciprocal, is within 2^-22 of 1 / step, so the
      // two products lie on either side of v / step and of its rounding, and the e2m1 rounding
      // is monotonic. Where both give the same codes, those are the quotient's codes; a block
      // where they differ (a quotient within about 2^-19 of an e2m1 midpoint), or whose
      // divisor has no normal reciprocal, keeps provisional codes and is redone with the IEEE
      // division after the row, with all lanes busy.
      const Divisor d(div);
      const float y_hi = __fmul_rn(d.y, 1.0f + 0x1p-19f), y_lo = __fmul_rn(d.y, 1.0f - 0x1p-19f);
      constexpr uint32_t kHalfInf = T == kBF16 ? 0x7F80u : 0x7C00u;
      const bool has_nan = bm[b] > kHalfInf;  // its NaN quotients become 0
      bool agree = d.fast;
#pragma unroll
      for (int c = 0; c < BLOCK / 8; ++c) {
        float eh[8], el[8];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 v = unpack2<T>(w[b][4 * c + j]);
          const float2 ph = mul2_rn(v, y_hi), pl = mul2_rn(v, y_lo);
          eh[2 * j] = ph.x;
          eh[2 * j + 1] = ph.y;
          el[2 * j] = pl.x;
          el[2 * j + 1] = pl.y;
        }
        if (has_nan) {
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            eh[j] = eh[j] == eh[j] ? eh[j] : 0.0f;
            el[j] = el[j] == el[j] ? el[j] : 0.0f;
          }
        }
        packed[c] = e2m1x8(eh);
        agree = agree && packed[c] == e2m1x8(el);
      }
      if (!agree) fixp[atomicAdd(&nfix, 1)] = bi;
    }
    uint8_t* dst = q + row * (k >> 1) + static_cast<int64_t>(bi) * (BLOCK / 2);
    if constexpr (BLOCK == 16) *reinterpret_cast<uint2*>(dst) = make_uint2(packed[0], packed[1]);
    else *reinterpret_cast<uint4*>(dst) = make_uint4(packed[0], packed[1], packed[2], packed[3]);
    const int64_t off = swizzle ? scale_offset_swizzled(row, bi, nblk) : row * nblk + bi;
    scales[off] = static_cast<uint8_t>(sbyte);
  }
  __syncthreads();  // every provisional code is written and the list is complete
  const int nf = nfix;
  for (int i = threadIdx.x; i < nf; i += blockDim.x) {
    const int bi = fixp[i];
    uint32_t wv[W];
#pragma unroll
    for (int c = 0; c < W / 4; ++c) {
      const uint4 r = NORM ? fp4_row_smem[bi * (W / 4) + c] : __ldg(xr + static_cast<int64_t>(bi) * (W / 4) + c);
      wv[4 * c] = r.x;
      wv[4 * c + 1] = r.y;
      wv[4 * c + 2] = r.z;
      wv[4 * c + 3] = r.w;
    }
    if constexpr (NORM) norm_words<T, W>(wv, reinterpret_cast<const uint4*>(nw) + static_cast<int64_t>(bi) * (W / 4), r_norm);
    const uint32_t bmi = block_absmax<T, W, NORM>(wv);
    uint32_t sbyte;
    float step;
    fp4_block_scale<T, FMT, MODE>(bmi, s_outer, by6, sbyte, step);
    const float div = (MODE == 2 && step < 1e-38f) ? 1e-38f : step;
    float t[BLOCK];
#pragma unroll
    for (int j = 0; j < W; ++j) {
      const float2 v = unpack2<T>(wv[j]);
      t[2 * j] = __fdiv_rn(v.x, div);
      t[2 * j + 1] = __fdiv_rn(v.y, div);
    }
    uint32_t packed[BLOCK / 8];
    fp4_block_pack<T, BLOCK>(t, bmi, packed);
    uint8_t* dst = q + row * (k >> 1) + static_cast<int64_t>(bi) * (BLOCK / 2);
    if constexpr (BLOCK == 16) *reinterpret_cast<uint2*>(dst) = make_uint2(packed[0], packed[1]);
    else *reinterpret_cast<uint4*>(dst) = make_uint4(packed[0], packed[1], packed[2], packed[3]);
  }
}

// ------------------------------------------------------------------ RMSNorm

// The RMSNorm of the fused producers (triton_fp8_producers.py:120-133,
// triton_fp4_producers.py:261-294; the arithmetic of Llama / Qwen / Mistral RMSNorm): per row
// r = rsqrt(sum(x^2) / k + eps) in fp32 (squares and sum each rounded, the sum as a tree),
// h = T(T(x * r) * w) in x's dtype T, written to h [rows, k]. One CTA per row: the sum of
// squares over 16-byte chunks and a block reduction, then a second read of the row (from L2)
// for h. The quantisers then read h, so the codes are exactly those of h.
template <int T>
__global__ void __launch_bounds__(256)
rmsnorm_rows_kernel(const void* __restrict__ x, int64_t ldx, int64_t k, const void* __restrict__ w, float eps,
                    void* __restrict__ h) {
  __shared__ float red[32];
  const int64_t row = blockIdx.x;
  const int64_t chunks = k >> 3;
  float ss = 0.0f;
  for (int64_t c = threadIdx.x; c < chunks; c += blockDim.x) {
    float v[8];
    load8<T>(x, row * ldx + c * 8, v);
#pragma unroll
    for (int j = 0; j < 8; ++j) ss = __fadd_rn(ss, __fmul_rn(v[j], v[j]));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, o));
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = (blockDim.x + 31) >> 5;
  if (lane == 0) red[warp] = ss;
  __syncthreads();
  float tot = lane < nwarps ? red[lane] : 0.0f;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) tot = __fadd_rn(tot, __shfl_xor_sync(0xffffffffu, tot, o));
  const float r = rsqrtf(__fadd_rn(__fdiv_rn(tot, static_cast<float>(k)), eps));
  for (int64_t c = threadIdx.x; c < chunks; c += blockDim.x) {
    float v[8], wv[8], o8[8];
    load8<T>(x, row * ldx + c * 8, v);
    load8<T>(w, c * 8, wv);
#pragma unroll
    for (int j = 0; j < 8; ++j) o8[j] = round_to_input<T>(__fmul_rn(round_to_input<T>(__fmul_rn(v[j], r)), wv[j]));
    store_h8<T>(h, row * k + c * 8, o8);
  }
}

// RMSNorm then FP8 in one pass over x (triton_fp8_producers.py:120-133, 191-202), launched
// for fp32 rows (2-byte rows: rmsnorm_quant_fp8_packed_kernel below): one CTA of 256 threads
// per row; the row's chunks stay in registers (MAXC per thread) from the sum of
// squares, taken in rmsnorm_rows_kernel's order so that r and h are bit for bit the two-pass
// ones, to the codes. MX 0: e4m3 per token (quant.py:361-377: scale amax / 448, 1 for a zero
// row); MX 1: MXFP8 (quant.py:479-526: the ceil rule's e8m0 per 32, four lanes per block),
// scales row-major or swizzled. h (nullable): the norm's output.
template <int T, int MAXC, int MX>
__global__ void __launch_bounds__(256, MAXC <= 2 ? 8 : MAXC <= 4 ? 4 : 2)
rmsnorm_quant_fp8_kernel(const void* __restrict__ x, int64_t ldx, int64_t k, const void* __restrict__ w, float eps,
                         int swizzle, uint8_t* __restrict__ q, void* __restrict__ scales, void* __restrict__ h) {
  __shared__ float red[32];
  const int64_t row = blockIdx.x;
  const int64_t chunks = k >> 3;
  float v[MAXC][8];
  float ss = 0.0f;
#pragma unroll
  for (int c = 0; c < MAXC; ++c) {
    const int64_t ci = threadIdx.x + static_cast<int64_t>(c) * 256;
    if (ci < chunks) {
      load8<T>(x, row * ldx + ci * 8, v[c]);
#pragma unroll
      for (int j = 0; j < 8; ++j) ss = __fadd_rn(ss, __fmul_rn(v[c][j], v[c][j]));
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, o));
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) red[warp] = ss;
  __syncthreads();
  float tot = lane < 8 ? red[lane] : 0.0f;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) tot = __fadd_rn(tot, __shfl_xor_sync(0xffffffffu, tot, o));
  const float r = rsqrtf(__fadd_rn(__fdiv_rn(tot, static_cast<float>(k)), eps));
  __syncthreads();  // red is reused below
  uint32_t abits = 0;
#pragma unroll
  for (int c = 0; c < MAXC; ++c) {
    const int64_t ci = threadIdx.x + static_cast<int64_t>(c) * 256;
    if (ci < chunks) {
      float wv[8];
      load8<T>(w, ci * 8, wv);
#pragma unroll
      for (int j = 0; j < 8; ++j)
        v[c][j] = round_to_input<T>(__fmul_rn(round_to_input<T>(__fmul_rn(v[c][j], r)), wv[j]));
      if (h != nullptr) store_h8<T>(h, row * k + ci * 8, v[c]);
      if constexpr (MX == 0) abits = abs_bits_max8(v[c], abits);
    }
  }
  if constexpr (MX == 0) {
    const float amax = block_amax(__uint_as_float(abits), red);
    const float sc = amax > 0.0f ? __fdiv_rn(amax, kFp8Max) : 1.0f;  // quant.py:374-375
    if (threadIdx.x == 0) reinterpret_cast<float*>(scales)[row] = sc;
    const Divisor div(sc);
#pragma unroll
    for (int c = 0; c < MAXC; ++c) {
      const int64_t ci = threadIdx.x + static_cast<int64_t>(c) * 256;
      if (ci < chunks) {
        *reinterpret_cast<uint2*>(q + row * k + ci * 8) = e4m3x8_quotients(v[c], div);
      }
    }
  } else {
#pragma unroll
    for (int c = 0; c < MAXC; ++c) {  // every lane of a block of 32 runs the same iterations
      const int64_t ci = threadIdx.x + static_cast<int64_t>(c) * 256;
      const bool live = ci < chunks;
      uint32_t b = live ? abs_bits_max8(v[c], 0u) : 0u;
      b = max(b, __shfl_xor_sync(0xffffffffu, b, 1));
      b = max(b, __shfl_xor_sync(0xffffffffu, b, 2));
      if (live) {
        const int e = mx_exponent(__uint_as_float(b), 0);
        const float inv = pow2_neg(e);
        float qv[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) qv[i] = __fmul_rn(v[c][i], inv);
        *reinterpret_cast<uint2*>(q + row * k + ci * 8) = e4m3x8(qv);
        if ((ci & 3) == 0) {
          const int64_t cols = k >> 5, col = ci >> 2;
          const int64_t off = swizzle ? scale_offset_swizzled(row, col, cols) : row * cols + col;
          reinterpret_cast<uint8_t*>(scales)[off] = static_cast<uint8_t>(e + 127);
        }
      }
    }
  }
}

// The same producer for bf16 / fp16 rows with NT threads per row (a divisor of 256) and NC
// 16-byte chunks each, kept packed (two values per register): more rows resident per SM.
// Thread t holds chunks t + NT * c, which are exactly the chunks of rmsnorm_rows_kernel's
// threads t + NT * u (u < 256 / NT, c = u + (256 / NT) * i), so the sum of squares is taken
// per such virtual thread in its order and reduced per virtual warp: r and h are bit for bit
// the two-pass ones. The norm is norm_words' packed arithmetic, a NaN re-patterned as stored.
template <int T, int NC, int MX, int NT>
__global__ void __launch_bounds__(NT)
rmsnorm_quant_fp8_packed_kernel(const void* __restrict__ x, int64_t ldx, int64_t k, const void* __restrict__ w,
                                float eps, int swizzle, uint8_t* __restrict__ q, void* __restrict__ scales,
                                void* __restrict__ h) {
  static_assert(T != kF32 && NT % 32 == 0 && 256 % NT == 0, "2-byte rows; NT divides 256");
  constexpr int U = 256 / NT;  // virtual threads per thread
  __shared__ float red[32];
  const int64_t row = blockIdx.x;
  const int chunks = static_cast<int>(k >> 3);
  const uint4* xr = reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(x) + row * ldx);
  uint32_t v[NC][4];
#pragma unroll
  for (int c = 0; c < NC; ++c) {
    const int ci = threadIdx.x + c * NT;
    if (ci < chunks) {
      const uint4 r = __ldg(xr + ci);
      v[c][0] = r.x; v[c][1] = r.y; v[c][2] = r.z; v[c][3] = r.w;
    } else {
      v[c][0] = v[c][1] = v[c][2] = v[c][3] = 0u;
    }
  }
  float ss[U];
#pragma unroll
  for (int u = 0; u < U; ++u) ss[u] = 0.0f;
#pragma unroll
  for (int c = 0; c < NC; ++c) {
    if (threadIdx.x + c * NT < chunks) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = unpack2<T>(v[c][i]);
        ss[c % U] = __fadd_rn(ss[c % U], __fmul_rn(f.x, f.x));
        ss[c % U] = __fadd_rn(ss[c % U], __fmul_rn(f.y, f.y));
      }
    }
  }
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int u = 0; u < U; ++u) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss[u] = __fadd_rn(ss[u], __shfl_xor_sync(0xffffffffu, ss[u], o));
    if (lane == 0) red[warp + (NT / 32) * u] = ss[u];
  }
  __syncthreads();
  float tot = lane < 8 ? red[lane] : 0.0f;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) tot = __fadd_rn(tot, __shfl_xor_sync(0xffffffffu, tot, o));
  const float r = rsqrtf(__fadd_rn(__fdiv_rn(tot, static_cast<float>(k)), eps));
  uint32_t abits = 0;
  const uint4* wr = reinterpret_cast<const uint4*>(w);
#pragma unroll
  for (int c = 0; c < NC; ++c) {
    const int ci = threadIdx.x + c * NT;
    if (ci < chunks) {
      norm_words<T, 4>(v[c], wr + ci, r);
      const uint32_t bm = block_absmax<T, 4, true>(v[c]);
      if (h != nullptr)
        reinterpret_cast<uint4*>(reinterpret_cast<uint16_t*>(h) + row * k)[ci] = make_uint4(v[c][0], v[c][1], v[c][2], v[c][3]);
      if constexpr (MX == 0) abits = max(abits, __float_as_uint(half_bits_to_float<T>(bm)) & 0x7FFFFFFFu);
    }
  }
  auto values = [&](int c, float (&f)[8]) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 p = unpack2<T>(v[c][i]);
      f[2 * i] = p.x;
      f[2 * i + 1] = p.y;
    }
  };
  if constexpr (MX == 0) {
    const float amax = block_amax(__uint_as_float(abits), red);  // (syncs before reusing red)
    const float sc = amax > 0.0f ? __fdiv_rn(amax, kFp8Max) : 1.0f;  // quant.py:374-375
    if (threadIdx.x == 0) reinterpret_cast<float*>(scales)[row] = sc;
    const Divisor div(sc);
#pragma unroll
    for (int c = 0; c < NC; ++c) {
      const int ci = threadIdx.x + c * NT;
      if (ci < chunks) {
        float f[8];
        values(c, f);
        *reinterpret_cast<uint2*>(q + row * k + static_cast<int64_t>(ci) * 8) = e4m3x8_quotients(f, div);
      }
    }
  } else {
#pragma unroll
    for (int c = 0; c < NC; ++c) {  // every lane of a block of 32 runs the same iterations
      const int ci = threadIdx.x + c * NT;
      const bool live = ci < chunks;
      uint32_t b = live ? __float_as_uint(half_bits_to_float<T>(block_absmax<T, 4, false>(v[c]))) & 0x7FFFFFFFu : 0u;
      b = max(b, __shfl_xor_sync(0xffffffffu, b, 1));
      b = max(b, __shfl_xor_sync(0xffffffffu, b, 2));
      if (live) {
        const int e = mx_exponent(__uint_as_float(b), 0);
        const float inv = pow2_neg(e);
        float f[8], qv[8];
        values(c, f);
#pragma unroll
        for (int i = 0; i < 8; ++i) qv[i] = __fmul_rn(f[i], inv);
        *reinterpret_cast<uint2*>(q + row * k + static_cast<int64_t>(ci) * 8) = e4m3x8(qv);
        if ((ci & 3) == 0) {
          const int64_t cols = k >> 5, col = ci >> 2;
          const int64_t off = swizzle ? scale_offset_swizzled(row, col, cols) : row * cols + col;
          reinterpret_cast<uint8_t*>(scales)[off] = static_cast<uint8_t>(e + 127);
        }
      }
    }
  }
}

// ------------------------------------------------------------------ global amax

// NaN-keeping max |x| of a [rows, k] matrix into *out (which holds 0 before the launch):
// non-negative floats order like their bits, and a NaN (0x7FC00000) beats +inf.
template <int T>
__global__ void __launch_bounds__(256)
amax_kernel(const void* __restrict__ x, int64_t ldx, int64_t rows, int64_t k, float* out) {
  __shared__ float red[32];
  float amax = 0.0f;
  const int64_t total = rows * k;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total; i += stride) {
    const int64_t r = i / k, c = i % k;
    amax = amax_step(amax, load_elem<T>(x, r * ldx + c));
  }
  amax = block_amax(amax, red);
  if (threadIdx.x == 0) {
    const uint32_t bits = amax != amax ? 0x7FC00000u : __float_as_uint(amax);
    atomicMax(reinterpret_cast<unsigned int*>(out), bits);
  }
}

// tensor_scale = fp32(double(amax) / (6 * 448)), 1 for a zero amax (quant.py:253-254).
__global__ void fp4_tensor_scale_kernel(const float* amax, float* ts) {
  const float a = *amax;
  *ts = a > 0.0f ? __double2float_rn(static_cast<double>(a) / 2688.0) : 1.0f;
}

// quant.py:479-495 mx_scale_exponents over a vector of block maxima.
__global__ void mx_exponents_kernel(const float* __restrict__ amax, int64_t n, int rule,
                                    int* __restrict__ out) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    out[i] = mx_exponent(amax[i], rule);
}

// ------------------------------------------------------------------ layout helpers

// quant.py:550-564: [rows, cols] bytes -> the flat 128 x 4 blocked layout (padding written
// as 0 by the caller's zeroed buffer).
__global__ void swizzle_scales_kernel(const uint8_t* __restrict__ s, int64_t rows, int64_t cols,
                                      uint8_t* __restrict__ out) {
  const int64_t total = rows * cols;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / cols, c = i % cols;
    out[scale_offset_swizzled(r, c, cols)] = s[i];
  }
}

// Exact fp32 values e2m1 * block scale [rows, K] of packed FP4 codes (quant.py:1110-1114).
__global__ void fp4_values_kernel(const uint8_t* __restrict__ codes, const uint8_t* __restrict__ scales,
                                  int64_t rows, int64_t k, int fmt, float* __restrict__ out) {
  const int block = fmt == 0 ? 16 : 32;
  const int64_t total = rows * k;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / k, c = i % k;
    const uint8_t byte = codes[r * (k >> 1) + (c >> 1)];
    const uint32_t code = (c & 1) ? (byte >> 4) : (byte & 0xF);
    const uint32_t idx = code & 7;
    const float mag = idx <= 4 ? 0.5f * static_cast<float>(idx) : static_cast<float>(idx - 2) + (idx == 7 ? 1.0f : 0.0f);
    const float v = (code & 8) ? -mag : mag;
    const uint8_t sb = scales[r * (k / block) + c / block];
    const float s = fmt == 0 ? e4m3_value(sb) : e8m0_value(sb);
    out[i] = __fmul_rn(v, s);
  }
}

// e2m1 code (sign in bit 3) -> its value.
__device__ __forceinline__ float e2m1_value(uint32_t code) {
  const uint32_t idx = code & 7;
  const float mag = idx <= 4 ? 0.5f * static_cast<float>(idx) : static_cast<float>(idx - 2) + (idx == 7 ? 1.0f : 0.0f);
  return (code & 8) ? -mag : mag;
}

// Block-diagonal Walsh-Hadamard rotation (quant.py:1150-1173 hadamard_rotate): every `block`
// consecutive elements of a row times the orthonormal Sylvester-Hadamard matrix, in fp32 (the
// butterflies of H x, then one multiplication by fp32(1 / sqrt(block))). One CTA per row, the
// row in shared memory; out fp32 [rows, k].
template <int T>
__global__ void __launch_bounds__(512)
hadamard_rotate_kernel(const void* __restrict__ x, int64_t ldx, int64_t k, int block, float inv_sqrt,
                       float* __restrict__ out) {
  extern __shared__ float hrow[];
  const int64_t r = blockIdx.x;
  for (int64_t i = threadIdx.x; i < k; i += blockDim.x) hrow[i] = load_elem<T>(x, r * ldx + i);
  __syncthreads();
  for (int h = 1; h < block; h <<= 1) {
    for (int64_t p = threadIdx.x; p < k / 2; p += blockDim.x) {
      const int64_t i = (p / h) * (2 * h) + (p % h);  // the pair (i, i + h) of one block
      const float a = hrow[i], b = hrow[i + h];
      hrow[i] = __fadd_rn(a, b);
      hrow[i + h] = __fsub_rn(a, b);
    }
    __syncthreads();
  }
  for (int64_t i = threadIdx.x; i < k; i += blockDim.x) out[r * k + i] = __fmul_rn(hrow[i], inv_sqrt);
}

// quant.py:1117-1148 fp4_bias_correction: per row c = sum x^2 / sum x x^ (float64 sums) with
// x^ = e2m1 * scale * outer; 1 when sum x x^ is not positive or c is not finite. One CTA per
// row; scales [rows, k / block] bytes, row-major or swizzled; outer per row, one value or null.
template <int T>
__global__ void __launch_bounds__(256)
fp4_bias_correction_kernel(const void* __restrict__ x, int64_t ldx, int64_t k, const uint8_t* __restrict__ codes,
                           const uint8_t* __restrict__ scales, int fmt, int swizzled, const float* __restrict__ outer,
                           int outer_per_row, float* __restrict__ out) {
  __shared__ double red[2][32];
  const int64_t r = blockIdx.x;
  const int block = fmt == 0 ? 16 : 32;
  const int64_t cols = k / block;
  const double o = outer == nullptr ? 1.0 : static_cast<double>(outer[outer_per_row ? r : 0]);
  double num = 0.0, den = 0.0;
  for (int64_t i = threadIdx.x; i < k; i += blockDim.x) {
    const double a = load_elem<T>(x, r * ldx + i);
    const uint8_t byte = codes[r * (k >> 1) + (i >> 1)];
    const uint32_t code = (i & 1) ? (byte >> 4) : (byte & 0xF);
    const int64_t c = i / block;
    const uint8_t sb = scales[swizzled ? scale_offset_swizzled(r, c, cols) : r * cols + c];
    const float s = fmt == 0 ? e4m3_value(sb) : e8m0_value(sb);
    const double xh = static_cast<double>(__fmul_rn(e2m1_value(code), s)) * o;
    num += a * a;
    den += a * xh;
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    num += __shfl_xor_sync(0xffffffffu, num, off);
    den += __shfl_xor_sync(0xffffffffu, den, off);
  }
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) { red[0][warp] = num; red[1][warp] = den; }
  __syncthreads();
  if (threadIdx.x == 0) {
    double n = 0.0, d = 0.0;
    for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) { n += red[0][w]; d += red[1][w]; }
    const double cval = n / fmax(d, 1e-300);
    out[r] = (d > 0.0 && isfinite(cval)) ? static_cast<float>(cval) : 1.0f;
  }
}

}  // namespace kab
