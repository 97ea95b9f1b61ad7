// Scale-rule checks of block-scaled activations (the evaluator's scale guard): one reduction
// pass over x and its block scales, counting the blocks each rule of kernel-agent's
// src/kernel_agent/kernels/quant.py flags and the largest block-max / step ratio.
//
//  * mxfp8_saturation_kernel: quant.py:623-660 (saturated, coarser, not_pow2, worst_ratio);
//  * fp4_scale_check_kernel:  quant.py:1325-1416 (saturated, underflow, nonfinite,
//    not_representable, coarser, worst_ratio) for NVFP4 (FMT 0) and MXFP4 (FMT 1).
//
// One thread per scale block; counts are summed per warp and added to the result with one
// 64-bit atomic per warp and count; the worst ratio (>= 0, NaN kept as the largest) with an
// atomic max of its bits.
#pragma once

#include "quant.cuh"

namespace kab {

constexpr float kMxSaturationLimit = 448.4375f;      // 448 * (1 + 2^-10), exact
constexpr float kNvfp4RoundingRatio = 6.375f;        // 6 * (1 + 2^-4), quant.py:1291
constexpr float kFp4SlackFactor = 1.0009765625f;     // 1 + 2^-10, quant.py:1294
constexpr float kLowTieFactor = 0.99999904632568359375f;  // fp32(1 - 2^-20)
constexpr float kE4m3MinNormal = 0.015625f;          // 2^-6
constexpr float kFp4PlainLimit = 6.0000057220458984375f;  // fp32(6 * (1 + 2^-20)), exact

__device__ __forceinline__ void check_add(unsigned long long* dst, unsigned v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  if ((threadIdx.x & 31) == 0 && v) atomicAdd(dst, static_cast<unsigned long long>(v));
}
__device__ __forceinline__ void check_max(unsigned* dst, float ratio) {
  uint32_t b = ratio != ratio ? 0x7FC00000u : __float_as_uint(ratio);  // ratio >= 0 or NaN
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) b = max(b, __shfl_xor_sync(0xffffffffu, b, o));
  if ((threadIdx.x & 31) == 0) atomicMax(dst, b);
}

// NaN-keeping max |x| of the BLOCK elements of block (row, col), as a float.
template <int T, int BLOCK>
__device__ __forceinline__ float block_max_of(const void* x, int64_t ldx, int64_t row, int64_t col) {
  uint32_t m = 0;
#pragma unroll
  for (int c = 0; c < BLOCK / 8; ++c) {
    float v[8];
    load8<T>(x, row * ldx + col * BLOCK + c * 8, v);
    m = abs_bits_max8(v, m);
  }
  return __uint_as_float(m);
}

// quant.py:623-660. `step`: fp32 scale values [rows, nb].
template <int T>
__global__ void __launch_bounds__(256)
mxfp8_saturation_kernel(const void* __restrict__ x, int64_t ldx, int64_t rows, int64_t nb,
                        const float* __restrict__ step, KabScaleCheck* out) {
  const int64_t total = rows * nb;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  unsigned saturated = 0, coarser = 0, not_pow2 = 0;
  float worst = 0.0f;
  for (int64_t base = blockIdx.x * static_cast<int64_t>(blockDim.x); base < total; base += stride) {
    const int64_t i = base + threadIdx.x;
    if (i < total) {
      const int64_t row = i / nb, col = i - row * nb;
      const float amax = block_max_of<T, 32>(x, ldx, row, col);
      const float s = step[i];
      int ex;
      bool half;
      frexp_parts(s, ex, half);
      not_pow2 += (!half && s > 0.0f) ? 1u : 0u;
      const float ratio = amax > 0.0f ? __fdiv_rn(amax, s != s ? s : fmaxf(s, 1e-38f)) : 0.0f;
      saturated += (ratio > kMxSaturationLimit || (s <= 0.0f && amax > 0.0f)) ? 1u : 0u;
      if (amax > 0.0f) {
        const int e = mx_exponent(amax, 0);
        coarser += (static_cast<double>(s) > ldexp(1.0, e)) ? 1u : 0u;
      }
      worst = (ratio > worst || ratio != ratio) ? ratio : worst;
    }
  }
  check_add(&out->saturated, saturated);
  check_add(&out->coarser, coarser);
  check_add(&out->not_pow2, not_pow2);
  check_max(&out->worst_ratio_bits, worst);
}

// quant.py:1325-1416. `scale`: fp32 block-scale values [rows, nb]; `outer`: [rows] or one
// value (outer_per_row 0), or null for 1.
template <int T, int FMT>
__global__ void __launch_bounds__(256)
fp4_scale_check_kernel(const void* __restrict__ x, int64_t ldx, int64_t rows, int64_t nb,
                       const float* __restrict__ scale, const float* __restrict__ outer, int outer_per_row,
                       KabScaleCheck* out) {
  constexpr int BLOCK = FMT == 0 ? 16 : 32;
  const int64_t total = rows * nb;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  unsigned saturated = 0, underflow = 0, nonfinite = 0, not_repr = 0, coarser = 0, plain = 0;
  float worst = 0.0f;
  for (int64_t base = blockIdx.x * static_cast<int64_t>(blockDim.x); base < total; base += stride) {
    const int64_t i = base + threadIdx.x;
    if (i < total) {
      const int64_t row = i / nb, col = i - row * nb;
      const float bmax = block_max_of<T, BLOCK>(x, ldx, row, col);
      const float s = scale[i];
      const float o = outer == nullptr ? 1.0f : outer[outer_per_row ? row : 0];
      const bool finite = isfinite(s) && isfinite(o) && o > 0.0f;
      const float step = finite ? __fmul_rn(s, o) : 0.0f;
      const bool live = finite && bmax > 0.0f;
      const float ratio = (live && step > 0.0f) ? __fdiv_rn(bmax, fmaxf(step, 1e-38f)) : 0.0f;
      const bool zero = live && step <= 0.0f;
      float bound;
      bool representable;
      if constexpr (FMT == 0) {
        const float safe = finite ? o : 1.0f;
        const float r = __fdiv_rn(bmax, __fmul_rn(safe, 6.0f));
        const float rn = e4m3_value_hw(e4m3_byte(min_keep_nan(r, 448.0f)));
        const float rn_low = e4m3_value_hw(e4m3_byte(min_keep_nan(__fmul_rn(r, kLowTieFactor), 448.0f)));
        bound = kNvfp4RoundingRatio;
#pragma unroll
        for (int t = 0; t < 2; ++t) {  // a subnormal scale's own rounding error
          const float ref = t == 0 ? rn : rn_low;
          const float ref_ratio = __fdiv_rn(bmax, fmaxf(__fmul_rn(ref, safe), 1e-38f));
          if (ref > 0.0f && ref < kE4m3MinNormal) bound = fmaxf(bound, ref_ratio);
        }
        underflow += (zero && rn_low > 0.0f) ? 1u : 0u;
        representable = e4m3_value_hw(e4m3_byte(s)) == s;
        coarser += (live && s > rn) ? 1u : 0u;
      } else {
        bound = 6.0f;
        underflow += zero ? 1u : 0u;
        int ex;
        bool half;
        frexp_parts(s, ex, half);
        representable = half && s > 0.0f;
        frexp_parts(bmax, ex, half);
        const float mant = bmax == 0.0f ? 0.0f : (isfinite(bmax) ? ldexpf(bmax, -ex) : bmax);  // frexp(inf) = inf
        const int c = ex - 3 + (mant > 0.75f ? 1 : 0);
        coarser += (live && s > __double2float_rn(ldexp(1.0, c))) ? 1u : 0u;
      }
      saturated += (live && ratio > __fmul_rn(bound, kFp4SlackFactor)) ? 1u : 0u;
      plain += ratio > kFp4PlainLimit ? 1u : 0u;  // quant.py:1290: ratio > 6 * (1 + 2^-20)
      nonfinite += finite ? 0u : 1u;
      not_repr += (finite && !representable) ? 1u : 0u;
      worst = (ratio > worst || ratio != ratio) ? ratio : worst;
    }
  }
  check_add(&out->saturated, saturated);
  check_add(&out->underflow, underflow);
  check_add(&out->nonfinite, nonfinite);
  check_add(&out->not_representable, not_repr);
  check_add(&out->coarser, coarser);
  check_add(&out->saturated_plain, plain);
  check_max(&out->worst_ratio_bits, worst);
}

// ------------------------------------------------------------------ error-report sums

__device__ __forceinline__ float to_float(float v) { return v; }
__device__ __forceinline__ float to_float(__nv_bfloat16 v) { return __bfloat162float(v); }
__device__ __forceinline__ float to_float(__half v) { return __half2float(v); }

// One CTA per row of a pair (x, y): float64 sums of x^2, y^2, (x - y)^2 and x * y, the NaN-
// keeping maxima of |x| and |y|, and the counts of x != 0 and of x != 0 with y == 0
// (quant.py:302-326 _error_metrics and the activation / output reports built on it).
template <typename TX, typename TY>
__global__ void __launch_bounds__(256)
row_pair_stats_kernel(const TX* __restrict__ x, int64_t ldx, const TY* __restrict__ y, int64_t ldy, int64_t k,
                      double* __restrict__ out) {
  __shared__ double sred[8][6];
  __shared__ uint32_t mred[8][2];
  const int64_t row = blockIdx.x;
  const TX* xr = x + row * ldx;
  const TY* yr = y + row * ldy;
  double sx = 0.0, sy = 0.0, sd = 0.0, sxy = 0.0, nz = 0.0, fl = 0.0;
  uint32_t mx = 0, my = 0;
  for (int64_t c = threadIdx.x; c < k; c += blockDim.x) {
    const float a = to_float(xr[c]), bb = to_float(yr[c]);
    const double da = a, db = bb;
    sx += da * da;
    sy += db * db;
    sd += (da - db) * (da - db);
    sxy += da * db;
    nz += a != 0.0f ? 1.0 : 0.0;
    fl += (a != 0.0f && bb == 0.0f) ? 1.0 : 0.0;
    mx = max(mx, __float_as_uint(a) & 0x7FFFFFFFu);
    my = max(my, __float_as_uint(bb) & 0x7FFFFFFFu);
  }
  double v[6] = {sx, sy, sd, sxy, nz, fl};
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
#pragma unroll
    for (int i = 0; i < 6; ++i) v[i] += __shfl_xor_sync(0xffffffffu, v[i], o);
    mx = max(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    my = max(my, __shfl_xor_sync(0xffffffffu, my, o));
  }
  const int w = threadIdx.x >> 5;
  if ((threadIdx.x & 31) == 0) {
#pragma unroll
    for (int i = 0; i < 6; ++i) sred[w][i] = v[i];
    mred[w][0] = mx;
    mred[w][1] = my;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const int nw = blockDim.x >> 5;
    double t[6] = {0, 0, 0, 0, 0, 0};
    uint32_t ax = 0, ay = 0;
    for (int i = 0; i < nw; ++i) {
#pragma unroll
      for (int j = 0; j < 6; ++j) t[j] += sred[i][j];
      ax = max(ax, mred[i][0]);
      ay = max(ay, mred[i][1]);
    }
    double* o = out + row * 8;
    o[0] = t[0];
    o[1] = t[1];
    o[2] = t[2];
    o[3] = t[3];
    o[4] = __uint_as_float(ax);
    o[5] = t[4];
    o[6] = t[5];
    o[7] = __uint_as_float(ay);
  }
}

}  // namespace kab

namespace kab {

// Outlier statistics of activations x [rows, k] (the scale guard's report,
// src/kernel_agent/kernels/scale_guard.py:103-118), one pass over x with non-finite values
// taken as 0: per row the sum of squares (float64) and the largest |x|; per column the
// largest |x|. A CTA covers kOutlierRows rows x 2048 columns (256 threads x 8 columns): each
// thread keeps the maxima of its 8 columns over the rows and adds them with one atomic max
// per column; the row partials are reduced over the CTA (warp shuffles, then shared memory)
// and added with one atomic per row. Maxima are non-negative floats, so their bit patterns
// order like the values and an unsigned atomic max is the float max. The outputs start at 0.
constexpr int kOutlierRows = 32;

template <int T>
__global__ void __launch_bounds__(256)
outlier_stats_kernel(const void* __restrict__ x, int64_t ldx, int64_t rows, int64_t k,
                     double* __restrict__ row_sumsq, unsigned* __restrict__ row_amax,
                     unsigned* __restrict__ col_amax) {
  __shared__ double s_sum[8][kOutlierRows];
  __shared__ unsigned s_max[8][kOutlierRows];
  const int64_t r0 = static_cast<int64_t>(blockIdx.y) * kOutlierRows;
  const int64_t c0 = (static_cast<int64_t>(blockIdx.x) * 256 + threadIdx.x) * 8;
  const int nr = static_cast<int>(rows - r0 < kOutlierRows ? rows - r0 : kOutlierRows);
  const bool live = c0 < k;
  float sum[kOutlierRows];
  unsigned rmax[kOutlierRows];
  unsigned cmax[8] = {0u, 0u, 0u, 0u, 0u, 0u, 0u, 0u};
#pragma unroll
  for (int r = 0; r < kOutlierRows; ++r) {
    sum[r] = 0.0f;
    rmax[r] = 0u;
    if (r < nr && live) {
      float v[8];
      load8<T>(x, (r0 + r) * ldx + c0, v);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float a = isfinite(v[j]) ? fabsf(v[j]) : 0.0f;
        sum[r] = fmaf(a, a, sum[r]);
        const unsigned b = __float_as_uint(a);
        rmax[r] = max(rmax[r], b);
        cmax[j] = max(cmax[j], b);
      }
    }
  }
  if (live) {
#pragma unroll
    for (int j = 0; j < 8; ++j)
      if (c0 + j < k && cmax[j] != 0u) atomicMax(col_amax + c0 + j, cmax[j]);
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
#pragma unroll
  for (int r = 0; r < kOutlierRows; ++r) {
    double s = sum[r];
    unsigned m = rmax[r];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      s += __shfl_xor_sync(0xffffffffu, s, o);
      m = max(m, __shfl_xor_sync(0xffffffffu, m, o));
    }
    if (lane == 0) {
      s_sum[warp][r] = s;
      s_max[warp][r] = m;
    }
  }
  __syncthreads();
  if (threadIdx.x < nr) {
    double s = 0.0;
    unsigned m = 0u;
#pragma unroll
    for (int w = 0; w < 8; ++w) {
      s += s_sum[w][threadIdx.x];
      m = max(m, s_max[w][threadIdx.x]);
    }
    atomicAdd(row_sumsq + r0 + threadIdx.x, s);
    if (m != 0u) atomicMax(row_amax + r0 + threadIdx.x, m);
  }
}

}  // namespace kab
