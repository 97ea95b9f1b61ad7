// Device helpers shared by the producers and the attention kernels: quotients by one divisor
// that match the IEEE division's codes, and the int8 / e4m3 / e2m1 code packers.
#pragma once

#include "kab_common.cuh"

namespace kab {

constexpr float kFp8Max = 448.0f;

// ------------------------------------------------------------------ quotients by one divisor

// The codes here (int8 rint, e4m3 and e2m1 round-to-nearest-even, each saturating) are step
// functions of the IEEE quotient RN(v / s) whose steps sit at "short" floats: the rounding
// boundaries (k + 1/2 for int8, the e4m3 and e2m1 midpoints) have at most 8, 4 and 3
// significant bits, so their low LOW = 16, 19, 21 mantissa bits are zero. With y the hardware
// reciprocal of s (relative error at most 2^-22), RN(v * y) is within 6 units in the last
// place of RN(v / s), so both give the same code unless the product lies within 16 units of a
// short float. Only then (about 33 quotients in 2^LOW) does the thread recompute its
// quotients with the IEEE division __fdiv_rn. The reciprocal path is taken only where 1 / s
// is a normal float, |s| in [2^-125, 2^125]; other divisors always divide.
// The hardware reciprocal (rcp.approx: within about one unit in the last place).
__device__ __forceinline__ float rcp_approx(float s) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(s));
  return y;
}
struct Divisor {
  float s, y;
  bool fast;
  __device__ __forceinline__ explicit Divisor(float s_) : s(s_) {
    const float a = fabsf(s_);
    fast = a >= 2.350988701644575e-38f && a <= 4.253529586511731e+37f;
    y = fast ? rcp_approx(s_) : 0.0f;
  }
};
// True when q is within 16 units in the last place of a float whose low LOW mantissa bits are
// zero (with y within 2 units of 1 / s, RN(v * y) is within 6 units of RN(v / s)).
template <int LOW>
__device__ __forceinline__ bool near_short(float q) {
  return ((__float_as_uint(q) + 16u) & ((1u << LOW) - 1u)) <= 32u;
}
template <int LOW, int N>
__device__ __forceinline__ void quotients(const float (&v)[N], const Divisor& d, float (&q)[N]) {
  float t[N];  // q may alias v
  bool slow = !d.fast;
#pragma unroll
  for (int i = 0; i < N; ++i) {
    t[i] = __fmul_rn(v[i], d.y);
    slow |= near_short<LOW>(t[i]);
  }
  if (slow) {
#pragma unroll
    for (int i = 0; i < N; ++i) t[i] = __fdiv_rn(v[i], d.s);
  }
#pragma unroll
  for (int i = 0; i < N; ++i) q[i] = t[i];
}
constexpr int kLowInt8 = 16, kLowE4m3 = 19, kLowE2m1 = 21;

// Eight e4m3fn codes of quotients (cvt.rn.satfinite: +-inf and finite overflow to +-448, NaN
// stays NaN: the reference's clamp(+-448) then cast), element 0 in the low byte.
__device__ __forceinline__ uint2 e4m3x8(const float (&q)[8]) {
  const uint32_t w0 = e4m3_pair(q[0], q[1]) | (static_cast<uint32_t>(e4m3_pair(q[2], q[3])) << 16);
  const uint32_t w1 = e4m3_pair(q[4], q[5]) | (static_cast<uint32_t>(e4m3_pair(q[6], q[7])) << 16);
  return make_uint2(w0, w1);
}
// e4m3 codes of the eight IEEE quotients RN(v / s) (d = Divisor(s)), element 0 in the low
// byte. The codes of v * y(1 + 2^-19) and of v * y(1 - 2^-19) bracket those of the quotient: y
// is within 2^-22 of 1 / s, so the two products lie on either side of v / s and of its
// rounding, and the e4m3 rounding is monotonic. Where both give the same codes, those are the
// quotient's; otherwise (a quotient within about 2^-19 of an e4m3 midpoint) and where s has
// no normal reciprocal, the eight quotients are divided. Unlike the short-float window of
// `quotients`, quotients that land on or near representable e4m3 values (frequent for ratios
// of bf16 values) do not divide.
__device__ __forceinline__ float2 fmul2_rn(float a, float b, float c) {  // (a * c, b * c)
  float2 r;
  asm("{\n .reg .b64 x, y, z;\n mov.b64 x, {%2, %3};\n mov.b64 y, {%4, %4};\n mul.rn.f32x2 z, x, y;\n"
      " mov.b64 {%0, %1}, z;\n}"
      : "=f"(r.x), "=f"(r.y)
      : "f"(a), "f"(b), "f"(c));
  return r;
}
__device__ __forceinline__ uint2 e4m3x8_quotients(const float (&v)[8], const Divisor& d) {
  if (d.fast) {
    const float yh = __fmul_rn(d.y, 1.0f + 0x1p-19f), yl = __fmul_rn(d.y, 1.0f - 0x1p-19f);
    float h[8], l[8];
#pragma unroll
    for (int i = 0; i < 8; i += 2) {
      const float2 ph = fmul2_rn(v[i], v[i + 1], yh), pl = fmul2_rn(v[i], v[i + 1], yl);
      h[i] = ph.x;
      h[i + 1] = ph.y;
      l[i] = pl.x;
      l[i + 1] = pl.y;
    }
    const uint2 ch = e4m3x8(h), cl = e4m3x8(l);
    if (ch.x == cl.x && ch.y == cl.y) return ch;
  }
  float t[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) t[i] = __fdiv_rn(v[i], d.s);
  return e4m3x8(t);
}

// Eight int8 codes: rint(q) to nearest even, clamped to +-127 (NaN -> 0), element 0 low.
__device__ __forceinline__ uint2 int8x8(const float (&q)[8]) {
  uint32_t w[2] = {0, 0};
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int r = max(-127, min(127, __float2int_rn(q[j])));
    w[j >> 2] |= static_cast<uint32_t>(r & 0xFF) << (8 * (j & 3));
  }
  return make_uint2(w[0], w[1]);
}
// Eight e2m1 codes (nibble j = element j) of quotients: cvt.rn.satfinite.e2m1x2 rounds to
// nearest even, which puts the ties where the reference's midpoint comparisons do (up at
// 0.75, 1.75, 3.5; down at 0.25, 1.25, 2.5, 5) and saturates at +-6 like its clamp. The
// reference has no negative zero: a zero magnitude drops its sign bit. It maps NaN to 0: the
// caller zeroes NaN quotients first.
__device__ __forceinline__ uint32_t e2m1x8(const float (&q)[8]) {
  uint32_t out;
  asm("{\n .reg .b8 b0, b1, b2, b3;\n"
      " cvt.rn.satfinite.e2m1x2.f32 b0, %2, %1;\n"
      " cvt.rn.satfinite.e2m1x2.f32 b1, %4, %3;\n"
      " cvt.rn.satfinite.e2m1x2.f32 b2, %6, %5;\n"
      " cvt.rn.satfinite.e2m1x2.f32 b3, %8, %7;\n"
      " mov.b32 %0, {b0, b1, b2, b3};\n}"
      : "=r"(out)
      : "f"(q[0]), "f"(q[1]), "f"(q[2]), "f"(q[3]), "f"(q[4]), "f"(q[5]), "f"(q[6]), "f"(q[7]));
  const uint32_t mag = out & 0x77777777u;
  const uint32_t nonzero = (mag + 0x77777777u) & 0x88888888u;  // bit 3 of each nibble with mag > 0
  return mag | (out & nonzero);
}

// NaN-keeping max |v| as the bits of |v|: non-negative floats order like their bit patterns
// and every NaN (0x7F800001 and up) is above +inf.
__device__ __forceinline__ uint32_t abs_bits_max8(const float (&v)[8], uint32_t acc) {
#pragma unroll
  for (int j = 0; j < 8; ++j) acc = max(acc, __float_as_uint(v[j]) & 0x7FFFFFFFu);
  return acc;
}

}  // namespace kab
