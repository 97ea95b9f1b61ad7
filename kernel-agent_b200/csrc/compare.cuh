// The comparator's element loop (kernel-agent src/kernel_agent/kernels/compare.py:684-739)
// as one fused reduction over (ref, new[, rerounded]): positions of NaN / +inf / -inf in
// each, the finite count, the mismatch count `diff > allowed`, the largest `diff / allowed`,
// the element ratio of the reduced tiers, and float64 sums of a^2, b^2, ab, d^2, d and
// (alt - ref)^2. Element-wise arithmetic is the reference's fp32 with explicit roundings
// (allowed = atol + rtol * |a| in two roundings, never an FMA), so counts and maxima equal
// torch's on the CPU bit for bit; the sums are float64 (more accurate than torch's fp32).
//
// Each block writes one partial into caller-provided scratch; a one-block kernel then adds
// the partials in index order, so the result does not depend on scheduling.
#pragma once

#include "kab_common.cuh"

namespace kab {

struct CmpPartial {
  long long cnt[KAB_CMP_NCOUNT];
  double sum[KAB_CMP_NSUM];
  float mx[KAB_CMP_NMAX];
  float pad[1];
};

__device__ __forceinline__ void warp_sum_partial(CmpPartial& p) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
#pragma unroll
    for (int i = 0; i < KAB_CMP_NCOUNT; ++i) p.cnt[i] += __shfl_xor_sync(0xffffffffu, p.cnt[i], o);
#pragma unroll
    for (int i = 0; i < KAB_CMP_NSUM; ++i) p.sum[i] += __shfl_xor_sync(0xffffffffu, p.sum[i], o);
#pragma unroll
    for (int i = 0; i < KAB_CMP_NMAX; ++i) p.mx[i] = amax_merge(p.mx[i], __shfl_xor_sync(0xffffffffu, p.mx[i], o));
  }
}

// Block reduction of a partial into shared memory slot 0 (fixed order: warp by warp).
__device__ __forceinline__ void block_sum_partial(CmpPartial& p, CmpPartial* sm) {
  warp_sum_partial(p);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  if (lane == 0) sm[warp] = p;
  __syncthreads();
  if (threadIdx.x == 0) {
    CmpPartial t = sm[0];
    for (int w = 1; w < nw; ++w) {
      for (int i = 0; i < KAB_CMP_NCOUNT; ++i) t.cnt[i] += sm[w].cnt[i];
      for (int i = 0; i < KAB_CMP_NSUM; ++i) t.sum[i] += sm[w].sum[i];
      for (int i = 0; i < KAB_CMP_NMAX; ++i) t.mx[i] = amax_merge(t.mx[i], sm[w].mx[i]);
    }
    sm[0] = t;
  }
  __syncthreads();
}

// One thread's running results: 32-bit counts (a thread sees far fewer than 2^31 elements),
// float64 sums, NaN-keeping maxima, and for the fast path the operands (bd, bal) of its
// largest diff / allowed, so that the one IEEE division happens at the end (rounding is
// monotonic, so the largest rounded ratio is the rounding of the largest exact one).
struct CmpThread {
  int cnt[KAB_CMP_NCOUNT];
  double sum[KAB_CMP_NSUM];
  float mx[KAB_CMP_NMAX];
  float bd, bal;
  float rb;  // the largest approximate ratio d * rcp(allowed) seen by the fast step
};

__device__ __forceinline__ void cmp_init(CmpThread& t) {
#pragma unroll
  for (int i = 0; i < KAB_CMP_NCOUNT; ++i) t.cnt[i] = 0;
#pragma unroll
  for (int i = 0; i < KAB_CMP_NSUM; ++i) t.sum[i] = 0.0;
#pragma unroll
  for (int i = 0; i < KAB_CMP_NMAX; ++i) t.mx[i] = 0.0f;
  t.bd = 0.0f;
  t.bal = 1.0f;
  t.rb = 0.0f;
}

// The hardware reciprocal (rcp.approx: within about one unit in the last place).
__device__ __forceinline__ float cmp_rcp(float x) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// (bd, bal) <- (d, al) when d / al > bd / bal exactly (finite d >= 0, al > 0): a float filter
// that never drops a larger ratio (its products are within 2^-23 of exact), then the exact
// comparison of the float64 products (exact for float operands).
__device__ __forceinline__ void ratio_max(float d, float al, float& bd, float& bal) {
  if (d * bal >= (bd * al) * 0.99999905f) {
    if (static_cast<double>(d) * bal > static_cast<double>(bd) * al) {
      bd = d;
      bal = al;
    }
  }
}

// The general element step (any mode, any value), compare.py:684-739.
__device__ __forceinline__ void cmp_element(const KabCompareParams& P, float a, float b, float alt, int64_t i,
                                            CmpThread& p) {
  const bool an = a != a, bn = b != b;
  const bool ap = a == INFINITY, bp = b == INFINITY, am = a == -INFINITY, bm = b == -INFINITY;
  p.cnt[KAB_CMP_NAN_REF] += an; p.cnt[KAB_CMP_NAN_NEW] += bn; p.cnt[KAB_CMP_NAN_DIFF] += an != bn;
  p.cnt[KAB_CMP_PINF_REF] += ap; p.cnt[KAB_CMP_PINF_NEW] += bp; p.cnt[KAB_CMP_PINF_DIFF] += ap != bp;
  p.cnt[KAB_CMP_NINF_REF] += am; p.cnt[KAB_CMP_NINF_NEW] += bm; p.cnt[KAB_CMP_NINF_DIFF] += am != bm;
  if (P.has_rerounded) {  // compare.py:622-624: diff where both ref and alt are finite
    const bool both = isfinite(a) && isfinite(alt);
    const float r = both ? __fsub_rn(alt, a) : 0.0f;
    p.sum[KAB_CMP_SUM_RR] += static_cast<double>(r) * r;
  }
  if (!isfinite(a)) return;  // compare.py:690-693: the finite elements of the reference
  p.cnt[KAB_CMP_FINITE] += 1;
  const float d = fabsf(__fsub_rn(a, b));
  const float aa = fabsf(a);
  p.sum[KAB_CMP_SUM_AA] += static_cast<double>(a) * a;
  p.sum[KAB_CMP_SUM_BB] += static_cast<double>(b) * b;
  p.sum[KAB_CMP_SUM_AB] += static_cast<double>(a) * b;
  p.sum[KAB_CMP_SUM_DD] += static_cast<double>(d) * d;
  p.sum[KAB_CMP_SUM_D] += d;
  p.mx[KAB_CMP_MAX_D] = amax_merge(p.mx[KAB_CMP_MAX_D], d);
  // compare.py:698: atol + rtol * |a| (fp32, two roundings)
  float allowed = __fadd_rn(P.atol, __fmul_rn(P.rtol, aa));
  if (P.alt_bound) allowed = fmaxf(allowed, __fadd_rn(P.alt_atol, __fmul_rn(P.alt_rtol, aa)));
  if (P.widen_mode == 1) allowed = __fadd_rn(allowed, P.widen_scalar);
  else if (P.widen_mode == 2) allowed = __fadd_rn(allowed, __ldg(P.widen_channel + i % P.channels));
  p.cnt[KAB_CMP_MISMATCH] += d > allowed;
  // compare.py:716: diff / allowed.clamp_min(1e-30)
  p.mx[KAB_CMP_MAX_RATIO] = amax_merge(p.mx[KAB_CMP_MAX_RATIO], __fdiv_rn(d, fmaxf(allowed, 1e-30f)));
  if (P.element_mode != 0) {  // compare.py:739: diff / (e_atol * scale + e_rtol * |a|)
    const float first = P.element_mode == 1 ? P.element_first
                                            : __fmul_rn(P.element_atol, __ldg(P.element_scale + i % P.channels));
    const float den = __fadd_rn(first, __fmul_rn(P.element_rtol, aa));
    p.mx[KAB_CMP_MAX_ELEMENT] = amax_merge(p.mx[KAB_CMP_MAX_ELEMENT], __fdiv_rn(d, den));
  }
}

// The common case of 8 elements (no rerounded / alternative bound / widening / element
// ratio; every a and b finite): the same counts and maxima with float partial sums over the
// 8 products added to the float64 totals, and the ratio kept as its operands. The exact
// ratio comparison runs only for a chunk that may hold a new largest ratio: its largest
// approximate ratio d * rcp(allowed) (within 2^-21 of the exact one) is at least 1 - 2^-20
// of the largest approximation seen before, which any chunk holding a larger exact ratio
// satisfies. That is a handful of chunks per thread, instead of a branch per element.
__device__ __forceinline__ void cmp_chunk_fast(const KabCompareParams& P, const float (&a)[8], const float (&b)[8],
                                               CmpThread& t) {
  float s_aa = 0.0f, s_bb = 0.0f, s_ab = 0.0f, s_dd = 0.0f, s_d = 0.0f;
  float mxd = t.mx[KAB_CMP_MAX_D];
  float rc = 0.0f;
  int mism = 0;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const float d = fabsf(__fsub_rn(a[j], b[j]));
    const float allowed = __fadd_rn(P.atol, __fmul_rn(P.rtol, fabsf(a[j])));
    mism += d > allowed;
    rc = fmaxf(rc, d * cmp_rcp(fmaxf(allowed, 1e-30f)));
    mxd = fmaxf(mxd, d);
    s_aa = fmaf(a[j], a[j], s_aa);
    s_bb = fmaf(b[j], b[j], s_bb);
    s_ab = fmaf(a[j], b[j], s_ab);
    s_dd = fmaf(d, d, s_dd);
    s_d += d;
  }
  if (rc >= t.rb * 0.99999905f) {  // 1 - 2^-20: this chunk may hold a new largest ratio
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float d = fabsf(__fsub_rn(a[j], b[j]));
      const float allowed = __fadd_rn(P.atol, __fmul_rn(P.rtol, fabsf(a[j])));
      ratio_max(d, fmaxf(allowed, 1e-30f), t.bd, t.bal);
    }
  }
  t.rb = fmaxf(t.rb, rc);
  t.mx[KAB_CMP_MAX_D] = mxd;
  t.cnt[KAB_CMP_FINITE] += 8;
  t.cnt[KAB_CMP_MISMATCH] += mism;
  t.sum[KAB_CMP_SUM_AA] += s_aa;
  t.sum[KAB_CMP_SUM_BB] += s_bb;
  t.sum[KAB_CMP_SUM_AB] += s_ab;
  t.sum[KAB_CMP_SUM_DD] += s_dd;
  t.sum[KAB_CMP_SUM_D] += s_d;
}

__device__ __forceinline__ bool all_finite8(const float (&a)[8], const float (&b)[8]) {
  bool ok = true;
#pragma unroll
  for (int j = 0; j < 8; ++j) ok = ok && fabsf(a[j]) < INFINITY && fabsf(b[j]) < INFINITY;
  return ok;
}

// SIMPLE: no rerounded tensor, alternative bound, widening or element ratio (the first pass
// of every tier): chunks whose values are all finite take the fast step.
template <int T, bool SIMPLE>
__global__ void __launch_bounds__(256)
compare_kernel(KabCompareParams P, CmpPartial* __restrict__ partials) {
  __shared__ CmpPartial sm[8];
  CmpThread t;
  cmp_init(t);
  const int64_t n = P.n;
  const int64_t tid = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  if (P.vector) {  // 8 elements per thread per step (16-byte loads of 2-byte types)
    const int64_t nv = n >> 3;
    int64_t c = tid;
    if constexpr (SIMPLE && T != kF32) {  // four chunks of raw 16-byte loads in flight per thread
      constexpr int U = 4;
      for (; c + (U - 1) * stride < nv; c += U * stride) {
        uint4 ra[U], rb[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
          ra[u] = __ldg(reinterpret_cast<const uint4*>(P.ref) + (c + u * stride));
          rb[u] = __ldg(reinterpret_cast<const uint4*>(P.new_) + (c + u * stride));
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
          float a[8], b[8];
          unpack8<T>(ra[u], a);
          unpack8<T>(rb[u], b);
          if (all_finite8(a, b)) {
            cmp_chunk_fast(P, a, b, t);
          } else {
            for (int j = 0; j < 8; ++j) cmp_element(P, a[j], b[j], 0.0f, (c + u * stride) * 8 + j, t);
          }
        }
      }
    }
    for (; c < nv; c += stride) {
      float a[8], b[8], r[8];
      load8<T>(P.ref, c * 8, a);
      load8<T>(P.new_, c * 8, b);
      if (!SIMPLE && P.has_rerounded) load8<T>(P.rerounded, c * 8, r);
      if (SIMPLE && all_finite8(a, b)) {
        cmp_chunk_fast(P, a, b, t);
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j)
          cmp_element(P, a[j], b[j], (!SIMPLE && P.has_rerounded) ? r[j] : 0.0f, c * 8 + j, t);
      }
    }
    for (int64_t i = nv * 8 + tid; i < n; i += stride)
      cmp_element(P, load_elem<T>(P.ref, i), load_elem<T>(P.new_, i),
                  P.has_rerounded ? load_elem<T>(P.rerounded, i) : 0.0f, i, t);
  } else {
    for (int64_t i = tid; i < n; i += stride)
      cmp_element(P, load_elem<T>(P.ref, i), load_elem<T>(P.new_, i),
                  P.has_rerounded ? load_elem<T>(P.rerounded, i) : 0.0f, i, t);
  }
  CmpPartial p;
#pragma unroll
  for (int i = 0; i < KAB_CMP_NCOUNT; ++i) p.cnt[i] = t.cnt[i];
#pragma unroll
  for (int i = 0; i < KAB_CMP_NSUM; ++i) p.sum[i] = t.sum[i];
#pragma unroll
  for (int i = 0; i < KAB_CMP_NMAX; ++i) p.mx[i] = t.mx[i];
  p.mx[KAB_CMP_MAX_RATIO] = amax_merge(p.mx[KAB_CMP_MAX_RATIO], __fdiv_rn(t.bd, t.bal));
  block_sum_partial(p, sm);
  if (threadIdx.x == 0) partials[blockIdx.x] = sm[0];
}

// Adds `count` partials in index order into *out (one block).
__global__ void __launch_bounds__(256)
compare_finalize_kernel(const CmpPartial* __restrict__ partials, int count, KabCompareResult* out) {
  __shared__ CmpPartial sm[8];
  CmpPartial p;
#pragma unroll
  for (int i = 0; i < KAB_CMP_NCOUNT; ++i) p.cnt[i] = 0;
#pragma unroll
  for (int i = 0; i < KAB_CMP_NSUM; ++i) p.sum[i] = 0.0;
#pragma unroll
  for (int i = 0; i < KAB_CMP_NMAX; ++i) p.mx[i] = 0.0f;
  for (int b = threadIdx.x; b < count; b += blockDim.x) {
    const CmpPartial& q = partials[b];
    for (int i = 0; i < KAB_CMP_NCOUNT; ++i) p.cnt[i] += q.cnt[i];
    for (int i = 0; i < KAB_CMP_NSUM; ++i) p.sum[i] += q.sum[i];
    for (int i = 0; i < KAB_CMP_NMAX; ++i) p.mx[i] = amax_merge(p.mx[i], q.mx[i]);
  }
  block_sum_partial(p, sm);
  if (threadIdx.x == 0) {
    for (int i = 0; i < KAB_CMP_NCOUNT; ++i) out->count[i] = sm[0].cnt[i];
    for (int i = 0; i < KAB_CMP_NSUM; ++i) out->sum[i] = sm[0].sum[i];
    for (int i = 0; i < KAB_CMP_NMAX; ++i) out->max[i] = sm[0].mx[i];
  }
}

// Per-channel (last dimension) float64 sums of squares of x (non-finite as 0) or of
// (alt - x) where both are finite, over `rows` rows of `channels`: compare.py:582-589 and
// 622-625. Grid (ceil(channels / 256), chunks); partial [chunk, channel] sums.
template <int T>
__global__ void __launch_bounds__(256)
channel_sumsq_kernel(const void* __restrict__ x, const void* __restrict__ alt, int64_t rows,
                     int64_t channels, int64_t rows_per_chunk, double* __restrict__ partial) {
  const int64_t c = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  if (c >= channels) return;
  const int64_t r0 = blockIdx.y * rows_per_chunk;
  const int64_t r1 = r0 + rows_per_chunk < rows ? r0 + rows_per_chunk : rows;
  double s = 0.0;
  for (int64_t r = r0; r < r1; ++r) {
    const float a = load_elem<T>(x, r * channels + c);
    float v;
    if (alt != nullptr) {
      const float b = load_elem<T>(alt, r * channels + c);
      v = (isfinite(a) && isfinite(b)) ? __fsub_rn(b, a) : 0.0f;
    } else {
      v = isfinite(a) ? a : 0.0f;
    }
    s += static_cast<double>(v) * v;
  }
  partial[blockIdx.y * channels + c] = s;
}

// rms[c] = sqrt(fp32(sum over chunks / rows)) (a mean then a square root in fp32).
__global__ void channel_rms_kernel(const double* __restrict__ partial, int64_t chunks,
                                   int64_t rows, int64_t channels, float* __restrict__ rms) {
  const int64_t c = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  if (c >= channels) return;
  double s = 0.0;
  for (int64_t k = 0; k < chunks; ++k) s += partial[k * channels + c];
  rms[c] = __fsqrt_rn(static_cast<float>(s / static_cast<double>(rows)));
}

}  // namespace kab

namespace kab {

// The difference census of the comparator's routing (src/kernel_agent/kernels/compare.py:
// 806-1182: grown caches, rows written into an input, in-place updates): which elements of a
// candidate tensor `a` (and, in union mode, of a second tensor `b` of the same layout) differ
// from a base tensor, over a region that may be a slice of each along one dimension. One
// pass; per differing element it sets its flag in `mask` and, per dimension, the flag of its
// index in `hits`; elements inside a given box (all of their indices flagged in `box`) are
// skipped. The count goes to `count` with one atomic per warp.
constexpr int kDiffF64 = 3;  // the census also reads float64 tensors
// ... and compares integer / boolean tensors by their bits (elements of 1, 2, 4 or 8 bytes)
constexpr int kDiffBits8 = 4, kDiffBits16 = 5, kDiffBits32 = 6, kDiffBits64 = 7;

template <int T>
__device__ __forceinline__ bool differs_at(const void* x, int64_t ix, const void* y, int64_t iy, bool nan_equal) {
  if constexpr (T == kDiffBits8) {
    return __ldg(reinterpret_cast<const uint8_t*>(x) + ix) != __ldg(reinterpret_cast<const uint8_t*>(y) + iy);
  } else if constexpr (T == kDiffBits16) {
    return __ldg(reinterpret_cast<const uint16_t*>(x) + ix) != __ldg(reinterpret_cast<const uint16_t*>(y) + iy);
  } else if constexpr (T == kDiffBits32) {
    return __ldg(reinterpret_cast<const uint32_t*>(x) + ix) != __ldg(reinterpret_cast<const uint32_t*>(y) + iy);
  } else if constexpr (T == kDiffBits64) {
    return __ldg(reinterpret_cast<const unsigned long long*>(x) + ix) !=
           __ldg(reinterpret_cast<const unsigned long long*>(y) + iy);
  } else if constexpr (T == kDiffF64) {
    const double a = __ldg(reinterpret_cast<const double*>(x) + ix), b = __ldg(reinterpret_cast<const double*>(y) + iy);
    return nan_equal ? !(a == b || (a != a && b != b)) : a != b;
  } else {
    const float a = load_elem<T>(x, ix), b = load_elem<T>(y, iy);  // exact for 2-byte types
    return nan_equal ? !(a == b || (a != a && b != b)) : a != b;
  }
}

template <int T>
__global__ void __launch_bounds__(256) diff_census_kernel(KabDiffParams P, unsigned long long* count) {
  const int64_t total = P.outer * P.len * P.inner;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  unsigned found = 0;
  for (int64_t r = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; r < total; r += stride) {
    const int64_t n = r % P.inner;
    const int64_t oi = r / P.inner;
    const int64_t i = oi % P.len, o = oi / P.len;
    const int64_t ia = (o * P.a_dim + P.a_off + i) * P.inner + n;
    const int64_t ib = (o * P.base_dim + P.base_off + i) * P.inner + n;
    bool d = differs_at<T>(P.a, ia, P.base, ib, P.nan_equal != 0);
    if (!d && P.b != nullptr) d = differs_at<T>(P.b, ia, P.base, ib, P.nan_equal != 0);
    if (d && (P.box != nullptr || P.hits != nullptr)) {
      // the element's index along each dimension of the region (row-major)
      int64_t rest = r, off = 0;
      int64_t idx[KAB_DIFF_MAXDIM];
      for (int k = P.ndim - 1; k >= 0; --k) {
        idx[k] = rest % P.shape[k];
        rest /= P.shape[k];
      }
      bool inside = P.box != nullptr;
      for (int k = 0; k < P.ndim; ++k) {
        if (P.box != nullptr && !P.box[off + idx[k]]) inside = false;
        off += P.shape[k];
      }
      if (inside) d = false;
      if (d && P.hits != nullptr) {
        off = 0;
        for (int k = 0; k < P.ndim; ++k) {
          P.hits[off + idx[k]] = 1;  // every writer stores the same byte
          off += P.shape[k];
        }
      }
    }
    if (P.mask != nullptr) P.mask[r] = d ? 1 : 0;
    found += d ? 1u : 0u;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) found += __shfl_xor_sync(0xffffffffu, found, o);
  if ((threadIdx.x & 31) == 0 && found) atomicAdd(count, static_cast<unsigned long long>(found));
}

}  // namespace kab
