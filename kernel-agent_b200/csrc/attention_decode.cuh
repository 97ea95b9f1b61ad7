// FP8 KV-cache decode attention and the cache's quantiser, the "fp8_kv" class of
// kernel-agent (src/kernel_agent/kernels/kv_quant.py, the example
// src/kernel_agent/agent/examples/triton_fp8_kv_decode.py).
//
//  * quant_kv_kernel (kv_quant.py:38-46 quantize_fp8_kv): one fp32 scale per row of D elements
//    (a token of one KV head), amax / 448 where amax > 0 else 1, codes e4m3(v / scale) clamped
//    to +-448, nearest even. Rows are addressed as (outer, inner) with separate strides for the
//    source, the codes and the scales, so that appending tokens writes straight into a
//    preallocated cache [batch, heads, max_tokens, D].
//  * kv_decode_kernel (kv_quant.py:56-83 fp8_kv_attention, split-KV as in
//    triton_fp8_kv_decode.py:195-260): one query token per sequence, grouped-query heads, an
//    e4m3 cache with one scale per (token, head). One CTA per (sequence, KV head, split of the
//    cache). The K and V codes enter the tensor core as they are: TMA brings 128-token tiles
//    of K [tokens, D] and V [tokens, D] (the same bytes serve as V^T, an MN-major operand),
//    and tcgen05.mma kind::f8f6f4 computes
//        S^T [128 tokens, 2 x GP] = K . (Q_hi | Q_lo)^T
//        O^T [D, 2 x GP]        += V^T . (P_hi | P_lo)^T
//    where each bf16 query row is carried exactly as two e4m3 terms (a power-of-two scale per
//    row puts the row's amax in [128, 256); Q_hi = e4m3(q), Q_lo = e4m3((q - Q_hi) * 16): a
//    bf16 value has 8 significant bits, each term 4), and P' = p * v_scale[token] likewise as
//    two e4m3 terms (one power-of-two scale per tile), about as fine as the reference's bf16
//    P. The K scale multiplies the scores, the V scale is folded into P (the reference's
//    split of the two scales, triton_fp8_kv_decode.py:142-155).
//    Warp 0 issues the TMA loads (5-7 stage ring); warp 14 issues each tile's S as soon as
//    the owning group has read the scores two tiles back, warp 1 each tile's P V once its P is
//    written (and owns the TMEM allocation); two groups of four softmax warps (warps 2-5 and
//    6-9, one token per thread) take the even and the odd tiles: scores, the tile max per
//    query head, p = 2^(s - max), the row sums, P' split and written in the no-swizzle
//    MN-major layout; warps 10-13 (one head-dim element per
//    thread) merge each tile's O with its own max in tile order (no rescaling in TMEM) and write
//    the split's partial (max, sum, O) or, with one split, the output. The splits' partials
//    are merged into the bf16 output (triton_fp8_kv_decode.py:163-186) either within a thread-
//    block cluster (the splits of a (sequence, KV head) as one cluster, each CTA merging a slice
//    of the output from the others' shared memory) or through a global workspace, where the CTA
//    that finishes a (sequence, KV head) last, by an atomic count, merges them all.
// No load uses cluster multicast; every wait is bounded and records kDevTimeout.
#pragma once

#include <cuda_fp8.h>

#include "codes.cuh"
#include "tcgen05.cuh"

namespace kab {

// g_attention_status: the device status word, defined by the including translation unit.

// ------------------------------------------------------------------ quantiser

// kv_quant.py:38-46. LANES = D / 8 threads share a row (8 elements each); rows = outer x inner.
template <int T, int LANES>
__global__ void __launch_bounds__(256)
quant_kv_kernel(const void* __restrict__ x, int64_t rows, int64_t inner, int64_t xs_o, int64_t xs_i,
                uint8_t* __restrict__ codes, int64_t cs_o, int64_t cs_i, float* __restrict__ scales, int64_t ss_o,
                int64_t ss_i) {
  const int64_t r = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) / LANES;
  const int j = static_cast<int>(threadIdx.x % LANES);
  const bool live = r < rows;
  const int64_t o = live ? r / inner : 0, t = live ? r % inner : 0;
  float v[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  if (live) load8<T>(x, o * xs_o + t * xs_i + j * 8, v);
  uint32_t abits = abs_bits_max8(v, 0u);
#pragma unroll
  for (int off = LANES / 2; off > 0; off >>= 1) abits = max(abits, __shfl_xor_sync(0xffffffffu, abits, off));
  if (!live) return;
  const float amax = __uint_as_float(abits);
  // kv_quant.py:44: torch.where(amax > 0, amax / 448, 1) (NaN -> 1; a positive amax whose
  // quotient underflows keeps the zero scale, as the reference does)
  const float s = amax > 0.0f ? __fdiv_rn(amax, kFp8Max) : 1.0f;
  *reinterpret_cast<uint2*>(codes + o * cs_o + t * cs_i + j * 8) = e4m3x8_quotients(v, Divisor(s));
  if (j == 0) scales[o * ss_o + t * ss_i] = s;
}

// ------------------------------------------------------------------ decode attention

struct DecodeArgs {
  int heads_kv, group;     // group = query heads per KV head
  int length;              // cached tokens of the view (L)
  int chunk, splits;       // tokens per split (a multiple of 128) and splits per (sequence, KV head)
  const void* q;           // [batch, heads_q, D]
  int64_t sqb, sqh;        // element strides of q
  const float* k_scale;    // [batch, heads_kv, L], unit last stride
  int64_t ksb, ksh;
  const float* v_scale;
  int64_t vsb, vsh;
  const int32_t* lengths;  // [batch] valid tokens per sequence, or null (all L)
  float scale_log2;        // softmax scale * log2(e)
  void* out;               // [batch, heads_q, D] bf16, contiguous
  float* part_o;           // [batch * heads_kv, splits, GP, D]
  float* part_ml;          // [batch * heads_kv, splits, 2, GP]: max (log2 domain), sum
  unsigned* counters;      // [batch * heads_kv], zero between launches
  int cluster;             // 1: the splits of a (sequence, KV head) are one thread-block cluster
                           // and merge through distributed shared memory (no workspace)
};

template <int D, int GP>
struct DecodeLayout {
  static constexpr int kRow = D;                  // bytes of a token row of codes
  static constexpr int kTile = 128 * kRow;        // one K or V tile
  static constexpr int kZero = D < 128 ? kTile : 0;  // zero rows M = D..127 of V^T (D = 64)
  static constexpr int kStage = 2 * kTile + kZero;
  static constexpr int kStages = D < 128 ? 7 : 5;
  static constexpr int kN = 2 * GP;               // MMA N: two terms per query head
  static constexpr int kQ = 0;                    // [kN rows, D bytes], K-major swizzled
  static constexpr int kP = kQ + ((kN * kRow + 1023) & ~1023);  // 2 x [kN / 16 blocks][128 tok][16 B]
  static constexpr int kPBytes = (kN / 16) * 2048;
  static constexpr int kRing = kP + 2 * kPBytes;  // stage s: K | V | zeros
  // [2 groups][2 slots][4 warps][GP + 4] floats: the warps' maxima of a tile
  static constexpr int kRed = kRing + kStages * kStage;
  // stats slot [2]: m[GP] (the tile's max per row, log2 domain), f (the tile's P scale
  // exponent) + 3 pad, l[4][GP] (the tile's row sums per softmax warp)
  static constexpr int kStats = kRed + 2 * 2 * 4 * (GP + 4) * 4;
  static constexpr int kSM = 0, kSF = GP, kSL = GP + 4;
  static constexpr int kStatsFloats = GP + 4 + 4 * GP;
  static constexpr int kQinv = kStats + 2 * kStatsFloats * 4;   // [2][GP] term factors of the scores
  static constexpr int kLfin = kQinv + 2 * GP * 4;              // [GP] final row sums
  static constexpr int kBars = (kLfin + GP * 4 + 7) & ~7;
  static constexpr int kNumBars = 2 * kStages + 2 * 6 + 2;
  static constexpr int kSmem = 1024 + kBars + kNumBars * 8 + 32;
  static constexpr int kThreads = 480;  // TMA, P V issuer, 2 x 4 softmax, 4 merge, S issuer
  static constexpr int kTmemCols = 4 * kN <= 128 ? 128 : 256;  // S x 2 and O x 2, kN columns each
};

// 2^e as fp32 for -149 <= e <= 127.
__device__ __forceinline__ float pow2f(int e) {
  if (e >= -126) return __uint_as_float(static_cast<uint32_t>(e + 127) << 23);
  return __uint_as_float(1u << (e + 149));
}
// The power-of-two exponent that puts a magnitude bound `a` (>= 0, may be inf / NaN) in
// [128, 256): 7 - floor(log2 a), clamped to [-121, 126] (a zero or subnormal bound: 126).
__device__ __forceinline__ int scale_exp(float a) {
  const int eb = static_cast<int>((__float_as_uint(a) >> 23) & 0xFF);
  const int e = eb == 0 ? 126 : 7 - (eb - 127);
  return min(126, max(-121, e));
}
// Values of two e4m3 codes (exact: e4m3 -> f16 -> f32).
__device__ __forceinline__ float2 e4m3x2_value(uint16_t pair) {
  const __half2_raw h = __nv_cvt_fp8x2_to_halfraw2(static_cast<__nv_fp8x2_storage_t>(pair), __NV_E4M3);
  return __half22float2(__half2(h));
}
// Two-term e4m3 split of x and y (|x|, |y| < 448 after scaling): hi = e4m3(v),
// lo = e4m3((v - hi) * 16). Returns the hi pair in the low half, the lo pair in the high half.
__device__ __forceinline__ uint32_t split2(float x, float y) {
  const uint16_t hi = e4m3_pair(x, y);
  const float2 hv = e4m3x2_value(hi);
  const uint16_t lo = e4m3_pair((x - hv.x) * 16.0f, (y - hv.y) * 16.0f);
  return static_cast<uint32_t>(hi) | (static_cast<uint32_t>(lo) << 16);
}

// 4-D tile load (coordinates innermost first) into this CTA's shared memory.
__device__ __forceinline__ void tma_load_4d(const CUtensorMap* map, uint64_t* bar, void* dst, int x, int y, int z,
                                            int w) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5, %6}], "
      "[%2];" ::"r"(tc::smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(tc::smem_u32(bar)), "r"(x), "r"(y), "r"(z), "r"(w)
      : "memory");
}

// Descriptor of the no-swizzle MN-major P operand: 16-byte x 8-token core matrices, K (token)
// groups 128 bytes apart, N blocks of 16 columns 2048 bytes apart.
__device__ __forceinline__ uint64_t desc_p(uint32_t saddr) {
  uint64_t d = static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4);
  d |= static_cast<uint64_t>(128 >> 4) << 16;    // leading byte offset: the K direction
  d |= static_cast<uint64_t>(2048 >> 4) << 32;   // stride byte offset: the N direction
  d |= static_cast<uint64_t>(1) << 46;
  return d;  // layout type 0: no swizzle
}
// The V^T operand (MN-major) of D = 64: 64-byte swizzled rows, 8-token groups 512 bytes apart,
// and the second 64 rows of M (zeros) `zero_off` bytes after the first.
__device__ __forceinline__ uint64_t desc_vt64(uint32_t saddr, uint32_t zero_off) {
  uint64_t d = static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4);
  d |= static_cast<uint64_t>(zero_off >> 4) << 16;  // leading byte offset: the M direction
  d |= static_cast<uint64_t>(512 >> 4) << 32;       // stride byte offset: the K direction
  d |= static_cast<uint64_t>(1) << 46;
  d |= static_cast<uint64_t>(4) << 61;              // 64-byte swizzle
  return d;
}

// N (16, 32 or 64) consecutive TMEM columns of this thread's lane.
template <int N>
__device__ __forceinline__ void tmem_ld_cols(uint32_t taddr, uint32_t (&r)[N]) {
  if constexpr (N == 16) {
    tc::tmem_ld16(taddr, r);
  } else {
#pragma unroll
    for (int c = 0; c < N / 32; ++c) tc::tmem_ld32(taddr + c * 32, *reinterpret_cast<uint32_t(*)[32]>(r + c * 32));
  }
}

// Loads from the shared memory of a CTA of this cluster (a shared::cluster address from mapa).
__device__ __forceinline__ float ld_cluster_f32(uint32_t addr) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
  return v;
}
__device__ __forceinline__ float4 ld_cluster_f32x4(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(addr)
               : "memory");
  return v;
}

__device__ __forceinline__ bool warp_wait_d(uint64_t* bar, uint32_t parity) {
  return __all_sync(0xffffffffu, tc::mbar_wait(bar, parity));
}
__device__ __forceinline__ void named_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}
// A named barrier that also ORs a predicate over the participating threads.
__device__ __forceinline__ bool named_sync_any(int id, int threads, bool pred) {
  uint32_t r;
  asm volatile(
      "{\n .reg .pred p, q;\n setp.ne.u32 p, %1, 0;\n bar.red.or.pred q, %2, %3, p;\n selp.u32 %0, 1, 0, q;\n}"
      : "=r"(r)
      : "r"(static_cast<uint32_t>(pred)), "r"(id), "r"(threads)
      : "memory");
  return r != 0;
}

// Per-lane reduction of N values across the warp by halving exchanges (N - 1 shuffles): on
// return v[0] holds the reduction over the warp of value index (lane >> (5 - log2 N)).
template <int N, bool MAX>
__device__ __forceinline__ float warp_reduce_scatter(float (&v)[N], int lane) {
  int n = N;
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) {
    if (n > 1) {
      const bool upper = (lane & off) != 0;
      const int h = n / 2;
#pragma unroll
      for (int j = 0; j < N / 2; ++j) {
        if (j < h) {
          const float send = upper ? v[j] : v[j + h];
          const float keep = upper ? v[j + h] : v[j];
          const float got = __shfl_xor_sync(0xffffffffu, send, off);
          v[j] = MAX ? fmaxf(keep, got) : keep + got;
        }
      }
      n = h;
    } else {
      const float got = __shfl_xor_sync(0xffffffffu, v[0], off);
      v[0] = MAX ? fmaxf(v[0], got) : v[0] + got;
    }
  }
  return v[0];
}

template <int D, int GP, int QT>
__global__ void __launch_bounds__(480, 1)
kv_decode_kernel(const __grid_constant__ CUtensorMap tma_k, const __grid_constant__ CUtensorMap tma_v, DecodeArgs g) {
  using L = DecodeLayout<D, GP>;
  constexpr int N = L::kN;
  constexpr int S = L::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem + L::kQ;
  uint8_t* sP = smem + L::kP;
  uint8_t* sRing = smem + L::kRing;
  float* red = reinterpret_cast<float*>(smem + L::kRed);
  float* stats = reinterpret_cast<float*>(smem + L::kStats);
  float* qinv = reinterpret_cast<float*>(smem + L::kQinv);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBars);
  uint64_t* kv_full = bars;
  uint64_t* kv_empty = kv_full + S;
  uint64_t* s_full = kv_empty + S;  // [2] MMA commit
  uint64_t* s_free = s_full + 2;    // [2] 4 softmax warps (the group has read S_i)
  uint64_t* p_full = s_free + 2;    // [2] 4 softmax warps
  uint64_t* p_free = p_full + 2;    // [2] MMA commit
  uint64_t* o_full = p_free + 2;    // [2] MMA commit
  uint64_t* o_free = o_full + 2;    // [2] 4 merge warps
  uint64_t* drain = o_free + 2;      // [2] the S issuer, the P V issuer
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 2);
  uint32_t* last_flag = tmem_slot + 1;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int sp = static_cast<int>(blockIdx.x);
  const int bh = static_cast<int>(blockIdx.y);  // b * heads_kv + h
  const int b = bh / g.heads_kv, h = bh % g.heads_kv;
  int n_valid = g.length;
  if (g.lengths != nullptr) n_valid = min(n_valid, static_cast<int>(__ldg(g.lengths + b)));
  const int t_begin = sp * g.chunk;
  const int t_end = min(t_begin + g.chunk, n_valid);
  const int n_tiles = t_end > t_begin ? (t_end - t_begin + 127) / 128 : 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      tc::mbar_init(&kv_full[s], 1);
      tc::mbar_init(&kv_empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      tc::mbar_init(&s_full[i], 1);
      tc::mbar_init(&s_free[i], 4);
      tc::mbar_init(&p_full[i], 4);
      tc::mbar_init(&p_free[i], 1);
      tc::mbar_init(&o_full[i], 1);
      tc::mbar_init(&o_free[i], 4);
    }
    tc::mbar_init(&drain[0], 1);
    tc::mbar_init(&drain[1], 1);
    tc::fence_barrier_init();
  }
  // The first tiles' loads go out at once (thread 0 initialised the barriers; the ring is
  // empty), so that their HBM latency overlaps the query's preparation.
  auto load_tile = [&](int i) {
    const int s = i % S;
    tc::mbar_arrive_expect_tx(&kv_full[s], 2 * L::kTile);
    uint8_t* st = sRing + s * L::kStage;
    const int t0 = t_begin + i * 128;
    tma_load_4d(&tma_k, &kv_full[s], st, 0, t0, h, b);
    tma_load_4d(&tma_v, &kv_full[s], st + L::kTile, 0, t0, h, b);
  };
  const int prefill = min(n_tiles, S);
  if (threadIdx.x == 0)
    for (int i = 0; i < prefill; ++i) load_tile(i);
  if (warp == 1) { tc::tmem_alloc(tmem_slot, L::kTmemCols); tc::tmem_relinquish(); }

  // ---- Q as two e4m3 terms per row (warps 2-13, one query head per warp at a time)
  if (warp >= 2) {
    constexpr int PER = D / 32;  // elements per lane
    for (int gi = warp - 2; warp < 14 && gi < GP; gi += 12) {
      float v[PER];
      if (gi < g.group) {
        const int64_t base = static_cast<int64_t>(b) * g.sqb + static_cast<int64_t>(h * g.group + gi) * g.sqh;
#pragma unroll
        for (int e = 0; e < PER; ++e) {
          const int64_t idx = base + lane * PER + e;
          if constexpr (QT == kBF16)
            v[e] = __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(g.q)[idx]);
          else if constexpr (QT == kF16)
            v[e] = __half2float(reinterpret_cast<const __half*>(g.q)[idx]);
          else
            v[e] = __bfloat162float(__float2bfloat16_rn(reinterpret_cast<const float*>(g.q)[idx]));
        }
      } else {
#pragma unroll
        for (int e = 0; e < PER; ++e) v[e] = 0.0f;
      }
      uint32_t ab = 0;
#pragma unroll
      for (int e = 0; e < PER; ++e) ab = max(ab, __float_as_uint(v[e]) & 0x7FFFFFFFu);
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) ab = max(ab, __shfl_xor_sync(0xffffffffu, ab, off));
      const int e2 = scale_exp(__uint_as_float(ab));
      const float up = pow2f(e2);
      uint32_t hi = 0, lo = 0;  // PER <= 4 codes of each term
#pragma unroll
      for (int e = 0; e < PER; e += 2) {
        const uint32_t w = split2(v[e] * up, v[e + 1] * up);
        hi |= (w & 0xFFFFu) << (8 * e);
        lo |= (w >> 16) << (8 * e);
      }
      // row n = term * GP + gi, byte d = lane * PER: 16-byte chunk d / 16 swizzled by the row
      const int d0 = lane * PER;
#pragma unroll
      for (int term = 0; term < 2; ++term) {
        const int n = term * GP + gi;
        const int c = d0 >> 4;
        int sw;
        if constexpr (D == 128) sw = c ^ (n & 7);
        else sw = c ^ ((n >> 1) & 3);
        uint8_t* dst = sQ + n * L::kRow + sw * 16 + (d0 & 15);
        if constexpr (PER == 4) *reinterpret_cast<uint32_t*>(dst) = term ? lo : hi;
        else *reinterpret_cast<uint16_t*>(dst) = static_cast<uint16_t>(term ? lo : hi);
      }
      if (lane == 0) {
        qinv[gi] = pow2f(-e2);
        qinv[GP + gi] = pow2f(-e2 - 4);
      }
    }
    if constexpr (L::kZero > 0) {  // the zero rows of V^T in every stage
      const int t = threadIdx.x - 64;
      for (int s = 0; s < S; ++s) {
        uint4* z = reinterpret_cast<uint4*>(sRing + s * L::kStage + 2 * L::kTile);
        for (int i = t; i < L::kZero / 16; i += L::kThreads - 64) z[i] = make_uint4(0, 0, 0, 0);
      }
    }
    tc::fence_proxy_async();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tS = tmem, tO = tmem + 2 * N;

  // The MMAs of tile i, each from a thread that does nothing else: S_i by warp 14 as soon as
  // the softmax group that owns the tile (its tiles are i, i + 2, ...; S, P and O buffers
  // i & 1 are the group's own) has read S_{i-2} out of TMEM, so that its latency hides under
  // tile i - 2's softmax; P V_i by warp 1 once P_i is written. (Issuing from a softmax warp
  // put the MMAs' issue and waits on the group's path: 1.2 us per tile instead of 0.9.)
  const uint32_t idesc_s = tc::idesc_f8(128, N);
  const uint32_t idesc_pv = tc::idesc_f8(128, N) | (1u << 15) | (1u << 16);  // A and B MN-major
  auto kdesc = [&](uint32_t a) { return D == 128 ? tc::desc_sw128(a) : tc::desc_sw64(a); };
  auto issue_s = [&](int i) {  // S^T_i = K_i (Q_hi | Q_lo)^T, once K_i has landed
    const int s = i % S;
    const uint64_t kd = kdesc(tc::smem_u32(sRing + s * L::kStage));
    const uint64_t qd = kdesc(tc::smem_u32(sQ));
#pragma unroll
    for (int kk = 0; kk < D / 32; ++kk)
      tc::mma_f8(tS + (i & 1) * N, kd + static_cast<uint64_t>(2 * kk), qd + static_cast<uint64_t>(2 * kk), idesc_s,
                 kk > 0 ? 1u : 0u);
    tc::commit(&s_full[i & 1]);
  };
  auto issue_pv = [&](int i) {  // O^T_i = V_i^T (P_hi | P_lo)^T, then release V, P and K
    const int s = i % S;
    const uint32_t v_addr = tc::smem_u32(sRing + s * L::kStage + L::kTile);
    const uint32_t p_addr = tc::smem_u32(sP + (i & 1) * L::kPBytes);
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {  // 32 tokens per MMA
      uint64_t vd;
      if constexpr (D == 128) vd = tc::desc_sw128(v_addr + kk * 32 * L::kRow);
      else vd = desc_vt64(v_addr + kk * 32 * L::kRow, static_cast<uint32_t>(L::kTile));
      tc::mma_f8(tO + (i & 1) * N, vd, desc_p(p_addr + kk * 512), idesc_pv, kk > 0 ? 1u : 0u);
    }
    tc::commit(&o_full[i & 1]);
    tc::commit(&p_free[i & 1]);
    tc::commit(&kv_empty[s]);
  };

  if (warp == 0) {
    if (lane == 0 && n_tiles > 0) {  // ---------------------------------------- TMA producer
      bool ok = true;
      int issued = prefill;
      for (int i = prefill; i < n_tiles; ++i) {
        if (!tc::mbar_wait(&kv_empty[i % S], static_cast<uint32_t>(((i / S) & 1) ^ 1))) { ok = false; break; }
        load_tile(i);
        issued = i + 1;
      }
      if (!ok) {
        atomicOr(&g_attention_status, kDevTimeout);
        for (int i = (issued > S ? issued - S : 0); i < issued; ++i)
          tc::mbar_wait(&kv_full[i % S], static_cast<uint32_t>((i / S) & 1));
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && n_tiles > 0) {  // ------------------------------------ P V issuer
      // P V_i once the group's four warps have written P_i and the merge warps have released
      // O buffer i & 1 (read tile i - 2); in tile order, off the softmax groups' path
      bool ok = true;
      for (int i = 0; i < n_tiles; ++i) {
        if (!tc::mbar_wait(&p_full[i & 1], static_cast<uint32_t>((i >> 1) & 1))) { ok = false; break; }
        if (!tc::mbar_wait(&o_free[i & 1], static_cast<uint32_t>(((i >> 1) & 1) ^ 1))) { ok = false; break; }
        tc::fence_after_sync();
        issue_pv(i);
      }
      tc::commit(&drain[1]);  // every P V issued has completed once this arrives
      if (!tc::mbar_wait(&drain[1], 0)) ok = false;
      if (!ok) atomicOr(&g_attention_status, kDevTimeout);
    }
  } else if (warp < 10) {  // ------------------------------------------------ softmax warps
    // two groups of four warps take the even and the odd tiles; a warp's TMEM lane quarter
    // (warp % 4) holds 32 of a tile's tokens
    const int grp = (warp - 2) >> 2;
    const int quarter = warp & 3;
    const int wi = (warp - 2) & 3;  // 0..3 within the group
    const uint32_t lane_base = static_cast<uint32_t>(32 * quarter) << 16;
    const int tok = 32 * quarter + lane;  // TMEM lane = token within the tile
    const float* ksp = g.k_scale + static_cast<int64_t>(b) * g.ksb + static_cast<int64_t>(h) * g.ksh;
    const float* vsp = g.v_scale + static_cast<int64_t>(b) * g.vsb + static_cast<int64_t>(h) * g.vsh;
    // A failed wait leaves `ok` false; the group's four warps agree on it at the next named
    // barrier (a reduction) and leave the loop together, so that none waits there for a warp
    // that left.
    bool ok = true;
    // the token scales two of the group's tiles ahead (a DRAM round trip per tile would sit on
    // the critical path); the raw values are kept until their tile so that no use waits early
    auto ld_scales = [&](int i, float& ks, float& vs) {
      const int t = t_begin + i * 128 + tok;
      const bool valid = i < n_tiles && t < t_end;
      ks = valid ? __ldg(ksp + t) : 0.0f;
      vs = valid ? __ldg(vsp + t) : 0.0f;
    };
    float ks_a, vs_a, ks_b, vs_b;
    ld_scales(grp, ks_a, vs_a);
    ld_scales(grp + 2, ks_b, vs_b);
    for (int i = grp; i < n_tiles; i += 2) {
      const int t = t_begin + i * 128 + tok;
      const bool valid = t < t_end;
      const float kq = ks_a * g.scale_log2;
      const float vs = vs_a;
      ks_a = ks_b;
      vs_a = vs_b;
      ld_scales(i + 4, ks_b, vs_b);
      if (ok) ok = warp_wait_d(&s_full[i & 1], static_cast<uint32_t>((i >> 1) & 1));
      float sl[GP];
#pragma unroll
      for (int j = 0; j < GP; ++j) sl[j] = -INFINITY;
      if (ok) {
        tc::fence_after_sync();
        uint32_t raw[N];
        tmem_ld_cols<N>(tS + lane_base + (i & 1) * N, raw);
        tc::tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < GP; ++j) {
          const float dot = __uint_as_float(raw[j]) * qinv[j] + __uint_as_float(raw[GP + j]) * qinv[GP + j];
          sl[j] = valid ? dot * kq : -INFINITY;  // scores in the log2 domain
        }
        tc::fence_before_sync();
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(&s_free[i & 1]);  // S buffer i & 1 may take S_{i+2}
      }
      // the tile's max per query head (and of the V scales): warp partials, then the 4 warps
      float part[GP];
#pragma unroll
      for (int j = 0; j < GP; ++j) part[j] = sl[j];
      const float wmax = warp_reduce_scatter<GP, true>(part, lane);
      float vmax = vs;
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) vmax = fmaxf(vmax, __shfl_xor_sync(0xffffffffu, vmax, off));
      const int slot = grp * 2 + ((i >> 1) & 1);  // two slots per group: tiles i and i + 2
      float* rd = red + (slot * 4 + wi) * (GP + 4);
      constexpr int kShift = GP == 8 ? 2 : GP == 16 ? 1 : 0;  // lane >> kShift: the row a lane reduced
      if ((lane & ((1 << kShift) - 1)) == 0) rd[lane >> kShift] = wmax;
      if (lane == 0) rd[GP] = vmax;
      if (named_sync_any(1 + grp, 128, !ok)) { ok = false; break; }
      float mt[GP];
      float vt = 0.0f;
#pragma unroll
      for (int j = 0; j < GP; ++j) mt[j] = -INFINITY;
#pragma unroll
      for (int w = 0; w < 4; ++w) {
        const float* rw = red + (slot * 4 + w) * (GP + 4);
#pragma unroll
        for (int j = 0; j < GP; j += 4) {
          const float4 m4 = *reinterpret_cast<const float4*>(rw + j);
          mt[j] = fmaxf(mt[j], m4.x);
          mt[j + 1] = fmaxf(mt[j + 1], m4.y);
          mt[j + 2] = fmaxf(mt[j + 2], m4.z);
          mt[j + 3] = fmaxf(mt[j + 3], m4.w);
        }
        vt = fmaxf(vt, rw[GP]);
      }
      const int f = scale_exp(vt);
      const float w8 = vs * pow2f(f);  // P' = p * v_scale * 2^f <= 256
      float p[GP];
#pragma unroll
      for (int j = 0; j < GP; ++j) p[j] = valid ? ex2(sl[j] - mt[j]) : 0.0f;
      uint32_t hi[GP / 4], lo[GP / 4];
#pragma unroll
      for (int j = 0; j < GP; j += 4) {
        const uint32_t a = split2(p[j] * w8, p[j + 1] * w8);
        const uint32_t c = split2(p[j + 2] * w8, p[j + 3] * w8);
        hi[j / 4] = (a & 0xFFFFu) | (c << 16);
        lo[j / 4] = (a >> 16) | (c & 0xFFFF0000u);
      }
      const float wsum = warp_reduce_scatter<GP, false>(p, lane);
      // P'_i into its buffer once P V_{i-2} has read it (a failed wait skips the rest of the
      // tile's work; the group leaves together at its next barrier)
      if (ok) ok = warp_wait_d(&p_free[i & 1], static_cast<uint32_t>(((i >> 1) & 1) ^ 1));
      if (ok) {
        uint8_t* pb = sP + (i & 1) * L::kPBytes + tok * 16;
        {  // the token's row of P: the hi codes of its GP columns, then the lo codes
          uint32_t w[GP / 2];
#pragma unroll
          for (int j = 0; j < GP / 4; ++j) { w[j] = hi[j]; w[GP / 4 + j] = lo[j]; }
#pragma unroll
          for (int blk = 0; blk < GP / 8; ++blk)
            *reinterpret_cast<uint4*>(pb + blk * 2048) = make_uint4(w[4 * blk], w[4 * blk + 1], w[4 * blk + 2], w[4 * blk + 3]);
        }
        // tokens in [n_valid, L) of the last tile: zero their V rows (the codes there are not
        // this sequence's; a NaN code times p = 0 would reach O)
        bool landed = true;
        if (t >= t_end && t < g.length) {
          landed = tc::mbar_wait(&kv_full[i % S], static_cast<uint32_t>((i / S) & 1));
          if (landed) {
            uint4* vrow = reinterpret_cast<uint4*>(sRing + (i % S) * L::kStage + L::kTile + tok * L::kRow);
#pragma unroll
            for (int c = 0; c < L::kRow / 16; ++c) vrow[c] = make_uint4(0, 0, 0, 0);
          }
        }
        ok = __all_sync(0xffffffffu, landed);
      }
      // the stats of tile i into slot i & 1 once the merge warps have read those of tile i - 2
      // (they read them before releasing O of tile i - 2; that phase of o_free cannot have
      // been overtaken, as the next one needs P V_i, issued after this group's barrier below)
      if (ok) ok = warp_wait_d(&o_free[i & 1], static_cast<uint32_t>(((i >> 1) & 1) ^ 1));
      if (ok) {
        float* st = stats + (i & 1) * L::kStatsFloats;
        if ((lane & ((1 << kShift) - 1)) == 0) st[L::kSL + wi * GP + (lane >> kShift)] = wsum;
        if (wi == 0) {
          if (lane < GP) {  // the tile's max of row `lane`
            float mi = -INFINITY;
#pragma unroll
            for (int w = 0; w < 4; ++w) mi = fmaxf(mi, red[(slot * 4 + w) * (GP + 4) + lane]);
            st[L::kSM + lane] = mi;
          }
          if (lane == 0) st[L::kSF] = __int_as_float(f);
        }
        tc::fence_proxy_async();
        tc::fence_before_sync();
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(&p_full[i & 1]);
      }
    }
    if (!ok && lane == 0) atomicOr(&g_attention_status, kDevTimeout);
  } else if (warp == 14) {
    if (lane == 0 && n_tiles > 0) {  // -------------------------------------- S issuer
      bool ok = true;
      for (int i = 0; i < n_tiles; ++i) {
        if (!tc::mbar_wait(&kv_full[i % S], static_cast<uint32_t>((i / S) & 1))) { ok = false; break; }
        if (!tc::mbar_wait(&s_free[i & 1], static_cast<uint32_t>(((i >> 1) & 1) ^ 1))) { ok = false; break; }
        tc::fence_after_sync();
        issue_s(i);
      }
      tc::commit(&drain[0]);  // every S issued has completed once this arrives
      if (!tc::mbar_wait(&drain[0], 0)) ok = false;
      if (!ok) atomicOr(&g_attention_status, kDevTimeout);
    }
  } else {  // --------------------------------------------------------------- merge warps
    const int quarter = warp & 3;
    const uint32_t lane_base = static_cast<uint32_t>(32 * quarter) << 16;
    const int d = 32 * quarter + lane;  // TMEM lane = head-dim element
    float o_run[GP], m_run[GP];  // the running output and max (log2 domain) per query row
#pragma unroll
    for (int j = 0; j < GP; ++j) { o_run[j] = 0.0f; m_run[j] = -INFINITY; }
    float l_run = 0.0f;  // thread d < GP: the running row sum of query row d
    bool ok = true;
    for (int i = 0; i < n_tiles; ++i) {
      if (!warp_wait_d(&o_full[i & 1], static_cast<uint32_t>((i >> 1) & 1))) { ok = false; break; }
      tc::fence_after_sync();
      uint32_t raw[N];
      tmem_ld_cols<N>(tO + lane_base + (i & 1) * N, raw);
      tc::tmem_ld_wait();
      // the stats of tile i: written before the softmax warps' arrival on p_full[i & 1], whose
      // phase of tile i cannot have been overtaken (the next needs this warp's o_free below)
      if (!warp_wait_d(&p_full[i & 1], static_cast<uint32_t>((i >> 1) & 1))) { ok = false; break; }
      const float* st = stats + (i & 1) * L::kStatsFloats;
      const float down = pow2f(-__float_as_int(st[L::kSF]));
      float la = 0.0f, lc = 0.0f;
#pragma unroll
      for (int j = 0; j < GP; ++j) {  // merge tile i with its own max into the running state
        const float mi = st[L::kSM + j];
        const float mn = fmaxf(m_run[j], mi);
        const float a = m_run[j] == -INFINITY ? 0.0f : ex2(m_run[j] - mn);
        const float c = ex2(mi - mn);
        const float oi = (__uint_as_float(raw[j]) + __uint_as_float(raw[GP + j]) * 0.0625f) * down;
        o_run[j] = o_run[j] * a + oi * c;
        m_run[j] = mn;
        if (j == d) { la = a; lc = c; }
      }
      if (d < GP)
        l_run = l_run * la +
                ((st[L::kSL + d] + st[L::kSL + GP + d]) + (st[L::kSL + 2 * GP + d] + st[L::kSL + 3 * GP + d])) * lc;
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(&o_free[i & 1]);
    }
    if (!ok && lane == 0) atomicOr(&g_attention_status, kDevTimeout);
    __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(g.out);
    const int64_t orow = static_cast<int64_t>(b) * g.heads_kv * g.group + static_cast<int64_t>(h) * g.group;
    float m_fin = -INFINITY;  // thread d < GP: the running max of row d (empty split: -inf)
#pragma unroll
    for (int j = 0; j < GP; ++j)
      if (j == d) m_fin = m_run[j];
    if (g.splits == 1) {
      float* lfin = reinterpret_cast<float*>(smem + L::kLfin);
      if (d < GP) lfin[d] = l_run;
      named_sync(3, 128);
      if (d < D) {
        for (int j = 0; j < GP; ++j)
          if (j < g.group) out[(orow + j) * D + d] = __float2bfloat16_rn(o_run[j] / lfin[j]);
      }
    } else if (g.cluster) {
      // this split's partial in this CTA's shared memory (the ring is free: every tile's P V
      // has completed), read by the cluster's CTAs after the launch's last barrier
      float* part = reinterpret_cast<float*>(sRing);  // [group][D], then max [GP], sum [GP]
      if (d < D) {
#pragma unroll
        for (int j = 0; j < GP; ++j)
          if (j < g.group) part[j * D + d] = o_run[j];
      }
      if (d < GP) {
        part[GP * D + d] = m_fin;
        part[GP * D + GP + d] = l_run;
      }
    } else {
      // this split's partial, then the last CTA of (sequence, KV head) merges them all
      const int64_t pbase = static_cast<int64_t>(bh) * g.splits + sp;
      if (d < D) {
        float* po = g.part_o + pbase * GP * D + d;
#pragma unroll
        for (int j = 0; j < GP; ++j)
          if (j < g.group) po[j * D] = o_run[j];
      }
      if (d < GP) {
        float* pml = g.part_ml + pbase * 2 * GP;
        pml[d] = m_fin;
        pml[GP + d] = l_run;
      }
      __threadfence();
      named_sync(3, 128);
      if (threadIdx.x == 320) {
        const unsigned old = atomicAdd(g.counters + bh, 1u);
        const bool last = old == static_cast<unsigned>(g.splits - 1);
        if (last) atomicExch(g.counters + bh, 0u);
        *last_flag = last ? 1u : 0u;
      }
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc::fence_after_sync();
    tc::tmem_dealloc(tmem, L::kTmemCols);
  }
  // ---- the cluster's CTAs merge the splits' partials from each other's shared memory, each
  // CTA a slice of the outputs; the second cluster barrier keeps every partial in place until
  // all slices are read (every thread of every CTA of the cluster reaches both barriers)
  if (g.splits > 1 && g.cluster) {
    tc::cluster_sync();
    const int cs = g.splits, rank = static_cast<int>(tc::cluster_ctarank());
    const int quads = g.group * (D / 4);
    const int per = (quads + cs - 1) / cs;
    const float* part = reinterpret_cast<const float*>(sRing);
    __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(g.out);
    const int64_t orow = static_cast<int64_t>(b) * g.heads_kv * g.group + static_cast<int64_t>(h) * g.group;
    for (int o = rank * per + static_cast<int>(threadIdx.x); o < min(quads, (rank + 1) * per); o += L::kThreads) {
      const int j = o / (D / 4), d4 = (o % (D / 4)) * 4;
      float ms[16], w[16];
      float mx = -INFINITY;
#pragma unroll
      for (int s2 = 0; s2 < 16; ++s2) {
        ms[s2] = s2 < cs ? ld_cluster_f32(tc::mapa(part + GP * D + j, s2)) : -INFINITY;
        mx = fmaxf(mx, ms[s2]);
      }
      float den = 0.0f;
#pragma unroll
      for (int s2 = 0; s2 < 16; ++s2) {
        w[s2] = ms[s2] == -INFINITY ? 0.0f : ex2(ms[s2] - mx);  // an empty split weighs 0
        if (s2 < cs) den += w[s2] * ld_cluster_f32(tc::mapa(part + GP * D + GP + j, s2));
      }
      float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
#pragma unroll
      for (int s2 = 0; s2 < 16; ++s2) {
        if (s2 < cs) {
          const float4 v = ld_cluster_f32x4(tc::mapa(part + j * D + d4, s2));
          acc.x += w[s2] * v.x;
          acc.y += w[s2] * v.y;
          acc.z += w[s2] * v.z;
          acc.w += w[s2] * v.w;
        }
      }
      const float inv = 1.0f / den;
      __nv_bfloat162* dst = reinterpret_cast<__nv_bfloat162*>(out + (orow + j) * D + d4);
      dst[0] = __floats2bfloat162_rn(acc.x * inv, acc.y * inv);
      dst[1] = __floats2bfloat162_rn(acc.z * inv, acc.w * inv);
    }
    __syncwarp();
    tc::cluster_sync();
  }
  // ---- the last CTA of (sequence, KV head) merges the splits' partials (all threads; the
  // ring's shared memory is free: every load landed and every MMA completed)
  if (g.splits > 1 && !g.cluster && *last_flag != 0u) {
    __threadfence();
    const int tid = threadIdx.x;
    const int64_t first = static_cast<int64_t>(bh) * g.splits;
    float* wts = reinterpret_cast<float*>(sRing);  // [splits][2][GP]: max, sum -> weight
    for (int i = tid; i < g.splits * 2 * GP; i += L::kThreads) wts[i] = __ldcg(g.part_ml + first * 2 * GP + i);
    __syncthreads();
    if (tid < GP) {  // weight of split s for row tid: 2^(m_s - M) / sum_s' 2^(m_s' - M) l_s'
      float mx = -INFINITY;
      for (int s2 = 0; s2 < g.splits; ++s2) mx = fmaxf(mx, wts[s2 * 2 * GP + tid]);
      float den = 0.0f;
      for (int s2 = 0; s2 < g.splits; ++s2) {
        const float ms = wts[s2 * 2 * GP + tid];
        const float w = ms == -INFINITY ? 0.0f : ex2(ms - mx);  // an empty split weighs 0
        wts[s2 * 2 * GP + tid] = w;
        den += w * wts[s2 * 2 * GP + GP + tid];
      }
      const float inv = 1.0f / den;
      for (int s2 = 0; s2 < g.splits; ++s2) wts[s2 * 2 * GP + tid] *= inv;
    }
    __syncthreads();
    __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(g.out);
    const int64_t orow = static_cast<int64_t>(b) * g.heads_kv * g.group + static_cast<int64_t>(h) * g.group;
    // one thread per 4 consecutive outputs of a row; the partials' float4 loads of 16 splits
    // are in flight together
    for (int o = tid; o < g.group * (D / 4); o += L::kThreads) {
      const int j = o / (D / 4), d4 = (o % (D / 4)) * 4;
      const float4* po = reinterpret_cast<const float4*>(g.part_o + (first * GP + j) * D + d4);
      const int64_t step = static_cast<int64_t>(GP) * D / 4;  // float4s between splits
      float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
      for (int s0 = 0; s0 < g.splits; s0 += 16) {
        float4 v[16];
#pragma unroll
        for (int u = 0; u < 16; ++u)
          v[u] = s0 + u < g.splits ? __ldcg(po + static_cast<int64_t>(s0 + u) * step) : make_float4(0, 0, 0, 0);
#pragma unroll
        for (int u = 0; u < 16; ++u) {
          const float w = s0 + u < g.splits ? wts[(s0 + u) * 2 * GP + j] : 0.0f;
          acc.x += w * v[u].x;
          acc.y += w * v[u].y;
          acc.z += w * v[u].z;
          acc.w += w * v[u].w;
        }
      }
      __nv_bfloat162* dst = reinterpret_cast<__nv_bfloat162*>(out + (orow + j) * D + d4);
      dst[0] = __floats2bfloat162_rn(acc.x, acc.y);
      dst[1] = __floats2bfloat162_rn(acc.z, acc.w);
    }
  }
}

}  // namespace kab
