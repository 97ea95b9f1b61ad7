// FP8 (e4m3) causal attention prefill with one scale per (batch, head), the "qkpv" emulation
// of kernel-agent's docs/research-scripts/fp8-sm120/fp8lib.py:184-215 (emulated_sdpa):
// Q, K, V quantised per head over [S, D] (_fq_last2, fp8lib.py:173-176: scale amax / 448,
// a zero scale replaced by 1), S = Q K^T on e4m3 codes, P = exp(S - max) carried as
// e4m3(P * 448) / 448 into P V, the row sum taken before P is rounded.
//
//  * quant_heads kernels: the per-head amax (one atomic max of the bits per block) and the
//    codes, row-major [S, D] for Q and K, transposed [D, S] for V so that V^T is the
//    K-major B operand of the P V product.
//  * attention_fp8_kernel: one CTA per 128-query tile, two CTAs per SM (256 TMEM columns and
//    ~97 KB of shared memory each), so the softmax of one CTA runs while the other's MMAs do.
//    Warp 0 loads Q once and K / V^T tiles of 128 keys through a 2-stage TMA ring; warp 1
//    issues the tcgen05 MMAs (kind::f8f6f4): S_j = Q K_j^T into a 128-column TMEM buffer
//    (released as soon as the softmax has read it), then O += P_j V_j into a second;
//    warps 2-5 (one query row per thread) run the online softmax in the exp2 domain: a
//    running row max m raised only when a tile's max exceeds it by more than 3 (so
//    p = 2^(t - m) <= 8), the row sum of the unrounded codes' values, P as e4m3(p * 448 / 8)
//    written into shared memory in the 128-byte swizzled layout the MMA reads, and the
//    rescaling of O in TMEM when m moves (after the previous P V has landed). The final O is
//    divided by the row sum, multiplied by the V scale and stored in bf16.
//
// The running max replaces the reference's global row max: P is rounded relative to the max
// seen so far (with 8x headroom), so its codes differ from the reference's, and the result is
// judged against fp32 attention by relative L2 and cosine, as the reference's own emulation
// is.
// No load uses cluster multicast; every wait is bounded and records kDevTimeout.
#pragma once

#include "codes.cuh"
#include "tcgen05.cuh"

namespace kab {

// g_attention_status: the device status word, defined by the including translation unit
// (kab_attention.cu) before this header.

// ------------------------------------------------------------------ per-head quantiser

// Per-head NaN-keeping amax as float bits: grid (blocks per head, heads); a head is a
// contiguous [S, D] slab of `per_head` elements. amax[] holds 0 before the launch.
template <int T>
__global__ void __launch_bounds__(256)
head_amax_kernel(const void* __restrict__ x, int64_t per_head, unsigned* __restrict__ amax) {
  __shared__ float red[32];
  const int64_t head = blockIdx.y;
  const int64_t chunks = per_head >> 3;
  uint32_t bits = 0;
  for (int64_t c = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; c < chunks;
       c += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    float v[8];
    load8<T>(x, head * per_head + c * 8, v);
    bits = abs_bits_max8(v, bits);
  }
  const float m = block_amax(__uint_as_float(bits), red);
  if (threadIdx.x == 0) atomicMax(amax + head, __float_as_uint(m) & 0x7FFFFFFFu);
}

// fp8lib.py:173-176: scale = amax / 448 (0 or NaN -> 1), codes e4m3(x / scale).
__device__ __forceinline__ float head_scale(unsigned amax_bits) {
  const float s = __fdiv_rn(__uint_as_float(amax_bits), kFp8Max);
  return s > 0.0f ? s : 1.0f;
}

// Codes of a [64 rows, D] tile of one head: grid (ceil(S / 64), heads), 256 threads. TRANSPOSE
// writes the tile into [D, S16] (S16 = S rounded up to 16, the columns past S zero: the row
// stride a TMA map needs), column block s0 .. s0 + 63 of each of the D rows.
template <int T, bool TRANSPOSE>
__global__ void __launch_bounds__(256)
quant_heads_kernel(const void* __restrict__ x, int64_t seq, int d, const unsigned* __restrict__ amax,
                   uint8_t* __restrict__ q, float* __restrict__ scales) {
  extern __shared__ uint8_t tile[];  // [64][d] codes (TRANSPOSE only)
  const int64_t head = blockIdx.y;
  const int64_t s0 = static_cast<int64_t>(blockIdx.x) * 64;
  const float sc = head_scale(amax[head]);
  if (blockIdx.x == 0 && threadIdx.x == 0) scales[head] = sc;
  const Divisor div(sc);
  const int cpr = d >> 3;  // chunks of 8 per row
  const int total = 64 * cpr;
  for (int c = threadIdx.x; c < total; c += blockDim.x) {
    const int r = c / cpr, col = (c % cpr) * 8;
    if (s0 + r >= seq) {
      if constexpr (TRANSPOSE) *reinterpret_cast<uint2*>(tile + r * d + col) = make_uint2(0u, 0u);
      continue;
    }
    float v[8];
    load8<T>(x, (head * seq + s0 + r) * d + col, v);
    const uint2 codes = e4m3x8_quotients(v, div);
    if constexpr (TRANSPOSE) *reinterpret_cast<uint2*>(tile + r * d + col) = codes;
    else *reinterpret_cast<uint2*>(q + (head * seq + s0 + r) * d + col) = codes;
  }
  if constexpr (TRANSPOSE) {
    __syncthreads();
    // [D, S16]: row dd gets the tile's 64 codes of column dd, 16 at a time
    const int64_t ld = (seq + 15) / 16 * 16;
    for (int c = threadIdx.x; c < d * 4; c += blockDim.x) {
      const int dd = c >> 2, part = c & 3;
      uint32_t w[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        uint32_t word = 0;
#pragma unroll
        for (int b = 0; b < 4; ++b) word |= static_cast<uint32_t>(tile[(part * 16 + i * 4 + b) * d + dd]) << (8 * b);
        w[i] = word;
      }
      const int64_t col = s0 + part * 16;
      if (col < ld) *reinterpret_cast<uint4*>(q + (head * d + dd) * ld + col) = make_uint4(w[0], w[1], w[2], w[3]);
    }
  }
}

// ------------------------------------------------------------------ attention

struct AttnArgs {
  int seq;            // keys = queries (any length: the last tile's keys past it are masked)
  int heads_q, heads_kv;
  int q_tiles;        // ceil(seq / 128)
  int causal;
  const float* q_scale;  // [batch * heads_q]
  const float* k_scale;  // [batch * heads_kv]
  const float* v_scale;
  float sm_scale_log2;   // softmax scale * log2(e)
  void* out;             // [batch, heads_q, seq, D] bf16
};

// Shared memory of one CTA for head dimension D (128 or 64): Q and the K ring hold
// [128 tokens, D] tiles (rows of D bytes, swizzled at D bytes), the V^T ring [D, 128 keys]
// tiles and P one [128, 128] tile (rows of 128 bytes, the 128-byte swizzle).
template <int D>
struct AttnLayout {
  static_assert(D == 128 || D == 64, "head_dim 128 or 64");
  static constexpr int kQKTile = 128 * D;
  static constexpr int kVTile = D * 128;
  static constexpr int kPTile = 128 * 128;
  static constexpr int kStages = 2;
  static constexpr int kThreads = 192;
  static constexpr int kQ = 0;
  static constexpr int kK = kQ + kQKTile;
  static constexpr int kV = kK + kStages * kQKTile;
  static constexpr int kP = kV + kStages * kVTile;
  static constexpr int kBars = kP + kPTile;
  static constexpr int kNumBars = 1 + 4 * kStages + 4 + 1;
  static constexpr int kTmemCols = 256;  // S at column 0, O (D columns) at 128
  static constexpr int kSmem = 1024 + kBars + kNumBars * 8 + 16;
};

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// max(a, b, c) in one instruction (the three-input form of sm_100; a NaN input is ignored,
// as by fmaxf).
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// Two fp32 lanes per instruction (packed f32x2 arithmetic of sm_100), each lane rounded to
// nearest like its scalar form.
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) {
  float2 d;
  asm("{\n .reg .b64 a, b, c, d;\n mov.b64 a, {%2, %3};\n mov.b64 b, {%4, %5};\n mov.b64 c, {%6, %7};\n"
      " fma.rn.f32x2 d, a, b, c;\n mov.b64 {%0, %1}, d;\n}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
  return d;
}
__device__ __forceinline__ float2 add2(float2 a, float2 b) {
  float2 d;
  asm("{\n .reg .b64 a, b, d;\n mov.b64 a, {%2, %3};\n mov.b64 b, {%4, %5};\n add.rn.f32x2 d, a, b;\n"
      " mov.b64 {%0, %1}, d;\n}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}
__device__ __forceinline__ float2 sub2(float2 a, float2 b) {
  float2 d;
  asm("{\n .reg .b64 a, b, d;\n mov.b64 a, {%2, %3};\n mov.b64 b, {%4, %5};\n sub.rn.f32x2 d, a, b;\n"
      " mov.b64 {%0, %1}, d;\n}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}

// 2^t for two lanes on the FMA pipe instead of the MUFU unit (which the softmax saturates with
// exp2 and the e4m3 conversions). Range reduction: t is clamped to >= -120 (so 2^t stays a
// normal float; masked -inf scores give ~1e-36, which rounds to the e4m3 code 0 and is nothing
// in a row sum >= 1), n = round(t) by adding and subtracting 1.5 * 2^23 (fp32 addition rounds
// to an integer there), r = t - n in [-1/2, 1/2]; 2^r by a degree-3 polynomial, the minimax
// fit of 2^r in relative error on [-1/2, 1/2] (coefficients computed for this kernel by linear
// programming on a dense grid; maximum relative error 7.5e-5 in fp32 Horner form, against
// e4m3's relative step of 1/16); then n is added to the exponent field: the bits of
// 1.5 * 2^23 + n shifted left by 23 are n << 23, modulo 2^32.
__device__ __forceinline__ float2 exp2_poly2(float2 t) {
  constexpr float kShift = 12582912.0f;  // 1.5 * 2^23
  t.x = fmaxf(t.x, -120.0f);
  t.y = fmaxf(t.y, -120.0f);
  const float2 f = add2(t, make_float2(kShift, kShift));
  const float2 r = sub2(t, sub2(f, make_float2(kShift, kShift)));
  float2 q = fma2(r, make_float2(0.0551716685295105f, 0.0551716685295105f),
                  make_float2(0.2426111251115799f, 0.2426111251115799f));
  q = fma2(q, r, make_float2(0.6932609677314758f, 0.6932609677314758f));
  q = fma2(q, r, make_float2(0.9999280571937561f, 0.9999280571937561f));
  return make_float2(__uint_as_float(__float_as_uint(q.x) + (__float_as_uint(f.x) << 23)),
                     __uint_as_float(__float_as_uint(q.y) + (__float_as_uint(f.y) << 23)));
}

// Which element pairs of the softmax take exp2_poly2 rather than the MUFU: of every group of
// eight scores, kPolyPairs of the four pairs (the MUFU also carries the e4m3 conversions).
constexpr int kPolyPairs = 1;

// A bounded wait whose outcome the whole warp shares (the softmax warps follow it with
// .sync.aligned TMEM accesses, which need every lane).
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity) {
  return __all_sync(0xffffffffu, tc::mbar_wait(bar, parity));
}

template <int D>
__global__ void __launch_bounds__(AttnLayout<D>::kThreads, 2)
attention_fp8_kernel(const __grid_constant__ CUtensorMap tma_q, const __grid_constant__ CUtensorMap tma_k,
                     const __grid_constant__ CUtensorMap tma_vt, AttnArgs g) {
  using L = AttnLayout<D>;
  constexpr int kChunks = D / 32;  // 32-column TMEM loads of O
  auto qk_desc = [](uint32_t a) { return D == 128 ? tc::desc_sw128(a) : tc::desc_sw64(a); };
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem + L::kQ;
  uint8_t* sK = smem + L::kK;
  uint8_t* sV = smem + L::kV;
  uint8_t* sP = smem + L::kP;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBars);
  uint64_t* q_full = bars;
  // K and V tiles have their own ring barriers: K_j's slot is free once S_j is computed, so the
  // next K loads while the softmax of tile j runs, V's once P_j V_j is
  uint64_t* k_full = bars + 1;
  uint64_t* k_empty = k_full + L::kStages;
  uint64_t* v_full = k_empty + L::kStages;
  uint64_t* v_empty = v_full + L::kStages;
  // one S buffer and one P buffer; use j of each completes phase j (parity j & 1)
  uint64_t* s_full = v_empty + L::kStages;
  uint64_t* s_empty = s_full + 1;  // 4 softmax warps
  uint64_t* p_full = s_empty + 1;  // 4 softmax warps
  uint64_t* p_empty = p_full + 1;
  uint64_t* drain = p_empty + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);

  // heavy (long causal) tiles first
  const int qt = g.q_tiles - 1 - static_cast<int>(blockIdx.x % g.q_tiles);
  const int bh = static_cast<int>(blockIdx.x / g.q_tiles);  // b * heads_q + h
  const int b = bh / g.heads_q, h = bh % g.heads_q;
  const int hk = h / (g.heads_q / g.heads_kv);
  const int bhk = b * g.heads_kv + hk;
  const int n_kv = g.causal ? qt + 1 : g.q_tiles;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    tc::mbar_init(q_full, 1);
    for (int s = 0; s < L::kStages; ++s) {
      tc::mbar_init(&k_full[s], 1);
      tc::mbar_init(&k_empty[s], 1);
      tc::mbar_init(&v_full[s], 1);
      tc::mbar_init(&v_empty[s], 1);
    }
    tc::mbar_init(s_full, 1);
    tc::mbar_init(s_empty, 4);
    tc::mbar_init(p_full, 4);
    tc::mbar_init(p_empty, 1);
    tc::mbar_init(drain, 1);
    tc::fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tc::prefetch_tensormap(&tma_q);
    tc::prefetch_tensormap(&tma_k);
    tc::prefetch_tensormap(&tma_vt);
  }
  if (warp == 1) { tc::tmem_alloc(tmem_slot, L::kTmemCols); tc::tmem_relinquish(); }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tS = tmem, tO = tmem + 128;  // S at column 0, O at 128

  if (warp == 0) {
    if (lane < 2) {  // --------------------------- TMA producers: lane 0 Q and K tiles, lane 1 V^T tiles
      bool ok = true;
      const bool is_k = lane == 0;
      uint64_t* full = is_k ? k_full : v_full;
      uint64_t* empty = is_k ? k_empty : v_empty;
      uint8_t* dst = is_k ? sK : sV;
      const int tile = is_k ? L::kQKTile : L::kVTile;
      if (is_k) {
        tc::mbar_arrive_expect_tx(q_full, L::kQKTile);
        tc::tma_load_2d(&tma_q, q_full, sQ, 0, bh * g.seq + qt * 128);
      }
      int issued = 0;
      for (int j = 0; j < n_kv; ++j) {
        const int s = j % L::kStages;
        const uint32_t ph = static_cast<uint32_t>((j / L::kStages) & 1);
        if (!tc::mbar_wait(&empty[s], ph ^ 1u)) { ok = false; break; }
        tc::mbar_arrive_expect_tx(&full[s], tile);
        if (is_k) tc::tma_load_2d(&tma_k, &full[s], dst + s * tile, 0, bhk * g.seq + j * 128);
        else tc::tma_load_2d(&tma_vt, &full[s], dst + s * tile, j * 128, bhk * D);
        issued = j + 1;
      }
      if (!ok) {
        atomicOr(&g_attention_status, kDevTimeout);
        if (is_k) tc::mbar_wait(q_full, 0);
        for (int j = (issued > L::kStages ? issued - L::kStages : 0); j < issued; ++j)
          tc::mbar_wait(&full[j % L::kStages], static_cast<uint32_t>((j / L::kStages) & 1));
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {  // ---------------------------------------------------- MMA issuer
      bool ok = tc::mbar_wait(q_full, 0);
      const uint32_t idesc = tc::idesc_f8(128, 128);  // S = Q K^T: 128 x 128, K = D
      const uint32_t idesc_pv = tc::idesc_f8(128, D);  // O += P V: 128 x D, K = 128 keys
      const uint64_t qdesc = qk_desc(tc::smem_u32(sQ));
      auto issue_pv = [&](int t) -> bool {
        if (!tc::mbar_wait(p_full, static_cast<uint32_t>(t & 1))) return false;
        const int s = t % L::kStages;
        if (!tc::mbar_wait(&v_full[s], static_cast<uint32_t>((t / L::kStages) & 1))) return false;
        tc::fence_after_sync();
        const uint64_t pdesc = tc::desc_sw128(tc::smem_u32(sP));
        const uint64_t vdesc = tc::desc_sw128(tc::smem_u32(sV + s * L::kVTile));
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          tc::mma_f8(tO, pdesc + static_cast<uint64_t>(2 * kk), vdesc + static_cast<uint64_t>(2 * kk), idesc_pv,
                     (t > 0 || kk > 0) ? 1u : 0u);
        tc::commit(p_empty);
        tc::commit(&v_empty[s]);
        return true;
      };
      for (int j = 0; ok && j < n_kv; ++j) {
        const int s = j % L::kStages;
        if (!tc::mbar_wait(&k_full[s], static_cast<uint32_t>((j / L::kStages) & 1))) { ok = false; break; }
        if (!tc::mbar_wait(s_empty, static_cast<uint32_t>((j & 1) ^ 1))) { ok = false; break; }
        tc::fence_after_sync();
        const uint64_t kdesc = qk_desc(tc::smem_u32(sK + s * L::kQKTile));
#pragma unroll
        for (int kk = 0; kk < D / 32; ++kk)
          tc::mma_f8(tS, qdesc + static_cast<uint64_t>(2 * kk), kdesc + static_cast<uint64_t>(2 * kk), idesc,
                     kk > 0 ? 1u : 0u);
        tc::commit(s_full);
        tc::commit(&k_empty[s]);
        if (j >= 1 && !issue_pv(j - 1)) { ok = false; break; }
      }
      if (ok && !issue_pv(n_kv - 1)) ok = false;
      tc::commit(drain);  // every MMA issued has completed once this arrives
      if (!tc::mbar_wait(drain, 0)) ok = false;
      if (!ok) atomicOr(&g_attention_status, kDevTimeout);
    }
  } else {  // ------------------------------------------------------------ softmax warps
    const int quarter = warp & 3;
    const uint32_t lane_base = static_cast<uint32_t>(32 * quarter) << 16;
    const int r = 32 * quarter + lane;  // query row within the tile
    const int qrow = qt * 128 + r;
    const float scale_log2 = g.q_scale[bh] * g.k_scale[bhk] * g.sm_scale_log2;
    // P is taken relative to a row max m that is only raised when a tile's max exceeds it by
    // more than kHeadroom (log2 units): p = 2^(t - m) <= 2^kHeadroom, and the codes hold
    // e4m3(p * 448 * 2^-kHeadroom) <= 448. O and the row sum are rescaled only when m moves,
    // so the softmax rarely waits for the previous P V.
    constexpr float kHeadroom = 3.0f;
    constexpr float kCodeLog2 = 8.807354922057604f - kHeadroom;  // log2(448) - headroom
    float m_run = -INFINITY, l_run = 0.0f;
    bool ok = true;
    for (int j = 0; j < n_kv; ++j) {
      if (!warp_wait(s_full, static_cast<uint32_t>(j & 1))) { ok = false; break; }
      tc::fence_after_sync();
      float sv[128];
      {  // the four loads in flight together, one wait
        uint32_t raw[4][32];
#pragma unroll
        for (int c = 0; c < 4; ++c) tc::tmem_ld32(tS + lane_base + c * 32, raw[c]);
        tc::tmem_ld_wait();
#pragma unroll
        for (int c = 0; c < 4; ++c)
#pragma unroll
          for (int i = 0; i < 32; ++i) sv[c * 32 + i] = __uint_as_float(raw[c][i]);
      }
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(s_empty);
      if (g.causal && j == qt) {  // keys after the query: -inf
#pragma unroll
        for (int i = 0; i < 128; ++i) sv[i] = i > r ? -INFINITY : sv[i];
      }
      if (j == g.q_tiles - 1 && (g.seq & 127)) {  // keys past the sequence (a ragged last tile): -inf
        const int valid = g.seq - j * 128;
#pragma unroll
        for (int i = 0; i < 128; ++i) sv[i] = i >= valid ? -INFINITY : sv[i];
      }
      float mxs[8];  // eight independent chains of three-input maxima, then a tree
#pragma unroll
      for (int a = 0; a < 8; ++a) mxs[a] = sv[a];
#pragma unroll
      for (int i = 8; i < 120; i += 2) mxs[(i >> 1) & 7] = fmax3(mxs[(i >> 1) & 7], sv[i], sv[i + 1]);
      mxs[4] = fmax3(mxs[4], sv[120], sv[121]);
      mxs[5] = fmax3(mxs[5], sv[122], sv[123]);
      mxs[6] = fmax3(mxs[6], sv[124], sv[125]);
      mxs[7] = fmax3(mxs[7], sv[126], sv[127]);
      const float mx = fmax3(fmax3(mxs[0], mxs[1], mxs[2]), fmax3(mxs[3], mxs[4], mxs[5]), fmaxf(mxs[6], mxs[7]));
      const float tmax = mx * scale_log2;  // the scale is positive: the max of the scaled scores
      const bool raise = !(tmax <= m_run + kHeadroom);
      const float m_new = raise ? tmax : m_run;
      const float alpha = m_run == -INFINITY ? 0.0f : (raise ? ex2(m_run - m_new) : 1.0f);
      const float bias = kCodeLog2 - m_new;
      // P_j goes into the buffer once P V_{j-1} has read it (and landed in O); that MMA was
      // issued when P_{j-1} was written and is done by now, so waiting here costs little and
      // each 16-byte chunk of codes is stored as soon as it is made: the row's 128 scores are
      // the only long-lived registers, which leaves room for the conversions of several chunks
      // to be in flight at once. Row r's chunk c sits at c ^ (r % 8).
      if (!warp_wait(p_empty, static_cast<uint32_t>((j & 1) ^ 1))) { ok = false; break; }
      float2 sums[2] = {make_float2(0.0f, 0.0f), make_float2(0.0f, 0.0f)};  // four independent chains
      const float2 sc2 = make_float2(scale_log2, scale_log2), bias2 = make_float2(bias, bias);
      uint8_t* prow = sP + r * 128;
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        uint32_t w[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int i = 4 * c + q;
          const float2 t01 = fma2(make_float2(sv[4 * i], sv[4 * i + 1]), sc2, bias2);
          const float2 t23 = fma2(make_float2(sv[4 * i + 2], sv[4 * i + 3]), sc2, bias2);
          // pair 2i of the row's 64 pairs, pair 2i + 1: the first kPolyPairs of each four on
          // the FMA pipe, the rest on the MUFU
          const float2 p01 = ((2 * i) & 3) < kPolyPairs ? exp2_poly2(t01) : make_float2(ex2(t01.x), ex2(t01.y));
          const float2 p23 = ((2 * i + 1) & 3) < kPolyPairs ? exp2_poly2(t23) : make_float2(ex2(t23.x), ex2(t23.y));
          sums[i & 1] = add2(sums[i & 1], add2(p01, p23));
          w[q] = static_cast<uint32_t>(e4m3_pair(p01.x, p01.y)) | (static_cast<uint32_t>(e4m3_pair(p23.x, p23.y)) << 16);
        }
        *reinterpret_cast<uint4*>(prow + ((c ^ (r & 7)) << 4)) = make_uint4(w[0], w[1], w[2], w[3]);
      }
      const float rowsum = (sums[0].x + sums[0].y) + (sums[1].x + sums[1].y);
      l_run = l_run * alpha + rowsum;
      m_run = m_new;
      tc::fence_proxy_async();
      // O holds P V up to tile j - 1 (landed: the wait for the P buffer above): rescale it when
      // a row's max moved
      if (j >= 1 && __any_sync(0xffffffffu, alpha != 1.0f)) {
        tc::fence_after_sync();
        {
#pragma unroll
          for (int c = 0; c < kChunks; ++c) {
            uint32_t o[32];
            tc::tmem_ld32(tO + lane_base + c * 32, o);
            tc::tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              uint32_t v8[8];
#pragma unroll
              for (int e = 0; e < 8; ++e) v8[e] = __float_as_uint(__uint_as_float(o[8 * i + e]) * alpha);
              tc::tmem_st8(tO + lane_base + c * 32 + 8 * i, v8);
            }
          }
          tc::tmem_st_wait();
        }
      }
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(p_full);
    }
    // the last P V, then O / rowsum * v_scale in bf16 (the code scale cancels)
    if (ok && !warp_wait(p_empty, static_cast<uint32_t>((n_kv - 1) & 1))) ok = false;
    if (ok) {  // (every lane loads: the TMEM loads are warp-wide; rows past a ragged sequence
               // are not stored)
      tc::fence_after_sync();
      const bool store = qrow < g.seq;
      const float f = g.v_scale[bhk] / l_run;
      __nv_bfloat16* orow = reinterpret_cast<__nv_bfloat16*>(g.out) + (static_cast<int64_t>(bh) * g.seq + qrow) * D;
#pragma unroll
      for (int c = 0; c < kChunks; ++c) {
        uint32_t o[32];
        tc::tmem_ld32(tO + lane_base + c * 32, o);
        tc::tmem_ld_wait();
        uint32_t w[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const __nv_bfloat162 hv = __floats2bfloat162_rn(__uint_as_float(o[2 * i]) * f, __uint_as_float(o[2 * i + 1]) * f);
          w[i] = *reinterpret_cast<const uint32_t*>(&hv);
        }
        if (store) {
#pragma unroll
          for (int i = 0; i < 4; ++i)
            reinterpret_cast<uint4*>(orow + c * 32)[i] = make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
        }
      }
    } else if (lane == 0) {
      atomicOr(&g_attention_status, kDevTimeout);
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc::fence_after_sync();
    tc::tmem_dealloc(tmem, L::kTmemCols);
  }
}

}  // namespace kab
