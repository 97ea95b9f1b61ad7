// Blockwise-scaled FP8 GEMM: A e4m3 [M, K] with one fp32 scale per 1 x 128 group along K,
// B e4m3 [N, K] with one fp32 scale per 128 x 128 block; for each 128-wide K step
// acc = fma(partial * sa[m, kb], sb[n / 128, kb], acc) in fp32, then (+ bias) one rounding to
// the output dtype (docs/research-scripts/fp8-sm120/gemm_bench.py:39-68, `acc += part * s_a *
// s_b`, which Triton compiles with its default fp fusion as a multiply and a fused
// multiply-add).
//
// The tensor core cannot apply a per-(row, K-step) fp32 scale, so each 128-wide K step is one
// fresh partial product in TMEM (4 kind::f8f6f4 MMAs of K = 32) and the epilogue warps promote
// it into fp32 registers while the MMA warp fills the next partial buffer (4 buffers of
// 128 x 128 fp32 = all 512 TMEM columns). Warp 0: TMA loads (one thread). Warp 1: MMAs (one
// thread), TMEM owner. Warps 2-9: promotion and the output epilogue, two warps per lane
// quarter, 64 columns each. No load uses cluster multicast; every wait is bounded.
#pragma once

#include "gemm.cuh"

namespace kab {

struct BlockwiseArgs {
  int64_t m, n;
  int k_blocks;             // K / 128
  int m_tiles, n_tiles;
  const float* sa;          // [m, k_blocks]
  const float* sb;          // [n / 128, k_blocks]
  const void* bias;         // [n] in bias_dtype, or null
  int bias_dtype;
};

// Two fp32 lanes in one 64-bit register (element 0 low): the promotion runs on packed
// f32x2 multiplies and adds, each lane rounded to nearest like its scalar form.
__device__ __forceinline__ unsigned long long f2_pack(float lo, float hi) {
  return (static_cast<unsigned long long>(__float_as_uint(hi)) << 32) | __float_as_uint(lo);
}
__device__ __forceinline__ unsigned long long f2_mul(unsigned long long a, unsigned long long b) {
  unsigned long long r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ unsigned long long f2_fma(unsigned long long a, unsigned long long b,
                                                     unsigned long long c) {
  unsigned long long r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}
// Two 32-bit registers as one 64-bit pair (element 0 low), without arithmetic.
__device__ __forceinline__ unsigned long long f2_regs(uint32_t lo, uint32_t hi) {
  unsigned long long r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "r"(lo), "r"(hi));
  return r;
}

// acc[i] = fma(p * sa, sb, acc[i]) over 32 columns of one K step's partial (16 pairs).
__device__ __forceinline__ void promote16(unsigned long long* acc, const uint32_t (&part)[32],
                                          unsigned long long sa2, unsigned long long sb2) {
#pragma unroll
  for (int i = 0; i < 16; ++i) acc[i] = f2_fma(f2_mul(f2_regs(part[2 * i], part[2 * i + 1]), sa2), sb2, acc[i]);
}

// A bounded wait whose outcome the whole warp shares (the promotion warps follow it with
// .sync.aligned TMEM loads, which need every lane).
__device__ __forceinline__ bool warp_wait_g(uint64_t* bar, uint32_t parity) {
  return __all_sync(0xffffffffu, tc::mbar_wait(bar, parity));
}

template <int OUT>
struct BlockwiseLayout {
  static constexpr int kBM = 128, kBN = 128, kBK = 128;  // bytes of K per stage = one scale group
  static constexpr int kABytes = kBM * kBK;
  static constexpr int kBBytes = kBN * kBK;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kPartials = 4;  // TMEM partial buffers of kBN columns
  static constexpr int kEpiWarps = 8;  // two per lane quarter, 64 columns each
  static constexpr int kThreads = 32 * (2 + kEpiWarps);
  static constexpr int kStageOutBytes = 32 * 32 * out_bytes(OUT);
  static constexpr int kStagingBytes = kEpiWarps * 2 * kStageOutBytes;
  static constexpr int kSmemLimit = 232448;
  static constexpr int kFixed = 1024 + kStagingBytes + 256;
  static constexpr int kStagesFit = (kSmemLimit - kFixed) / kStageBytes;
  static constexpr int kStages = kStagesFit > 6 ? 6 : kStagesFit;
  static constexpr int kBarriers = 2 * kStages + 2 * kPartials + 1;
  static constexpr int kSmem = 1024 + kStages * kStageBytes + kStagingBytes + kBarriers * 8 + 16;
  static_assert(kStages >= 2, "shared memory does not fit two stages");
  static_assert(kPartials * kBN <= 512, "TMEM overflow");
  static_assert(kSmem <= kSmemLimit, "shared memory overflow");
};

template <int OUT>
__global__ void __launch_bounds__(BlockwiseLayout<OUT>::kThreads, 1)
gemm_blockwise_kernel(const __grid_constant__ CUtensorMap tma_a, const __grid_constant__ CUtensorMap tma_b,
                      const __grid_constant__ CUtensorMap tma_out, BlockwiseArgs g) {
  using L = BlockwiseLayout<OUT>;
  constexpr int STAGES = L::kStages;
  constexpr int BN = L::kBN;
  constexpr int NP = L::kPartials;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = sA + STAGES * L::kABytes;
  uint8_t* sOut = sB + STAGES * L::kBBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sOut + L::kStagingBytes);
  uint64_t* full = bars;
  uint64_t* empty = bars + STAGES;
  uint64_t* part_full = bars + 2 * STAGES;   // partial buffer p holds a finished K step
  uint64_t* part_empty = part_full + NP;     // ... and has been read by all epilogue warps
  uint64_t* drain = part_empty + NP;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      tc::mbar_init(&full[s], 1);
      tc::mbar_init(&empty[s], 1);
    }
    for (int p = 0; p < NP; ++p) {
      tc::mbar_init(&part_full[p], 1);
      tc::mbar_init(&part_empty[p], L::kEpiWarps);
    }
    tc::mbar_init(drain, 1);
    tc::fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tc::prefetch_tensormap(&tma_a);
    tc::prefetch_tensormap(&tma_b);
    tc::prefetch_tensormap(&tma_out);
  }
  if (warp == 1) { tc::tmem_alloc(tmem_slot, 512); tc::tmem_relinquish(); }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *tmem_slot;
  const int total = g.m_tiles * g.n_tiles;
  const int KB = g.k_blocks;

  if (warp == 0) {
    if (lane == 0) {  // ---------------------------------------------------- TMA producer
      int s = 0;
      uint32_t ph = 0;
      bool ok = true;
      uint32_t issued_ph[STAGES];
      bool issued[STAGES];
      for (int i = 0; i < STAGES; ++i) issued[i] = false;
      for (int t = blockIdx.x; ok && t < total; t += gridDim.x) {
        int mt, nt;
        tile_coords(t, g.m_tiles, g.n_tiles, 0, mt, nt);
        for (int kb = 0; kb < KB; ++kb) {
          if (!tc::mbar_wait(&empty[s], ph ^ 1u)) { ok = false; break; }
          tc::mbar_arrive_expect_tx(&full[s], L::kStageBytes);
          tc::tma_load_2d(&tma_a, &full[s], sA + s * L::kABytes, kb * L::kBK, mt * 128);
          tc::tma_load_2d(&tma_b, &full[s], sB + s * L::kBBytes, kb * L::kBK, nt * BN);
          issued[s] = true;
          issued_ph[s] = ph;
          if (++s == STAGES) { s = 0; ph ^= 1u; }
        }
      }
      if (!ok) {
        atomicOr(&g_gemm_status, kDevTimeout);
        for (int i = 0; i < STAGES; ++i)  // let the loads already issued land first
          if (issued[i]) tc::mbar_wait(&full[i], issued_ph[i]);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {  // ---------------------------------------------------- MMA issuer
      int s = 0, p = 0;
      uint32_t ph = 0, pph = 0;
      bool ok = true;
      const uint32_t idesc = tc::idesc_f8(128, BN);
      for (int t = blockIdx.x; ok && t < total; t += gridDim.x) {
        for (int kb = 0; kb < KB; ++kb) {
          if (!tc::mbar_wait(&part_empty[p], pph ^ 1u)) { ok = false; break; }
          if (!tc::mbar_wait(&full[s], ph)) { ok = false; break; }
          tc::fence_after_sync();
          const uint64_t adesc = tc::desc_sw128(tc::smem_u32(sA + s * L::kABytes));
          const uint64_t bdesc = tc::desc_sw128(tc::smem_u32(sB + s * L::kBBytes));
          const uint32_t d = tmem + p * BN;
#pragma unroll
          for (int j = 0; j < 4; ++j)  // a fresh partial: the first MMA overwrites
            tc::mma_f8(d, adesc + static_cast<uint64_t>(2 * j), bdesc + static_cast<uint64_t>(2 * j), idesc,
                       j > 0 ? 1u : 0u);
          tc::commit(&empty[s]);
          tc::commit(&part_full[p]);
          if (++s == STAGES) { s = 0; ph ^= 1u; }
          if (++p == NP) { p = 0; pph ^= 1u; }
        }
      }
      tc::commit(drain);  // every MMA this thread issued has completed once this arrives
      if (!tc::mbar_wait(drain, 0)) ok = false;
      if (!ok) atomicOr(&g_gemm_status, kDevTimeout);
    }
  } else {  // ------------------------------------------------- promotion + epilogue warps
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;  // columns half * 64 .. + 63 of the tile
    const uint32_t lane_base = static_cast<uint32_t>(32 * quarter) << 16;
    uint8_t* stage0 = sOut + (warp - 2) * 2 * L::kStageOutBytes;
    int p = 0;
    uint32_t pph = 0;
    int chunk = 0;
    bool ok = true;
    for (int t = blockIdx.x; ok && t < total; t += gridDim.x) {
      int mt, nt;
      tile_coords(t, g.m_tiles, g.n_tiles, 0, mt, nt);
      const int row0 = mt * 128 + 32 * quarter;
      const int64_t row = static_cast<int64_t>(row0) + lane;
      const bool live = row < g.m;
      const int col0 = nt * BN + half * 64;
      const float* sa_row = g.sa + (live ? row : 0) * static_cast<int64_t>(KB);
      const float* sb_col = g.sb + static_cast<int64_t>(nt) * KB;
      unsigned long long acc[32];  // columns 2i, 2i + 1
#pragma unroll
      for (int i = 0; i < 32; ++i) acc[i] = 0ull;
      const uint32_t col = lane_base + half * 64;
      // The scales of four K steps are fetched together: independent loads, one L2 latency
      // per four steps instead of one per step (the L1 is mostly given to shared memory here
      // and does not keep the rows' scale sectors between steps).
      for (int k4 = 0; ok && k4 < KB; k4 += 4) {
        float sa4[4], sb4[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const bool in = k4 + j < KB;
          sa4[j] = live && in ? __ldg(sa_row + k4 + j) : 0.0f;
          sb4[j] = in ? __ldg(sb_col + k4 + j) : 0.0f;
        }
        const int steps = KB - k4 < 4 ? KB - k4 : 4;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          if (j >= steps) break;
          if (!warp_wait_g(&part_full[p], pph)) { ok = false; break; }
          tc::fence_after_sync();
          uint32_t r0[32], r1[32];
          tc::tmem_ld32(tmem + col + p * BN, r0);
          tc::tmem_ld32(tmem + col + p * BN + 32, r1);
          tc::tmem_ld_wait();
          tc::fence_before_sync();
          __syncwarp();
          if (lane == 0) tc::mbar_arrive(&part_empty[p]);
          if (++p == NP) { p = 0; pph ^= 1u; }
          const unsigned long long sa2 = f2_pack(sa4[j], sa4[j]), sb2 = f2_pack(sb4[j], sb4[j]);
          promote16(acc, r0, sa2, sb2);
          promote16(acc + 16, r1, sa2, sb2);
        }
      }
      if (!ok) break;
      // output: (+ bias) and one rounding, through the staging buffers and TMA stores
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        uint32_t y[32];
        float bv = 0.0f;
        if (g.bias != nullptr && col0 + c * 32 + lane < g.n) bv = load_bias(g.bias, g.bias_dtype, col0 + c * 32 + lane);
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const unsigned long long a2 = acc[c * 16 + i / 2];
          float v = __uint_as_float(static_cast<uint32_t>(i & 1 ? a2 >> 32 : a2));
          const float b = __shfl_sync(0xffffffffu, bv, i);
          if (g.bias != nullptr) v = __fadd_rn(v, b);
          y[i] = __float_as_uint(v);
        }
        uint8_t* buf = stage0 + (chunk & 1) * L::kStageOutBytes;
        if (chunk >= 2) {  // the store two chunks ago has finished reading this buffer
          if (lane == 0) tc::bulk_wait_read<1>();
          __syncwarp();
        }
        stage_row<OUT>(buf, lane, y);
        tc::fence_proxy_async();
        __syncwarp();
        if (lane == 0) {
          tc::tma_store_2d(&tma_out, buf, col0 + c * 32, row0);
          tc::bulk_commit();
        }
        ++chunk;
      }
    }
    if (!ok && lane == 0) atomicOr(&g_gemm_status, kDevTimeout);
    if (lane == 0) tc::bulk_wait_all();
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc::fence_after_sync();
    tc::tmem_dealloc(tmem, 512);
  }
}

// ------------------------------------------------------------------ decode sizes (M <= 32)
//
// For a few tokens the weight stream is the whole cost (config 2 at M = 1 / 16: 3 MB of codes)
// and one CTA per 128 x 128 output tile leaves most SMs idle. Here the weight is the MMA's
// 128-row A operand and the tokens its N (NT = 16 or 32, the rows past M zero-filled by TMA),
// and the K steps of one 128-channel panel are split over a thread-block cluster of C <= 8 CTAs
// (`per` consecutive K steps each). Each CTA loads its K steps' weight and token tiles at once,
// issues their MMAs into separate TMEM partials, and four warps (one channel per thread) write
// t = partial * sa[token, kb] (fp32) into shared memory over the weight tile that MMA has
// finished reading. After a cluster barrier the CTAs reduce the panel's [M, 128] outputs in
// slices: acc = fma(t_kb, sb[panel, kb], acc) in K order, reading t from the owning CTA's
// shared memory (distributed shared memory): the tiled kernel's promotion sequence (the
// partials come from the tensor core with the operands swapped). A second barrier keeps every
// CTA's shared memory alive until read. Shared memory and TMEM are sized by `per`, so a
// cluster of one-step CTAs packs many to an SM.

struct BlockwiseSkinnyArgs {
  int64_t m, n, ldo;
  int k_blocks;        // K / 128
  int per;             // K steps per CTA of a cluster
  const float* sa;     // [m, k_blocks]
  const float* sb;     // [n / 128, k_blocks]
  const void* bias;    // [n] in bias_dtype, or null
  int bias_dtype;
  void* out;           // [m, ldo]
};

template <int NT>
struct BlockwiseSkinnyLayout {
  static constexpr int kMaxPer = 8;
  static constexpr int kWBytes = 128 * 128;        // one K step of the panel's weight
  static constexpr int kXBytes = NT * 128;         // one K step of the tokens
  static constexpr int kThreads = 32 * 6;          // TMA, MMA, four promotion warps
  static constexpr int kNumBars = 2 * kMaxPer + 1;  // full[i], part_full[i], drain
  static constexpr int kMaxKb = 8 * kMaxPer;         // K steps of a panel (K <= 8192)
  // per K steps: the weight tiles, then the token tiles (both 1024-byte aligned), then the
  // barriers, the panel's weight scales sb[kb] and the TMEM address
  __host__ __device__ static constexpr int x_offset(int per) { return per * kWBytes; }
  __host__ __device__ static constexpr int bar_offset(int per) { return per * (kWBytes + kXBytes); }
  __host__ __device__ static constexpr int smem(int per) {
    return 1024 + bar_offset(per) + kNumBars * 8 + kMaxKb * 4 + 16;
  }
  __host__ __device__ static constexpr uint32_t tmem_cols(int per) {
    return per * NT <= 32 ? 32u : (per * NT <= 64 ? 64u : (per * NT <= 128 ? 128u : 256u));
  }
  static_assert(NT * 128 * 4 <= kWBytes, "a promoted step must fit over its weight tile");
  static_assert(1024 + kMaxPer * (kWBytes + kXBytes) + kNumBars * 8 + 16 <= 232448, "shared memory overflow");
};

template <int NT, int OUT>
__global__ void __launch_bounds__(BlockwiseSkinnyLayout<NT>::kThreads, 1)
gemm_blockwise_skinny_kernel(const __grid_constant__ CUtensorMap tma_w, const __grid_constant__ CUtensorMap tma_x,
                             BlockwiseSkinnyArgs g) {
  using L = BlockwiseSkinnyLayout<NT>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sW = smem;
  uint8_t* sX = smem + L::x_offset(g.per);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::bar_offset(g.per));
  const uint32_t tmem_cols = L::tmem_cols(g.per);
  uint64_t* part_full = full + L::kMaxPer;
  uint64_t* drain = part_full + L::kMaxPer;
  float* s_sb = reinterpret_cast<float*>(drain + 1);  // [kMaxKb] this panel's weight scales
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(s_sb + L::kMaxKb);

  const uint32_t rank = tc::cluster_ctarank();
  const int csize = static_cast<int>(gridDim.x / (g.n / 128));  // CTAs per cluster (one panel)
  const int panel = static_cast<int>(blockIdx.x) / csize;
  const int kb0 = static_cast<int>(rank) * g.per;
  const int nk = max(0, min(g.per, g.k_blocks - kb0));  // this CTA's K steps
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int i = 0; i < L::kMaxPer; ++i) {
      tc::mbar_init(&full[i], 1);
      tc::mbar_init(&part_full[i], 1);
    }
    tc::mbar_init(drain, 1);
    tc::fence_barrier_init();
    tc::fence_proxy_async();
    // every K step of this CTA at once, before the TMEM allocation and the block barrier: the
    // weight's HBM latency is the longest wait of the kernel
    for (int i = 0; i < nk; ++i) {
      tc::mbar_arrive_expect_tx(&full[i], L::kWBytes + L::kXBytes);
      tc::tma_load_2d(&tma_w, &full[i], sW + i * L::kWBytes, (kb0 + i) * 128, panel * 128);
      tc::tma_load_2d(&tma_x, &full[i], sX + i * L::kXBytes, (kb0 + i) * 128, 0);
    }
  }
  if (warp == 1) { tc::tmem_alloc(tmem_slot, tmem_cols); tc::tmem_relinquish(); }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *tmem_slot;
  bool ok = true;

  if (warp == 1) {
    if (lane == 0) {  // ------------------------------------ MMA: one partial per K step
      const uint32_t idesc = tc::idesc_f8(128, NT);
      int landed = 0;
      for (int i = 0; i < nk; ++i) {
        if (!tc::mbar_wait(&full[i], 0)) { ok = false; break; }
        landed = i + 1;
        tc::fence_after_sync();
        const uint64_t wdesc = tc::desc_sw128(tc::smem_u32(sW + i * L::kWBytes));
        const uint64_t xdesc = tc::desc_sw128(tc::smem_u32(sX + i * L::kXBytes));
#pragma unroll
        for (int j = 0; j < 4; ++j)
          tc::mma_f8(tmem + i * NT, wdesc + static_cast<uint64_t>(2 * j), xdesc + static_cast<uint64_t>(2 * j), idesc,
                     j > 0 ? 1u : 0u);
        tc::commit(&part_full[i]);
      }
      tc::commit(drain);  // every MMA issued has completed once this arrives
      if (!tc::mbar_wait(drain, 0)) ok = false;
      if (!ok) {
        atomicOr(&g_gemm_status, kDevTimeout);
        for (int i = landed; i < nk; ++i) tc::mbar_wait(&full[i], 0);  // loads still in flight land first
      }
    }
  } else if (warp >= 2) {  // ---------------------------------- promotion: t = partial * sa
    const int quarter = warp & 3;
    const int ch = 32 * quarter + lane;  // the weight row (output channel) of this TMEM lane
    const uint32_t lane_base = static_cast<uint32_t>(32 * quarter) << 16;
    // the reduction's weight scales, fetched while the tiles are in flight
    for (int kb = threadIdx.x - 64; kb < g.k_blocks; kb += 128)
      s_sb[kb] = __ldg(g.sb + static_cast<int64_t>(panel) * g.k_blocks + kb);
    for (int i = 0; i < nk; ++i) {
      float sa[NT];
#pragma unroll
      for (int t = 0; t < NT; ++t) sa[t] = t < g.m ? __ldg(g.sa + static_cast<int64_t>(t) * g.k_blocks + kb0 + i) : 0.0f;
      if (!__all_sync(0xffffffffu, tc::mbar_wait(&part_full[i], 0))) {
        ok = false;
        if (lane == 0) atomicOr(&g_gemm_status, kDevTimeout);
        break;
      }
      tc::fence_after_sync();
      uint32_t r[NT];
      if constexpr (NT == 16) tc::tmem_ld16(tmem + lane_base + i * NT, r);
      else tc::tmem_ld32(tmem + lane_base + i * NT, *reinterpret_cast<uint32_t(*)[32]>(r));
      tc::tmem_ld_wait();
      // [NT tokens][128 channels] fp32 over weight tile i (its MMAs have completed)
      float* part = reinterpret_cast<float*>(sW + i * L::kWBytes);
#pragma unroll
      for (int t = 0; t < NT; ++t) part[t * 128 + ch] = __fmul_rn(__uint_as_float(r[t]), sa[t]);
    }
  }
  tc::fence_before_sync();
  tc::cluster_sync();  // every CTA's t values are written (release / acquire)
  tc::fence_after_sync();

  // ------------------------------------------------------------ reduction in K order
  // four consecutive channels per thread (16-byte distributed-shared-memory loads), the
  // panel's M x 128 outputs in equal slices over the cluster's CTAs
  const int quads = static_cast<int>(g.m) * 32;
  const int slice = (quads + csize - 1) / csize;
  const int q_end = min(quads, (static_cast<int>(rank) + 1) * slice);
  for (int qd = static_cast<int>(rank) * slice + threadIdx.x; qd < q_end; qd += blockDim.x) {
    const int t = qd >> 5, ch = (qd & 31) * 4;
    float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    for (int k8 = 0; k8 < g.k_blocks; k8 += 8) {  // eight loads in flight, then the fmas in order
      float4 v[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int kb = k8 + j;
        v[j] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        if (kb < g.k_blocks) {
          const int owner = kb / g.per, i = kb - owner * g.per;
          const float* src = reinterpret_cast<const float*>(sW + i * L::kWBytes) + t * 128 + ch;
          asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
                       : "=f"(v[j].x), "=f"(v[j].y), "=f"(v[j].z), "=f"(v[j].w)
                       : "r"(tc::mapa(src, static_cast<uint32_t>(owner)))
                       : "memory");
        }
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        if (k8 + j < g.k_blocks) {
          const float w = s_sb[k8 + j];
          acc.x = __fmaf_rn(v[j].x, w, acc.x);
          acc.y = __fmaf_rn(v[j].y, w, acc.y);
          acc.z = __fmaf_rn(v[j].z, w, acc.z);
          acc.w = __fmaf_rn(v[j].w, w, acc.w);
        }
      }
    }
    const int64_t col = static_cast<int64_t>(panel) * 128 + ch;
    if (g.bias != nullptr) {
      acc.x = __fadd_rn(acc.x, load_bias(g.bias, g.bias_dtype, col));
      acc.y = __fadd_rn(acc.y, load_bias(g.bias, g.bias_dtype, col + 1));
      acc.z = __fadd_rn(acc.z, load_bias(g.bias, g.bias_dtype, col + 2));
      acc.w = __fadd_rn(acc.w, load_bias(g.bias, g.bias_dtype, col + 3));
    }
    const int64_t idx = static_cast<int64_t>(t) * g.ldo + col;  // a multiple of 4 (ldo % 8 == 0)
    if constexpr (OUT == KAB_BF16) {
      const __nv_bfloat162 lo = __floats2bfloat162_rn(acc.x, acc.y), hi = __floats2bfloat162_rn(acc.z, acc.w);
      *reinterpret_cast<uint2*>(reinterpret_cast<__nv_bfloat16*>(g.out) + idx) =
          make_uint2(*reinterpret_cast<const uint32_t*>(&lo), *reinterpret_cast<const uint32_t*>(&hi));
    } else if constexpr (OUT == KAB_F16) {
      const __half2 lo = __floats2half2_rn(acc.x, acc.y), hi = __floats2half2_rn(acc.z, acc.w);
      *reinterpret_cast<uint2*>(reinterpret_cast<__half*>(g.out) + idx) =
          make_uint2(*reinterpret_cast<const uint32_t*>(&lo), *reinterpret_cast<const uint32_t*>(&hi));
    } else {
      *reinterpret_cast<float4*>(reinterpret_cast<float*>(g.out) + idx) = acc;
    }
  }
  tc::cluster_sync();  // no CTA leaves while another may still read its shared memory
  if (warp == 1) {
    __syncwarp();
    tc::fence_after_sync();
    tc::tmem_dealloc(tmem, tmem_cols);
  }
}

}  // namespace kab
