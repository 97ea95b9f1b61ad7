// Blockwise-scaled FP8 GEMM: A e4m3 [M, K] with one fp32 scale per 1 x 128 group along K,
// B e4m3 [N, K] with one fp32 scale per 128 x 128 block; D[m, n] = sum over 128-wide K steps
// of (partial * sa[m, kb]) * sb[n / 128, kb] in fp32 (+ bias), one rounding to the output
// dtype (docs/research-scripts/fp8-sm120/gemm_bench.py:39-68, the promotion rule of the
// 1x128 / 128x128 recipe).
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
__device__ __forceinline__ unsigned long long f2_add(unsigned long long a, unsigned long long b) {
  unsigned long long r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}

template <int OUT>
struct BlockwiseLayout {
  static constexpr int kBM = 128, kBN = 128, kBK = 128;  // bytes of K per stage = one scale group
  static constexpr int kABytes = kBM * kBK;
  static constexpr int kBBytes = kBN * kBK;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kPartials = 4;  // TMEM partial buffers of kBN columns
  static constexpr int kEpiWarps = 8;
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
    const int half = (warp - 2) >> 2;
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
      for (int kb = 0; kb < KB; ++kb) {
        const float sa = live ? __ldg(sa_row + kb) : 0.0f;
        const float sb = __ldg(sb_col + kb);
        if (!tc::mbar_wait(&part_full[p], pph)) { ok = false; break; }
        tc::fence_after_sync();
        uint32_t r0[32], r1[32];
        const uint32_t src = tmem + lane_base + p * BN + half * 64;
        tc::tmem_ld32(src, r0);
        tc::tmem_ld32(src + 32, r1);
        tc::tmem_ld_wait();
        tc::fence_before_sync();
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(&part_empty[p]);
        if (++p == NP) { p = 0; pph ^= 1u; }
        // gemm_bench.py:39-68: acc += (partial * sa[m, kb]) * sb[n / 128, kb], each rounded
        const unsigned long long sa2 = f2_pack(sa, sa), sb2 = f2_pack(sb, sb);
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const unsigned long long p0 = f2_pack(__uint_as_float(r0[2 * i]), __uint_as_float(r0[2 * i + 1]));
          const unsigned long long p1 = f2_pack(__uint_as_float(r1[2 * i]), __uint_as_float(r1[2 * i + 1]));
          acc[i] = f2_add(acc[i], f2_mul(f2_mul(p0, sa2), sb2));
          acc[16 + i] = f2_add(acc[16 + i], f2_mul(f2_mul(p1, sa2), sb2));
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

}  // namespace kab
