// Scaled GEMMs D[m, n] = sum_k A[m, k] * B[n, k] on the 5th-generation tensor cores
// (tcgen05.mma, accumulators in TMEM), fed by a TMA multistage shared-memory ring, with the
// dequantisation / bias / cast epilogue fused.
//
//   KIND 0  kind::i8        int8 x int8 -> int32 (exact); epilogue acc * sa[m] * sb[n] (+ bias)
//   KIND 1  kind::f8f6f4    e4m3 x e4m3 -> fp32; epilogue acc * sa[m] * sb[n] (+ bias)
//   KIND 2  kind::mxf8f6f4  e4m3 x e4m3 with e8m0 scales per 32 applied by the tensor core
//   KIND 3  kind::mxf4nvf4  e2m1 x e2m1 with e4m3 scales per 16 applied by the tensor core;
//                            epilogue acc * (outer[m] * ts[n or one]) (+ bias)
//
// One persistent CTA per SM: warp 0 issues the TMA loads (one thread), warp 1 the MMAs (one
// thread) and owns the TMEM allocation, warps 2-9 drain the accumulator (tcgen05.ld, one TMEM
// lane = one output row per thread; two warps per lane quarter, each taking half the columns),
// and for the block-scaled kinds warps 10-13 move the scale factors into TMEM. Output tiles are 128 x BN; the
// operand ring holds STAGES k-steps of 128 bytes of K per row (128 int8 / e4m3 elements, 256
// e2m1). Block scales arrive in cuBLASLt's 128 x 4 blocked layout (quant.py:540-564), whose
// 512-byte chunks are exactly the 32 x 128-bit sources tcgen05.cp expects; they are copied
// into TMEM next to the accumulators. No load uses cluster multicast.
#pragma once

#include "kab_common.cuh"
#include "tcgen05.cuh"

namespace kab {

__device__ unsigned g_gemm_status = 0;

struct GemmArgs {
  int64_t m, n;
  int k_stages;                 // K bytes per row / 128
  int m_tiles, n_tiles;
  const uint8_t* sfa;           // swizzled block scales of A (KIND 2, 3)
  const uint8_t* sfb;           // ... of B
  int64_t sfa_ncb, sfb_ncb;     // 4-column blocks per 128-row block of each
  const float* a_scale;         // per row of A: token scale (KIND 0, 1), outer (KIND 3)
  const float* b_scale;         // per row of B (KIND 0, 1), tensor scale(s) (KIND 3)
  int b_scale_per_col;          // KIND 3: b_scale[n] instead of b_scale[0]
  const void* bias;             // [n] in bias_dtype, or null
  int bias_dtype;
  void* out;                    // [m, ldo] in out_dtype
  int out_dtype;
  int64_t ldo;
  int32_t* acc_out;             // KIND 0: raw int32 products [m, ldo] instead of `out`
};

template <int KIND>
struct GemmTraits {
  static constexpr bool kScaled = KIND >= 2;
};

// Output element types of the epilogue (KAB_BF16 / KAB_F16 / KAB_F32, or the raw int32
// products of KIND 0).
constexpr int kOutI32 = 7;
__host__ __device__ constexpr int out_bytes(int out) { return out == KAB_F32 || out == kOutI32 ? 4 : 2; }

// BKB: bytes of K per row per pipeline stage (128: 128-byte swizzle, 64: 64-byte swizzle);
// each stage holds BKB / 32 MMAs (32 bytes of K each).
template <int KIND, int BN, int BKB, int OUT>
struct GemmLayout {
  static constexpr int kBM = 128;
  static constexpr int kKSteps = BKB / 32;
  static constexpr bool kScaled = KIND >= 2;
  static constexpr int kABytes = kBM * BKB;
  static constexpr int kBBytes = BN * BKB;
  // block scales per 128 rows per stage: NVFP4 one 512-byte chunk per MMA (K = 64), MXFP8 one
  // chunk per 4 MMAs (K = 128: the stage)
  static constexpr int kSfaBytes = KIND == 3 ? 512 * kKSteps : (KIND == 2 ? 512 : 0);
  static constexpr int kSfbBytes = kSfaBytes * (BN / 128);
  static constexpr int kStageBytes = kABytes + kBBytes + kSfaBytes + kSfbBytes;
  // TMEM columns of block scales per stage: each 512-byte chunk (32 rows of 16 bytes: row
  // r % 32 holds rows {r, r + 32, r + 64, r + 96}) lands in 4 columns of every lane quarter,
  // lane l holding chunk row l (the layout tcgen05.cp.32x128b.warpx4 makes); the
  // scale-factor warps write it with tcgen05.st, each into its own quarter.
  static constexpr int kSfaCols = KIND == 3 ? 4 * kKSteps : (KIND == 2 ? 4 : 0);
  static constexpr int kSfbCols = kSfaCols * (BN / 128);
  static constexpr int kSfColsPerStage = kSfaCols + kSfbCols;
  static constexpr int kEpiWarps = 8;  // two per TMEM lane quarter
  static constexpr int kThreads = 32 * (2 + kEpiWarps + (kScaled ? 4 : 0));
  static constexpr int kAccBufs = kScaled ? 1 : 2;
  static constexpr int kSfCol = kAccBufs * BN;
  // epilogue staging: 8 warps x 2 buffers x [32 rows, 32 columns]
  static constexpr int kStageOutBytes = 32 * 32 * out_bytes(OUT);
  static constexpr int kStagingBytes = kEpiWarps * 2 * kStageOutBytes;
  static constexpr int kSmemLimit = 232448;
  static constexpr int kFixed = 1024 + kStagingBytes + 320;
  static constexpr int kStagesFit = (kSmemLimit - kFixed) / kStageBytes;
  static constexpr int kStages = kStagesFit > 8 ? 8 : kStagesFit;
  static constexpr int kBarriers = 3 * kStages + 2 * kAccBufs + 1;
  static constexpr int kSmem = 1024 + kStages * kStageBytes + kStagingBytes + kBarriers * 8 + 16;
  static_assert(kStages >= 2, "shared memory does not fit two stages");
  static_assert(kSfCol + kStages * kSfColsPerStage <= 512, "TMEM overflow");
  static_assert(kSmem <= kSmemLimit, "shared memory overflow");
};

__device__ __forceinline__ float load_bias(const void* bias, int dtype, int64_t i) {
  if (dtype == KAB_BF16) return __bfloat162float(__ldg(reinterpret_cast<const __nv_bfloat16*>(bias) + i));
  if (dtype == KAB_F16) return __half2float(__ldg(reinterpret_cast<const __half*>(bias) + i));
  return __ldg(reinterpret_cast<const float*>(bias) + i);
}

// Rounds to the output dtype and back (the bf16 / fp16 result of F.scaled_mm before a bias).
template <int OUT>
__device__ __forceinline__ float round_out(float f) {
  if constexpr (OUT == KAB_BF16) return round_bf16(f);
  else if constexpr (OUT == KAB_F16) return __half2float(__float2half_rn(f));
  else return f;
}

// The epilogue of 32 accumulator columns of one row: y[i] in fp32 (or raw int32 bits).
// `sa`: this row's scale (token scale, or NVFP4 outer scale); `cs` / `cb`: lane i holds the
// column scale / bias of column col0 + i (broadcast by shuffles).
template <int KIND, int OUT>
__device__ __forceinline__ void epilogue_math(const GemmArgs& g, const uint32_t (&r)[32], float sa, float cs,
                                              float cb, uint32_t (&y)[32]) {
  const bool bias = g.bias != nullptr;
  if constexpr (OUT == kOutI32) {
#pragma unroll
    for (int i = 0; i < 32; ++i) y[i] = r[i];
  } else if constexpr (KIND == 0 || KIND == 1) {
    // quant.py:920-922: acc.float() * xs[m] * sw[n] (+ bias), left to right in fp32
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      const float acc = KIND == 0 ? __int2float_rn(static_cast<int>(r[i])) : __uint_as_float(r[i]);
      const float sb = __shfl_sync(0xffffffffu, cs, i);
      const float bi = __shfl_sync(0xffffffffu, cb, i);
      float v = __fmul_rn(__fmul_rn(acc, sa), sb);
      if (bias) v = __fadd_rn(v, bi);
      y[i] = __float_as_uint(v);
    }
  } else if constexpr (KIND == 2) {
    // quant.py:602-614: F.scaled_mm's output in the output dtype, then + bias in that dtype
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      const float bi = __shfl_sync(0xffffffffu, cb, i);
      float v = round_out<OUT>(__uint_as_float(r[i]));
      if (bias) v = __fadd_rn(v, bi);
      y[i] = __float_as_uint(v);
    }
  } else {
    // quant.py:1254-1256: acc * (outer[m] * ts) (+ bias.float())
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      const float ts = __shfl_sync(0xffffffffu, cs, i);
      const float bi = __shfl_sync(0xffffffffu, cb, i);
      float v = __fmul_rn(__uint_as_float(r[i]), __fmul_rn(sa, ts));
      if (bias) v = __fadd_rn(v, bi);
      y[i] = __float_as_uint(v);
    }
  }
}

// Writes one row of 32 outputs (this lane's row) into a [32 rows, 32 columns] staging tile.
template <int OUT>
__device__ __forceinline__ void stage_row(uint8_t* buf, int lane, const uint32_t (&y)[32]) {
  if constexpr (out_bytes(OUT) == 4) {
    uint4* p = reinterpret_cast<uint4*>(buf + lane * 128);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int j = (i + lane) & 7;  // rotate the 16-byte chunks: fewer bank conflicts
      p[j] = make_uint4(y[4 * j], y[4 * j + 1], y[4 * j + 2], y[4 * j + 3]);
    }
  } else {
    uint32_t w[16];  // round to nearest even, two per conversion instruction
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const float a = __uint_as_float(y[2 * i]), b = __uint_as_float(y[2 * i + 1]);
      if constexpr (OUT == KAB_BF16) {
        const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
        w[i] = *reinterpret_cast<const uint32_t*>(&h);
      } else {
        const __half2 h = __floats2half2_rn(a, b);
        w[i] = *reinterpret_cast<const uint32_t*>(&h);
      }
    }
    uint4* p = reinterpret_cast<uint4*>(buf + lane * 64);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int j = (i + lane) & 3;
      p[j] = make_uint4(w[4 * j], w[4 * j + 1], w[4 * j + 2], w[4 * j + 3]);
    }
  }
}

// Tile t of the persistent schedule -> (m tile, n tile): groups of 8 m-tiles sweep n.
__device__ __forceinline__ void tile_coords(int t, int m_tiles, int n_tiles, int& mt, int& nt) {
  constexpr int kGroup = 8;
  const int group_size = kGroup * n_tiles;
  const int g = t / group_size;
  const int first = g * kGroup;
  const int gm = min(m_tiles - first, kGroup);
  const int r = t % group_size;
  mt = first + r % gm;
  nt = r / gm;
}

template <int KIND, int BN, int BKB, int OUT>
__global__ void __launch_bounds__(GemmLayout<KIND, BN, BKB, OUT>::kThreads, 1)
gemm_kernel(const __grid_constant__ CUtensorMap tma_a, const __grid_constant__ CUtensorMap tma_b,
            const __grid_constant__ CUtensorMap tma_out, GemmArgs g) {
  using L = GemmLayout<KIND, BN, BKB, OUT>;
  constexpr int STAGES = L::kStages;
  constexpr int KS = L::kKSteps;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = sA + STAGES * L::kABytes;
  uint8_t* sSFA = sB + STAGES * L::kBBytes;
  uint8_t* sSFB = sSFA + STAGES * L::kSfaBytes;
  uint8_t* sOut = sSFB + STAGES * L::kSfbBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sOut + L::kStagingBytes);
  uint64_t* full = bars;
  uint64_t* empty = bars + STAGES;
  uint64_t* sf_full = bars + 2 * STAGES;  // scale factors of stage s are in TMEM (4 arrivals)
  uint64_t* acc_full = bars + 3 * STAGES;
  uint64_t* acc_empty = acc_full + L::kAccBufs;
  uint64_t* drain = acc_empty + L::kAccBufs;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      tc::mbar_init(&full[s], 1);
      tc::mbar_init(&empty[s], 1);
      tc::mbar_init(&sf_full[s], 4);
    }
    for (int b = 0; b < L::kAccBufs; ++b) { tc::mbar_init(&acc_full[b], 1); tc::mbar_init(&acc_empty[b], L::kEpiWarps); }
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
  constexpr uint32_t kTx = L::kStageBytes;

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
        tile_coords(t, g.m_tiles, g.n_tiles, mt, nt);
        for (int kb = 0; kb < g.k_stages; ++kb) {
          if (!tc::mbar_wait(&empty[s], ph ^ 1u)) { ok = false; break; }
          tc::mbar_arrive_expect_tx(&full[s], kTx);
          tc::tma_load_2d(&tma_a, &full[s], sA + s * L::kABytes, kb * BKB, mt * 128);
          tc::tma_load_2d(&tma_b, &full[s], sB + s * L::kBBytes, kb * BKB, nt * BN);
          if constexpr (KIND == 3) {  // KS chunks of 512 bytes per 128 rows: contiguous
            tc::bulk_load(sSFA + s * L::kSfaBytes, g.sfa + (mt * g.sfa_ncb + KS * kb) * 512, L::kSfaBytes, &full[s]);
#pragma unroll
            for (int h = 0; h < BN / 128; ++h)
              tc::bulk_load(sSFB + s * L::kSfbBytes + h * L::kSfaBytes,
                            g.sfb + ((nt * (BN / 128) + h) * g.sfb_ncb + KS * kb) * 512, L::kSfaBytes, &full[s]);
          } else if constexpr (KIND == 2) {
            tc::bulk_load(sSFA + s * L::kSfaBytes, g.sfa + (mt * g.sfa_ncb + kb) * 512, 512, &full[s]);
#pragma unroll
            for (int h = 0; h < BN / 128; ++h)
              tc::bulk_load(sSFB + s * L::kSfbBytes + h * 512,
                            g.sfb + ((nt * (BN / 128) + h) * g.sfb_ncb + kb) * 512, 512, &full[s]);
          }
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
      int s = 0, ab = 0;
      uint32_t ph = 0, aph = 0;
      bool ok = true;
      for (int t = blockIdx.x; ok && t < total; t += gridDim.x) {
        if (!tc::mbar_wait(&acc_empty[ab], aph ^ 1u)) { ok = false; break; }
        tc::fence_after_sync();
        const uint32_t d = tmem + ab * BN;
        for (int kb = 0; kb < g.k_stages; ++kb) {
          if (!tc::mbar_wait(&full[s], ph)) { ok = false; break; }
          if constexpr (L::kScaled) {
            if (!tc::mbar_wait(&sf_full[s], ph)) { ok = false; break; }
          }
          tc::fence_after_sync();
          const uint32_t abase = tc::smem_u32(sA + s * L::kABytes);
          const uint32_t bbase = tc::smem_u32(sB + s * L::kBBytes);
          const uint64_t adesc = BKB == 128 ? tc::desc_sw128(abase) : tc::desc_sw64(abase);
          const uint64_t bdesc = BKB == 128 ? tc::desc_sw128(bbase) : tc::desc_sw64(bbase);
          const uint32_t sf = tmem + L::kSfCol + s * L::kSfColsPerStage;
#pragma unroll
          for (int j = 0; j < KS; ++j) {
            const uint32_t acc = (kb > 0 || j > 0) ? 1u : 0u;
            const uint64_t a = adesc + static_cast<uint64_t>(2 * j);  // +32 bytes of K
            const uint64_t b = bdesc + static_cast<uint64_t>(2 * j);
            if constexpr (KIND == 0) {
              tc::mma_i8(d, a, b, tc::idesc_i8(128, BN), acc);
            } else if constexpr (KIND == 1) {
              tc::mma_f8(d, a, b, tc::idesc_f8(128, BN), acc);
            } else if constexpr (KIND == 2) {  // one scale byte per row per MMA (sf_id = j)
              tc::mma_mxf8(d, a, b, tc::idesc_mxf8(128, BN, j), sf, sf + L::kSfaCols, acc);
            } else {  // this MMA's chunk: 4 columns for A, 4 per 128 rows of B
              tc::mma_nvf4(d, a, b, tc::idesc_nvf4(128, BN), sf + 4 * j, sf + L::kSfaCols + 4 * (BN / 128) * j, acc);
            }
          }
          tc::commit(&empty[s]);
          if (++s == STAGES) { s = 0; ph ^= 1u; }
        }
        if (!ok) break;
        tc::commit(&acc_full[ab]);
        if (++ab == L::kAccBufs) { ab = 0; aph ^= 1u; }
      }
      tc::commit(drain);  // every MMA this thread issued has completed once this arrives
      if (!tc::mbar_wait(drain, 0)) ok = false;
      if (!ok) atomicOr(&g_gemm_status, kDevTimeout);
    }
  } else if (warp >= 2 + L::kEpiWarps) {  // ---------------------------------- scale-factor warps
    if constexpr (L::kScaled) {
      const int q = warp & 3;
      const uint32_t lane_base = static_cast<uint32_t>(32 * q) << 16;
      int s = 0;
      uint32_t ph = 0;
      bool ok = true;
      for (int t = blockIdx.x; ok && t < total; t += gridDim.x) {
        for (int kb = 0; kb < g.k_stages; ++kb) {
          if (!tc::mbar_wait(&full[s], ph)) { ok = false; break; }
          const uint32_t col = tmem + lane_base + L::kSfCol + s * L::kSfColsPerStage;
          const uint8_t* ca = sSFA + s * L::kSfaBytes + lane * 16;
          const uint8_t* cb = sSFB + s * L::kSfbBytes + lane * 16;
          if constexpr (KIND == 3) {  // MMA j: A chunk j at +4 j, B chunks (j, h) at +4 (BN/128) j + 4 h
#pragma unroll
            for (int j = 0; j < KS; ++j) {
              tc::tmem_st4(col + 4 * j, *reinterpret_cast<const uint4*>(ca + j * 512));
#pragma unroll
              for (int h = 0; h < BN / 128; ++h)
                tc::tmem_st4(col + L::kSfaCols + 4 * (BN / 128) * j + 4 * h,
                             *reinterpret_cast<const uint4*>(cb + h * L::kSfaBytes + j * 512));
            }
          } else {  // one chunk per 128 rows covers the stage's 4 MMAs
            tc::tmem_st4(col, *reinterpret_cast<const uint4*>(ca));
#pragma unroll
            for (int h = 0; h < BN / 128; ++h)
              tc::tmem_st4(col + L::kSfaCols + 4 * h, *reinterpret_cast<const uint4*>(cb + h * 512));
          }
          tc::tmem_st_wait();
          tc::fence_before_sync();
          __syncwarp();
          if (lane == 0) tc::mbar_arrive(&sf_full[s]);
          if (++s == STAGES) { s = 0; ph ^= 1u; }
        }
      }
      if (!ok && lane == 0) atomicOr(&g_gemm_status, kDevTimeout);
    }
  } else {  // ------------------------------------------------------------- epilogue warps
    // warps 2..9: lane quarter = warp % 4 (the quarter a warp may read), column half = (warp - 2) / 4
    constexpr int HC = BN / 64;  // 32-column chunks per warp per tile
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;
    const uint32_t lane_base = static_cast<uint32_t>(32 * quarter) << 16;
    uint8_t* stage0 = sOut + (warp - 2) * 2 * L::kStageOutBytes;
    int ab = 0;
    uint32_t aph = 0;
    int chunk = 0;  // chunks this warp has staged (selects the staging buffer)
    for (int t = blockIdx.x; t < total; t += gridDim.x) {
      int mt, nt;
      tile_coords(t, g.m_tiles, g.n_tiles, mt, nt);
      if (!tc::mbar_wait(&acc_full[ab], aph)) {
        if (lane == 0) atomicOr(&g_gemm_status, kDevTimeout);
        break;
      }
      tc::fence_after_sync();
      const int row0 = mt * 128 + 32 * quarter;
      const int64_t row = static_cast<int64_t>(row0) + lane;
      const int colh = nt * BN + half * (BN / 2);
      const uint32_t tbase = tmem + lane_base + ab * BN + half * (BN / 2);
      // this tile's row scale and (lane i of chunk c) column scale / bias, loaded once
      float sa = 0.0f;
      if constexpr (KIND != 2 && OUT != kOutI32) sa = row < g.m ? __ldg(g.a_scale + row) : 0.0f;
      float cs[HC], cbv[HC];
#pragma unroll
      for (int c = 0; c < HC; ++c) {
        const int64_t col = static_cast<int64_t>(colh) + c * 32 + lane;
        cs[c] = 0.0f;
        cbv[c] = 0.0f;
        if constexpr (OUT != kOutI32) {
          if constexpr (KIND == 0 || KIND == 1) cs[c] = col < g.n ? __ldg(g.b_scale + col) : 0.0f;
          if constexpr (KIND == 3) cs[c] = g.b_scale_per_col ? (col < g.n ? __ldg(g.b_scale + col) : 0.0f) : __ldg(g.b_scale);
          if (g.bias != nullptr && col < g.n) cbv[c] = load_bias(g.bias, g.bias_dtype, col);
        }
      }
      uint32_t r[32];
      tc::tmem_ld32(tbase, r);
      tc::tmem_ld_wait();
#pragma unroll
      for (int c = 0; c < HC; ++c) {
        uint32_t y[32];
        epilogue_math<KIND, OUT>(g, r, sa, cs[c], cbv[c], y);
        if (c + 1 < HC) {
          tc::tmem_ld32(tbase + (c + 1) * 32, r);
        } else {  // this warp's columns are read: hand the accumulator back to the MMA warp
          tc::fence_before_sync();
          __syncwarp();
          if (lane == 0) tc::mbar_arrive(&acc_empty[ab]);
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
          tc::tma_store_2d(&tma_out, buf, colh + c * 32, row0);
          tc::bulk_commit();
        }
        ++chunk;
        if (c + 1 < HC) tc::tmem_ld_wait();
      }
      if (++ab == L::kAccBufs) { ab = 0; aph ^= 1u; }
    }
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
