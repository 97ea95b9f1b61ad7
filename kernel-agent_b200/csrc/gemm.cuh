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
// One persistent CTA per SM (192 threads): warp 0 issues the TMA loads (one thread), warp 1
// the MMAs (one thread) and owns the TMEM allocation, warps 2-5 drain the accumulator
// (tcgen05.ld, one TMEM lane = one output row per thread). Output tiles are 128 x BN; the
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
  // bytes of block scales per 128 rows per k-step (128 bytes of K per row)
  static constexpr int kSfBytes = KIND == 3 ? 2048 : (KIND == 2 ? 512 : 0);
  // TMEM columns of block scales per k-step for A (B: twice as many per 256 rows)
  static constexpr int kSfColsA = KIND == 3 ? 16 : (KIND == 2 ? 4 : 0);
};

template <int BN, int STAGES, int KIND>
struct GemmLayout {
  static constexpr int kBM = 128;
  static constexpr int kABytes = kBM * 128;
  static constexpr int kBBytes = BN * 128;
  static constexpr int kSfaBytes = GemmTraits<KIND>::kSfBytes;
  static constexpr int kSfbBytes = GemmTraits<KIND>::kSfBytes * (BN / 128);
  static constexpr int kStageBytes = kABytes + kBBytes + kSfaBytes + kSfbBytes;
  static constexpr int kAccBufs = GemmTraits<KIND>::kScaled ? (BN == 256 ? 1 : 2) : 2;
  static constexpr int kSfCol = kAccBufs * BN;
  static constexpr int kSfColsPerStage = GemmTraits<KIND>::kSfColsA * (1 + BN / 128);
  static constexpr int kBarriers = 2 * STAGES + 2 * kAccBufs + 1;
  static constexpr int kSmem = 1024 + STAGES * kStageBytes + kBarriers * 8 + 16;
  static_assert(kSfCol + STAGES * kSfColsPerStage <= 512, "TMEM overflow");
};

template <int OUT>
__device__ __forceinline__ void store32(void* out, int64_t off, const float (&y)[32]) {
  if constexpr (OUT == KAB_F32) {
    float4* p = reinterpret_cast<float4*>(reinterpret_cast<float*>(out) + off);
#pragma unroll
    for (int i = 0; i < 8; ++i) p[i] = make_float4(y[4 * i], y[4 * i + 1], y[4 * i + 2], y[4 * i + 3]);
  } else {
    uint32_t w[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const uint16_t lo = OUT == KAB_BF16 ? f32_to_bf16_bits(y[2 * i]) : f32_to_f16_bits(y[2 * i]);
      const uint16_t hi = OUT == KAB_BF16 ? f32_to_bf16_bits(y[2 * i + 1]) : f32_to_f16_bits(y[2 * i + 1]);
      w[i] = static_cast<uint32_t>(lo) | (static_cast<uint32_t>(hi) << 16);
    }
    uint4* p = reinterpret_cast<uint4*>(reinterpret_cast<uint16_t*>(out) + off);
#pragma unroll
    for (int i = 0; i < 4; ++i) p[i] = make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
  }
}

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

template <int KIND, int BN, int OUT>
__device__ __forceinline__ void epilogue_chunk(const GemmArgs& g, const uint32_t (&r)[32], int64_t row,
                                               int64_t col0) {
  float y[32];
  if constexpr (KIND == 0 || KIND == 1) {
    // quant.py:920-922: acc.float() * xs[m] * sw[n] (+ bias), left to right in fp32
    const float sa = row < g.m ? __ldg(g.a_scale + row) : 0.0f;
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      const float acc = KIND == 0 ? __int2float_rn(static_cast<int>(r[i])) : __uint_as_float(r[i]);
      const int64_t c = col0 + i;
      const float sb = c < g.n ? __ldg(g.b_scale + c) : 0.0f;
      float v = __fmul_rn(__fmul_rn(acc, sa), sb);
      if (g.bias != nullptr && c < g.n) v = __fadd_rn(v, load_bias(g.bias, g.bias_dtype, c));
      y[i] = v;
    }
  } else if constexpr (KIND == 2) {
    // quant.py:602-614: F.scaled_mm's output in the output dtype, then + bias in that dtype
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      const int64_t c = col0 + i;
      float v = round_out<OUT>(__uint_as_float(r[i]));
      if (g.bias != nullptr && c < g.n) v = __fadd_rn(v, load_bias(g.bias, g.bias_dtype, c));
      y[i] = v;
    }
  } else {
    // quant.py:1254-1256: acc * (outer[m] * ts) (+ bias.float())
    const float outer = row < g.m ? __ldg(g.a_scale + row) : 0.0f;
    const float ts0 = g.b_scale_per_col ? 0.0f : __ldg(g.b_scale);
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      const int64_t c = col0 + i;
      const float ts = g.b_scale_per_col ? (c < g.n ? __ldg(g.b_scale + c) : 0.0f) : ts0;
      float v = __fmul_rn(__uint_as_float(r[i]), __fmul_rn(outer, ts));
      if (g.bias != nullptr && c < g.n) v = __fadd_rn(v, load_bias(g.bias, g.bias_dtype, c));
      y[i] = v;
    }
  }
  if (row >= g.m) return;
  if (col0 + 32 <= g.n) {
    store32<OUT>(g.out, row * g.ldo + col0, y);
  } else {
    for (int i = 0; i < 32 && col0 + i < g.n; ++i) {
      const int64_t o = row * g.ldo + col0 + i;
      if constexpr (OUT == KAB_F32) reinterpret_cast<float*>(g.out)[o] = y[i];
      else if constexpr (OUT == KAB_BF16) reinterpret_cast<uint16_t*>(g.out)[o] = f32_to_bf16_bits(y[i]);
      else reinterpret_cast<uint16_t*>(g.out)[o] = f32_to_f16_bits(y[i]);
    }
  }
}

__device__ __forceinline__ void store_acc32(const GemmArgs& g, const uint32_t (&r)[32], int64_t row, int64_t col0) {
  if (row >= g.m) return;
  int32_t* p = g.acc_out + row * g.ldo + col0;
  if (col0 + 32 <= g.n) {
    int4* q = reinterpret_cast<int4*>(p);
#pragma unroll
    for (int i = 0; i < 8; ++i)
      q[i] = make_int4(static_cast<int>(r[4 * i]), static_cast<int>(r[4 * i + 1]), static_cast<int>(r[4 * i + 2]),
                       static_cast<int>(r[4 * i + 3]));
  } else {
    for (int i = 0; i < 32 && col0 + i < g.n; ++i) p[i] = static_cast<int>(r[i]);
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

template <int KIND, int BN, int STAGES, int OUT>
__global__ void __launch_bounds__(192, 1)
gemm_kernel(const __grid_constant__ CUtensorMap tma_a, const __grid_constant__ CUtensorMap tma_b, GemmArgs g) {
  using L = GemmLayout<BN, STAGES, KIND>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = sA + STAGES * L::kABytes;
  uint8_t* sSFA = sB + STAGES * L::kBBytes;
  uint8_t* sSFB = sSFA + STAGES * L::kSfaBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sSFB + STAGES * L::kSfbBytes);
  uint64_t* full = bars;
  uint64_t* empty = bars + STAGES;
  uint64_t* acc_full = bars + 2 * STAGES;
  uint64_t* acc_empty = acc_full + L::kAccBufs;
  uint64_t* drain = acc_empty + L::kAccBufs;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) { tc::mbar_init(&full[s], 1); tc::mbar_init(&empty[s], 1); }
    for (int b = 0; b < L::kAccBufs; ++b) { tc::mbar_init(&acc_full[b], 1); tc::mbar_init(&acc_empty[b], 4); }
    tc::mbar_init(drain, 1);
    tc::fence_barrier_init();
  }
  if (warp == 0 && lane == 0) { tc::prefetch_tensormap(&tma_a); tc::prefetch_tensormap(&tma_b); }
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
          tc::tma_load_2d(&tma_a, &full[s], sA + s * L::kABytes, kb * 128, mt * 128);
          tc::tma_load_2d(&tma_b, &full[s], sB + s * L::kBBytes, kb * 128, nt * BN);
          if constexpr (KIND == 3) {
            tc::bulk_load(sSFA + s * L::kSfaBytes, g.sfa + (mt * g.sfa_ncb + 4 * kb) * 512, 2048, &full[s]);
#pragma unroll
            for (int h = 0; h < BN / 128; ++h)
              tc::bulk_load(sSFB + s * L::kSfbBytes + h * 2048,
                            g.sfb + ((nt * (BN / 128) + h) * g.sfb_ncb + 4 * kb) * 512, 2048, &full[s]);
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
          tc::fence_after_sync();
          const uint64_t adesc = tc::desc_sw128(tc::smem_u32(sA + s * L::kABytes));
          const uint64_t bdesc = tc::desc_sw128(tc::smem_u32(sB + s * L::kBBytes));
          const uint32_t sf = tmem + L::kSfCol + s * L::kSfColsPerStage;
          if constexpr (KIND == 3) {
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              tc::cp_sf(sf + j * 4, tc::desc_sf(tc::smem_u32(sSFA + s * L::kSfaBytes + j * 512)));
#pragma unroll
              for (int h = 0; h < BN / 128; ++h)
                tc::cp_sf(sf + 16 + j * (4 * (BN / 128)) + h * 4,
                          tc::desc_sf(tc::smem_u32(sSFB + s * L::kSfbBytes + h * 2048 + j * 512)));
            }
          } else if constexpr (KIND == 2) {
            tc::cp_sf(sf, tc::desc_sf(tc::smem_u32(sSFA + s * L::kSfaBytes)));
#pragma unroll
            for (int h = 0; h < BN / 128; ++h)
              tc::cp_sf(sf + 4 + h * 4, tc::desc_sf(tc::smem_u32(sSFB + s * L::kSfbBytes + h * 512)));
          }
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const uint32_t acc = (kb > 0 || j > 0) ? 1u : 0u;
            const uint64_t a = adesc + static_cast<uint64_t>(2 * j);  // +32 bytes of K
            const uint64_t b = bdesc + static_cast<uint64_t>(2 * j);
            if constexpr (KIND == 0) tc::mma_i8(d, a, b, tc::idesc_i8(128, BN), acc);
            else if constexpr (KIND == 1) tc::mma_f8(d, a, b, tc::idesc_f8(128, BN), acc);
            else if constexpr (KIND == 2) tc::mma_mxf8(d, a, b, tc::idesc_mxf8(128, BN, j), sf, sf + 4, acc);
            else tc::mma_nvf4(d, a, b, tc::idesc_nvf4(128, BN), sf + j * 4, sf + 16 + j * (4 * (BN / 128)), acc);
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
  } else {  // ------------------------------------------------------------- epilogue warps
    const int quarter = warp & 3;
    const uint32_t lane_base = static_cast<uint32_t>(32 * quarter) << 16;
    int ab = 0;
    uint32_t aph = 0;
    for (int t = blockIdx.x; t < total; t += gridDim.x) {
      int mt, nt;
      tile_coords(t, g.m_tiles, g.n_tiles, mt, nt);
      if (!tc::mbar_wait(&acc_full[ab], aph)) {
        if (lane == 0) atomicOr(&g_gemm_status, kDevTimeout);
        break;
      }
      tc::fence_after_sync();
      const int64_t row = static_cast<int64_t>(mt) * 128 + 32 * quarter + lane;
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        uint32_t r[32];
        tc::tmem_ld32(tmem + lane_base + ab * BN + c * 32, r);
        tc::tmem_ld_wait();
        const int64_t col0 = static_cast<int64_t>(nt) * BN + c * 32;
        if (KIND == 0 && g.acc_out != nullptr) store_acc32(g, r, row, col0);
        else epilogue_chunk<KIND, BN, OUT>(g, r, row, col0);
      }
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(&acc_empty[ab]);
      if (++ab == L::kAccBufs) { ab = 0; aph ^= 1u; }
    }
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
