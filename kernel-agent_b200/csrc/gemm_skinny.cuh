// Decode-size W8A8 GEMMs (M <= 32 tokens): the weight streams through the tensor core as the
// MMA's 128-row A operand and the tokens are its N (16 or 32), the role swap of kernel-agent's
// skinny examples (src/kernel_agent/agent/examples/cuda_int8_skinny_gemm.py,
// cuda_fp8_skinny_gemm.py) on tcgen05: D[channel, token] = W[channel, :] . X[token, :].
//
// One CTA per 128-channel panel of W: warp 0 loads W [128 x 128 bytes] and X [NT x 128 bytes]
// stages by TMA (rows of X past M read as zeros) into a 10- or 5-stage ring, warp 1 issues
// tcgen05.mma (kind::i8 exact int32, or kind::f8f6f4 fp32) into a [128 lanes x NT] TMEM
// accumulator, warps 2-5 read it back (lane = channel) and apply the epilogue of the tiled
// kernel, quant.py:920-922's acc.float() * xs[m] * sw[n] (+ bias), left to right in fp32, one
// rounding to the output type; each warp stores 32 consecutive channels of one token per
// instruction. The weight is read from HBM once; the tokens' 128-byte stages come from L2.
// No load uses cluster multicast; every wait is bounded.
#pragma once

#include "gemm.cuh"

namespace kab {

// STAGES 10 when the grid fits on the SMs (one CTA each, the deepest ring), 5 otherwise (two
// CTAs per SM).
template <int NT, int OUT, int STAGES>
struct SkinnyLayout {
  static constexpr int kWBytes = 128 * 128;
  static constexpr int kXBytes = NT * 128;
  static constexpr int kStageBytes = kWBytes + kXBytes;
  static constexpr int kStages = STAGES;
  static constexpr int kThreads = 192;
  static constexpr int kSmem = 1024 + kStages * kStageBytes + (2 * kStages + 1) * 8 + 16;
  static_assert(kSmem <= (STAGES > 5 ? 232448 : 232448 / 2), "shared memory per CTA");
};

template <int KIND, int NT, int OUT, int STAGES_>
__global__ void __launch_bounds__(192, 2)
gemm_skinny_kernel(const __grid_constant__ CUtensorMap tma_w, const __grid_constant__ CUtensorMap tma_x, GemmArgs g) {
  using L = SkinnyLayout<NT, OUT, STAGES_>;
  constexpr int STAGES = L::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sW = smem;
  uint8_t* sX = sW + STAGES * L::kWBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sX + STAGES * L::kXBytes);
  uint64_t* full = bars;
  uint64_t* empty = full + STAGES;
  uint64_t* done = empty + STAGES;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = static_cast<int>(blockIdx.x) * 128;
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      tc::mbar_init(&full[s], 1);
      tc::mbar_init(&empty[s], 1);
    }
    tc::mbar_init(done, 1);
    tc::fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tc::prefetch_tensormap(&tma_w);
    tc::prefetch_tensormap(&tma_x);
  }
  if (warp == 1) { tc::tmem_alloc(tmem_slot, 32); tc::tmem_relinquish(); }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {  // ---------------------------------------------------- TMA producer
      bool ok = true;
      int issued = 0;
      for (int kb = 0; kb < g.k_stages; ++kb) {
        const int s = kb % STAGES;
        if (!tc::mbar_wait(&empty[s], static_cast<uint32_t>(((kb / STAGES) & 1) ^ 1))) { ok = false; break; }
        tc::mbar_arrive_expect_tx(&full[s], L::kStageBytes);
        tc::tma_load_2d(&tma_w, &full[s], sW + s * L::kWBytes, kb * 128, n0);
        tc::tma_load_2d(&tma_x, &full[s], sX + s * L::kXBytes, kb * 128, 0);
        issued = kb + 1;
      }
      if (!ok) {
        atomicOr(&g_gemm_status, kDevTimeout);
        for (int kb = (issued > STAGES ? issued - STAGES : 0); kb < issued; ++kb)  // let issued loads land
          tc::mbar_wait(&full[kb % STAGES], static_cast<uint32_t>((kb / STAGES) & 1));
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {  // ---------------------------------------------------- MMA issuer
      bool ok = true;
      for (int kb = 0; kb < g.k_stages; ++kb) {
        const int s = kb % STAGES;
        if (!tc::mbar_wait(&full[s], static_cast<uint32_t>((kb / STAGES) & 1))) { ok = false; break; }
        tc::fence_after_sync();
        const uint64_t adesc = tc::desc_sw128(tc::smem_u32(sW + s * L::kWBytes));
        const uint64_t bdesc = tc::desc_sw128(tc::smem_u32(sX + s * L::kXBytes));
#pragma unroll
        for (int j = 0; j < 4; ++j) {  // 32 bytes of K each
          const uint32_t acc = (kb > 0 || j > 0) ? 1u : 0u;
          if constexpr (KIND == 0)
            tc::mma_i8(tmem, adesc + 2 * j, bdesc + 2 * j, tc::idesc_i8(128, NT), acc);
          else
            tc::mma_f8(tmem, adesc + 2 * j, bdesc + 2 * j, tc::idesc_f8(128, NT), acc);
        }
        tc::commit(&empty[s]);
      }
      tc::commit(done);  // the accumulator is final (or, after a timeout, the MMAs issued are done)
      if (!ok) atomicOr(&g_gemm_status, kDevTimeout);
    }
  } else {  // ------------------------------------------------------------- epilogue warps 2-5
    const int quarter = warp & 3;
    const int64_t n = static_cast<int64_t>(n0) + 32 * quarter + lane;  // this lane's channel
    const bool live = n < g.n;
    if (!tc::mbar_wait(done, 0)) {
      if (lane == 0) atomicOr(&g_gemm_status, kDevTimeout);
    } else {
      tc::fence_after_sync();
      uint32_t r[32];
      tc::tmem_ld32(tmem + (static_cast<uint32_t>(32 * quarter) << 16), r);
      tc::tmem_ld_wait();
      float sw = 0.0f, bi = 0.0f;
      if constexpr (OUT != kOutI32) {
        sw = live ? __ldg(g.b_scale + n) : 0.0f;
        if (g.bias != nullptr && live) bi = load_bias(g.bias, g.bias_dtype, n);
      }
#pragma unroll
      for (int m = 0; m < NT; ++m) {
        if (m >= g.m) break;
        if constexpr (OUT == kOutI32) {
          if (live) g.acc_out[m * g.ldo + n] = static_cast<int32_t>(r[m]);
        } else {
          // quant.py:920-922: acc.float() * xs[m] * sw[n] (+ bias), left to right in fp32
          const float acc = KIND == 0 ? __int2float_rn(static_cast<int>(r[m])) : __uint_as_float(r[m]);
          float v = __fmul_rn(__fmul_rn(acc, __ldg(g.a_scale + m)), sw);
          if (g.bias != nullptr) v = __fadd_rn(v, bi);
          if (live) {
            if constexpr (OUT == KAB_BF16)
              reinterpret_cast<uint16_t*>(g.out)[m * g.ldo + n] = f32_to_bf16_bits(v);
            else if constexpr (OUT == KAB_F16)
              reinterpret_cast<uint16_t*>(g.out)[m * g.ldo + n] = f32_to_f16_bits(v);
            else
              reinterpret_cast<float*>(g.out)[m * g.ldo + n] = v;
          }
        }
      }
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc::fence_after_sync();
    tc::tmem_dealloc(tmem, 32);
  }
}

}  // namespace kab
