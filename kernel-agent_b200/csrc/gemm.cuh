// Scaled GEMMs D[m, n] = sum_k A[m, k] * B[n, k] on the 5th-generation tensor cores
// (tcgen05.mma, accumulators in TMEM), fed by a TMA multistage shared-memory ring, with the
// dequantisation / bias / cast epilogue fused.
//
//   KIND 0  kind::i8        int8 x int8 -> int32 (exact); epilogue acc * sa[m] * sb[n] (+ bias)
//   KIND 1  kind::f8f6f4    e4m3 x e4m3 -> fp32; epilogue acc * sa[m] * sb[n] (+ bias)
//   KIND 2  kind::mxf8f6f4  e4m3 x e4m3 with e8m0 scales per 32 applied by the tensor core
//   KIND 3  kind::mxf4nvf4  e2m1 x e2m1 with e4m3 scales per 16 applied by the tensor core;
//                            epilogue acc * (outer[m] * ts[n or one]) (+ bias)
//   KIND 4  kind::mxf4nvf4  e2m1 x e2m1 with e8m0 scales per 32 (MXFP4, scale_vec::2X);
//                            epilogue acc * (1 * ts) (+ bias): MXFP4 activations have outer 1
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

constexpr int kMaxPeers = 7;  // peer outputs one GEMM epilogue writes (8 GPUs of a box)

struct GemmArgs {
  int64_t m, n;
  int k_stages;                 // K bytes per row / 128
  int m_tiles, n_tiles;
  int group_n;                  // tile order: see tile_coords
  const uint8_t* sfa;           // swizzled block scales of A (KIND 2, 3)
  const uint8_t* sfb;           // ... of B
  int64_t sfa_ncb, sfb_ncb;     // 4-column blocks per 128-row block of each
  int64_t sfb_chunks;           // 128-row blocks of B's scales (ceil(n / 128))
  const float* a_scale;         // per row of A: token scale (KIND 0, 1), outer (KIND 3)
  const float* b_scale;         // per row of B (KIND 0, 1), tensor scale(s) (KIND 3)
  int b_scale_per_col;          // KIND 3: b_scale[n] instead of b_scale[0]
  const void* bias;             // [n] in bias_dtype, or null
  int bias_dtype;
  void* out;                    // [m, ldo] in out_dtype
  int out_dtype;
  int64_t ldo;
  int32_t* acc_out;             // KIND 0: raw int32 products [m, ldo] instead of `out`
  void* peer_out[kMaxPeers];     // other ranks' output origins ([m, ldo] like `out`), or none
  int npeers;
};

// Tensor maps of the other ranks' outputs (CUDA IPC mappings of buffers laid out like `out`):
// the epilogue stores each staged tile to them with TMA, like the local output.
struct PeerMaps {
  CUtensorMap m[kMaxPeers];
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
  static constexpr int kGroups = BN / 32;  // 32-row groups of B per tile
  // Block scales per 128 rows per stage (one 512-byte chunk of the swizzled layout per 64
  // elements of K for NVFP4, per 128 for MXFP8) and the 128-row chunks a B tile can span
  // (BN need not be a multiple of 128).
  static constexpr int kSfChunkBytes = KIND == 3 ? 512 * kKSteps : (KIND == 4 ? 256 * kKSteps : 512);
  static constexpr int kSfaBytes = kScaled ? kSfChunkBytes : 0;
  // groups start at word 0 or 2 of a chunk (BN a multiple of 64), so a tile spans
  // ceil((2 + kGroups) / 4) chunks at most (kGroups / 4 when BN is a multiple of 128)
  static constexpr int kSfbChunks = !kScaled ? 0 : (kGroups % 4 == 0 ? kGroups / 4 : (kGroups + 2 + 3) / 4);
  static constexpr int kSfbBytes = kSfbChunks * kSfChunkBytes;
  static constexpr int kStageBytes = kABytes + kBBytes + kSfaBytes + kSfbBytes;
  // TMEM columns of block scales per stage. Each 512-byte chunk (32 rows of 16 bytes: row
  // r % 32 holds the scale words of rows {r, r + 32, r + 64, r + 96}) lands in 4 columns of
  // every lane quarter, lane l holding chunk row l (the layout tcgen05.cp.32x128b.warpx4
  // makes); the scale-factor warps 10-13 write it with tcgen05.st, each into its own quarter.
  // A: 4 columns per scale set; B: one per 32 rows. NVFP4 has one set per MMA (K = 64),
  // MXFP8 one per stage (the MMA picks its byte by sf_id).
  static constexpr int kSfSets = KIND == 3 ? kKSteps : (KIND == 4 ? kKSteps / 2 : 1);
  static constexpr int kSfaCols = kScaled ? 4 * kSfSets : 0;
  static constexpr int kSfbCols = kScaled ? kGroups * kSfSets : 0;
  static constexpr int kSfColsPerStage = kSfaCols + kSfbCols;
  static constexpr int kEpiWarps = 8;  // two per TMEM lane quarter
  // warps: 0 TMA, 1 MMA, 2-9 epilogue; block-scaled kinds add warps 10-13 for the scale factors
  static constexpr int kThreads = 32 * (2 + kEpiWarps + (kScaled ? 4 : 0));
  // stages whose scale factors the warp writes before one wait for the stores to land
  static constexpr int kSfBatch = 1;
  static constexpr int kAccBufs = 2;  // the epilogue drains one accumulator while the MMAs fill the other
  static constexpr int kSfCol = kAccBufs * BN;
  // the scale-factor ring in the columns the accumulators leave
  static constexpr int kSfSlotsFit = kScaled ? (512 - kSfCol) / kSfColsPerStage : 0;
  static constexpr int kSfSlots = kSfSlotsFit > 8 ? 8 : kSfSlotsFit;
  // epilogue staging: 8 warps x 2 buffers x [32 rows, 32 columns]
  static constexpr int kStageOutBytes = 32 * 32 * out_bytes(OUT);
  static constexpr int kStagingBytes = kEpiWarps * 2 * kStageOutBytes;
  static_assert(kStagingBytes % 1024 == 0, "the operand tiles after the staging tiles need 1024-byte alignment");
  static constexpr int kSmemLimit = 232448;
  static constexpr int kFixed = 1024 + kStagingBytes + 384;
  static constexpr int kStagesFit = (kSmemLimit - kFixed) / kStageBytes;
  static constexpr int kStages = kStagesFit > 8 ? 8 : kStagesFit;
  static constexpr int kBarriers = 2 * kStages + 2 * kSfSlots + 2 * kAccBufs + 1;
  static constexpr int kSmem = 1024 + kStages * kStageBytes + kStagingBytes + kBarriers * 8 + 16;
  static_assert(BN % 64 == 0 && BN <= 256, "BN must be a multiple of 64, at most 256");
  static_assert(kStages >= 2, "shared memory does not fit two stages");
  static_assert(!kScaled || kSfSlots >= 2 * kSfBatch, "TMEM does not fit two batches of scale-factor slots");
  static_assert(kSfCol + kSfSlots * kSfColsPerStage <= 512, "TMEM overflow");
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
    // quant.py:1254-1256: acc * (outer[m] * ts) (+ bias.float()); MXFP4's outer is 1
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

// One row of 32 outputs packed in the output type: 32 words (4-byte types) or 16 (2-byte
// types, rounded to nearest even, two per conversion instruction).
template <int OUT>
__device__ __forceinline__ void pack_row(const uint32_t (&y)[32], uint32_t (&w)[32]) {
  if constexpr (out_bytes(OUT) == 4) {
#pragma unroll
    for (int i = 0; i < 32; ++i) w[i] = y[i];
  } else {
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
  }
}

// Writes one packed row (this lane's row) into a [32 rows, 32 columns] staging tile in the
// layout of the output tensor map's swizzle (64-byte rows: SWIZZLE_64B, 16-byte chunk i of row
// r at i ^ ((r >> 1) & 3); 128-byte rows: SWIZZLE_128B, at i ^ (r & 7)), so each quarter-warp
// phase of the stores covers all 32 banks. The tile must be 1024-byte aligned.
template <int OUT>
__device__ __forceinline__ void stage_packed(uint8_t* buf, int lane, const uint32_t (&w)[32]) {
  constexpr int kChunks = 32 * out_bytes(OUT) / 16;
  const int sw = kChunks == 8 ? (lane & 7) : ((lane >> 1) & 3);
  uint4* p = reinterpret_cast<uint4*>(buf + lane * (32 * out_bytes(OUT)));
#pragma unroll
  for (int i = 0; i < kChunks; ++i) p[i ^ sw] = make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
}

template <int OUT>
__device__ __forceinline__ void stage_row(uint8_t* buf, int lane, const uint32_t (&y)[32]) {
  uint32_t w[32];
  pack_row<OUT>(y, w);
  stage_packed<OUT>(buf, lane, w);
}

// Tile t of the persistent schedule -> (m tile, n tile). group_n == 0: groups of 8 m-tiles
// sweep n (an A panel stays in L2 while B streams); group_n > 0: groups of group_n n-tiles
// sweep m (for a B larger than L2: each B panel is read from HBM once while A, the smaller
// operand, stays in L2).
__device__ __forceinline__ void tile_coords(int t, int m_tiles, int n_tiles, int group_n, int& mt, int& nt) {
  if (group_n > 0) {
    const int group_size = group_n * m_tiles;
    const int first = (t / group_size) * group_n;
    const int gn = min(n_tiles - first, group_n);
    const int r = t % group_size;
    nt = first + r % gn;
    mt = r / gn;
    return;
  }
  constexpr int kGroup = 8;
  const int group_size = kGroup * n_tiles;
  const int first = (t / group_size) * kGroup;
  const int gm = min(m_tiles - first, kGroup);
  const int r = t % group_size;
  mt = first + r % gm;
  nt = r / gm;
}

// One epilogue warp's share of a finished accumulator tile: rows row0 + lane (its TMEM lane
// quarter), HC chunks of 32 columns from colh, read from TMEM at tbase. Each chunk is scaled
// (epilogue_math), staged in shared memory and stored by TMA to the output and to each of the
// g.npeers peer outputs in `peers` (over NVLink: the copies run on the TMA unit while the warp
// goes on); `release` runs (lane 0, after a warp sync) once the last chunk has been read from
// TMEM.
template <int KIND, int OUT, int HC, class Release>
__device__ __forceinline__ void epilogue_tile(const GemmArgs& g, const CUtensorMap* tma_out, const PeerMaps* peers,
                                              uint32_t tbase, int row0, int colh, uint8_t* stage0, int& chunk, int lane,
                                              Release release) {
  constexpr int kStageOutBytes = 32 * 32 * out_bytes(OUT);
  const int64_t row = static_cast<int64_t>(row0) + lane;
  // this tile's row scale and (lane i of chunk c) column scale / bias, loaded once
  float sa = 0.0f;
  if constexpr (KIND == 4) sa = g.a_scale == nullptr ? 1.0f : (row < g.m ? __ldg(g.a_scale + row) : 0.0f);
  else if constexpr (KIND != 2 && OUT != kOutI32) sa = row < g.m ? __ldg(g.a_scale + row) : 0.0f;
  float cs[HC], cbv[HC];
#pragma unroll
  for (int c = 0; c < HC; ++c) {
    const int64_t col = static_cast<int64_t>(colh) + c * 32 + lane;
    cs[c] = 0.0f;
    cbv[c] = 0.0f;
    if constexpr (OUT != kOutI32) {
      if constexpr (KIND == 0 || KIND == 1) cs[c] = col < g.n ? __ldg(g.b_scale + col) : 0.0f;
      if constexpr (KIND == 3 || KIND == 4) {
        if (KIND == 4 && g.b_scale == nullptr) cs[c] = 1.0f;
        else cs[c] = g.b_scale_per_col ? (col < g.n ? __ldg(g.b_scale + col) : 0.0f) : __ldg(g.b_scale);
      }
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
      if (lane == 0) release();
    }
    uint8_t* buf = stage0 + (chunk & 1) * kStageOutBytes;
    if (chunk >= 2) {  // the store two chunks ago has finished reading this buffer
      if (lane == 0) tc::bulk_wait_read<1>();
      __syncwarp();
    }
    uint32_t w[32];
    pack_row<OUT>(y, w);
    stage_packed<OUT>(buf, lane, w);
    tc::fence_proxy_async();
    __syncwarp();
    if (lane == 0) {
      tc::tma_store_2d(tma_out, buf, colh + c * 32, row0);
      if (peers != nullptr) {
#pragma unroll
        for (int p = 0; p < kMaxPeers; ++p) {
          if (p >= g.npeers) break;
          tc::tma_store_2d(&peers->m[p], buf, colh + c * 32, row0);
        }
      }
      tc::bulk_commit();  // one group per chunk: the buffer is free once its reads are done
    }
    ++chunk;
    if (c + 1 < HC) tc::tmem_ld_wait();
  }
}

// The per-tile scale operands of one epilogue warp's share (rows row0 + lane, HC chunks of 32
// columns from colh): the row scale and, lane i of chunk c, the column scale and bias of
// column colh + 32 c + i. Loaded before the accumulator is ready.
template <int KIND, int OUT, int HC>
struct EpilogueOperands {
  float sa;
  float cs[HC], cb[HC];
  __device__ __forceinline__ void load(const GemmArgs& g, int row0, int colh, int lane) {
    const int64_t row = static_cast<int64_t>(row0) + lane;
    sa = 0.0f;
    if constexpr (KIND == 4) sa = g.a_scale == nullptr ? 1.0f : (row < g.m ? __ldg(g.a_scale + row) : 0.0f);
    else if constexpr (KIND != 2 && OUT != kOutI32) sa = row < g.m ? __ldg(g.a_scale + row) : 0.0f;
#pragma unroll
    for (int c = 0; c < HC; ++c) {
      const int64_t col = static_cast<int64_t>(colh) + c * 32 + lane;
      cs[c] = 0.0f;
      cb[c] = 0.0f;
      if constexpr (OUT != kOutI32) {
        if constexpr (KIND == 0 || KIND == 1) cs[c] = col < g.n ? __ldg(g.b_scale + col) : 0.0f;
        if constexpr (KIND == 3 || KIND == 4) {
          if (KIND == 4 && g.b_scale == nullptr) cs[c] = 1.0f;
          else cs[c] = g.b_scale_per_col ? (col < g.n ? __ldg(g.b_scale + col) : 0.0f) : __ldg(g.b_scale);
        }
        if (g.bias != nullptr && col < g.n) cb[c] = load_bias(g.bias, g.bias_dtype, col);
      }
    }
  }
};

// epilogue_tile for an accumulator that only one buffer holds: every column of the warp's
// share is read from TMEM first (HC x 32 registers) and the accumulator is released before
// any of the epilogue arithmetic, so the next tile's MMAs wait only for the TMEM reads.
template <int KIND, int OUT, int HC, class Release>
__device__ __forceinline__ void epilogue_tile_early(const GemmArgs& g, const EpilogueOperands<KIND, OUT, HC>& ops,
                                                    const CUtensorMap* tma_out, const PeerMaps* peers, uint32_t tbase,
                                                    int row0, int colh, uint8_t* stage0, int& chunk, int lane,
                                                    Release release) {
  constexpr int kStageOutBytes = 32 * 32 * out_bytes(OUT);
  uint32_t r[HC][32];
#pragma unroll
  for (int c = 0; c < HC; ++c) tc::tmem_ld32(tbase + c * 32, r[c]);
  tc::tmem_ld_wait();
  tc::fence_before_sync();
  __syncwarp();
  if (lane == 0) release();
#pragma unroll
  for (int c = 0; c < HC; ++c) {
    uint32_t y[32];
    epilogue_math<KIND, OUT>(g, r[c], ops.sa, ops.cs[c], ops.cb[c], y);
    uint8_t* buf = stage0 + (chunk & 1) * kStageOutBytes;
    if (chunk >= 2) {  // the store two chunks ago has finished reading this buffer
      if (lane == 0) tc::bulk_wait_read<1>();
      __syncwarp();
    }
    uint32_t w[32];
    pack_row<OUT>(y, w);
    stage_packed<OUT>(buf, lane, w);
    tc::fence_proxy_async();
    __syncwarp();
    if (lane == 0) {
      tc::tma_store_2d(tma_out, buf, colh + c * 32, row0);
      if (peers != nullptr) {
#pragma unroll
        for (int p = 0; p < kMaxPeers; ++p) {
          if (p >= g.npeers) break;
          tc::tma_store_2d(&peers->m[p], buf, colh + c * 32, row0);
        }
      }
      tc::bulk_commit();
    }
    ++chunk;
  }
}

// epilogue_tile_early with 128-byte staged rows: each store is [32 rows, 128 bytes] (64
// columns of a 2-byte output, 32 of a 4-byte one) in the TMA store's 128-byte swizzle (16-byte
// chunk i of row r at i ^ (r & 7)), so every row a store writes, to the local output and over
// NVLink to each peer, is a full 128 bytes (B200: a probe of peer TMA stores moved 570 GB/s
// with 64-byte rows and 698 GB/s with 128-byte ones). One 4 KB staging buffer per warp: before
// it is rewritten, the previous store has finished reading it.
template <int KIND, int OUT, int HC, class Release>
__device__ __forceinline__ void epilogue_tile_wide(const GemmArgs& g, const EpilogueOperands<KIND, OUT, HC>& ops,
                                                   const CUtensorMap* tma_out, const PeerMaps* peers, uint32_t tbase,
                                                   int row0, int colh, uint8_t* stage, int lane, Release release) {
  constexpr int kPer = out_bytes(OUT) == 2 ? 2 : 1;  // 32-column sub-chunks per 128-byte row
  static_assert(HC % kPer == 0, "whole 128-byte rows");
  uint32_t r[HC][32];
#pragma unroll
  for (int c = 0; c < HC; ++c) tc::tmem_ld32(tbase + c * 32, r[c]);
  tc::tmem_ld_wait();
  tc::fence_before_sync();
  __syncwarp();
  if (lane == 0) release();
  const int sw = lane & 7;
  uint4* row = reinterpret_cast<uint4*>(stage + lane * 128);
#pragma unroll
  for (int c = 0; c < HC; c += kPer) {
    uint32_t w[32];  // the row's 128 bytes
#pragma unroll
    for (int h = 0; h < kPer; ++h) {
      uint32_t y[32], p[32];
      epilogue_math<KIND, OUT>(g, r[c + h], ops.sa, ops.cs[c + h], ops.cb[c + h], y);
      pack_row<OUT>(y, p);
#pragma unroll
      for (int i = 0; i < 32 / kPer; ++i) w[h * (32 / kPer) + i] = p[i];
    }
    if (lane == 0) tc::bulk_wait_read<0>();  // the previous store has read the buffer
    __syncwarp();
#pragma unroll
    for (int i = 0; i < 8; ++i) row[i ^ sw] = make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
    tc::fence_proxy_async();
    __syncwarp();
    if (lane == 0) {
      tc::tma_store_2d(tma_out, stage, colh + c * 32, row0);
      if (peers != nullptr) {
#pragma unroll
        for (int p = 0; p < kMaxPeers; ++p) {
          if (p >= g.npeers) break;
          tc::tma_store_2d(&peers->m[p], stage, colh + c * 32, row0);
        }
      }
      tc::bulk_commit();
    }
  }
}

template <int KIND, int BN, int BKB, int OUT>
__global__ void __launch_bounds__(GemmLayout<KIND, BN, BKB, OUT>::kThreads, 1)
gemm_kernel(const __grid_constant__ CUtensorMap tma_a, const __grid_constant__ CUtensorMap tma_b,
            const __grid_constant__ CUtensorMap tma_out, GemmArgs g, const __grid_constant__ PeerMaps peers) {
  using L = GemmLayout<KIND, BN, BKB, OUT>;
  constexpr int STAGES = L::kStages;
  constexpr int KS = L::kKSteps;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sOut = smem;  // first: the swizzled staging tiles need 1024-byte alignment
  uint8_t* sA = sOut + L::kStagingBytes;
  uint8_t* sB = sA + STAGES * L::kABytes;
  uint8_t* sSFA = sB + STAGES * L::kBBytes;
  uint8_t* sSFB = sSFA + STAGES * L::kSfaBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sSFB + STAGES * L::kSfbBytes);
  constexpr int SLOTS = L::kSfSlots;
  uint64_t* full = bars;
  uint64_t* empty = bars + STAGES;
  uint64_t* sf_full = bars + 2 * STAGES;   // a stage's scale factors are in TMEM slot (4 arrivals)
  uint64_t* sf_empty = sf_full + SLOTS;    // the MMAs that read the slot have completed
  uint64_t* acc_full = sf_empty + SLOTS;
  uint64_t* acc_empty = acc_full + L::kAccBufs;
  uint64_t* drain = acc_empty + L::kAccBufs;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      tc::mbar_init(&full[s], 1);
      tc::mbar_init(&empty[s], 1);
    }
    for (int s = 0; s < SLOTS; ++s) {
      tc::mbar_init(&sf_full[s], 4);
      tc::mbar_init(&sf_empty[s], 1);
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
        tile_coords(t, g.m_tiles, g.n_tiles, g.group_n, mt, nt);
        // the 128-row scale chunks B's rows [nt * BN, nt * BN + BN) span (those that exist)
        const int64_t c0 = static_cast<int64_t>(nt) * L::kGroups / 4;
        int64_t c1 = (static_cast<int64_t>(nt) * L::kGroups + L::kGroups - 1) / 4;
        if (c1 > g.sfb_chunks - 1) c1 = g.sfb_chunks - 1;
        const uint32_t tx = kTx - static_cast<uint32_t>(L::kSfbChunks - (c1 - c0 + 1)) * L::kSfChunkBytes;
        for (int kb = 0; kb < g.k_stages; ++kb) {
          if (!tc::mbar_wait(&empty[s], ph ^ 1u)) { ok = false; break; }
          tc::mbar_arrive_expect_tx(&full[s], L::kScaled ? tx : kTx);
          tc::tma_load_2d(&tma_a, &full[s], sA + s * L::kABytes, kb * BKB, mt * 128);
          tc::tma_load_2d(&tma_b, &full[s], sB + s * L::kBBytes, kb * BKB, nt * BN);
          if constexpr (L::kScaled) {  // one chunk per 128 rows per stage (KS chunks for NVFP4: contiguous)
            const int64_t kc = KIND == 3 ? static_cast<int64_t>(KS) * kb : (KIND == 4 ? static_cast<int64_t>(KS / 2) * kb : kb);
            tc::bulk_load(sSFA + s * L::kSfaBytes, g.sfa + (mt * g.sfa_ncb + kc) * 512, L::kSfChunkBytes, &full[s]);
            for (int64_t c = c0; c <= c1; ++c)
              tc::bulk_load(sSFB + s * L::kSfbBytes + (c - c0) * L::kSfChunkBytes, g.sfb + (c * g.sfb_ncb + kc) * 512,
                            L::kSfChunkBytes, &full[s]);
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
      int s = 0, ab = 0, slot = 0;
      uint32_t ph = 0, aph = 0, sph = 0;
      bool ok = true;
      for (int t = blockIdx.x; ok && t < total; t += gridDim.x) {
        if (!tc::mbar_wait(&acc_empty[ab], aph ^ 1u)) { ok = false; break; }
        tc::fence_after_sync();
        const uint32_t d = tmem + ab * BN;
        for (int kb = 0; kb < g.k_stages; ++kb) {
          if (!tc::mbar_wait(&full[s], ph)) { ok = false; break; }
          if constexpr (L::kScaled) {
            if (!tc::mbar_wait(&sf_full[slot], sph)) { ok = false; break; }
          }
          tc::fence_after_sync();
          const uint32_t abase = tc::smem_u32(sA + s * L::kABytes);
          const uint32_t bbase = tc::smem_u32(sB + s * L::kBBytes);
          const uint64_t adesc = BKB == 128 ? tc::desc_sw128(abase) : tc::desc_sw64(abase);
          const uint64_t bdesc = BKB == 128 ? tc::desc_sw128(bbase) : tc::desc_sw64(bbase);
          const uint32_t sf = tmem + L::kSfCol + slot * L::kSfColsPerStage;
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
            } else if constexpr (KIND == 3) {  // this MMA's scale set: 4 columns for A, one per 32 rows of B
              tc::mma_nvf4(d, a, b, tc::idesc_nvf4(128, BN), sf + 4 * j, sf + L::kSfaCols + L::kGroups * j, acc);
            } else {  // MXFP4: set j / 2 covers two MMAs, sf_id 0 / 2 picks the pair of scale bytes
              tc::mma_mxf4(d, a, b, tc::idesc_mxf4(128, BN, 2 * (j & 1)), sf + 4 * (j >> 1),
                           sf + L::kSfaCols + L::kGroups * (j >> 1), acc);
            }
          }
          tc::commit(&empty[s]);
          if (++s == STAGES) { s = 0; ph ^= 1u; }
          if constexpr (L::kScaled) {
            tc::commit(&sf_empty[slot]);
            if (++slot == SLOTS) { slot = 0; sph ^= 1u; }
          }
        }
        if (!ok) break;
        tc::commit(&acc_full[ab]);
        if (++ab == L::kAccBufs) { ab = 0; aph ^= 1u; }
      }
      tc::commit(drain);  // every MMA this thread issued has completed once this arrives
      if (!tc::mbar_wait(drain, 0)) ok = false;
      if (!ok) atomicOr(&g_gemm_status, kDevTimeout);
    }
  } else if (warp >= 2 + L::kEpiWarps) {  // ----------------------------------- scale-factor warps
    if constexpr (L::kScaled) {
      {
        constexpr int NB = L::kSfBatch;
        const uint32_t lane_base = static_cast<uint32_t>(32 * (warp & 3)) << 16;
        int s = 0, slot = 0, pending = 0;
        uint32_t ph = 0, sph = 0;
        bool ok = true;
        for (int t = blockIdx.x; ok && t < total; t += gridDim.x) {
          int mt, nt;
          tile_coords(t, g.m_tiles, g.n_tiles, g.group_n, mt, nt);
          const int64_t g0 = static_cast<int64_t>(nt) * L::kGroups;
          const bool last_tile = t + static_cast<int>(gridDim.x) >= total;
          // B's 32-row groups g0 .. g0 + kGroups - 1 start at word p = g0 % 4 (0, or 2 when
          // kGroups % 4 == 2) of chunk g0 / 4 and run over the following chunks; a chunk past the
          // end of B reads as zeros
          const int p = static_cast<int>(g0 & 3);
          bool live[L::kSfbChunks];
#pragma unroll
          for (int c = 0; c < L::kSfbChunks; ++c) live[c] = g0 / 4 + c < g.sfb_chunks;
          for (int kb = 0; kb < g.k_stages; ++kb) {
            if (!tc::mbar_wait(&full[s], ph)) { ok = false; break; }
            if (!tc::mbar_wait(&sf_empty[slot], sph ^ 1u)) { ok = false; break; }
            tc::fence_after_sync();
            const uint32_t col = tmem + lane_base + L::kSfCol + slot * L::kSfColsPerStage;
            const uint8_t* ca = sSFA + s * L::kSfaBytes + lane * 16;
            const uint8_t* cb = sSFB + s * L::kSfbBytes + lane * 16;
            // every load first (chunk row `lane` of A's chunk and of B's chunks, per scale set)
            uint4 av[L::kSfSets], bv[L::kSfSets][L::kSfbChunks];
#pragma unroll
            for (int j = 0; j < L::kSfSets; ++j) {
              av[j] = *reinterpret_cast<const uint4*>(ca + j * 512);
#pragma unroll
              for (int c = 0; c < L::kSfbChunks; ++c)
                bv[j][c] = live[c] ? *reinterpret_cast<const uint4*>(cb + c * L::kSfChunkBytes + j * 512)
                                   : make_uint4(0u, 0u, 0u, 0u);
            }
            // the stage's columns in order (A's sets, then B's sets) in a few wide stores
            uint32_t sw[L::kSfColsPerStage];
#pragma unroll
            for (int j = 0; j < L::kSfSets; ++j) {
              sw[4 * j] = av[j].x;  // A: the words of rows lane, lane + 32, + 64, + 96
              sw[4 * j + 1] = av[j].y;
              sw[4 * j + 2] = av[j].z;
              sw[4 * j + 3] = av[j].w;
            }
#pragma unroll
            for (int j = 0; j < L::kSfSets; ++j) {
              uint32_t w[4 * L::kSfbChunks];
#pragma unroll
              for (int c = 0; c < L::kSfbChunks; ++c) {
                w[4 * c] = bv[j][c].x;
                w[4 * c + 1] = bv[j][c].y;
                w[4 * c + 2] = bv[j][c].z;
                w[4 * c + 3] = bv[j][c].w;
              }
#pragma unroll
              for (int gi = 0; gi < L::kGroups; ++gi) {
                uint32_t v = w[gi];
                if constexpr (L::kGroups % 4 == 2) v = p == 0 ? w[gi] : w[gi + 2];
                sw[L::kSfaCols + L::kGroups * j + gi] = v;
              }
            }
            tc::tmem_st_n<L::kSfColsPerStage>(col, sw);
            if (++s == STAGES) { s = 0; ph ^= 1u; }
            if (++slot == SLOTS) { slot = 0; sph ^= 1u; }
            // one wait for the stores of NB stages (or of the last ones), then their signals
            if (++pending == NB || (last_tile && kb == g.k_stages - 1)) {
              tc::tmem_st_wait();
              tc::fence_before_sync();
              __syncwarp();
              if (lane == 0)
                for (int b = pending; b >= 1; --b) tc::mbar_arrive(&sf_full[(slot - b + SLOTS) % SLOTS]);
              pending = 0;
            }
          }
        }
        if (!ok && lane == 0) atomicOr(&g_gemm_status, kDevTimeout);
      }
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
      tile_coords(t, g.m_tiles, g.n_tiles, g.group_n, mt, nt);
      if (!tc::mbar_wait(&acc_full[ab], aph)) {
        if (lane == 0) atomicOr(&g_gemm_status, kDevTimeout);
        break;
      }
      tc::fence_after_sync();
      const int row0 = mt * 128 + 32 * quarter;
      const int colh = nt * BN + half * (BN / 2);
      const uint32_t tbase = tmem + lane_base + ab * BN + half * (BN / 2);
      uint64_t* release_bar = &acc_empty[ab];
      epilogue_tile<KIND, OUT, HC>(g, &tma_out, g.npeers > 0 ? &peers : nullptr, tbase, row0, colh, stage0, chunk,
                                   lane, [release_bar] { tc::mbar_arrive(release_bar); });
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
