// extern "C" entry points of the scaled GEMMs (gemm.cuh): argument checks, TMA tensor maps,
// the persistent launch, and this translation unit's device status word.
#include <cudaTypedefs.h>

#include <cstdlib>
#include <mutex>

#include "gemm.cuh"
#include "gemm_blockwise.cuh"
#include "gemm_pair.cuh"
#include "gemm_skinny.cuh"
#include "kab_host.h"

namespace kab {

unsigned gemm_device_status(bool clear, cudaStream_t stream) {
  unsigned v = 0;
  cudaMemcpyFromSymbolAsync(&v, g_gemm_status, sizeof v, 0, cudaMemcpyDeviceToHost, stream);
  cudaStreamSynchronize(stream);
  if (clear) {
    const unsigned zero = 0;
    cudaMemcpyToSymbolAsync(g_gemm_status, &zero, sizeof zero, 0, cudaMemcpyHostToDevice, stream);
    cudaStreamSynchronize(stream);
  }
  return v;
}

namespace {

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static std::once_flag once;
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// A 2-D byte matrix [rows, cols_bytes] (row stride ld_bytes) read in boxes of
// [box_rows, box_bytes] with the swizzle of that row width (128 or 64 bytes).
int make_map(CUtensorMap* map, const void* ptr, uint64_t rows, uint64_t cols_bytes, uint64_t ld_bytes,
             uint32_t box_rows, uint32_t box_bytes, const char* name) {
  auto fn = encode_fn();
  if (fn == nullptr) return fail(KAB_EUNSUPPORTED, "cuTensorMapEncodeTiled is unavailable (driver too old?)");
  cuuint64_t dims[2] = {cols_bytes, rows};
  cuuint64_t strides[1] = {ld_bytes};
  cuuint32_t box[2] = {box_bytes, box_rows};
  cuuint32_t estr[2] = {1, 1};
  const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE,
                        box_bytes == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(KAB_EINVAL, "tensor map of %s failed (CUresult %d)", name, static_cast<int>(r));
  return KAB_OK;
}

// The output [m, n] (row stride ldo elements) written by TMA stores from staging tiles swizzled
// at the width of their rows: [32 rows, 32 columns] boxes (the one-CTA kernel's stores; 64- or
// 128-byte rows), or with `wide` [32 rows, 128 bytes] boxes (the pair kernel's).
int make_out_map(CUtensorMap* map, void* ptr, int out, uint64_t m, uint64_t n, uint64_t ldo, bool wide = false) {
  auto fn = encode_fn();
  if (fn == nullptr) return fail(KAB_EUNSUPPORTED, "cuTensorMapEncodeTiled is unavailable (driver too old?)");
  const CUtensorMapDataType dt = out == KAB_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                 : out == KAB_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                 : out == KAB_F32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                                  : CU_TENSOR_MAP_DATA_TYPE_INT32;
  cuuint64_t dims[2] = {n, m};
  cuuint64_t strides[1] = {ldo * static_cast<uint64_t>(out_bytes(out))};
  cuuint32_t box[2] = {wide ? 128u / out_bytes(out) : 32u, 32};
  cuuint32_t estr[2] = {1, 1};
  const CUresult r = fn(map, dt, 2, ptr, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        (wide || out_bytes(out) == 4) ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B,
                        CU_TENSOR_MAP_L2_PROMOTION_NONE,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(KAB_EINVAL, "tensor map of the output failed (CUresult %d)", static_cast<int>(r));
  return KAB_OK;
}

template <int KIND, int BN, int BKB, int OUT>
int launch_one(const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& mo, const GemmArgs& g,
               const PeerMaps& pm, cudaStream_t s) {
  using L = GemmLayout<KIND, BN, BKB, OUT>;
  auto kernel = gemm_kernel<KIND, BN, BKB, OUT>;
  static bool configured[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !configured[dev]) {
    if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kSmem) != cudaSuccess)
      return fail(KAB_ECUDA, "cannot set %d bytes of shared memory", L::kSmem);
    configured[dev] = true;
  }
  const int tiles = g.m_tiles * g.n_tiles;
  const int grid = tiles < sm_count() ? tiles : sm_count();
  kernel<<<grid, L::kThreads, L::kSmem, s>>>(ma, mb, mo, g, pm);
  return check_launch("gemm kernel");
}

template <int KIND, int BN>
int launch_out(int out, const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& mo, const GemmArgs& g,
               const PeerMaps& pm, cudaStream_t s) {
  constexpr int BKB = 128;
  if constexpr (KIND == 0) {
    if (out == kOutI32) return launch_one<KIND, BN, BKB, kOutI32>(ma, mb, mo, g, pm, s);
  }
  if (out == KAB_BF16) return launch_one<KIND, BN, BKB, KAB_BF16>(ma, mb, mo, g, pm, s);
  if (out == KAB_F16) return launch_one<KIND, BN, BKB, KAB_F16>(ma, mb, mo, g, pm, s);
  return launch_one<KIND, BN, BKB, KAB_F32>(ma, mb, mo, g, pm, s);
}

// A swizzled block-scale tensor of `bytes` bytes as [bytes / 256, 256] read in boxes of
// `box_rows` rows (one stage's chunk of one 128-row block), no swizzle.
int make_sf_map(CUtensorMap* map, const void* ptr, uint64_t bytes, uint32_t box_rows, const char* name) {
  auto fn = encode_fn();
  if (fn == nullptr) return fail(KAB_EUNSUPPORTED, "cuTensorMapEncodeTiled is unavailable (driver too old?)");
  cuuint64_t dims[2] = {256, bytes / 256};
  cuuint64_t strides[1] = {256};
  cuuint32_t box[2] = {256, box_rows};
  cuuint32_t estr[2] = {1, 1};
  const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(KAB_EINVAL, "tensor map of %s failed (CUresult %d)", name, static_cast<int>(r));
  return KAB_OK;
}

// The CTA-pair kernel (gemm_pair.cuh): one cluster of 2 per SM pair, as many pairs as can be
// resident at once (persistent), at most one per tile.
template <int KIND, int OUT>
int launch_pair_one(const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& msa, const CUtensorMap& msb,
                    const CUtensorMap& mo, const GemmArgs& g, const PeerMaps& pm, cudaStream_t s) {
  using L = PairLayout<KIND, OUT>;
  auto kernel = gemm_pair_kernel<KIND, OUT>;
  static int pairs_of[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  int pairs = dev < 64 ? pairs_of[dev] : 0;
  if (pairs == 0) {
    if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kSmem) != cudaSuccess)
      return fail(KAB_ECUDA, "cannot set %d bytes of shared memory", L::kSmem);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * (sm_count() / 2));
    cfg.blockDim = dim3(L::kThreads);
    cfg.dynamicSmemBytes = L::kSmem;
    int clusters = 0;
    if (cudaOccupancyMaxActiveClusters(&clusters, kernel, &cfg) != cudaSuccess || clusters < 1) {
      cudaGetLastError();
      clusters = sm_count() / 2;
    }
    pairs = clusters;
    if (dev < 64) pairs_of[dev] = pairs;
  }
  const int tiles = g.m_tiles * g.n_tiles;
  const int grid = 2 * (tiles < pairs ? tiles : pairs);
  kernel<<<grid, L::kThreads, L::kSmem, s>>>(ma, mb, msa, msb, mo, g, pm);
  return check_launch("gemm pair kernel");
}

template <int KIND>
int launch_pair(int out, const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& msa, const CUtensorMap& msb,
                const CUtensorMap& mo, const GemmArgs& g, const PeerMaps& pm, cudaStream_t s) {
  if constexpr (KIND == 0) {
    if (out == kOutI32) return launch_pair_one<KIND, kOutI32>(ma, mb, msa, msb, mo, g, pm, s);
  }
  if (out == KAB_BF16) return launch_pair_one<KIND, KAB_BF16>(ma, mb, msa, msb, mo, g, pm, s);
  if (out == KAB_F16) return launch_pair_one<KIND, KAB_F16>(ma, mb, msa, msb, mo, g, pm, s);
  return launch_pair_one<KIND, KAB_F32>(ma, mb, msa, msb, mo, g, pm, s);
}

// The skinny kernel (gemm_skinny.cuh) for M <= 32: one CTA per 128-channel panel of W.
template <int KIND, int NT, int OUT, int STAGES>
int launch_skinny_one(const CUtensorMap& mw, const CUtensorMap& mx, const GemmArgs& g, cudaStream_t s) {
  using L = SkinnyLayout<NT, OUT, STAGES>;
  auto kernel = gemm_skinny_kernel<KIND, NT, OUT, STAGES>;
  static bool configured[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !configured[dev]) {
    if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kSmem) != cudaSuccess)
      return fail(KAB_ECUDA, "cannot set %d bytes of shared memory", L::kSmem);
    configured[dev] = true;
  }
  const unsigned grid = static_cast<unsigned>((g.n + 127) / 128);
  kernel<<<grid, L::kThreads, L::kSmem, s>>>(mw, mx, g);
  return check_launch("skinny gemm kernel");
}

template <int KIND, int NT, int OUT>
int launch_skinny_stages(const CUtensorMap& mw, const CUtensorMap& mx, const GemmArgs& g, cudaStream_t s) {
  if ((g.n + 127) / 128 <= sm_count()) return launch_skinny_one<KIND, NT, OUT, 10>(mw, mx, g, s);
  return launch_skinny_one<KIND, NT, OUT, 5>(mw, mx, g, s);
}

template <int KIND, int NT>
int launch_skinny_nt(int out, const CUtensorMap& mw, const CUtensorMap& mx, const GemmArgs& g, cudaStream_t s) {
  if constexpr (KIND == 0) {
    if (out == kOutI32) return launch_skinny_stages<KIND, NT, kOutI32>(mw, mx, g, s);
  }
  if (out == KAB_BF16) return launch_skinny_stages<KIND, NT, KAB_BF16>(mw, mx, g, s);
  if (out == KAB_F16) return launch_skinny_stages<KIND, NT, KAB_F16>(mw, mx, g, s);
  return launch_skinny_stages<KIND, NT, KAB_F32>(mw, mx, g, s);
}

// Tile kernel choice. The CTA-pair kernel (256 x 256 tiles on two SMs) moves half the bytes
// per FLOP through L2 and shared memory that the one-CTA kernel's 128 x 192 / 256 tiles do:
// on B200 at 8192^3 it ran NVFP4 at 4.53 vs 3.82 PFLOP/s, MXFP4 4.89 vs 4.09, MXFP8 2.50 vs
// 2.01, INT8 3.19 vs 2.85 POPS and FP8 2.87 vs 2.62, and the config-4 NVFP4 linear (8192 x
// 28672 x 8192) at 4.73 vs 3.85. With fewer than two pair tiles per SM pair the one-CTA
// kernel's smaller tiles fill the GPU better (2048 x 3072 x 1024: FP8 0.55 vs 0.49). So the
// pair kernel takes shapes with M > 128, N >= 256 (padding N to 256 costing at most 1/16)
// and at least two waves of pair tiles. KAB_GEMM_PAIR=0 / 1 (read once per process) forces
// the one-CTA kernel / the pair kernel wherever its shape conditions hold.
int pair_mode() {
  static const int mode = [] {
    const char* v = std::getenv("KAB_GEMM_PAIR");
    if (v == nullptr || v[0] == 0) return -1;
    return v[0] == '1' ? 1 : 0;
  }();
  return mode;
}

bool use_pair(int64_t m, int64_t n) {
  const int64_t pad256 = (n + 255) / 256 * 256 - n;
  if (m <= 128 || n < 256 || pad256 * 16 > n) return false;
  const int mode = pair_mode();
  if (mode >= 0) return mode == 1;
  const int64_t pair_tiles = ((m + 255) / 256) * ((n + 255) / 256);
  return pair_tiles >= 2 * (sm_count() / 2);
}

// Common checks and launch: a [m, k_bytes] and b [n, k_bytes] K-major byte matrices.
template <int KIND>
int run(const void* a, const void* b, int64_t m, int64_t n, int64_t k_bytes, GemmArgs g, int out_dtype,
        cudaStream_t s) {
  KAB_REQUIRE(m >= 0 && n >= 0 && k_bytes >= 0, "negative shape");
  if (m == 0 || n == 0) return KAB_OK;
  KAB_REQUIRE(a != nullptr && b != nullptr, "operand is null");
  KAB_REQUIRE(aligned(a, 16) && aligned(b, 16), "operands must be 16-byte aligned");
  const int bkb = 128;
  KAB_REQUIRE(k_bytes > 0 && k_bytes % bkb == 0,
              "K must be a positive multiple of %d bytes per row (128 int8 / e4m3, 256 e2m1); got %lld bytes",
              bkb, (long long)k_bytes);
  KAB_REQUIRE(out_dtype == KAB_BF16 || out_dtype == KAB_F16 || out_dtype == KAB_F32 || out_dtype == kOutI32,
              "unknown out dtype %d", out_dtype);
  void* out = out_dtype == kOutI32 ? static_cast<void*>(g.acc_out) : g.out;
  KAB_REQUIRE(out != nullptr, "output is null");
  KAB_REQUIRE(g.ldo >= n && g.ldo % 8 == 0, "ldo %lld must be >= n and a multiple of 8", (long long)g.ldo);
  KAB_REQUIRE(aligned(out, 16), "output must be 16-byte aligned");
  KAB_REQUIRE(m <= (int64_t(1) << 30) && n <= (int64_t(1) << 30), "shape too large");
  // decode sizes of the W8A8 kinds: the weight streams as the MMA's A operand, the tokens are
  // its N (16 or 32)
  if constexpr (KIND == 0 || KIND == 1) {
    if (m <= 32 && g.npeers == 0) {
      const int nt = m <= 16 ? 16 : 32;
      g.m = m;
      g.n = n;
      g.k_stages = static_cast<int>(k_bytes / bkb);
      CUtensorMap mw, mx;
      if (int e = make_map(&mw, b, n, k_bytes, k_bytes, 128, bkb, "W")) return e;
      if (int e = make_map(&mx, a, m, k_bytes, k_bytes, nt, bkb, "X")) return e;
      if (nt == 16) return launch_skinny_nt<KIND, 16>(out_dtype, mw, mx, g, s);
      return launch_skinny_nt<KIND, 32>(out_dtype, mw, mx, g, s);
    }
  }
  // 256 x 256 tiles on SM pairs (use_pair: large shapes)
  if (use_pair(m, n)) {
    g.m = m;
    g.n = n;
    g.k_stages = static_cast<int>(k_bytes / bkb);
    g.m_tiles = static_cast<int>((m + 255) / 256);
    g.n_tiles = static_cast<int>((n + 255) / 256);
    g.group_n = n > m && g.m_tiles > 4 ? 16 : 0;
    g.sfb_chunks = (n + 127) / 128;
    CUtensorMap ma, mb, msa, msb, mo;
    if (int e = make_map(&ma, a, m, k_bytes, k_bytes, 128, bkb, "A")) return e;
    if (int e = make_map(&mb, b, n, k_bytes, k_bytes, 128, bkb, "B")) return e;
    if (int e = make_out_map(&mo, out, out_dtype, m, n, g.ldo, true)) return e;
    msa = ma;
    msb = mb;
    if constexpr (GemmTraits<KIND>::kScaled) {
      constexpr uint32_t rows = PairLayout<KIND, KAB_BF16>::kSfRows;
      const uint64_t a_blocks = static_cast<uint64_t>((m + 127) / 128);
      if (int e = make_sf_map(&msa, g.sfa, a_blocks * g.sfa_ncb * 512, rows, "A's block scales")) return e;
      if (int e = make_sf_map(&msb, g.sfb, static_cast<uint64_t>(g.sfb_chunks) * g.sfb_ncb * 512, rows,
                              "B's block scales"))
        return e;
    }
    PeerMaps pm{};
    for (int p = 0; p < g.npeers; ++p)
      if (int e = make_out_map(&pm.m[p], g.peer_out[p], out_dtype, m, n, g.ldo, true)) return e;
    return launch_pair<KIND>(out_dtype, ma, mb, msa, msb, mo, g, pm, s);
  }
  // one-CTA tiles, width 256 (two 256-column accumulators) for int8 / fp8; the block-scaled
  // kinds keep room for their scale-factor ring next to two accumulators: 192 unless that pads
  // N by more than 1/16, else 128
  int bn;
  if (!GemmTraits<KIND>::kScaled) {
    bn = n >= 256 ? 256 : 128;
    // a small problem (config 1: 128 x 1024 x 1024 is 4 tiles of 128 x 256) is bound by each
    // CTA's serial operand stream: twice the tiles at half the width halve that stream
    if (bn == 256 && ((m + 127) / 128) * ((n + 255) / 256) * 2 <= sm_count()) bn = 128;
  } else {
    const int64_t pad192 = (n + 191) / 192 * 192 - n;
    bn = (n >= 192 && pad192 * 16 <= n) ? 192 : 128;
  }
  g.m = m;
  g.n = n;
  g.k_stages = static_cast<int>(k_bytes / bkb);
  g.m_tiles = static_cast<int>((m + 127) / 128);
  g.n_tiles = static_cast<int>((n + bn - 1) / bn);
  // B larger than A (a weight panel sweep): keep A in L2 and stream each B panel once
  g.group_n = n > m && g.m_tiles > 8 ? 16 : 0;
  CUtensorMap ma, mb, mo;
  if (int e = make_map(&ma, a, m, k_bytes, k_bytes, 128, bkb, "A")) return e;
  if (int e = make_map(&mb, b, n, k_bytes, k_bytes, bn, bkb, "B")) return e;
  if (int e = make_out_map(&mo, out, out_dtype, m, n, g.ldo)) return e;
  PeerMaps pm{};
  for (int p = 0; p < g.npeers; ++p)
    if (int e = make_out_map(&pm.m[p], g.peer_out[p], out_dtype, m, n, g.ldo)) return e;
  if constexpr (GemmTraits<KIND>::kScaled) {
    g.sfb_chunks = (n + 127) / 128;
    if (bn == 192) return launch_out<KIND, 192>(out_dtype, ma, mb, mo, g, pm, s);
  } else {
    if (bn == 256) return launch_out<KIND, 256>(out_dtype, ma, mb, mo, g, pm, s);
  }
  return launch_out<KIND, 128>(out_dtype, ma, mb, mo, g, pm, s);
}

// Whether the decode-size blockwise GEMM's CTAs, as many as fit an SM by shared memory and
// threads, can all hold their TMEM at once (a CTA that waited for TMEM held by a cluster peer
// on the same SM would wait forever).
bool blockwise_skinny_fits(int64_t m, int per) {
  const bool small = m <= 16;
  const int smem = small ? BlockwiseSkinnyLayout<16>::smem(per) : BlockwiseSkinnyLayout<32>::smem(per);
  const uint32_t cols = small ? BlockwiseSkinnyLayout<16>::tmem_cols(per) : BlockwiseSkinnyLayout<32>::tmem_cols(per);
  const int by_smem = (228 * 1024) / (smem + 1024);
  const int by_threads = 2048 / BlockwiseSkinnyLayout<16>::kThreads;
  const int resident = by_smem < by_threads ? by_smem : by_threads;
  return resident >= 1 && static_cast<uint32_t>(resident) * cols <= 512u;
}

// The decode-size blockwise GEMM (M <= 32): one cluster of `csize` CTAs per 128-channel panel.
template <int NT, int OUT>
int launch_blockwise_skinny(const CUtensorMap& mw, const CUtensorMap& mx, const BlockwiseSkinnyArgs& g, int csize,
                            cudaStream_t s) {
  using L = BlockwiseSkinnyLayout<NT>;
  auto kernel = gemm_blockwise_skinny_kernel<NT, OUT>;
  static bool configured[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  const int max_smem = L::smem(L::kMaxPer);
  if (dev < 64 && !configured[dev]) {
    if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem) != cudaSuccess)
      return fail(KAB_ECUDA, "cannot set %d bytes of shared memory", max_smem);
    configured[dev] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(g.n / 128 * csize));
  cfg.blockDim = dim3(L::kThreads);
  cfg.dynamicSmemBytes = static_cast<size_t>(L::smem(g.per));
  cfg.stream = s;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = static_cast<unsigned>(csize);
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, kernel, mw, mx, g) != cudaSuccess) return check_launch("blockwise gemm (decode size)");
  return check_launch("blockwise gemm (decode size)");
}

template <int OUT>
int launch_blockwise(const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& mo, const BlockwiseArgs& g,
                     cudaStream_t s) {
  using L = BlockwiseLayout<OUT>;
  auto kernel = gemm_blockwise_kernel<OUT>;
  static bool configured[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !configured[dev]) {
    if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kSmem) != cudaSuccess)
      return fail(KAB_ECUDA, "cannot set %d bytes of shared memory", L::kSmem);
    configured[dev] = true;
  }
  const int tiles = g.m_tiles * g.n_tiles;
  const int grid = tiles < sm_count() ? tiles : sm_count();
  kernel<<<grid, L::kThreads, L::kSmem, s>>>(ma, mb, mo, g);
  return check_launch("blockwise gemm kernel");
}

GemmArgs args_of(const void* bias, int bias_dtype, void* out, int out_dtype, int64_t ldo) {
  GemmArgs g{};
  g.bias = bias;
  g.bias_dtype = bias_dtype;
  g.out = out;
  g.out_dtype = out_dtype;
  g.ldo = ldo;
  return g;
}

}  // namespace
}  // namespace kab

using namespace kab;

extern "C" {

int kab_gemm_i8(const int8_t* a, const int8_t* b, int64_t m, int64_t n, int64_t k, const float* a_scale,
                const float* b_scale, const void* bias, int bias_dtype, void* out, int out_dtype, int64_t ldo,
                int32_t* acc_out, void* stream) {
  GemmArgs g = args_of(bias, bias_dtype, out, out_dtype, ldo);
  g.acc_out = acc_out;
  g.a_scale = a_scale;
  g.b_scale = b_scale;
  if (acc_out == nullptr)
    KAB_REQUIRE(a_scale != nullptr && b_scale != nullptr, "scales are null");
  else
    g.out = nullptr;
  KAB_REQUIRE(bias == nullptr || valid_dtype(bias_dtype), "unknown bias dtype %d", bias_dtype);
  return run<0>(a, b, m, n, k, g, acc_out != nullptr ? kOutI32 : out_dtype, as_stream(stream));
}

int kab_gemm_f8(const uint8_t* a, const uint8_t* b, int64_t m, int64_t n, int64_t k, const float* a_scale,
                const float* b_scale, const void* bias, int bias_dtype, void* out, int out_dtype, int64_t ldo,
                void* stream) {
  GemmArgs g = args_of(bias, bias_dtype, out, out_dtype, ldo);
  g.a_scale = a_scale;
  g.b_scale = b_scale;
  KAB_REQUIRE(a_scale != nullptr && b_scale != nullptr, "scales are null");
  KAB_REQUIRE(bias == nullptr || valid_dtype(bias_dtype), "unknown bias dtype %d", bias_dtype);
  return run<1>(a, b, m, n, k, g, out_dtype, as_stream(stream));
}

int kab_gemm_mxf8(const uint8_t* a, const uint8_t* a_sf, const uint8_t* b, const uint8_t* b_sf, int64_t m,
                  int64_t n, int64_t k, const void* bias, int bias_dtype, void* out, int out_dtype, int64_t ldo,
                  void* stream) {
  GemmArgs g = args_of(bias, bias_dtype, out, out_dtype, ldo);
  KAB_REQUIRE(a_sf != nullptr && b_sf != nullptr && aligned(a_sf, 16) && aligned(b_sf, 16),
              "block scales are null or not 16-byte aligned");
  KAB_REQUIRE(bias == nullptr || valid_dtype(bias_dtype), "unknown bias dtype %d", bias_dtype);
  g.sfa = a_sf;
  g.sfb = b_sf;
  g.sfa_ncb = g.sfb_ncb = (k / 32 + 3) / 4;
  return run<2>(a, b, m, n, k, g, out_dtype, as_stream(stream));
}

int kab_gemm_nvf4(const uint8_t* a, const uint8_t* a_sf, const float* a_outer, const uint8_t* b,
                  const uint8_t* b_sf, const float* b_scale, int b_scale_per_col, int64_t m, int64_t n, int64_t k,
                  const void* bias, int bias_dtype, void* out, int out_dtype, int64_t ldo, void* stream) {
  GemmArgs g = args_of(bias, bias_dtype, out, out_dtype, ldo);
  KAB_REQUIRE(a_sf != nullptr && b_sf != nullptr && aligned(a_sf, 16) && aligned(b_sf, 16),
              "block scales are null or not 16-byte aligned");
  KAB_REQUIRE(a_outer != nullptr && b_scale != nullptr, "outer / tensor scales are null");
  KAB_REQUIRE(k % 2 == 0, "K must be even");
  KAB_REQUIRE(bias == nullptr || valid_dtype(bias_dtype), "unknown bias dtype %d", bias_dtype);
  g.sfa = a_sf;
  g.sfb = b_sf;
  g.sfa_ncb = g.sfb_ncb = (k / 16 + 3) / 4;
  g.a_scale = a_outer;
  g.b_scale = b_scale;
  g.b_scale_per_col = b_scale_per_col;
  return run<3>(a, b, m, n, k / 2, g, out_dtype, as_stream(stream));
}

int kab_gemm_nvf4_scatter(const uint8_t* a, const uint8_t* a_sf, const float* a_outer, const uint8_t* b,
                          const uint8_t* b_sf, const float* b_scale, int b_scale_per_col, int64_t m, int64_t n,
                          int64_t k, const void* bias, int bias_dtype, void* out, int out_dtype, int64_t ldo,
                          void* const* peer_out, int npeers, void* stream) {
  KAB_REQUIRE(npeers >= 0 && npeers <= kMaxPeers, "npeers %d not in 0..%d", npeers, kMaxPeers);
  KAB_REQUIRE(npeers == 0 || peer_out != nullptr, "peer_out is null");
  GemmArgs g = args_of(bias, bias_dtype, out, out_dtype, ldo);
  for (int p = 0; p < npeers; ++p) {
    KAB_REQUIRE(peer_out[p] != nullptr && aligned(peer_out[p], 16), "peer output %d is null or not 16-byte aligned", p);
    g.peer_out[p] = peer_out[p];
  }
  g.npeers = npeers;
  KAB_REQUIRE(a_sf != nullptr && b_sf != nullptr && aligned(a_sf, 16) && aligned(b_sf, 16),
              "block scales are null or not 16-byte aligned");
  KAB_REQUIRE(a_outer != nullptr && b_scale != nullptr, "outer / tensor scales are null");
  KAB_REQUIRE(k % 2 == 0, "K must be even");
  KAB_REQUIRE(bias == nullptr || valid_dtype(bias_dtype), "unknown bias dtype %d", bias_dtype);
  g.sfa = a_sf;
  g.sfb = b_sf;
  g.sfa_ncb = g.sfb_ncb = (k / 16 + 3) / 4;
  g.a_scale = a_outer;
  g.b_scale = b_scale;
  g.b_scale_per_col = b_scale_per_col;
  return run<3>(a, b, m, n, k / 2, g, out_dtype, as_stream(stream));
}

int kab_gemm_mxf4(const uint8_t* a, const uint8_t* a_sf, const float* a_outer, const uint8_t* b,
                  const uint8_t* b_sf, const float* b_scale, int b_scale_per_col, int64_t m, int64_t n, int64_t k,
                  const void* bias, int bias_dtype, void* out, int out_dtype, int64_t ldo, void* stream) {
  GemmArgs g = args_of(bias, bias_dtype, out, out_dtype, ldo);
  g.a_scale = a_outer;
  g.b_scale = b_scale;
  g.b_scale_per_col = b_scale != nullptr && b_scale_per_col;
  KAB_REQUIRE(a_sf != nullptr && b_sf != nullptr && aligned(a_sf, 16) && aligned(b_sf, 16),
              "block scales are null or not 16-byte aligned");
  KAB_REQUIRE(k % 2 == 0, "K must be even");
  KAB_REQUIRE(bias == nullptr || valid_dtype(bias_dtype), "unknown bias dtype %d", bias_dtype);
  g.sfa = a_sf;
  g.sfb = b_sf;
  g.sfa_ncb = g.sfb_ncb = (k / 32 + 3) / 4;
  return run<4>(a, b, m, n, k / 2, g, out_dtype, as_stream(stream));
}

int kab_gemm_f8_blockwise(const uint8_t* a, const float* a_scale, const uint8_t* b, const float* b_scale,
                          int64_t m, int64_t n, int64_t k, const void* bias, int bias_dtype, void* out,
                          int out_dtype, int64_t ldo, void* stream) {
  KAB_REQUIRE(m >= 0 && n >= 0 && k >= 0, "negative shape");
  if (m == 0 || n == 0) return KAB_OK;
  KAB_REQUIRE(a != nullptr && b != nullptr && a_scale != nullptr && b_scale != nullptr,
              "operand or scale is null");
  KAB_REQUIRE(aligned(a, 16) && aligned(b, 16), "operands must be 16-byte aligned");
  KAB_REQUIRE(k > 0 && k % 128 == 0, "K (%lld) must be a positive multiple of 128 (the scale group)", (long long)k);
  KAB_REQUIRE(n % 128 == 0, "N (%lld) must be a multiple of 128 (the weight block)", (long long)n);
  KAB_REQUIRE(out_dtype == KAB_BF16 || out_dtype == KAB_F16 || out_dtype == KAB_F32, "unknown out dtype %d",
              out_dtype);
  KAB_REQUIRE(bias == nullptr || valid_dtype(bias_dtype), "unknown bias dtype %d", bias_dtype);
  KAB_REQUIRE(out != nullptr && aligned(out, 16), "output is null or not 16-byte aligned");
  KAB_REQUIRE(ldo >= n && ldo % 8 == 0, "ldo %lld must be >= n and a multiple of 8", (long long)ldo);
  KAB_REQUIRE(m <= (int64_t(1) << 30) && n <= (int64_t(1) << 30), "shape too large");
  const int k_blocks = static_cast<int>(k / 128);
  const cudaStream_t s = as_stream(stream);
  // decode sizes: the K steps of each 128-channel panel split over a cluster of up to 8 CTAs,
  // as many as keep the grid within one CTA per SM (the weight stream needs no more)
  const int64_t panels = n / 128;
  int want = static_cast<int>(sm_count() / (panels > 0 ? panels : 1));
  want = want < 1 ? 1 : (want > 8 ? 8 : want);
  const int per = (k_blocks + want - 1) / want;
  if (m <= 32 && per <= BlockwiseSkinnyLayout<16>::kMaxPer && blockwise_skinny_fits(m, per)) {
    BlockwiseSkinnyArgs q{};
    q.m = m;
    q.n = n;
    q.ldo = ldo;
    q.k_blocks = k_blocks;
    q.per = per;
    const int csize = (k_blocks + per - 1) / per;
    q.sa = a_scale;
    q.sb = b_scale;
    q.bias = bias;
    q.bias_dtype = bias_dtype;
    q.out = out;
    const uint32_t nt = m <= 16 ? 16 : 32;
    CUtensorMap mw, mx;
    if (int e = make_map(&mw, b, n, k, k, 128, 128, "B")) return e;
    if (int e = make_map(&mx, a, m, k, k, nt, 128, "A")) return e;
#define KAB_SKINNY(NT)                                                                    \
  if (out_dtype == KAB_BF16) return launch_blockwise_skinny<NT, KAB_BF16>(mw, mx, q, csize, s); \
  if (out_dtype == KAB_F16) return launch_blockwise_skinny<NT, KAB_F16>(mw, mx, q, csize, s);   \
  return launch_blockwise_skinny<NT, KAB_F32>(mw, mx, q, csize, s)
    if (nt == 16) { KAB_SKINNY(16); }
    KAB_SKINNY(32);
#undef KAB_SKINNY
  }
  BlockwiseArgs g{};
  g.m = m;
  g.n = n;
  g.k_blocks = k_blocks;
  g.m_tiles = static_cast<int>((m + 127) / 128);
  g.n_tiles = static_cast<int>(n / 128);
  g.sa = a_scale;
  g.sb = b_scale;
  g.bias = bias;
  g.bias_dtype = bias_dtype;
  CUtensorMap ma, mb, mo;
  if (int e = make_map(&ma, a, m, k, k, 128, 128, "A")) return e;
  if (int e = make_map(&mb, b, n, k, k, 128, 128, "B")) return e;
  if (int e = make_out_map(&mo, out, out_dtype, m, n, ldo)) return e;
  if (out_dtype == KAB_BF16) return launch_blockwise<KAB_BF16>(ma, mb, mo, g, s);
  if (out_dtype == KAB_F16) return launch_blockwise<KAB_F16>(ma, mb, mo, g, s);
  return launch_blockwise<KAB_F32>(ma, mb, mo, g, s);
}

}  // extern "C"
