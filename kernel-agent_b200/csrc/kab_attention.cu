// extern "C" entry points of the FP8 attention prefill (attention.cuh): the per-head
// quantiser, the attention kernel's TMA maps and launch, and this translation unit's
// device status word.
#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>

#include "kab_host.h"

namespace kab {
__device__ unsigned g_attention_status = 0;
}  // namespace kab

#include "attention.cuh"
#include "attention_decode.cuh"

namespace kab {

unsigned attention_device_status(bool clear, cudaStream_t stream) {
  unsigned v = 0;
  cudaMemcpyFromSymbolAsync(&v, g_attention_status, sizeof v, 0, cudaMemcpyDeviceToHost, stream);
  cudaStreamSynchronize(stream);
  if (clear) {
    const unsigned zero = 0;
    cudaMemcpyToSymbolAsync(g_attention_status, &zero, sizeof zero, 0, cudaMemcpyHostToDevice, stream);
  }
  return v;
}

namespace {

PFN_cuTensorMapEncodeTiled_v12000 attn_encode_fn() {
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

// A [rows, cols] byte matrix read in boxes of box_rows x box_cols bytes (box_cols 128 or 64),
// swizzled at the box's row length like the MMA operands.
int byte_map(CUtensorMap* map, const void* ptr, uint64_t rows, uint64_t cols, const char* name,
             uint32_t box_cols = 128, uint32_t box_rows = 128) {
  auto fn = attn_encode_fn();
  if (fn == nullptr) return fail(KAB_EUNSUPPORTED, "cuTensorMapEncodeTiled is unavailable (driver too old?)");
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {cols};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE,
                        box_cols == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(KAB_EINVAL, "tensor map of %s failed (CUresult %d)", name, static_cast<int>(r));
  return KAB_OK;
}

// A [B, H, L, D] e4m3 cache (element strides sb, sh, sl; unit last stride) read in boxes of
// 128 tokens x D bytes of one (sequence, head), swizzled like the MMA operands (D = 128: the
// 128-byte swizzle, D = 64: the 64-byte one); tokens at or past L read as zeros.
int cache_map(CUtensorMap* map, const void* ptr, int64_t b, int64_t hh, int64_t l, int64_t d, int64_t sb, int64_t sh,
              int64_t sl, const char* name) {
  auto fn = attn_encode_fn();
  if (fn == nullptr) return fail(KAB_EUNSUPPORTED, "cuTensorMapEncodeTiled is unavailable (driver too old?)");
  cuuint64_t dims[4] = {static_cast<cuuint64_t>(d), static_cast<cuuint64_t>(l), static_cast<cuuint64_t>(hh),
                        static_cast<cuuint64_t>(b)};
  cuuint64_t strides[3] = {static_cast<cuuint64_t>(sl), static_cast<cuuint64_t>(sh), static_cast<cuuint64_t>(sb)};
  cuuint32_t box[4] = {static_cast<cuuint32_t>(d), 128, 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, const_cast<void*>(ptr), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, d == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(KAB_EINVAL, "tensor map of %s failed (CUresult %d)", name, static_cast<int>(r));
  return KAB_OK;
}

template <int D, int GP>
auto decode_kernel_for(int qt) {
  return qt == KAB_BF16 ? kv_decode_kernel<D, GP, kBF16>
         : qt == KAB_F16 ? kv_decode_kernel<D, GP, kF16>
                         : kv_decode_kernel<D, GP, kF32>;
}

// Opts the kernel instance into its shared memory (once per device) and returns the CTAs of
// it that fit on one SM.
template <int D, int GP>
int decode_prepare(int qt) {
  using L = DecodeLayout<D, GP>;
  static int resident[3][64] = {};
  const int ti = qt == KAB_BF16 ? 0 : qt == KAB_F16 ? 1 : 2;
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 64) return 1;
  if (resident[ti][dev] == 0) {
    auto kern = decode_kernel_for<D, GP>(qt);
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kSmem) != cudaSuccess) return -1;
    int n = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kern, L::kThreads, L::kSmem) != cudaSuccess) return -1;
    resident[ti][dev] = n > 0 ? n : 1;
  }
  return resident[ti][dev];
}

// How many clusters of `cs` CTAs of the kernel instance can be resident at once (0 when the
// cluster cannot be formed); cached per device and size.
template <int D, int GP>
int decode_clusters(int qt, int cs) {
  using L = DecodeLayout<D, GP>;
  static int fits[3][64][17] = {};  // value + 1; 0: not asked yet
  const int ti = qt == KAB_BF16 ? 0 : qt == KAB_F16 ? 1 : 2;
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 64 || cs < 2 || cs > 16) return 0;
  if (fits[ti][dev][cs] == 0) {
    auto kern = decode_kernel_for<D, GP>(qt);
    int n = 0;
    if (cs <= 8 || cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) == cudaSuccess) {
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(static_cast<unsigned>(cs));
      cfg.blockDim = dim3(L::kThreads);
      cfg.dynamicSmemBytes = L::kSmem;
      cudaLaunchAttribute at[1];
      at[0].id = cudaLaunchAttributeClusterDimension;
      at[0].val.clusterDim.x = static_cast<unsigned>(cs);
      at[0].val.clusterDim.y = 1;
      at[0].val.clusterDim.z = 1;
      cfg.attrs = at;
      cfg.numAttrs = 1;
      if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess) n = 0;
    }
    cudaGetLastError();  // a size the device refuses is not an error of the caller
    fits[ti][dev][cs] = n + 1;
  }
  return fits[ti][dev][cs] - 1;
}

int decode_cluster_fit(int64_t d, int gp, int qt, int cs) {
  if (d == 128)
    return gp == 8 ? decode_clusters<128, 8>(qt, cs) : gp == 16 ? decode_clusters<128, 16>(qt, cs)
                                                      : decode_clusters<128, 32>(qt, cs);
  return gp == 8 ? decode_clusters<64, 8>(qt, cs) : gp == 16 ? decode_clusters<64, 16>(qt, cs)
                                                  : decode_clusters<64, 32>(qt, cs);
}

int decode_resident(int64_t d, int gp, int qt) {
  if (d == 128)
    return gp == 8 ? decode_prepare<128, 8>(qt) : gp == 16 ? decode_prepare<128, 16>(qt) : decode_prepare<128, 32>(qt);
  return gp == 8 ? decode_prepare<64, 8>(qt) : gp == 16 ? decode_prepare<64, 16>(qt) : decode_prepare<64, 32>(qt);
}

// Splits per (sequence, KV head) and tokens per split (a multiple of 128): the asked splits,
// or with 0 one wave of the CTAs that fit on the GPU (triton_fp8_kv_decode.py:232-235 asks
// for ~4 programs per SM).
void decode_split(const KabKvDecodeParams* p, int resident, int* splits, int* chunk) {
  const int64_t tiles = (p->length + 127) / 128;
  int64_t s = p->splits;
  if (s <= 0) {
    const int64_t pairs = p->batch * p->heads_kv;
    s = static_cast<int64_t>(resident) * sm_count() / pairs;  // at most one wave
  }
  s = std::max<int64_t>(1, std::min<int64_t>(std::min<int64_t>(s, tiles), 256));  // the merge's weights fit in the ring
  const int64_t per = (p->length + s - 1) / s;
  const int64_t c = (per + 127) / 128 * 128;
  *chunk = static_cast<int>(c);
  *splits = static_cast<int>((p->length + c - 1) / c);
}

// The launch's splits, tokens per split and merge: the splits of a (sequence, KV head) form
// one thread-block cluster and merge through distributed shared memory when a cluster of
// that many CTAs fits and one wave of them runs at once; otherwise the partials go through
// the global workspace and the last CTA merges them. (Fewer splits to make a cluster fit was
// slower: at batch 4, 16 / 2 heads, 4096 tokens, 8 splits in clusters took 11.2 us per step
// against 10.3 us for 16 splits merged through the workspace.)
struct DecodePlan {
  int splits = 1, chunk = 128, cluster = 0;
};
int decode_plan(const KabKvDecodeParams* p, int gp, DecodePlan* plan) {
  const int qt = valid_dtype(p->q_dtype) ? p->q_dtype : KAB_BF16;
  const int resident = decode_resident(p->head_dim, gp, qt);
  if (resident < 0) return fail(KAB_ECUDA, "cannot configure the decode kernel");
  decode_split(p, resident, &plan->splits, &plan->chunk);
  const int64_t pairs = p->batch * p->heads_kv;
  plan->cluster = 0;
  if (plan->splits > 1 && plan->splits <= 16 && decode_cluster_fit(p->head_dim, gp, qt, plan->splits) >= pairs)
    plan->cluster = 1;
  return KAB_OK;
}

size_t decode_workspace_bytes(const KabKvDecodeParams* p, int splits, int gp) {
  if (splits <= 1) return 0;
  const size_t pairs = static_cast<size_t>(p->batch * p->heads_kv);
  const size_t counters = (pairs * 4 + 255) / 256 * 256;
  const size_t ml = (pairs * splits * 2 * gp * 4 + 255) / 256 * 256;
  return counters + ml + pairs * splits * gp * static_cast<size_t>(p->head_dim) * 4;
}

int decode_check(const KabKvDecodeParams* p, int* gp) {
  KAB_REQUIRE(p != nullptr, "null parameters");
  KAB_REQUIRE(p->batch >= 0 && p->heads_q >= 0 && p->heads_kv > 0 && p->length >= 0 && p->q_len >= 1,
              "bad shape");
  KAB_REQUIRE(p->head_dim == 64 || p->head_dim == 128, "head_dim %lld: the kernel takes 64 or 128",
              (long long)p->head_dim);
  KAB_REQUIRE(p->heads_q % p->heads_kv == 0, "heads_q %lld is not a multiple of heads_kv %lld",
              (long long)p->heads_q, (long long)p->heads_kv);
  const int64_t rows = p->heads_q / p->heads_kv * p->q_len;
  KAB_REQUIRE(rows <= 32, "%lld query rows per KV head (query heads per KV head x query tokens): at most 32",
              (long long)rows);
  *gp = rows <= 8 ? 8 : rows <= 16 ? 16 : 32;
  return KAB_OK;
}

template <int D, int GP>
int launch_decode_t(const CUtensorMap& mk, const CUtensorMap& mv, const DecodeArgs& g, int qt, int64_t pairs,
                    cudaStream_t s) {
  using L = DecodeLayout<D, GP>;
  auto kern = decode_kernel_for<D, GP>(qt);
  const dim3 grid(static_cast<unsigned>(g.splits), static_cast<unsigned>(pairs));
  if (!g.cluster) {
    kern<<<grid, L::kThreads, L::kSmem, s>>>(mk, mv, g);
    return check_launch("kab_kv_decode_fp8");
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(L::kThreads);
  cfg.dynamicSmemBytes = L::kSmem;
  cfg.stream = s;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = static_cast<unsigned>(g.splits);
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, kern, mk, mv, g) != cudaSuccess) return check_launch("kab_kv_decode_fp8 (cluster)");
  return check_launch("kab_kv_decode_fp8 (cluster)");
}

template <int D>
int launch_attention(const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv, const AttnArgs& g,
                     int64_t ctas, void* stream) {
  using L = AttnLayout<D>;
  static bool configured[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !configured[dev]) {
    if (cudaFuncSetAttribute(attention_fp8_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kSmem) !=
        cudaSuccess)
      return fail(KAB_ECUDA, "cannot set %d bytes of shared memory", L::kSmem);
    configured[dev] = true;
  }
  attention_fp8_kernel<D><<<static_cast<unsigned>(ctas), L::kThreads, L::kSmem, as_stream(stream)>>>(mq, mk, mv, g);
  return check_launch("kab_attention_fp8");
}

}  // namespace
}  // namespace kab

using namespace kab;

extern "C" {

int kab_quant_heads_fp8(const void* x, int dtype, int64_t heads, int64_t seq, int64_t d, int transpose,
                        unsigned* amax, uint8_t* q, float* scales, void* stream) {
  KAB_REQUIRE(valid_dtype(dtype), "unknown dtype %d", dtype);
  KAB_REQUIRE(heads >= 0 && seq >= 0 && d >= 0, "negative shape");
  if (heads == 0 || seq == 0 || d == 0) return KAB_OK;
  KAB_REQUIRE(x != nullptr && amax != nullptr && q != nullptr && scales != nullptr, "null pointer");
  KAB_REQUIRE(aligned(x, 16) && aligned(q, 16), "x and q must be 16-byte aligned");
  KAB_REQUIRE(d % 8 == 0 && d <= 256, "head_dim %lld must be a multiple of 8, at most 256", (long long)d);
  KAB_REQUIRE(heads < 65536, "too many heads (%lld)", (long long)heads);
  const cudaStream_t s = as_stream(stream);
  if (cudaMemsetAsync(amax, 0, heads * sizeof(unsigned), s) != cudaSuccess) return check_launch("amax reset");
  const int64_t per = seq * d;
  int64_t bx = (per / 8 + 255) / 256;
  if (bx > 64) bx = 64;
  const dim3 ga(static_cast<unsigned>(bx), static_cast<unsigned>(heads));
  if (dtype == KAB_BF16) head_amax_kernel<kBF16><<<ga, 256, 0, s>>>(x, per, amax);
  else if (dtype == KAB_F16) head_amax_kernel<kF16><<<ga, 256, 0, s>>>(x, per, amax);
  else head_amax_kernel<kF32><<<ga, 256, 0, s>>>(x, per, amax);
  if (int e = check_launch("kab_quant_heads_fp8 amax")) return e;
  const dim3 gq(static_cast<unsigned>((seq + 63) / 64), static_cast<unsigned>(heads));
  const size_t sm = transpose ? static_cast<size_t>(64 * d) : 0;
#define KAB_HEADS(TT)                                                                                 \
  if (transpose) quant_heads_kernel<TT, true><<<gq, 256, sm, s>>>(x, seq, static_cast<int>(d), amax, q, scales); \
  else quant_heads_kernel<TT, false><<<gq, 256, 0, s>>>(x, seq, static_cast<int>(d), amax, q, scales)
  if (dtype == KAB_BF16) { KAB_HEADS(kBF16); }
  else if (dtype == KAB_F16) { KAB_HEADS(kF16); }
  else { KAB_HEADS(kF32); }
#undef KAB_HEADS
  return check_launch("kab_quant_heads_fp8");
}

int kab_attention_fp8(const uint8_t* q, const float* q_scale, const uint8_t* k, const float* k_scale,
                      const uint8_t* vt, const float* v_scale, int64_t batch, int64_t heads_q, int64_t heads_kv,
                      int64_t seq, int64_t head_dim, int causal, float sm_scale, void* out, void* stream) {
  KAB_REQUIRE(batch >= 0 && heads_q >= 0 && heads_kv >= 0 && seq >= 0, "negative shape");
  if (batch == 0 || heads_q == 0 || seq == 0) return KAB_OK;
  KAB_REQUIRE(q && k && vt && q_scale && k_scale && v_scale && out, "null pointer");
  KAB_REQUIRE(aligned(q, 16) && aligned(k, 16) && aligned(vt, 16) && aligned(out, 16), "pointers must be 16-byte aligned");
  KAB_REQUIRE(head_dim == 128 || head_dim == 64, "head_dim %lld: the kernel takes 128 or 64", (long long)head_dim);
  KAB_REQUIRE(heads_kv > 0 && heads_q % heads_kv == 0, "heads_q %lld is not a multiple of heads_kv %lld",
              (long long)heads_q, (long long)heads_kv);
  const int64_t q_tiles = (seq + 127) / 128;
  const int64_t ld_vt = (seq + 15) / 16 * 16;  // V^T rows: seq rounded up to 16 (kab_quant_heads_fp8)
  const int64_t ctas = batch * heads_q * q_tiles;
  KAB_REQUIRE(ctas < (int64_t(1) << 31) && batch * heads_q * seq < (int64_t(1) << 31), "problem too large");
  const uint32_t d = static_cast<uint32_t>(head_dim);
  CUtensorMap mq, mk, mv;
  if (int e = byte_map(&mq, q, static_cast<uint64_t>(batch * heads_q * seq), d, "Q", d, 128)) return e;
  if (int e = byte_map(&mk, k, static_cast<uint64_t>(batch * heads_kv * seq), d, "K", d, 128)) return e;
  if (int e = byte_map(&mv, vt, static_cast<uint64_t>(batch * heads_kv * head_dim), static_cast<uint64_t>(ld_vt),
                       "V^T", 128, d))
    return e;
  AttnArgs g{};
  g.seq = static_cast<int>(seq);
  g.heads_q = static_cast<int>(heads_q);
  g.heads_kv = static_cast<int>(heads_kv);
  g.q_tiles = static_cast<int>(q_tiles);
  g.causal = causal;
  g.q_scale = q_scale;
  g.k_scale = k_scale;
  g.v_scale = v_scale;
  g.sm_scale_log2 = sm_scale * 1.4426950408889634f;
  g.out = out;
  return head_dim == 128 ? launch_attention<128>(mq, mk, mv, g, ctas, stream)
                          : launch_attention<64>(mq, mk, mv, g, ctas, stream);
}

int kab_quant_kv_fp8(const void* x, int dtype, int64_t outer, int64_t inner, int64_t d, int64_t xs_o, int64_t xs_i,
                     uint8_t* codes, int64_t cs_o, int64_t cs_i, float* scales, int64_t ss_o, int64_t ss_i,
                     void* stream) {
  KAB_REQUIRE(valid_dtype(dtype), "unknown dtype %d", dtype);
  KAB_REQUIRE(outer >= 0 && inner >= 0 && d >= 0, "negative shape");
  if (outer == 0 || inner == 0) return KAB_OK;
  KAB_REQUIRE(x != nullptr && codes != nullptr && scales != nullptr, "null pointer");
  KAB_REQUIRE(d == 16 || d == 32 || d == 64 || d == 128 || d == 256, "head_dim %lld: a power of two in 16..256",
              (long long)d);
  KAB_REQUIRE(aligned(x, 16) && aligned(codes, 8) && xs_o % 8 == 0 && xs_i % 8 == 0 && cs_o % 8 == 0 &&
                  cs_i % 8 == 0,
              "x must be 16-byte aligned, codes 8-byte aligned, and every row start a multiple of 8 elements");
  const int64_t rows = outer * inner;
  const int64_t lanes = d / 8;
  const int64_t blocks = (rows * lanes + 255) / 256;
  KAB_REQUIRE(blocks < (int64_t(1) << 31), "too many rows");
  const cudaStream_t s = as_stream(stream);
#define KAB_KV(TT, LN)                                                                                      \
  quant_kv_kernel<TT, LN><<<static_cast<unsigned>(blocks), 256, 0, s>>>(x, rows, inner, xs_o, xs_i, codes, \
                                                                         cs_o, cs_i, scales, ss_o, ss_i)
#define KAB_KV_D(TT)                  \
  switch (lanes) {                    \
    case 2: KAB_KV(TT, 2); break;     \
    case 4: KAB_KV(TT, 4); break;     \
    case 8: KAB_KV(TT, 8); break;     \
    case 16: KAB_KV(TT, 16); break;   \
    default: KAB_KV(TT, 32); break;   \
  }
  if (dtype == KAB_BF16) { KAB_KV_D(kBF16) }
  else if (dtype == KAB_F16) { KAB_KV_D(kF16) }
  else { KAB_KV_D(kF32) }
#undef KAB_KV_D
#undef KAB_KV
  return check_launch("kab_quant_kv_fp8");
}

int kab_kv_decode_workspace(const KabKvDecodeParams* p, int* splits, size_t* bytes) {
  int gp = 16;
  if (int e = decode_check(p, &gp)) return e;
  KAB_REQUIRE(bytes != nullptr, "null pointer");
  DecodePlan plan;
  if (p->length > 0)
    if (int e = decode_plan(p, gp, &plan)) return e;
  if (splits != nullptr) *splits = plan.splits;
  *bytes = plan.cluster ? 0 : decode_workspace_bytes(p, plan.splits, gp);
  return KAB_OK;
}

int kab_kv_decode_fp8(const KabKvDecodeParams* p, void* workspace, size_t workspace_bytes, void* stream) {
  int gp = 16;
  if (int e = decode_check(p, &gp)) return e;
  if (p->batch == 0 || p->heads_q == 0) return KAB_OK;
  KAB_REQUIRE(p->length >= 1, "an empty cache: at least one token is needed");
  KAB_REQUIRE(valid_dtype(p->q_dtype), "unknown q dtype %d", p->q_dtype);
  KAB_REQUIRE(p->q && p->k_codes && p->k_scales && p->v_codes && p->v_scales && p->out, "null pointer");
  KAB_REQUIRE(aligned(p->k_codes, 16) && aligned(p->v_codes, 16), "the codes must be 16-byte aligned");
  const int64_t d = p->head_dim;
  KAB_REQUIRE(p->kc_stride_l % 16 == 0 && p->kc_stride_h % 16 == 0 && p->kc_stride_b % 16 == 0 &&
                  p->vc_stride_l % 16 == 0 && p->vc_stride_h % 16 == 0 && p->vc_stride_b % 16 == 0,
              "code strides must be multiples of 16 bytes");
  KAB_REQUIRE(p->length < (int64_t(1) << 30) && p->batch * p->heads_kv < 65536, "problem too large");
  DecodePlan plan;
  if (int e = decode_plan(p, gp, &plan)) return e;
  const int splits = plan.splits, chunk = plan.chunk;
  const size_t need = plan.cluster ? 0 : decode_workspace_bytes(p, splits, gp);
  KAB_REQUIRE(need == 0 || (workspace != nullptr && workspace_bytes >= need && aligned(workspace, 256)),
              "the workspace needs %zu bytes, 256-byte aligned (kab_kv_decode_workspace)", need);
  CUtensorMap mk, mv;
  if (int e = cache_map(&mk, p->k_codes, p->batch, p->heads_kv, p->length, d, p->kc_stride_b, p->kc_stride_h,
                        p->kc_stride_l, "K codes"))
    return e;
  if (int e = cache_map(&mv, p->v_codes, p->batch, p->heads_kv, p->length, d, p->vc_stride_b, p->vc_stride_h,
                        p->vc_stride_l, "V codes"))
    return e;
  DecodeArgs g{};
  g.heads_kv = static_cast<int>(p->heads_kv);
  g.group = static_cast<int>(p->heads_q / p->heads_kv * p->q_len);
  g.length = static_cast<int>(p->length);
  g.chunk = chunk;
  g.splits = splits;
  g.q = p->q;
  g.sqb = p->q_stride_b;
  g.sqh = p->q_stride_row;
  g.k_scale = p->k_scales;
  g.ksb = p->ks_stride_b;
  g.ksh = p->ks_stride_h;
  g.v_scale = p->v_scales;
  g.vsb = p->vs_stride_b;
  g.vsh = p->vs_stride_h;
  g.lengths = p->lengths;
  g.scale_log2 = p->sm_scale * 1.4426950408889634f;
  g.out = p->out;
  g.cluster = plan.cluster;
  const int64_t pairs = p->batch * p->heads_kv;
  if (need > 0) {
    uint8_t* w = static_cast<uint8_t*>(workspace);
    const size_t counters = (static_cast<size_t>(pairs) * 4 + 255) / 256 * 256;
    const size_t ml = (static_cast<size_t>(pairs) * splits * 2 * gp * 4 + 255) / 256 * 256;
    g.counters = reinterpret_cast<unsigned*>(w);
    g.part_ml = reinterpret_cast<float*>(w + counters);
    g.part_o = reinterpret_cast<float*>(w + counters + ml);
  }
  const cudaStream_t s = as_stream(stream);
  if (d == 128)
    return gp == 8    ? launch_decode_t<128, 8>(mk, mv, g, p->q_dtype, pairs, s)
           : gp == 16 ? launch_decode_t<128, 16>(mk, mv, g, p->q_dtype, pairs, s)
                      : launch_decode_t<128, 32>(mk, mv, g, p->q_dtype, pairs, s);
  return gp == 8    ? launch_decode_t<64, 8>(mk, mv, g, p->q_dtype, pairs, s)
         : gp == 16 ? launch_decode_t<64, 16>(mk, mv, g, p->q_dtype, pairs, s)
                    : launch_decode_t<64, 32>(mk, mv, g, p->q_dtype, pairs, s);
}

}  // extern "C"
