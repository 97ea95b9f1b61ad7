// extern "C" entry points of the FP8 attention prefill (attention.cuh): the per-head
// quantiser, the attention kernel's TMA maps and launch, and this translation unit's
// device status word.
#include <cudaTypedefs.h>

#include <mutex>

#include "kab_host.h"

namespace kab {
__device__ unsigned g_attention_status = 0;
}  // namespace kab

#include "attention.cuh"

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

// A [rows, cols] byte matrix read in 128 x 128-byte boxes with the 128-byte swizzle.
int byte_map(CUtensorMap* map, const void* ptr, uint64_t rows, uint64_t cols, const char* name) {
  auto fn = attn_encode_fn();
  if (fn == nullptr) return fail(KAB_EUNSUPPORTED, "cuTensorMapEncodeTiled is unavailable (driver too old?)");
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {cols};
  cuuint32_t box[2] = {128, 128};
  cuuint32_t estr[2] = {1, 1};
  const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(KAB_EINVAL, "tensor map of %s failed (CUresult %d)", name, static_cast<int>(r));
  return KAB_OK;
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
  KAB_REQUIRE(!transpose || seq % 64 == 0, "the transposed layout needs seq a multiple of 64");
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
  KAB_REQUIRE(head_dim == 128, "head_dim %lld: the kernel takes 128", (long long)head_dim);
  KAB_REQUIRE(seq % 128 == 0, "seq %lld must be a multiple of 128", (long long)seq);
  KAB_REQUIRE(heads_kv > 0 && heads_q % heads_kv == 0, "heads_q %lld is not a multiple of heads_kv %lld",
              (long long)heads_q, (long long)heads_kv);
  const int64_t ctas = batch * heads_q * (seq / 128);
  KAB_REQUIRE(ctas < (int64_t(1) << 31) && batch * heads_q * seq < (int64_t(1) << 31), "problem too large");
  CUtensorMap mq, mk, mv;
  if (int e = byte_map(&mq, q, static_cast<uint64_t>(batch * heads_q * seq), 128, "Q")) return e;
  if (int e = byte_map(&mk, k, static_cast<uint64_t>(batch * heads_kv * seq), 128, "K")) return e;
  if (int e = byte_map(&mv, vt, static_cast<uint64_t>(batch * heads_kv * 128), static_cast<uint64_t>(seq), "V^T"))
    return e;
  AttnArgs g{};
  g.seq = static_cast<int>(seq);
  g.heads_q = static_cast<int>(heads_q);
  g.heads_kv = static_cast<int>(heads_kv);
  g.q_tiles = static_cast<int>(seq / 128);
  g.causal = causal;
  g.q_scale = q_scale;
  g.k_scale = k_scale;
  g.v_scale = v_scale;
  g.sm_scale_log2 = sm_scale * 1.4426950408889634f;
  g.out = out;
  static bool configured[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !configured[dev]) {
    if (cudaFuncSetAttribute(attention_fp8_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, AttnLayout::kSmem) !=
        cudaSuccess)
      return fail(KAB_ECUDA, "cannot set %d bytes of shared memory", AttnLayout::kSmem);
    configured[dev] = true;
  }
  attention_fp8_kernel<<<static_cast<unsigned>(ctas), AttnLayout::kThreads, AttnLayout::kSmem, as_stream(stream)>>>(
      mq, mk, mv, g);
  return check_launch("kab_attention_fp8");
}

}  // extern "C"
