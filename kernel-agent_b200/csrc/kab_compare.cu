// extern "C" entry points of the comparator (compare.cuh).
#include <mutex>
#include <vector>

#include "compare.cuh"
#include "kab_host.h"

namespace kab {
namespace {
int compare_grid(int64_t n) {
  const int64_t per = 256 * 8 * 4;  // elements per block per pass before capping
  int64_t g = (n + per - 1) / per;
  const int64_t cap = static_cast<int64_t>(sm_count()) * 4;
  if (g < 1) g = 1;
  if (g > cap) g = cap;
  return static_cast<int>(g);
}
constexpr int64_t kChannelChunkRows = 64;

// The per-block partials of kab_compare_noalloc. compare_grid caps the grid at 4 blocks per
// SM, so these 1024 slots (152 KB per device) serve any element count on devices of up to
// 256 SMs (a B200 uses at most 592). Every launched block overwrites its own slot before the
// finalize kernel reads it: nothing here has to start at zero, and nothing is cleared.
constexpr int kStaticPartials = 1024;
static __device__ __align__(256) CmpPartial g_compare_partials[kStaticPartials];

// The device address of g_compare_partials on the current device, looked up once per device
// (cudaGetSymbolAddress, which may load the module on that device).
int static_partials(CmpPartial** out) {
  static std::mutex mu;
  static std::vector<CmpPartial*> cache;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(KAB_ECUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
  std::lock_guard<std::mutex> lock(mu);
  if (static_cast<int>(cache.size()) <= dev) cache.resize(dev + 1, nullptr);
  if (cache[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_compare_partials);
    if (e != cudaSuccess) return fail(KAB_ECUDA, "cudaGetSymbolAddress: %s", cudaGetErrorString(e));
    cache[dev] = static_cast<CmpPartial*>(p);
  }
  *out = cache[dev];
  return KAB_OK;
}
}  // namespace
}  // namespace kab

using namespace kab;

extern "C" {

size_t kab_compare_scratch_bytes(int64_t n) {
  return static_cast<size_t>(compare_grid(n < 0 ? 0 : n)) * sizeof(CmpPartial);
}

int kab_compare(const KabCompareParams* params, void* scratch, size_t scratch_bytes,
                KabCompareResult* result, void* stream) {
  KAB_REQUIRE(params != nullptr && result != nullptr, "null pointer");
  const KabCompareParams& P = *params;
  KAB_REQUIRE(valid_dtype(P.dtype), "unknown dtype %d", P.dtype);
  KAB_REQUIRE(P.n >= 0, "negative element count");
  KAB_REQUIRE(P.n == 0 || (P.ref != nullptr && P.new_ != nullptr), "ref / new is null");
  KAB_REQUIRE(!P.has_rerounded || P.rerounded != nullptr, "rerounded is null");
  KAB_REQUIRE((P.widen_mode != 2 && P.element_mode != 2) || P.channels > 0,
              "per-channel bounds need channels > 0");
  KAB_REQUIRE(P.widen_mode != 2 || P.widen_channel != nullptr, "widen_channel is null");
  KAB_REQUIRE(P.element_mode != 2 || P.element_scale != nullptr, "element_scale is null");
  if (P.vector) {
    KAB_REQUIRE(aligned(P.ref, 16) && aligned(P.new_, 16) && (!P.has_rerounded || aligned(P.rerounded, 16)),
                "vector loads need 16-byte aligned tensors");
  }
  const int grid = compare_grid(P.n);
  KAB_REQUIRE(scratch != nullptr && scratch_bytes >= static_cast<size_t>(grid) * sizeof(CmpPartial),
              "scratch of %zu bytes is smaller than the %zu needed", scratch_bytes,
              static_cast<size_t>(grid) * sizeof(CmpPartial));
  const cudaStream_t s = as_stream(stream);
  CmpPartial* partials = static_cast<CmpPartial*>(scratch);
  const bool simple = !P.has_rerounded && !P.alt_bound && P.widen_mode == 0 && P.element_mode == 0;
#define KAB_CMP(TT)                                                        \
  if (simple) compare_kernel<TT, true><<<grid, 256, 0, s>>>(P, partials);  \
  else compare_kernel<TT, false><<<grid, 256, 0, s>>>(P, partials)
  if (P.dtype == KAB_BF16) { KAB_CMP(kBF16); }
  else if (P.dtype == KAB_F16) { KAB_CMP(kF16); }
  else { KAB_CMP(kF32); }
#undef KAB_CMP
  if (int e = check_launch("kab_compare")) return e;
  compare_finalize_kernel<<<1, 256, 0, s>>>(partials, grid, result);
  return check_launch("kab_compare finalize");
}

// kab_compare with its partials in g_compare_partials instead of caller scratch. For callers
// that cannot allocate device memory at the point of the check: a harness judging a candidate
// that has just filled HBM (an out-of-memory candidate still gets its verdict), or a host
// binding with no device allocator of its own. It allocates and frees nothing, and adds no
// code path: the same kernels run, through kab_compare, on the same grid, so the result is
// bit-identical to kab_compare's. Calls that overlap on one device (two streams, two host
// threads) share the slots and race: order them on one stream.
int kab_compare_noalloc(const KabCompareParams* params, KabCompareResult* result, void* stream) {
  KAB_REQUIRE(params != nullptr && result != nullptr, "null pointer");
  KAB_REQUIRE(params->n >= 0, "negative element count");
  const int grid = compare_grid(params->n);
  KAB_REQUIRE(grid <= kStaticPartials,
              "kab_compare_noalloc: %d blocks need %d partial slots, the static scratch holds %d "
              "(a device of more than %d SMs); use kab_compare with caller scratch",
              grid, grid, kStaticPartials, kStaticPartials / 4);
  CmpPartial* partials = nullptr;
  if (int e = static_partials(&partials)) return e;
  return kab_compare(params, partials, sizeof(CmpPartial) * kStaticPartials, result, stream);
}

size_t kab_channel_rms_scratch_bytes(int64_t rows, int64_t channels) {
  if (rows <= 0 || channels <= 0) return 0;
  const int64_t chunks = (rows + kChannelChunkRows - 1) / kChannelChunkRows;
  return static_cast<size_t>(chunks * channels) * sizeof(double);
}

int kab_channel_rms(const void* x, const void* alt, int dtype, int64_t rows,
                    int64_t channels, float* rms, void* scratch, size_t scratch_bytes,
                    void* stream) {
  KAB_REQUIRE(valid_dtype(dtype), "unknown dtype %d", dtype);
  KAB_REQUIRE(rows > 0 && channels > 0, "empty [%lld, %lld]", (long long)rows, (long long)channels);
  KAB_REQUIRE(x != nullptr && rms != nullptr, "null pointer");
  const int64_t chunks = (rows + kChannelChunkRows - 1) / kChannelChunkRows;
  KAB_REQUIRE(scratch != nullptr && scratch_bytes >= kab_channel_rms_scratch_bytes(rows, channels),
              "scratch too small");
  KAB_REQUIRE(chunks < 65536, "too many rows (%lld)", (long long)rows);
  const cudaStream_t s = as_stream(stream);
  double* partial = static_cast<double*>(scratch);
  const dim3 grid(static_cast<unsigned>((channels + 255) / 256), static_cast<unsigned>(chunks));
  if (dtype == KAB_BF16) channel_sumsq_kernel<kBF16><<<grid, 256, 0, s>>>(x, alt, rows, channels, kChannelChunkRows, partial);
  else if (dtype == KAB_F16) channel_sumsq_kernel<kF16><<<grid, 256, 0, s>>>(x, alt, rows, channels, kChannelChunkRows, partial);
  else channel_sumsq_kernel<kF32><<<grid, 256, 0, s>>>(x, alt, rows, channels, kChannelChunkRows, partial);
  if (int e = check_launch("kab_channel_rms")) return e;
  channel_rms_kernel<<<static_cast<unsigned>((channels + 255) / 256), 256, 0, s>>>(partial, chunks, rows, channels, rms);
  return check_launch("kab_channel_rms finalize");
}

int kab_diff_census(const KabDiffParams* params, unsigned long long* count, void* stream) {
  KAB_REQUIRE(params != nullptr && count != nullptr, "null pointer");
  const KabDiffParams& P = *params;
  KAB_REQUIRE(valid_dtype(P.dtype) || (P.dtype >= kDiffF64 && P.dtype <= kDiffBits64), "unknown dtype %d", P.dtype);
  KAB_REQUIRE(P.outer >= 0 && P.len >= 0 && P.inner >= 0, "negative region");
  KAB_REQUIRE(P.a_off >= 0 && P.base_off >= 0 && P.a_off + P.len <= P.a_dim && P.base_off + P.len <= P.base_dim,
              "the slice [%lld, %lld) / [%lld, %lld) leaves the dimension (%lld / %lld)", (long long)P.a_off,
              (long long)(P.a_off + P.len), (long long)P.base_off, (long long)(P.base_off + P.len),
              (long long)P.a_dim, (long long)P.base_dim);
  const int64_t total = P.outer * P.len * P.inner;
  KAB_REQUIRE(total == 0 || (P.a != nullptr && P.base != nullptr), "null tensor");
  if (P.hits != nullptr || P.box != nullptr) {
    KAB_REQUIRE(P.ndim >= 1 && P.ndim <= KAB_DIFF_MAXDIM, "ndim %d not in 1..%d", P.ndim, KAB_DIFF_MAXDIM);
    int64_t n = 1;
    for (int k = 0; k < P.ndim; ++k) {
      KAB_REQUIRE(P.shape[k] > 0, "empty dimension %d", k);
      n *= P.shape[k];
    }
    KAB_REQUIRE(n == total, "the region's shape holds %lld elements, not %lld", (long long)n, (long long)total);
  }
  const cudaStream_t s = as_stream(stream);
  if (cudaMemsetAsync(count, 0, sizeof(unsigned long long), s) != cudaSuccess) return check_launch("census reset");
  if (total == 0) return KAB_OK;
  const int64_t blocks = (total + 255) / 256;
  const int cap = sm_count() * 8;
  const int grid = static_cast<int>(blocks < cap ? blocks : cap);
  if (P.dtype == KAB_BF16) diff_census_kernel<kBF16><<<grid, 256, 0, s>>>(P, count);
  else if (P.dtype == KAB_F16) diff_census_kernel<kF16><<<grid, 256, 0, s>>>(P, count);
  else if (P.dtype == kDiffF64) diff_census_kernel<kDiffF64><<<grid, 256, 0, s>>>(P, count);
  else if (P.dtype == kDiffBits8) diff_census_kernel<kDiffBits8><<<grid, 256, 0, s>>>(P, count);
  else if (P.dtype == kDiffBits16) diff_census_kernel<kDiffBits16><<<grid, 256, 0, s>>>(P, count);
  else if (P.dtype == kDiffBits32) diff_census_kernel<kDiffBits32><<<grid, 256, 0, s>>>(P, count);
  else if (P.dtype == kDiffBits64) diff_census_kernel<kDiffBits64><<<grid, 256, 0, s>>>(P, count);
  else diff_census_kernel<kF32><<<grid, 256, 0, s>>>(P, count);
  return check_launch("kab_diff_census");
}

}  // extern "C"
