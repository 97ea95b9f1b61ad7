// extern "C" entry points of the comparator (compare.cuh).
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
  if (P.dtype == KAB_BF16) compare_kernel<kBF16><<<grid, 256, 0, s>>>(P, partials);
  else if (P.dtype == KAB_F16) compare_kernel<kF16><<<grid, 256, 0, s>>>(P, partials);
  else compare_kernel<kF32><<<grid, 256, 0, s>>>(P, partials);
  if (int e = check_launch("kab_compare")) return e;
  compare_finalize_kernel<<<1, 256, 0, s>>>(partials, grid, result);
  return check_launch("kab_compare finalize");
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

}  // extern "C"
