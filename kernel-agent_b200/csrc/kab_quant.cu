// extern "C" entry points of the quantise producers (quant.cuh): argument checks, launch
// shapes and template dispatch.
#include "checks.cuh"
#include "kab_host.h"
#include "quant.cuh"

namespace kab {
namespace {

// Threads per row and chunks per thread for a row of `nchunks` chunks of 8.
void row_shape(int64_t nchunks, int& threads, int& maxc) {
  threads = nchunks <= 128 ? 128 : 256;
  const int64_t per = (nchunks + threads - 1) / threads;
  maxc = per <= 1 ? 1 : per <= 2 ? 2 : per <= 4 ? 4 : per <= 8 ? 8 : per <= 16 ? 16 : 0;
}

// One row per grid x index, chunks of 8 along the row over grid y blocks of `threads`
// (a multiple of 32 that covers a short row in one block).
void chunk_grid(int64_t rows, int64_t k, int& threads, dim3& grid) {
  const int64_t chunks = k / 8;
  threads = chunks >= 256 ? 256 : static_cast<int>((chunks + 31) / 32 * 32);
  grid = dim3(static_cast<unsigned>(rows), static_cast<unsigned>((chunks + threads - 1) / threads));
}

int grid_for(int64_t work_items, int threads) {
  const int64_t blocks = (work_items + threads - 1) / threads;
  const int64_t cap = static_cast<int64_t>(sm_count()) * 16;
  return static_cast<int>(blocks < 1 ? 1 : (blocks > cap ? cap : blocks));
}

template <int T, int OUT, int SMOOTH, bool SILU>
void launch_rows(int maxc, dim3 grid, int threads, cudaStream_t s, const void* x, int64_t ldx,
                 const void* up, int64_t ldu, int64_t k, const float* smooth, void* q,
                 float* scale, void* h) {
#define KAB_ROWS(MC) quant_rows_kernel<T, MC, OUT, SMOOTH, SILU><<<grid, threads, 0, s>>>(x, ldx, up, ldu, k, smooth, q, scale, h)
  switch (maxc) {
    case 1: KAB_ROWS(1); break;
    case 2: KAB_ROWS(2); break;
    case 4: KAB_ROWS(4); break;
    case 8: KAB_ROWS(8); break;
    case 16: KAB_ROWS(16); break;
    default: KAB_ROWS(0); break;
  }
#undef KAB_ROWS
}

int check_matrix(const void* x, int dtype, int64_t rows, int64_t k, int64_t ldx, const char* name) {
  KAB_REQUIRE(valid_dtype(dtype), "%s: unknown dtype %d", name, dtype);
  KAB_REQUIRE(rows >= 0 && k >= 0, "%s: negative shape [%lld, %lld]", name, (long long)rows, (long long)k);
  KAB_REQUIRE(rows == 0 || x != nullptr, "%s is null", name);
  KAB_REQUIRE(ldx >= k, "%s: leading dimension %lld < width %lld", name, (long long)ldx, (long long)k);
  KAB_REQUIRE(k % 8 == 0, "%s: width %lld is not a multiple of 8", name, (long long)k);
  KAB_REQUIRE(ldx % 8 == 0, "%s: leading dimension %lld is not a multiple of 8", name, (long long)ldx);
  KAB_REQUIRE(aligned(x, 16), "%s is not 16-byte aligned", name);
  return KAB_OK;
}

template <int T, int FMT, int MODE, bool SILU>
void launch_fp4(int maxc, unsigned rows, int threads, cudaStream_t s, const void* x, int64_t ldx,
                const void* up, int64_t ldu, int64_t nrows, int64_t k, const float* amax,
                const float* ts, int swizzle, uint8_t* q, uint8_t* scales, float* outer, void* h) {
#define KAB_FP4(MC) quant_fp4_kernel<T, MC, FMT, MODE, SILU><<<rows, threads, 0, s>>>(x, ldx, up, ldu, nrows, k, amax, ts, swizzle, q, scales, outer, h)
  if constexpr (FMT == 0) {
    if (maxc == 1) KAB_FP4(1);
    else if (maxc == 2) KAB_FP4(2);
    else KAB_FP4(4);
  } else {
    if (maxc == 1) KAB_FP4(1);
    else KAB_FP4(2);
  }
#undef KAB_FP4
}
template <int T, int F, int M>
void launch_fp4_fast_nb(int maxc, unsigned rows, int threads, cudaStream_t s, const void* x, int64_t ldx, int64_t k,
                        const float* amax, const float* ts, int swizzle, uint8_t* q, uint8_t* scales, float* outer) {
  constexpr int kNbMax = F == 0 ? 4 : 2;
  if (maxc == 1) quant_fp4_fast_kernel<T, 1, F, M><<<rows, threads, 0, s>>>(x, ldx, k, amax, ts, swizzle, q, scales, outer);
  else if (maxc == 2) quant_fp4_fast_kernel<T, 2, F, M><<<rows, threads, 0, s>>>(x, ldx, k, amax, ts, swizzle, q, scales, outer);
  else quant_fp4_fast_kernel<T, kNbMax, F, M><<<rows, threads, 0, s>>>(x, ldx, k, amax, ts, swizzle, q, scales, outer);
}
// The kernel's dynamic shared memory (the staged row and the fix list) passes the default 48 KB
// for rows above ~21.8K NVFP4 elements; the attribute is a per-device setting, so it is made
// once on every device that launches the kernel.
template <typename Kernel>
int allow_row_smem(Kernel kernel, bool (&configured)[64]) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return fail(KAB_ECUDA, "cudaGetDevice failed");
  if (dev >= 64 || configured[dev]) return KAB_OK;
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 32768 * 2 + 2048 * 4) != cudaSuccess)
    return fail(KAB_ECUDA, "cannot raise the RMSNorm FP4 producer's shared memory to %d bytes", 32768 * 2 + 2048 * 4);
  configured[dev] = true;
  return KAB_OK;
}
template <int T, int F, int NB>
int launch_rmsnorm_fp4_nb(unsigned rows, int threads, size_t smem, cudaStream_t s, const void* x, int64_t ldx,
                          int64_t k, const void* w, float eps, int swizzle, uint8_t* q, uint8_t* scales, float* outer,
                          void* h) {
  static bool configured[64] = {};
  auto kernel = quant_fp4_fast_kernel<T, NB, F, 0, true>;
  if (smem > 48 * 1024)
    if (int e = allow_row_smem(kernel, configured)) return e;
  kernel<<<rows, threads, smem, s>>>(x, ldx, k, nullptr, nullptr, swizzle, q, scales, outer, w, eps, h);
  return KAB_OK;
}
template <int T, int F>
int launch_rmsnorm_fp4(int maxc, unsigned rows, int threads, cudaStream_t s, const void* x, int64_t ldx, int64_t k,
                       const void* w, float eps, int swizzle, uint8_t* q, uint8_t* scales, float* outer, void* h) {
  constexpr int kNbMax = F == 0 ? 4 : 2;
  const size_t smem = static_cast<size_t>(k) * 2 + static_cast<size_t>(k / (F == 0 ? 16 : 32)) * 4;  // row, fix list
  if (maxc == 1) return launch_rmsnorm_fp4_nb<T, F, 1>(rows, threads, smem, s, x, ldx, k, w, eps, swizzle, q, scales, outer, h);
  if (maxc == 2) return launch_rmsnorm_fp4_nb<T, F, 2>(rows, threads, smem, s, x, ldx, k, w, eps, swizzle, q, scales, outer, h);
  return launch_rmsnorm_fp4_nb<T, F, kNbMax>(rows, threads, smem, s, x, ldx, k, w, eps, swizzle, q, scales, outer, h);
}
template <int T>
void launch_fp4_fast(int fmt, int mode, int maxc, unsigned rows, int threads, cudaStream_t s, const void* x,
                     int64_t ldx, int64_t k, const float* amax, const float* ts, int swizzle, uint8_t* q,
                     uint8_t* scales, float* outer) {
#define KAB_FP4F(F, M) launch_fp4_fast_nb<T, F, M>(maxc, rows, threads, s, x, ldx, k, amax, ts, swizzle, q, scales, outer)
  if (fmt == KAB_NVFP4) {
    if (mode == KAB_FP4_TOKEN) KAB_FP4F(0, 0);
    else if (mode == KAB_FP4_TENSOR) KAB_FP4F(0, 1);
    else KAB_FP4F(0, 2);
  } else {
    if (mode == KAB_FP4_WEIGHT) KAB_FP4F(1, 2);
    else KAB_FP4F(1, 0);
  }
#undef KAB_FP4F
}
template <int T, bool SILU>
void launch_fp4_fmt(int fmt, int mode, int maxc, unsigned rows, int threads, cudaStream_t s,
                    const void* x, int64_t ldx, const void* up, int64_t ldu, int64_t nrows,
                    int64_t k, const float* amax, const float* ts, int swizzle, uint8_t* q,
                    uint8_t* scales, float* outer, void* h) {
#define KAB_FP4M(F, M) launch_fp4<T, F, M, SILU>(maxc, rows, threads, s, x, ldx, up, ldu, nrows, k, amax, ts, swizzle, q, scales, outer, h)
  if (fmt == KAB_NVFP4) {
    if (mode == KAB_FP4_TOKEN) KAB_FP4M(0, 0);
    else if (mode == KAB_FP4_TENSOR) KAB_FP4M(0, 1);
    else KAB_FP4M(0, 2);
  } else {
    if (mode == KAB_FP4_WEIGHT) KAB_FP4M(1, 2);
    else KAB_FP4M(1, 0);
  }
#undef KAB_FP4M
}
}  // namespace
}  // namespace kab

using namespace kab;

extern "C" {

int kab_quant_rows_int8(const void* x, int dtype, int64_t rows, int64_t k, int64_t ldx,
                        const float* smooth, int smooth_mode, int8_t* q, float* scale,
                        void* stream) {
  if (int e = check_matrix(x, dtype, rows, k, ldx, "x")) return e;
  KAB_REQUIRE(smooth_mode >= 0 && smooth_mode <= 2, "smooth_mode %d not in 0..2", smooth_mode);
  KAB_REQUIRE(smooth_mode == 0 || (smooth != nullptr && aligned(smooth, 16)),
              "smooth factors are null or not 16-byte aligned");
  KAB_REQUIRE(rows == 0 || (q != nullptr && scale != nullptr && aligned(q, 8)), "outputs are null or misaligned");
  if (rows == 0) return KAB_OK;
  int threads, maxc;
  row_shape(k / 8, threads, maxc);
  const cudaStream_t s = as_stream(stream);
  const dim3 grid(static_cast<unsigned>(rows));
#define KAB_INT8(TT, SM) launch_rows<TT, 0, SM, false>(maxc, grid, threads, s, x, ldx, nullptr, 0, k, smooth, q, scale, nullptr)
#define KAB_INT8_SM(TT) \
  if (smooth_mode == 0) KAB_INT8(TT, 0); else if (smooth_mode == 1) KAB_INT8(TT, 1); else KAB_INT8(TT, 2)
  if (dtype == KAB_BF16) { KAB_INT8_SM(kBF16); }
  else if (dtype == KAB_F16) { KAB_INT8_SM(kF16); }
  else { KAB_INT8_SM(kF32); }
#undef KAB_INT8_SM
#undef KAB_INT8
  return check_launch("kab_quant_rows_int8");
}

int kab_quant_rows_fp8(const void* x, int dtype, int64_t rows, int64_t k, int64_t ldx,
                       const void* up, int64_t ldu, uint8_t* q, float* scale, void* h,
                       void* stream) {
  if (int e = check_matrix(x, dtype, rows, k, ldx, "x")) return e;
  if (up != nullptr) {
    if (int e = check_matrix(up, dtype, rows, k, ldu, "up")) return e;
    KAB_REQUIRE(dtype != KAB_F32, "the fused SiLU * up producer takes bf16 or fp16");
  }
  KAB_REQUIRE(h == nullptr || aligned(h, 16), "h is not 16-byte aligned");
  KAB_REQUIRE(rows == 0 || (q != nullptr && scale != nullptr && aligned(q, 8)), "outputs are null or misaligned");
  if (rows == 0) return KAB_OK;
  int threads, maxc;
  row_shape(k / 8, threads, maxc);
  const cudaStream_t s = as_stream(stream);
  const dim3 grid(static_cast<unsigned>(rows));
  if (up != nullptr) {
    if (dtype == KAB_BF16) launch_rows<kBF16, 1, 0, true>(maxc, grid, threads, s, x, ldx, up, ldu, k, nullptr, q, scale, h);
    else launch_rows<kF16, 1, 0, true>(maxc, grid, threads, s, x, ldx, up, ldu, k, nullptr, q, scale, h);
  } else {
    if (dtype == KAB_BF16) launch_rows<kBF16, 1, 0, false>(maxc, grid, threads, s, x, ldx, nullptr, 0, k, nullptr, q, scale, nullptr);
    else if (dtype == KAB_F16) launch_rows<kF16, 1, 0, false>(maxc, grid, threads, s, x, ldx, nullptr, 0, k, nullptr, q, scale, nullptr);
    else launch_rows<kF32, 1, 0, false>(maxc, grid, threads, s, x, ldx, nullptr, 0, k, nullptr, q, scale, nullptr);
  }
  return check_launch("kab_quant_rows_fp8");
}

int kab_quant_groups_fp8(const void* x, int dtype, int64_t rows, int64_t k, int64_t ldx,
                         int group, uint8_t* q, float* scales, void* stream) {
  if (int e = check_matrix(x, dtype, rows, k, ldx, "x")) return e;
  KAB_REQUIRE(group == 32 || group == 64 || group == 128, "group %d is not 32, 64 or 128", group);
  KAB_REQUIRE(k % group == 0, "width %lld is not a multiple of the group %d", (long long)k, group);
  KAB_REQUIRE(rows == 0 || (q != nullptr && scales != nullptr && aligned(q, 8)), "outputs are null or misaligned");
  if (rows == 0 || k == 0) return KAB_OK;
  KAB_REQUIRE(rows < (int64_t(1) << 31), "too many rows (%lld)", (long long)rows);
  int threads;
  dim3 grid;
  chunk_grid(rows, k, threads, grid);
  const cudaStream_t s = as_stream(stream);
#define KAB_GROUPS(TT)                                                                          \
  if (group == 32) quant_groups_kernel<TT, 4><<<grid, threads, 0, s>>>(x, ldx, k, q, scales); \
  else if (group == 64) quant_groups_kernel<TT, 8><<<grid, threads, 0, s>>>(x, ldx, k, q, scales); \
  else quant_groups_kernel<TT, 16><<<grid, threads, 0, s>>>(x, ldx, k, q, scales)
  if (dtype == KAB_BF16) { KAB_GROUPS(kBF16); }
  else if (dtype == KAB_F16) { KAB_GROUPS(kF16); }
  else { KAB_GROUPS(kF32); }
#undef KAB_GROUPS
  return check_launch("kab_quant_groups_fp8");
}

int kab_quant_blocks_fp8(const void* w, int dtype, int64_t n, int64_t k, int64_t ldw,
                         uint8_t* q, float* scales, void* stream) {
  if (int e = check_matrix(w, dtype, n, k, ldw, "w")) return e;
  KAB_REQUIRE(n % 128 == 0 && k % 128 == 0, "weight [%lld, %lld] is not whole 128 x 128 blocks",
              (long long)n, (long long)k);
  KAB_REQUIRE(n == 0 || (q != nullptr && scales != nullptr && aligned(q, 8)), "outputs are null or misaligned");
  if (n == 0 || k == 0) return KAB_OK;
  const dim3 grid(static_cast<unsigned>(k / 128), static_cast<unsigned>(n / 128));
  const cudaStream_t s = as_stream(stream);
  if (dtype == KAB_BF16) quant_blocks128_kernel<kBF16><<<grid, 256, 0, s>>>(w, ldw, k, q, scales);
  else if (dtype == KAB_F16) quant_blocks128_kernel<kF16><<<grid, 256, 0, s>>>(w, ldw, k, q, scales);
  else quant_blocks128_kernel<kF32><<<grid, 256, 0, s>>>(w, ldw, k, q, scales);
  return check_launch("kab_quant_blocks_fp8");
}

int kab_quant_mxfp8(const void* x, int dtype, int64_t rows, int64_t k, int64_t ldx,
                    const void* up, int64_t ldu, int rule, uint8_t* q, uint8_t* scales,
                    int swizzle, void* h, void* stream) {
  if (int e = check_matrix(x, dtype, rows, k, ldx, "x")) return e;
  KAB_REQUIRE(k % 32 == 0, "width %lld is not a multiple of the MXFP8 block (32)", (long long)k);
  KAB_REQUIRE(rule == 0 || rule == 1, "rule %d is not 0 (ceil) or 1 (floor)", rule);
  if (up != nullptr) {
    if (int e = check_matrix(up, dtype, rows, k, ldu, "up")) return e;
    KAB_REQUIRE(dtype != KAB_F32, "the fused SiLU * up producer takes bf16 or fp16");
  }
  KAB_REQUIRE(h == nullptr || aligned(h, 16), "h is not 16-byte aligned");
  KAB_REQUIRE(rows == 0 || (q != nullptr && scales != nullptr && aligned(q, 8)), "outputs are null or misaligned");
  if (rows == 0 || k == 0) return KAB_OK;
  KAB_REQUIRE(rows < (int64_t(1) << 31), "too many rows (%lld)", (long long)rows);
  int threads;
  dim3 grid;
  chunk_grid(rows, k, threads, grid);
  const cudaStream_t s = as_stream(stream);
  if (up != nullptr) {
    if (dtype == KAB_BF16) quant_mxfp8_kernel<kBF16, true><<<grid, threads, 0, s>>>(x, ldx, up, ldu, k, rule, swizzle, q, scales, h);
    else quant_mxfp8_kernel<kF16, true><<<grid, threads, 0, s>>>(x, ldx, up, ldu, k, rule, swizzle, q, scales, h);
  } else {
    if (dtype == KAB_BF16) quant_mxfp8_kernel<kBF16, false><<<grid, threads, 0, s>>>(x, ldx, nullptr, 0, k, rule, swizzle, q, scales, nullptr);
    else if (dtype == KAB_F16) quant_mxfp8_kernel<kF16, false><<<grid, threads, 0, s>>>(x, ldx, nullptr, 0, k, rule, swizzle, q, scales, nullptr);
    else quant_mxfp8_kernel<kF32, false><<<grid, threads, 0, s>>>(x, ldx, nullptr, 0, k, rule, swizzle, q, scales, nullptr);
  }
  return check_launch("kab_quant_mxfp8");
}


int kab_quant_fp4(const void* x, int dtype, int64_t rows, int64_t k, int64_t ldx,
                  const void* up, int64_t ldu, int fmt, int mode, const float* amax,
                  const float* tensor_scale, uint8_t* q, uint8_t* scales, int swizzle,
                  float* outer, void* h, void* stream) {
  if (int e = check_matrix(x, dtype, rows, k, ldx, "x")) return e;
  KAB_REQUIRE(fmt == KAB_NVFP4 || fmt == KAB_MXFP4, "fmt %d is not NVFP4 (0) or MXFP4 (1)", fmt);
  KAB_REQUIRE(mode >= 0 && mode <= 2, "mode %d not in 0..2", mode);
  const int block = fmt == KAB_NVFP4 ? 16 : 32;
  KAB_REQUIRE(k % block == 0, "width %lld is not a multiple of the block (%d)", (long long)k, block);
  KAB_REQUIRE(!(fmt == KAB_NVFP4 && mode == KAB_FP4_TENSOR && amax == nullptr), "amax is null");
  KAB_REQUIRE(!(fmt == KAB_NVFP4 && mode == KAB_FP4_WEIGHT && tensor_scale == nullptr), "tensor_scale is null");
  KAB_REQUIRE(k / 8 <= 256 * 16, "width %lld exceeds the register-resident row (32768)", (long long)k);
  KAB_REQUIRE(rows < (int64_t(1) << 31), "too many rows (%lld)", (long long)rows);
  if (up != nullptr) {
    if (int e = check_matrix(up, dtype, rows, k, ldu, "up")) return e;
    KAB_REQUIRE(dtype != KAB_F32, "the fused SiLU * up producer takes bf16 or fp16");
  }
  KAB_REQUIRE(h == nullptr || aligned(h, 16), "h is not 16-byte aligned");
  KAB_REQUIRE(rows == 0 || (q != nullptr && scales != nullptr && aligned(q, 4)), "outputs are null or misaligned");
  if (rows == 0 || k == 0) return KAB_OK;
  // threads per row and scale blocks per thread: 256 threads where that suffices, up to 512
  // with 4 (NVFP4) or 2 (MXFP4) register-resident blocks each
  const int64_t nblk = k / block;
  const int nb_max = fmt == KAB_NVFP4 ? 4 : 2;
  int threads = static_cast<int>(nblk < 256 ? (nblk + 31) / 32 * 32 : 256);
  // 2-byte NVFP4 rows of 257-512 blocks: 128 threads x 4 blocks (x [8192, 8192] bf16: 51.3 us
  // against 52.9 us at 256 x 2 and 68.8 us at 512 x 1; one B200, the same box)
  if (up == nullptr && dtype != KAB_F32 && fmt == KAB_NVFP4 && nblk > 256 && nblk <= 512) threads = 128;
  if (nblk > static_cast<int64_t>(threads) * nb_max)
    threads = static_cast<int>(((nblk + nb_max - 1) / nb_max + 31) / 32 * 32);
  const int64_t per = (nblk + threads - 1) / threads;
  const int maxc = per <= 1 ? 1 : per <= 2 ? 2 : 4;
  const cudaStream_t s = as_stream(stream);
  const unsigned grid = static_cast<unsigned>(rows);
  if (up != nullptr) {
    if (dtype == KAB_BF16) launch_fp4_fmt<kBF16, true>(fmt, mode, maxc, grid, threads, s, x, ldx, up, ldu, rows, k, amax, tensor_scale, swizzle, q, scales, outer, h);
    else launch_fp4_fmt<kF16, true>(fmt, mode, maxc, grid, threads, s, x, ldx, up, ldu, rows, k, amax, tensor_scale, swizzle, q, scales, outer, h);
  } else {
    if (dtype == KAB_BF16) launch_fp4_fast<kBF16>(fmt, mode, maxc, grid, threads, s, x, ldx, k, amax, tensor_scale, swizzle, q, scales, outer);
    else if (dtype == KAB_F16) launch_fp4_fast<kF16>(fmt, mode, maxc, grid, threads, s, x, ldx, k, amax, tensor_scale, swizzle, q, scales, outer);
    else launch_fp4_fmt<kF32, false>(fmt, mode, maxc, grid, threads, s, x, ldx, nullptr, 0, rows, k, amax, tensor_scale, swizzle, q, scales, outer, nullptr);
  }
  return check_launch("kab_quant_fp4");
}

int kab_rmsnorm_quant_fp4(const void* x, int dtype, int64_t rows, int64_t k, int64_t ldx, const void* weight,
                          float eps, int fmt, int swizzle, uint8_t* q, uint8_t* scales, float* outer, void* h,
                          void* stream) {
  if (int e = check_matrix(x, dtype, rows, k, ldx, "x")) return e;
  KAB_REQUIRE(dtype != KAB_F32, "the fused RMSNorm FP4 producer takes bf16 or fp16 (fp32: kab_rmsnorm, then kab_quant_fp4)");
  KAB_REQUIRE(fmt == KAB_NVFP4 || fmt == KAB_MXFP4, "fmt %d is not NVFP4 (0) or MXFP4 (1)", fmt);
  const int block = fmt == KAB_NVFP4 ? 16 : 32;
  KAB_REQUIRE(k % block == 0, "width %lld is not a multiple of the block (%d)", (long long)k, block);
  KAB_REQUIRE(k <= 32768, "width %lld exceeds the register-resident row (32768)", (long long)k);
  KAB_REQUIRE(rows == 0 || (weight != nullptr && aligned(weight, 16)), "weight is null or not 16-byte aligned");
  KAB_REQUIRE(h == nullptr || aligned(h, 16), "h is not 16-byte aligned");
  KAB_REQUIRE(rows == 0 || (q != nullptr && scales != nullptr && outer != nullptr && aligned(q, block / 2)),
              "outputs are null or misaligned");
  KAB_REQUIRE(eps >= 0.0f, "eps must be non-negative");
  if (rows == 0 || k == 0) return KAB_OK;
  KAB_REQUIRE(rows < (int64_t(1) << 31), "too many rows (%lld)", (long long)rows);
  // at least 128 threads, more (a multiple of 32) where the row needs them at 4 (NVFP4) or 2
  // (MXFP4) blocks each: x [16384, 4096] bf16 ran in 81 us at 128 threads x 2 blocks per
  // row, 88 us at 64 x 4 and 102 us at 256 x 1 (one B200, the same box)
  const int64_t nblk = k / block;
  const int nb_max = fmt == KAB_NVFP4 ? 4 : 2;
  const int threads = max(128, static_cast<int>(((nblk + nb_max - 1) / nb_max + 31) / 32 * 32));
  const int64_t per = (nblk + threads - 1) / threads;
  const int maxc = per <= 1 ? 1 : per <= 2 ? 2 : 4;
  const cudaStream_t s = as_stream(stream);
  const unsigned grid = static_cast<unsigned>(rows);
#define KAB_RF4(TT)                                                                                     \
  (fmt == KAB_NVFP4 ? launch_rmsnorm_fp4<TT, 0>(maxc, grid, threads, s, x, ldx, k, weight, eps, swizzle, q, scales, outer, h) \
                    : launch_rmsnorm_fp4<TT, 1>(maxc, grid, threads, s, x, ldx, k, weight, eps, swizzle, q, scales, outer, h))
  const int e = dtype == KAB_BF16 ? KAB_RF4(kBF16) : KAB_RF4(kF16);
#undef KAB_RF4
  if (e) return e;
  return check_launch("kab_rmsnorm_quant_fp4");
}

int kab_amax(const void* x, int dtype, int64_t rows, int64_t k, int64_t ldx, float* out,
             void* stream) {
  KAB_REQUIRE(valid_dtype(dtype), "unknown dtype %d", dtype);
  KAB_REQUIRE(rows >= 0 && k >= 0 && ldx >= k, "bad shape");
  KAB_REQUIRE(out != nullptr && (rows * k == 0 || x != nullptr), "null pointer");
  if (rows * k == 0) return KAB_OK;
  const int threads = 256;
  const int grid = grid_for(rows * k / 8 + 1, threads);
  const cudaStream_t s = as_stream(stream);
  if (dtype == KAB_BF16) amax_kernel<kBF16><<<grid, threads, 0, s>>>(x, ldx, rows, k, out);
  else if (dtype == KAB_F16) amax_kernel<kF16><<<grid, threads, 0, s>>>(x, ldx, rows, k, out);
  else amax_kernel<kF32><<<grid, threads, 0, s>>>(x, ldx, rows, k, out);
  return check_launch("kab_amax");
}

int kab_fp4_tensor_scale(const float* amax, float* tensor_scale, void* stream) {
  KAB_REQUIRE(amax != nullptr && tensor_scale != nullptr, "null pointer");
  fp4_tensor_scale_kernel<<<1, 1, 0, as_stream(stream)>>>(amax, tensor_scale);
  return check_launch("kab_fp4_tensor_scale");
}

int kab_mx_exponents(const float* amax, int64_t n, int rule, int32_t* out, void* stream) {
  KAB_REQUIRE(rule == 0 || rule == 1, "rule %d is not 0 (ceil) or 1 (floor)", rule);
  KAB_REQUIRE(n >= 0, "negative count");
  if (n == 0) return KAB_OK;
  KAB_REQUIRE(amax != nullptr && out != nullptr, "null pointer");
  mx_exponents_kernel<<<grid_for(n, 256), 256, 0, as_stream(stream)>>>(amax, n, rule, out);
  return check_launch("kab_mx_exponents");
}

int kab_swizzle_scales(const uint8_t* scales, int64_t rows, int64_t cols, uint8_t* out,
                       void* stream) {
  KAB_REQUIRE(rows >= 0 && cols >= 0, "negative shape");
  if (rows * cols == 0) return KAB_OK;
  KAB_REQUIRE(scales != nullptr && out != nullptr, "null pointer");
  const int grid = grid_for(rows * cols, 256);
  swizzle_scales_kernel<<<grid, 256, 0, as_stream(stream)>>>(scales, rows, cols, out);
  return check_launch("kab_swizzle_scales");
}

int kab_fp4_values(const uint8_t* codes, const uint8_t* scales, int64_t rows, int64_t k,
                   int fmt, float* out, void* stream) {
  KAB_REQUIRE(fmt == KAB_NVFP4 || fmt == KAB_MXFP4, "fmt %d is not NVFP4 (0) or MXFP4 (1)", fmt);
  const int block = fmt == KAB_NVFP4 ? 16 : 32;
  KAB_REQUIRE(rows >= 0 && k >= 0 && k % block == 0, "bad shape [%lld, %lld]", (long long)rows, (long long)k);
  if (rows * k == 0) return KAB_OK;
  KAB_REQUIRE(codes != nullptr && scales != nullptr && out != nullptr, "null pointer");
  const int grid = grid_for(rows * k, 256);
  fp4_values_kernel<<<grid, 256, 0, as_stream(stream)>>>(codes, scales, rows, k, fmt, out);
  return check_launch("kab_fp4_values");
}

int kab_mxfp8_saturation(const void* x, int dtype, int64_t rows, int64_t k, int64_t ldx,
                         const float* step, KabScaleCheck* result, void* stream) {
  if (int e = check_matrix(x, dtype, rows, k, ldx, "x")) return e;
  KAB_REQUIRE(k % 32 == 0, "width %lld is not a multiple of the MXFP8 block (32)", (long long)k);
  KAB_REQUIRE(result != nullptr && (rows == 0 || step != nullptr), "null pointer");
  const cudaStream_t s = as_stream(stream);
  if (cudaMemsetAsync(result, 0, sizeof(KabScaleCheck), s) != cudaSuccess) return check_launch("check reset");
  const int64_t total = rows * (k / 32);
  if (total == 0) return KAB_OK;
  const int grid = grid_for(total, 256);
  if (dtype == KAB_BF16) mxfp8_saturation_kernel<kBF16><<<grid, 256, 0, s>>>(x, ldx, rows, k / 32, step, result);
  else if (dtype == KAB_F16) mxfp8_saturation_kernel<kF16><<<grid, 256, 0, s>>>(x, ldx, rows, k / 32, step, result);
  else mxfp8_saturation_kernel<kF32><<<grid, 256, 0, s>>>(x, ldx, rows, k / 32, step, result);
  return check_launch("kab_mxfp8_saturation");
}

int kab_fp4_scale_check(const void* x, int dtype, int64_t rows, int64_t k, int64_t ldx, int fmt,
                        const float* scale, const float* outer, int outer_per_row,
                        KabScaleCheck* result, void* stream) {
  if (int e = check_matrix(x, dtype, rows, k, ldx, "x")) return e;
  KAB_REQUIRE(fmt == KAB_NVFP4 || fmt == KAB_MXFP4, "fmt %d is not NVFP4 (0) or MXFP4 (1)", fmt);
  const int block = fmt == KAB_NVFP4 ? 16 : 32;
  KAB_REQUIRE(k % block == 0, "width %lld is not a multiple of the block (%d)", (long long)k, block);
  KAB_REQUIRE(result != nullptr && (rows == 0 || scale != nullptr), "null pointer");
  const cudaStream_t s = as_stream(stream);
  if (cudaMemsetAsync(result, 0, sizeof(KabScaleCheck), s) != cudaSuccess) return check_launch("check reset");
  const int64_t nb = k / block, total = rows * nb;
  if (total == 0) return KAB_OK;
  const int grid = grid_for(total, 256);
#define KAB_CHECK(TT, F) fp4_scale_check_kernel<TT, F><<<grid, 256, 0, s>>>(x, ldx, rows, nb, scale, outer, outer_per_row, result)
#define KAB_CHECK_T(F) \
  if (dtype == KAB_BF16) KAB_CHECK(kBF16, F); else if (dtype == KAB_F16) KAB_CHECK(kF16, F); else KAB_CHECK(kF32, F)
  if (fmt == KAB_NVFP4) { KAB_CHECK_T(0); } else { KAB_CHECK_T(1); }
#undef KAB_CHECK_T
#undef KAB_CHECK
  return check_launch("kab_fp4_scale_check");
}

int kab_outlier_stats(const void* x, int dtype, int64_t rows, int64_t k, int64_t ldx, double* row_sumsq,
                      float* row_amax, float* col_amax, void* stream) {
  if (int e = check_matrix(x, dtype, rows, k, ldx, "x")) return e;
  KAB_REQUIRE(rows == 0 || k == 0 || (row_sumsq != nullptr && row_amax != nullptr && col_amax != nullptr),
              "null output");
  KAB_REQUIRE(rows <= static_cast<int64_t>(kOutlierRows) * 65535, "too many rows (%lld)", (long long)rows);
  const cudaStream_t s = as_stream(stream);
  if (rows > 0 && (cudaMemsetAsync(row_sumsq, 0, rows * sizeof(double), s) != cudaSuccess ||
                   cudaMemsetAsync(row_amax, 0, rows * sizeof(float), s) != cudaSuccess))
    return check_launch("outlier stats reset");
  if (k > 0 && cudaMemsetAsync(col_amax, 0, k * sizeof(float), s) != cudaSuccess)
    return check_launch("outlier stats reset");
  if (rows == 0 || k == 0) return KAB_OK;
  const dim3 grid(static_cast<unsigned>((k + 2047) / 2048), static_cast<unsigned>((rows + kOutlierRows - 1) / kOutlierRows));
  auto* rm = reinterpret_cast<unsigned*>(row_amax);
  auto* cm = reinterpret_cast<unsigned*>(col_amax);
  if (dtype == KAB_BF16) outlier_stats_kernel<kBF16><<<grid, 256, 0, s>>>(x, ldx, rows, k, row_sumsq, rm, cm);
  else if (dtype == KAB_F16) outlier_stats_kernel<kF16><<<grid, 256, 0, s>>>(x, ldx, rows, k, row_sumsq, rm, cm);
  else outlier_stats_kernel<kF32><<<grid, 256, 0, s>>>(x, ldx, rows, k, row_sumsq, rm, cm);
  return check_launch("kab_outlier_stats");
}

int kab_row_pair_stats(const void* x, int x_dtype, int64_t ldx, const void* y, int y_dtype, int64_t ldy,
                       int64_t rows, int64_t k, double* out, void* stream) {
  KAB_REQUIRE(valid_dtype(x_dtype) && valid_dtype(y_dtype), "unknown dtype %d / %d", x_dtype, y_dtype);
  KAB_REQUIRE(rows >= 0 && k >= 0, "negative shape");
  if (rows == 0) return KAB_OK;
  KAB_REQUIRE(out != nullptr && (k == 0 || (x != nullptr && y != nullptr)), "null pointer");
  KAB_REQUIRE(ldx >= k && ldy >= k, "row strides %lld / %lld are below the width %lld", (long long)ldx,
              (long long)ldy, (long long)k);
  KAB_REQUIRE(rows < (int64_t(1) << 31), "too many rows");
  const cudaStream_t s = as_stream(stream);
  const dim3 grid(static_cast<unsigned>(rows));
#define KAB_PAIR(TXX, TYY)                                                                                     \
  row_pair_stats_kernel<TXX, TYY><<<grid, 256, 0, s>>>(static_cast<const TXX*>(x), ldx, static_cast<const TYY*>(y), \
                                                       ldy, k, out)
#define KAB_PAIR_Y(TXX)                                     \
  if (y_dtype == KAB_F32) KAB_PAIR(TXX, float);             \
  else if (y_dtype == KAB_BF16) KAB_PAIR(TXX, __nv_bfloat16); \
  else KAB_PAIR(TXX, __half)
  if (x_dtype == KAB_F32) { KAB_PAIR_Y(float); }
  else if (x_dtype == KAB_BF16) { KAB_PAIR_Y(__nv_bfloat16); }
  else { KAB_PAIR_Y(__half); }
#undef KAB_PAIR_Y
#undef KAB_PAIR
  return check_launch("kab_row_pair_stats");
}

int kab_rmsnorm(const void* x, int dtype, int64_t rows, int64_t k, int64_t ldx, const void* weight, float eps,
                void* out, void* stream) {
  if (int e = check_matrix(x, dtype, rows, k, ldx, "x")) return e;
  KAB_REQUIRE(k % 8 == 0, "the last dimension %lld is not a multiple of 8", (long long)k);
  KAB_REQUIRE(rows == 0 || (weight != nullptr && out != nullptr && aligned(weight, 16) && aligned(out, 16)),
              "weight or out is null or not 16-byte aligned");
  KAB_REQUIRE(eps >= 0.0f, "eps must be non-negative");
  if (rows == 0 || k == 0) return KAB_OK;
  const cudaStream_t s = as_stream(stream);
  const unsigned grid = static_cast<unsigned>(rows);
  if (dtype == KAB_BF16) rmsnorm_rows_kernel<kBF16><<<grid, 256, 0, s>>>(x, ldx, k, weight, eps, out);
  else if (dtype == KAB_F16) rmsnorm_rows_kernel<kF16><<<grid, 256, 0, s>>>(x, ldx, k, weight, eps, out);
  else rmsnorm_rows_kernel<kF32><<<grid, 256, 0, s>>>(x, ldx, k, weight, eps, out);
  return check_launch("kab_rmsnorm");
}

int kab_rmsnorm_quant_fp8(const void* x, int dtype, int64_t rows, int64_t k, int64_t ldx, const void* weight,
                          float eps, int mx, int swizzle, uint8_t* q, void* scales, void* h, void* stream) {
  if (int e = check_matrix(x, dtype, rows, k, ldx, "x")) return e;
  KAB_REQUIRE(k % (mx ? 32 : 8) == 0, "the last dimension %lld is not a multiple of %d", (long long)k, mx ? 32 : 8);
  KAB_REQUIRE(k <= 16384, "rows of %lld elements exceed the fused kernel's 16384 (use kab_rmsnorm, then quantise)",
              (long long)k);
  KAB_REQUIRE(rows == 0 || (weight != nullptr && aligned(weight, 16) && q != nullptr && aligned(q, 8) &&
                            scales != nullptr),
              "weight, q or scales is null or misaligned");
  KAB_REQUIRE(h == nullptr || aligned(h, 16), "h is not 16-byte aligned");
  KAB_REQUIRE(eps >= 0.0f, "eps must be non-negative");
  if (rows == 0 || k == 0) return KAB_OK;
  KAB_REQUIRE(rows < (int64_t(1) << 31), "too many rows (%lld)", (long long)rows);
  const int64_t per = (k / 8 + 255) / 256;
  const int maxc = per <= 1 ? 1 : per <= 2 ? 2 : per <= 4 ? 4 : 8;
  const cudaStream_t s = as_stream(stream);
  const unsigned grid = static_cast<unsigned>(rows);
#define KAB_RQ(TT, MC, M) \
  rmsnorm_quant_fp8_kernel<TT, MC, M><<<grid, 256, 0, s>>>(x, ldx, k, weight, eps, swizzle, q, scales, h)
#define KAB_RQ_M(TT, MC) \
  if (mx) KAB_RQ(TT, MC, 1); else KAB_RQ(TT, MC, 0)
#define KAB_RQ_C(TT)                               \
  switch (maxc) {                                  \
    case 1: KAB_RQ_M(TT, 1); break;                \
    case 2: KAB_RQ_M(TT, 2); break;                \
    case 4: KAB_RQ_M(TT, 4); break;                \
    default: KAB_RQ_M(TT, 8); break;               \
  }
  if (dtype != KAB_F32) {
    // 2-byte rows: the packed kernel, 128 threads per row up to 8 chunks each, 256 beyond
    // (x [16384, 4096] bf16: 81 us at 128 threads x 4 chunks, 85 us at 64 x 8, 88 us at
    // 256 x 2; one B200, the same box)
    const int64_t chunks = k / 8;
    const int nt = chunks <= 1024 ? 128 : 256;
    const int64_t pc = (chunks + nt - 1) / nt;
    const int nc = pc <= 1 ? 1 : pc <= 2 ? 2 : pc <= 4 ? 4 : 8;
#define KAB_RP(TT, NC, NT)                                                                                     \
  do {                                                                                                         \
    if (mx) rmsnorm_quant_fp8_packed_kernel<TT, NC, 1, NT><<<grid, NT, 0, s>>>(x, ldx, k, weight, eps, swizzle, q, scales, h); \
    else rmsnorm_quant_fp8_packed_kernel<TT, NC, 0, NT><<<grid, NT, 0, s>>>(x, ldx, k, weight, eps, swizzle, q, scales, h); \
  } while (0)
#define KAB_RP_T(TT)                          \
  if (nt == 256) KAB_RP(TT, 8, 256);          \
  else if (nc == 8) KAB_RP(TT, 8, 128);       \
  else if (nc == 4) KAB_RP(TT, 4, 128);       \
  else if (nc == 2) KAB_RP(TT, 2, 128);       \
  else KAB_RP(TT, 1, 128)
    if (dtype == KAB_BF16) { KAB_RP_T(kBF16); }
    else { KAB_RP_T(kF16); }
#undef KAB_RP_T
#undef KAB_RP
  } else {
    KAB_RQ_C(kF32)
  }
#undef KAB_RQ_C
#undef KAB_RQ_M
#undef KAB_RQ
  return check_launch("kab_rmsnorm_quant_fp8");
}

int kab_hadamard_rotate(const void* x, int dtype, int64_t rows, int64_t k, int64_t ldx, int block, float* out,
                        void* stream) {
  KAB_REQUIRE(valid_dtype(dtype), "unknown dtype %d", dtype);
  KAB_REQUIRE(rows >= 0 && k >= 0 && ldx >= k, "bad shape [%lld, %lld] (ld %lld)", (long long)rows, (long long)k,
              (long long)ldx);
  KAB_REQUIRE(block >= 1 && (block & (block - 1)) == 0, "the Hadamard order must be a power of two, got %d", block);
  KAB_REQUIRE(k % block == 0, "the last dimension %lld is not a multiple of the rotation (%d)", (long long)k, block);
  KAB_REQUIRE(k <= 32768, "rows of %lld elements exceed the shared-memory row (32768)", (long long)k);
  KAB_REQUIRE(rows == 0 || (x != nullptr && out != nullptr), "null pointer");
  if (rows == 0 || k == 0) return KAB_OK;
  const size_t smem = static_cast<size_t>(k) * sizeof(float);
  const float inv = static_cast<float>(1.0 / sqrt(static_cast<double>(block)));
  const cudaStream_t s = as_stream(stream);
#define KAB_HAD(TT)                                                                                   \
  do {                                                                                                \
    cudaFuncSetAttribute(hadamard_rotate_kernel<TT>, cudaFuncAttributeMaxDynamicSharedMemorySize, 32768 * 4); \
    hadamard_rotate_kernel<TT><<<static_cast<unsigned>(rows), 512, smem, s>>>(x, ldx, k, block, inv, out); \
  } while (0)
  if (dtype == KAB_BF16) KAB_HAD(kBF16);
  else if (dtype == KAB_F16) KAB_HAD(kF16);
  else KAB_HAD(kF32);
#undef KAB_HAD
  return check_launch("kab_hadamard_rotate");
}

int kab_fp4_bias_correction(const void* x, int dtype, int64_t rows, int64_t k, int64_t ldx, const uint8_t* codes,
                            const uint8_t* scales, int fmt, int swizzled, const float* outer, int outer_per_row,
                            float* out, void* stream) {
  if (int e = check_matrix(x, dtype, rows, k, ldx, "x")) return e;
  KAB_REQUIRE(fmt == KAB_NVFP4 || fmt == KAB_MXFP4, "fmt %d is not NVFP4 (0) or MXFP4 (1)", fmt);
  const int block = fmt == KAB_NVFP4 ? 16 : 32;
  KAB_REQUIRE(k % block == 0, "width %lld is not a multiple of the block (%d)", (long long)k, block);
  KAB_REQUIRE(rows == 0 || (codes != nullptr && scales != nullptr && out != nullptr), "null pointer");
  if (rows == 0) return KAB_OK;
  const cudaStream_t s = as_stream(stream);
  const unsigned grid = static_cast<unsigned>(rows);
  if (dtype == KAB_BF16) fp4_bias_correction_kernel<kBF16><<<grid, 256, 0, s>>>(x, ldx, k, codes, scales, fmt, swizzled, outer, outer_per_row, out);
  else if (dtype == KAB_F16) fp4_bias_correction_kernel<kF16><<<grid, 256, 0, s>>>(x, ldx, k, codes, scales, fmt, swizzled, outer, outer_per_row, out);
  else fp4_bias_correction_kernel<kF32><<<grid, 256, 0, s>>>(x, ldx, k, codes, scales, fmt, swizzled, outer, outer_per_row, out);
  return check_launch("kab_fp4_bias_correction");
}

}  // extern "C"
