/*
 * kab.h: the C ABI of the B200-native low-precision library (libkab.so).
 *
 * It replaces the numeric core of kernel-agent's low-precision path: the quantisers and
 * scaled linears of src/kernel_agent/kernels/quant.py, the research blockwise / FP8
 * attention math of docs/research-scripts/fp8-sm120/fp8lib.py, and the element loop of the
 * comparator src/kernel_agent/kernels/compare.py:631-790. Each entry point below names the
 * reference function it stands in for.
 *
 * Conventions
 *  - Plain device pointers, element counts and strides (in elements); matrices are
 *    row-major with a leading dimension `ld*` >= their width. Outputs are contiguous.
 *  - `stream` is a cudaStream_t passed as void* (NULL: the legacy default stream). Every
 *    call is asynchronous on it: no host synchronisation, no allocation, so the calls can
 *    be captured in a CUDA graph.
 *  - The return value is a KAB_* status. On failure kab_last_error() gives the reason
 *    (thread-local). Arguments are validated before any launch.
 *  - Floating-point inputs are fp32, bf16 or fp16 (KAB_F32 / KAB_BF16 / KAB_F16).
 *  - FP8 codes are e4m3fn bytes, MX scales e8m0 bytes (exponent + 127), NVFP4 block scales
 *    e4m3fn bytes, FP4 codes two e2m1 per byte with the even element in the low nibble.
 *  - "Swizzled" scales use the 128 x 4 blocked layout of cuBLASLt (quant.py:540-564,
 *    mx_scale_offset): rows padded to 128, columns to 4, blocks of 512 bytes; the caller
 *    provides a zeroed buffer of that padded size when padding exists.
 */
#ifndef KAB_H_
#define KAB_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------------ status */

#define KAB_OK 0
#define KAB_EINVAL 1       /* an argument is out of range, misaligned or null */
#define KAB_EUNSUPPORTED 2 /* no sm_100 device, or a shape this build does not handle */
#define KAB_ECUDA 3        /* the CUDA runtime reported an error (launch, attribute, ...) */
#define KAB_ETIMEOUT 4     /* a device-side wait gave up (see kab_device_status) */

#define KAB_F32 0
#define KAB_BF16 1
#define KAB_F16 2

/* The message of the last failing call on this thread ("" when none). */
const char* kab_last_error(void);
/* The library's ABI version (KAB_ABI_VERSION). */
int kab_abi_version(void);
#define KAB_ABI_VERSION 1
/* KAB_OK when `device` is an sm_100 GPU this build runs on. */
int kab_device_check(int device);
/* Error bits kernels raised on the current device since the last clear (1: a wait timed
 * out, 2: an index check failed); synchronises the stream. `clear` resets them. */
int kab_device_status(unsigned* bits, int clear, void* stream);

/* ------------------------------------------------------------------ producers */

/* Per-row INT8: scale = amax * fp32(1/127) (1 for a zero row), codes round(v / scale) to
 * nearest even clamped to +-127. smooth_mode 0: v = x; 1: v = x / smooth[col]
 * (activations, quant.py:823-839 quantize_int8_activations); 2: v = x * smooth[col]
 * (weights, quant.py:794-813 quantize_int8). k % 8 == 0, 16-byte aligned rows. */
int kab_quant_rows_int8(const void* x, int dtype, int64_t rows, int64_t k, int64_t ldx,
                        const float* smooth, int smooth_mode, int8_t* q, float* scale,
                        void* stream);

/* Per-row FP8 e4m3: scale = amax / 448 (1 for a zero row), codes (v / scale) clamped to
 * +-448, nearest even (quant.py:361-377 quantize_fp8_activations, quant.py:101-119
 * quantize_fp8). With `up` non-null the row is silu(x) * up in x's dtype, and `h` (nullable,
 * x's dtype, [rows, k]) receives it (triton_fp8_producers.py:136-147). */
int kab_quant_rows_fp8(const void* x, int dtype, int64_t rows, int64_t k, int64_t ldx,
                       const void* up, int64_t ldu, uint8_t* q, float* scale, void* h,
                       void* stream);

/* FP8 per 1 x group along rows (group 32, 64 or 128): scale = amax / 448, 0 -> 1, scales
 * fp32 [rows, k / group] (fp8lib.py:22-27 fq_groups). */
int kab_quant_groups_fp8(const void* x, int dtype, int64_t rows, int64_t k, int64_t ldx,
                         int group, uint8_t* q, float* scales, void* stream);

/* FP8 per 128 x 128 block of a weight [n, k]: scales fp32 [n / 128, k / 128]
 * (fp8lib.py:35-39 fq_block). */
int kab_quant_blocks_fp8(const void* w, int dtype, int64_t n, int64_t k, int64_t ldw,
                         uint8_t* q, float* scales, void* stream);

/* MXFP8: per block of 32 along rows, e = the rule's exponent (rule 0: ceil
 * 2^ceil(log2(amax / 448)), 1: floor, the OCP rule), codes (v / 2^e) clamped to +-448,
 * scale byte e + 127, row-major [rows, k / 32] or swizzled (quant.py:479-526
 * mx_scale_exponents / quantize_mxfp8). `up`, `h`: the fused SiLU * up producer. */
int kab_quant_mxfp8(const void* x, int dtype, int64_t rows, int64_t k, int64_t ldx,
                    const void* up, int64_t ldu, int rule, uint8_t* q, uint8_t* scales,
                    int swizzle, void* h, void* stream);

#define KAB_NVFP4 0
#define KAB_MXFP4 1
#define KAB_FP4_TOKEN 0  /* activations, outer scale per row */
#define KAB_FP4_TENSOR 1 /* activations, one outer scale per call (from *amax) */
#define KAB_FP4_WEIGHT 2 /* a weight with its tensor scale *tensor_scale */

/* FP4 activations (quant.py:1056-1107 quantize_fp4_activations) or weights (quant.py:217-272
 * quantize_fp4): codes [rows, k / 2], block scales [rows, k / block] row-major or swizzled,
 * outer fp32 [rows] (nullable). mode KAB_FP4_TENSOR reads the call's amax from *amax
 * (kab_amax); KAB_FP4_WEIGHT reads *tensor_scale (kab_fp4_tensor_scale). `up`, `h`: the
 * fused SiLU * up producer (triton_fp4_producers.py:297-328). */
int kab_quant_fp4(const void* x, int dtype, int64_t rows, int64_t k, int64_t ldx,
                  const void* up, int64_t ldu, int fmt, int mode, const float* amax,
                  const float* tensor_scale, uint8_t* q, uint8_t* scales, int swizzle,
                  float* outer, void* h, void* stream);

/* NaN-keeping max |x| of a [rows, k] matrix into *out, which must hold 0 (or a smaller
 * value to fold in) before the call. */
int kab_amax(const void* x, int dtype, int64_t rows, int64_t k, int64_t ldx, float* out,
             void* stream);

/* The NVFP4 weight tensor scale fp32(double(*amax) / 2688), 1 for 0 (quant.py:253-254). */
int kab_fp4_tensor_scale(const float* amax, float* tensor_scale, void* stream);

/* The unbiased exponents (int32, clamped to [-127, 127], -127 for 0) of block maxima
 * amax[n] under rule 0 (ceil) or 1 (floor) (quant.py:479-495 mx_scale_exponents). */
int kab_mx_exponents(const float* amax, int64_t n, int rule, int32_t* out, void* stream);

/* [rows, cols] scale bytes into the swizzled layout (quant.py:550-564 swizzle_mx_scales,
 * 1176-1182 swizzle_fp4_scales); `out` is zeroed by the caller where padding exists. */
int kab_swizzle_scales(const uint8_t* scales, int64_t rows, int64_t cols, uint8_t* out,
                       void* stream);

/* Exact fp32 e2m1 * block scale [rows, k] of FP4 codes (quant.py:1110-1114 fp4_values). */
int kab_fp4_values(const uint8_t* codes, const uint8_t* scales, int64_t rows, int64_t k,
                   int fmt, float* out, void* stream);

/* ------------------------------------------------------------------ scaled GEMMs (tcgen05) */

/* A [m, k] and B [n, k] are K-major (row-major, K contiguous; B is an nn.Linear weight),
 * 16-byte aligned, with k * (bytes per element) a positive multiple of 128. The output
 * [m, ldo] (ldo >= n, a multiple of 8) is bf16 / fp16 / fp32 (out_dtype); `bias` (nullable,
 * [n], bias_dtype) is added in the epilogue. One persistent CTA per SM. */

/* int8 x int8 -> exact int32 (kind::i8). With acc_out non-null: the raw int32 products
 * [m, ldo] (quant.py:854-885 int8_matmul); else out = acc * a_scale[m] * b_scale[n]
 * (+ bias) in fp32, one rounding (quant.py:901-923 int8_w8a8_linear's epilogue). */
int kab_gemm_i8(const int8_t* a, const int8_t* b, int64_t m, int64_t n, int64_t k,
                const float* a_scale, const float* b_scale, const void* bias, int bias_dtype,
                void* out, int out_dtype, int64_t ldo, int32_t* acc_out, void* stream);

/* e4m3 x e4m3 -> fp32 (kind::f8f6f4); out = acc * a_scale[m] * b_scale[n] (+ bias)
 * (quant.py:390-417 fp8_w8a8_linear, torch._scaled_mm with row-wise scales). */
int kab_gemm_f8(const uint8_t* a, const uint8_t* b, int64_t m, int64_t n, int64_t k,
                const float* a_scale, const float* b_scale, const void* bias, int bias_dtype,
                void* out, int out_dtype, int64_t ldo, void* stream);

/* kab_gemm_nvf4 whose epilogue also writes every output tile into `npeers` (<= 7) other
 * buffers of the same layout (peer_out[p]: the [m, ldo] origin in another rank's output,
 * mapped by kab_ipc_open) with 16-byte stores over NVLink; columns past n are not written.
 * The caller orders the peers' uses of those buffers (a barrier before and after). */
int kab_gemm_nvf4_scatter(const uint8_t* a, const uint8_t* a_sf, const float* a_outer, const uint8_t* b,
                          const uint8_t* b_sf, const float* b_scale, int b_scale_per_col, int64_t m,
                          int64_t n, int64_t k, const void* bias, int bias_dtype, void* out, int out_dtype,
                          int64_t ldo, void* const* peer_out, int npeers, void* stream);

/* MXFP4: packed e2m1 A [m, k / 2], B [n, k / 2] with e8m0 scales per 32 along K (swizzled),
 * applied by the tensor core (kind::mxf4nvf4.block_scale.scale_vec::2X); out = acc * (outer[m]
 * * ts) (+ bias), outer = a_outer[m] or 1 (null: MXFP4 activations), ts = b_scale[0],
 * b_scale[n] (b_scale_per_col) or 1 (null) (quant.py:1201-1257 fp4_w4a4_linear, fmt
 * "mxfp4"). k % 256 == 0. */
int kab_gemm_mxf4(const uint8_t* a, const uint8_t* a_sf, const float* a_outer, const uint8_t* b,
                  const uint8_t* b_sf, const float* b_scale, int b_scale_per_col, int64_t m, int64_t n,
                  int64_t k, const void* bias, int bias_dtype, void* out, int out_dtype, int64_t ldo,
                  void* stream);

/* Blockwise FP8: e4m3 A [m, k] with fp32 scales a_scale [m, k / 128] (1 x 128 groups), e4m3
 * B [n, k] with fp32 scales b_scale [n / 128, k / 128] (128 x 128 blocks); out = sum over
 * 128-wide K steps of (partial * a_scale[m, kb]) * b_scale[n / 128, kb] in fp32 (+ bias), one
 * rounding to out_dtype (docs/research-scripts/fp8-sm120/gemm_bench.py:39-68, the promotion
 * of the blockwise recipe; F.scaled_mm BlockWise1x128 / BlockWise128x128 on the GPU).
 * k % 128 == 0, n % 128 == 0. */
int kab_gemm_f8_blockwise(const uint8_t* a, const float* a_scale, const uint8_t* b,
                          const float* b_scale, int64_t m, int64_t n, int64_t k, const void* bias,
                          int bias_dtype, void* out, int out_dtype, int64_t ldo, void* stream);

/* MXFP8: e4m3 with e8m0 scales per 32 along K on both operands (swizzled layout), applied
 * by the tensor core (kind::mxf8f6f4.block_scale); out = round(acc) (+ bias) in out_dtype
 * (quant.py:581-620 mxfp8_linear, F.scaled_mm BlockWise1x32 then + bias). n % 128 == 0. */
int kab_gemm_mxf8(const uint8_t* a, const uint8_t* a_sf, const uint8_t* b, const uint8_t* b_sf,
                  int64_t m, int64_t n, int64_t k, const void* bias, int bias_dtype, void* out,
                  int out_dtype, int64_t ldo, void* stream);

/* NVFP4 W4A4: packed e2m1 A [m, k/2], B [n, k/2] with e4m3 scales per 16 (swizzled), applied
 * by the tensor core (kind::mxf4nvf4.block_scale.scale_vec::4X), fp32 accumulation;
 * out = acc * (a_outer[m] * b_scale[0 or n]) (+ bias) in fp32, one rounding
 * (quant.py:1201-1257 fp4_w4a4_linear). k % 256 == 0, n % 128 == 0. */
int kab_gemm_nvf4(const uint8_t* a, const uint8_t* a_sf, const float* a_outer, const uint8_t* b,
                  const uint8_t* b_sf, const float* b_scale, int b_scale_per_col, int64_t m,
                  int64_t n, int64_t k, const void* bias, int bias_dtype, void* out,
                  int out_dtype, int64_t ldo, void* stream);

/* ------------------------------------------------------------------ comparator */

/* Count slots of KabCompareResult.count */
#define KAB_CMP_NAN_REF 0
#define KAB_CMP_NAN_NEW 1
#define KAB_CMP_NAN_DIFF 2
#define KAB_CMP_PINF_REF 3
#define KAB_CMP_PINF_NEW 4
#define KAB_CMP_PINF_DIFF 5
#define KAB_CMP_NINF_REF 6
#define KAB_CMP_NINF_NEW 7
#define KAB_CMP_NINF_DIFF 8
#define KAB_CMP_FINITE 9
#define KAB_CMP_MISMATCH 10
#define KAB_CMP_NCOUNT 11
/* Sum slots (float64, over the finite elements of ref; RR over both-finite (ref, alt)) */
#define KAB_CMP_SUM_AA 0
#define KAB_CMP_SUM_BB 1
#define KAB_CMP_SUM_AB 2
#define KAB_CMP_SUM_DD 3
#define KAB_CMP_SUM_D 4
#define KAB_CMP_SUM_RR 5
#define KAB_CMP_NSUM 6
/* Max slots (fp32): |a - b|, |a - b| / allowed, the element ratio */
#define KAB_CMP_MAX_D 0
#define KAB_CMP_MAX_RATIO 1
#define KAB_CMP_MAX_ELEMENT 2
#define KAB_CMP_NMAX 3

typedef struct KabCompareResult {
  long long count[KAB_CMP_NCOUNT];
  double sum[KAB_CMP_NSUM];
  float max[KAB_CMP_NMAX];
  float pad_;
} KabCompareResult;

/* One pass of compare_tensors' element loop (compare.py:684-739) over `n` elements of
 * ref / new (and rerounded when has_rerounded). With a = ref[i], b = new[i], d = |a - b|
 * in fp32 and the reference's roundings:
 *   allowed = atol + rtol * |a|                      (compare.py:698)
 *   alt_bound:    allowed = max(allowed, alt_atol + alt_rtol * |a|)    (699-700)
 *   widen_mode 1: allowed += widen_scalar; 2: allowed += widen_channel[i % channels] (713)
 *   element_mode 1: den = element_first + element_rtol * |a|;
 *                2: den = element_atol * element_scale[i % channels] + element_rtol * |a| (739)
 * `vector` selects 16-byte loads (ref / new / rerounded 16-byte aligned). */
typedef struct KabCompareParams {
  const void* ref;
  const void* new_;
  const void* rerounded;
  int64_t n;
  int64_t channels;
  int dtype;
  int has_rerounded;
  int vector;
  int alt_bound;
  float atol, rtol;
  float alt_atol, alt_rtol;
  int widen_mode;
  float widen_scalar;
  const float* widen_channel;
  int element_mode;
  float element_first, element_atol, element_rtol;
  const float* element_scale;
} KabCompareParams;

/* Bytes of scratch kab_compare needs (device memory the caller provides). */
size_t kab_compare_scratch_bytes(int64_t n);
/* The element loop into *result (device). `scratch`: kab_compare_scratch_bytes(n) bytes. */
int kab_compare(const KabCompareParams* params, void* scratch, size_t scratch_bytes,
                KabCompareResult* result, void* stream);
/* kab_compare without caller scratch: the per-block partials live in a static device array
 * of the library (1024 slots of 152 bytes per device; enough for any `n` on a device of up to
 * 256 SMs, KAB_EINVAL beyond that). No counterpart in the reference, whose comparator runs in
 * PyTorch: it exists for callers that cannot allocate device memory when they check a result
 * (a harness judging a candidate that has just exhausted HBM, a host binding without a device
 * allocator). It allocates nothing; nothing must start at zero (each block overwrites its slot;
 * every field of *result is written). Results are bit-identical to kab_compare's. Calls overlapping on
 * one device share the array and race: order them on one stream. The first call on each device
 * looks up the array's address (cudaGetSymbolAddress, which may load the module); make it
 * before capturing a stream. */
int kab_compare_noalloc(const KabCompareParams* params, KabCompareResult* result, void* stream);

/* Per-channel RMS over the last dimension (compare.py:582-589 _channels): rms[c] =
 * sqrt(mean over rows of v^2) with v = x (non-finite as 0) or, with `alt` non-null,
 * v = alt - x where both are finite (compare.py:622-625). Scratch:
 * kab_channel_rms_scratch_bytes(rows, channels) bytes. */
size_t kab_channel_rms_scratch_bytes(int64_t rows, int64_t channels);
int kab_channel_rms(const void* x, const void* alt, int dtype, int64_t rows,
                    int64_t channels, float* rms, void* scratch, size_t scratch_bytes,
                    void* stream);

/* quant.py:1150-1173 hadamard_rotate: each `block` (a power of two) consecutive elements of
 * the rows of x [rows, k] times the orthonormal Sylvester-Hadamard matrix, fp32 out
 * [rows, k] (k <= 32768). */
int kab_hadamard_rotate(const void* x, int dtype, int64_t rows, int64_t k, int64_t ldx, int block,
                        float* out, void* stream);

/* The RMSNorm of the fused producers rmsnorm_fp8 / rmsnorm_fp4
 * (src/kernel_agent/agent/examples/triton_fp8_producers.py:120-133, 191-202;
 * triton_fp4_producers.py:261-294, 384-405): per row r = rsqrt(sum(x^2) / k + eps) in fp32,
 * out = dtype(dtype(x * r) * weight) [rows, k] (k % 8 == 0, weight [k] in x's dtype). The
 * producers then quantise out with the quantisers above, so codes and scales are exactly
 * those of out. */
int kab_rmsnorm(const void* x, int dtype, int64_t rows, int64_t k, int64_t ldx, const void* weight, float eps,
                void* out, void* stream);

/* The same RMSNorm and its FP8 quantisation in one pass over x (the fused producers of
 * triton_fp8_producers.py:120-133, 191-202): h (nullable: written when given) and the codes of
 * h, bit for bit those of kab_rmsnorm followed by kab_quant_rows_fp8 (mx 0: fp32 scales
 * [rows]) or kab_quant_mxfp8 with the ceil rule (mx 1: e8m0 bytes [rows, k / 32], in the
 * 128 x 4 swizzled layout with `swizzle`). k <= 16384 (a multiple of 8, of 32 with mx). */
int kab_rmsnorm_quant_fp8(const void* x, int dtype, int64_t rows, int64_t k, int64_t ldx,
                          const void* weight, float eps, int mx, int swizzle, uint8_t* q,
                          void* scales, void* h, void* stream);

/* The same RMSNorm and its FP4 quantisation in one pass over x (triton_fp4_producers.py:
 * 261-294, 384-405): the codes, block scales and per-row outer scales of h, bit for bit those
 * of kab_rmsnorm followed by kab_quant_fp4 with mode KAB_FP4_TOKEN (same outputs and layouts);
 * h (nullable) receives the norm's output. x bf16 or fp16, k <= 32768 (a multiple of the
 * format's block). */
int kab_rmsnorm_quant_fp4(const void* x, int dtype, int64_t rows, int64_t k, int64_t ldx,
                          const void* weight, float eps, int fmt, int swizzle, uint8_t* q,
                          uint8_t* scales, float* outer, void* h, void* stream);

/* quant.py:1117-1148 fp4_bias_correction: per row of x [rows, k] quantised to (codes,
 * scales [rows, k / block] bytes, row-major or `swizzled`, outer [rows] / one value / null),
 * c = sum x^2 / sum x x^ in float64 (1 when sum x x^ <= 0 or c is not finite); fp32 out [rows]. */
int kab_fp4_bias_correction(const void* x, int dtype, int64_t rows, int64_t k, int64_t ldx,
                            const uint8_t* codes, const uint8_t* scales, int fmt, int swizzled,
                            const float* outer, int outer_per_row, float* out, void* stream);

/* ------------------------------------------------------------------ peer output buffers */

/* CUDA IPC of a device buffer for the column-sharded GEMM (each rank writes its tiles into
 * every rank's output over NVLink). kab_ipc_handle: the 64-byte handle of the allocation that
 * holds `ptr` and ptr's byte offset in it; kab_ipc_open: that allocation mapped into this
 * process (*base; add the offset); kab_ipc_close: unmaps it. */
#define KAB_IPC_HANDLE_BYTES 64
int kab_ipc_handle(const void* ptr, void* handle, int64_t* offset);
int kab_ipc_open(const void* handle, void** base);
int kab_ipc_close(void* base);

/* ------------------------------------------------------------------ scale-rule checks */

/* What one scale-rule check found (device memory; zeroed by the call): block counts and the
 * bits of the largest block-max / step ratio (a non-negative float; NaN kept). */
typedef struct KabScaleCheck {
  unsigned long long saturated, underflow, nonfinite, not_representable, coarser, not_pow2;
  unsigned worst_ratio_bits;
  unsigned pad;
  /* kab_fp4_scale_check: blocks whose ratio exceeds 6 * (1 + 2^-20), quant.py:1260-1297
   * fp4_saturation's count */
  unsigned long long saturated_plain;
} KabScaleCheck;

/* quant.py:623-660 mxfp8_saturation: x [rows, k] against fp32 MXFP8 scale values `step`
 * [rows, k / 32] (unswizzled): saturated (ratio above 448 * (1 + 2^-10), or a zero step under a
 * non-zero block), coarser (above the ceil rule's scale), not_pow2, worst ratio. */
int kab_mxfp8_saturation(const void* x, int dtype, int64_t rows, int64_t k, int64_t ldx,
                         const float* step, KabScaleCheck* result, void* stream);

/* quant.py:1325-1416 fp4_scale_check: x [rows, k] against fp32 block-scale values `scale`
 * [rows, k / block] (fmt KAB_NVFP4: e4m3 per 16; KAB_MXFP4: e8m0 per 32) and the outer scale
 * (`outer`: [rows] with outer_per_row, else one value; null: 1): saturated, underflow,
 * nonfinite, not_representable, coarser, worst ratio. */
int kab_fp4_scale_check(const void* x, int dtype, int64_t rows, int64_t k, int64_t ldx, int fmt,
                        const float* scale, const float* outer, int outer_per_row,
                        KabScaleCheck* result, void* stream);

/* src/kernel_agent/kernels/scale_guard.py:103-118 outliers(): one pass over activations
 * x [rows, k] with non-finite values as 0: row_sumsq [rows] (float64 sums of x^2), row_amax
 * [rows] and col_amax [k] (largest |x| per row and per column). The outputs are reset here. */
int kab_outlier_stats(const void* x, int dtype, int64_t rows, int64_t k, int64_t ldx, double* row_sumsq,
                      float* row_amax, float* col_amax, void* stream);

/* Per-row sums of a pair of [rows, k] matrices x, y (x and y each fp32 / bf16 / fp16, rows
 * ldx / ldy elements apart), the reductions of the error reports (quant.py:133-181, 302-326,
 * 420-476, 707-768, 926-1000, 1511-1573; kv_quant.py:86-101): out[row * 8 + i] for
 * i = 0..7: sum x^2, sum y^2, sum (x - y)^2, sum x * y, max |x|, count(x != 0),
 * count(x != 0 and y == 0), max |y|; float64, NaN propagating. */
int kab_row_pair_stats(const void* x, int x_dtype, int64_t ldx, const void* y, int y_dtype, int64_t ldy,
                       int64_t rows, int64_t k, double* out, void* stream);

/* ------------------------------------------------------------------ comparator routing */

#define KAB_DIFF_MAXDIM 8

/* The difference census of the comparator's routing (src/kernel_agent/kernels/compare.py:
 * 806-1182: compare_grown, written_box, compare_written, compare_side_effects_flat). The
 * compared region is [outer, len, inner] elements: element (o, i, n) of `a` (and of `b`,
 * laid out like `a`) is a[(o * a_dim + a_off + i) * inner + n], of `base`
 * base[(o * base_dim + base_off + i) * inner + n] (contiguous tensors sliced along one
 * dimension; dtype KAB_F32 / KAB_BF16 / KAB_F16, 3 for float64, or 4 / 5 / 6 / 7 for integer
 * or boolean elements of 1 / 2 / 4 / 8 bytes, compared by their bits). An element differs when
 * a's (or, with `b` non-null, a's or b's) value differs
 * from base's: `nan_equal` 1 takes NaN as equal to NaN (x == y or both NaN), 0 is IEEE `!=`.
 * Optional outputs: `mask` (one byte per region element, row-major: 1 where it differs) and
 * `hits` (per dimension k of the region's shape, shape[k] bytes laid end to end, set to 1 at
 * each index where an element differs; the caller zeroes them). `box` (the same layout as
 * `hits`): elements whose every index is flagged are not counted. */
typedef struct KabDiffParams {
  const void* a;
  const void* b;
  const void* base;
  int dtype;
  int nan_equal;
  int64_t outer, len, inner;
  int64_t a_dim, a_off, base_dim, base_off;
  int ndim;
  int64_t shape[KAB_DIFF_MAXDIM];
  unsigned char* hits;
  const unsigned char* box;
  unsigned char* mask;
} KabDiffParams;

/* Runs the census; `count` (device, one 64-bit word) receives the number of differing
 * elements (reset here). */
int kab_diff_census(const KabDiffParams* params, unsigned long long* count, void* stream);

/* ------------------------------------------------------------------ FP8 attention prefill */

/* Per-head e4m3 quantisation of x [heads, seq, d] (docs/research-scripts/fp8-sm120/
 * fp8lib.py:173-176 _fq_last2: scale = amax / 448 per head, 0 -> 1; codes e4m3(x / scale)):
 * q [heads, seq, d], or with `transpose` [heads, d, seq16] (the V^T operand of the attention;
 * seq16 = seq rounded up to a multiple of 16, the columns past seq written as zeros), scales
 * fp32 [heads]. `amax`: [heads] words of device scratch (reset here). */
int kab_quant_heads_fp8(const void* x, int dtype, int64_t heads, int64_t seq, int64_t d,
                        int transpose, unsigned* amax, uint8_t* q, float* scales, void* stream);

/* FP8 attention prefill (fp8lib.py:184-215 emulated_sdpa, mode "qkpv"): e4m3 Q [batch,
 * heads_q, seq, 128], K [batch, heads_kv, seq, 128], V^T [batch, heads_kv, 128, seq16] with one
 * fp32 scale per (batch, head); S = Q K^T * scale, causal mask, online softmax with P as
 * e4m3(p * 448) / 448, out = (P V) / rowsum in bf16 [batch, heads_q, seq, 128]. GQA by head
 * index (heads_q % heads_kv == 0); any seq (keys past it in the last 128-row tile are masked,
 * V^T's row stride seq16 as kab_quant_heads_fp8 writes it). */
int kab_attention_fp8(const uint8_t* q, const float* q_scale, const uint8_t* k, const float* k_scale,
                      const uint8_t* vt, const float* v_scale, int64_t batch, int64_t heads_q,
                      int64_t heads_kv, int64_t seq, int64_t head_dim, int causal, float sm_scale,
                      void* out, void* stream);

/* ------------------------------------------------------------------ FP8 KV cache */

/* kv_quant.py:38-46 quantize_fp8_kv (and triton_fp8_kv_decode.py:51-64 _quant_kv_kernel):
 * one fp32 scale per row of d elements (a token of one KV head), amax / 448 where amax > 0
 * else 1, codes e4m3(v / scale) clamped to +-448, nearest even. Rows are outer x inner; row
 * (o, i) reads x + o * xs_o + i * xs_i, writes codes + o * cs_o + i * cs_i and
 * scales + o * ss_o + i * ss_i (element strides): an append writes straight into the slots
 * of a preallocated cache (kv_quant.py:133-151 Fp8KVCache.append). d a power of two in
 * 16..256; x 16-byte aligned; row starts multiples of 8 elements. */
int kab_quant_kv_fp8(const void* x, int dtype, int64_t outer, int64_t inner, int64_t d, int64_t xs_o,
                     int64_t xs_i, uint8_t* codes, int64_t cs_o, int64_t cs_i, float* scales,
                     int64_t ss_o, int64_t ss_i, void* stream);

/* Decode attention over an e4m3 KV cache (kv_quant.py:56-83 fp8_kv_attention;
 * triton_fp8_kv_decode.py:195-260 fp8_kv_decode): softmax(Q K^T * sm_scale) V with
 * K = k_codes * k_scales[..., None], V likewise, grouped-query heads (heads_q a multiple of
 * heads_kv), optional per-sequence lengths (the first lengths[b] tokens, >= 1), every query
 * token seeing every valid cached token. q [batch, heads_q, q_len, head_dim] (element
 * strides: q_stride_b between sequences, q_stride_row between the rows of one KV head's group,
 * which are the query heads x query tokens, contiguous in that order), codes [batch, heads_kv,
 * length, head_dim] (byte strides, multiples of 16), scales [batch, heads_kv, length] fp32
 * (unit last stride); out [batch, heads_q, q_len, head_dim] bf16, contiguous. head_dim 64 or
 * 128; heads_q / heads_kv * q_len <= 32. `splits`: chunks of the cache per (sequence,
 * KV head), at most 256; 0 for one wave of the CTAs that fit on the GPU. */
typedef struct KabKvDecodeParams {
  const void* q;
  int q_dtype;
  int64_t q_stride_b, q_stride_row;
  const uint8_t* k_codes;
  const float* k_scales;
  const uint8_t* v_codes;
  const float* v_scales;
  int64_t kc_stride_b, kc_stride_h, kc_stride_l;
  int64_t vc_stride_b, vc_stride_h, vc_stride_l;
  int64_t ks_stride_b, ks_stride_h;
  int64_t vs_stride_b, vs_stride_h;
  const int32_t* lengths; /* [batch] or NULL */
  int64_t batch, heads_q, heads_kv, q_len, length, head_dim;
  float sm_scale;
  int splits;
  void* out;
} KabKvDecodeParams;

/* The splits the launch will use and the workspace bytes it needs (0 with one split). The
 * workspace holds the per-split partials and one counter per (sequence, KV head): zero it
 * once when it is allocated; every launch leaves the counters at zero. */
int kab_kv_decode_workspace(const KabKvDecodeParams* params, int* splits, size_t* bytes);
int kab_kv_decode_fp8(const KabKvDecodeParams* params, void* workspace, size_t workspace_bytes,
                      void* stream);

#ifdef __cplusplus
}
#endif

#endif /* KAB_H_ */
