/*
 * fp8_b200.h — C ABI of the B200 (sm_100a) FP8/FP4 conversion and scaled-GEMM
 * library (libfp8_b200.so).
 *
 * This is the boundary the Python plugin (package fp4_fp8_for_torch_mps)
 * binds with ctypes. It replaces the reference plugin's kernel boundary: the
 * Metal library compiled by torch.mps.compile_shader and dispatched as
 * `lib.<kernel>(..., threads=, group_size=)` from fp8_mps_native.py. Each
 * entry point below cites the reference kernel and launcher it replaces.
 *
 * Conventions
 *  - All data pointers are device pointers on the current CUDA device, owned
 *    by the caller; the library never allocates or frees. `stream` is a
 *    cudaStream_t (NULL = legacy default stream).
 *  - Scales are device pointers to float32 so that no host synchronisation is
 *    needed (the reference reads amax with .item(), fp8_mps_native.py:107).
 *  - Every function returns 0 on success or a negative FP8B200_E* status;
 *    fp8b200_last_error() gives a message for the calling thread.
 *  - n == 0 is valid and launches nothing.
 */
#ifndef FP8_B200_H_
#define FP8_B200_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* status codes */
#define FP8B200_OK 0
#define FP8B200_EINVAL (-1)   /* bad argument (dtype, size, alignment, stride) */
#define FP8B200_ELAUNCH (-2)  /* CUDA launch or runtime error */
#define FP8B200_EDEVICE (-3)  /* current device is not sm_100 (B200) */
#define FP8B200_ETIMEOUT (-4) /* a bounded device-side wait gave up */

/* dtype codes */
#define FP8B200_F32 0
#define FP8B200_BF16 1
#define FP8B200_F16 2
#define FP8B200_E4M3 3 /* torch.float8_e4m3fn */
#define FP8B200_E5M2 4 /* torch.float8_e5m2 */
#define FP8B200_E2M1 5 /* torch.float4_e2m1fn_x2: two e2m1 values per byte, element
                          2i in the low nibble (GEMM operands only) */

/* scale modes for the decoders */
#define FP8B200_SCALE_NONE 0     /* exact conversion, scale ignored */
#define FP8B200_SCALE_F32 1      /* out = round_out(round_f32(value * scale)) */
#define FP8B200_SCALE_F16_REF 2  /* out = f16(f16(value) * f16(scale)), the
                                    reference dequantize semantics (f16 out only) */

/* scale layouts for fp8b200_scaled_mm */
#define FP8B200_SCALE_TENSOR 0   /* one float */
#define FP8B200_SCALE_ROWWISE 1  /* scale_a: M floats; scale_b: N floats */

/* Library version (major*10000 + minor*100 + patch). */
int fp8b200_version(void);

/* Message describing the last failure on the calling thread ("" if none). */
const char *fp8b200_last_error(void);

/*
 * float32/bfloat16/float16 -> float8 (e4m3fn or e5m2) encode of n contiguous
 * elements: round to nearest even; e4m3fn: |x| rounding past 448, inf and NaN
 * give 0x7F|sign; e5m2: rounding past 57344 and inf give 0x7C|sign, NaN
 * 0x7F|sign. If `scale` is non-NULL each element is first multiplied by
 * *scale in float32.
 * Replaces float_to_fp8_kernel (shaders/fp8_matmul.metal:240-248, encoder
 * :105-142) launched by fp8_encode (fp8_mps_native.py:85-98).
 */
int fp8b200_encode_fp8(const void *src, int src_dtype, void *dst, int fp8_dtype,
                       int64_t n, const float *scale, void *stream);

/*
 * float8 -> float32/bfloat16/float16 decode of n contiguous codes, bit-exact
 * with CPU PyTorch (NaN payloads included), optionally scaled (scale_mode).
 * Replaces fp8_to_half_kernel (shaders/fp8_matmul.metal:229-237) plus the
 * scale and cast passes of fp8_dequantize (fp8_mps_native.py:65-82) and
 * ops.py:113-120.
 */
int fp8b200_decode_fp8(const void *src, int fp8_dtype, void *dst, int out_dtype,
                       int64_t n, const float *scale, int scale_mode, void *stream);

/*
 * float4_e2m1fn_x2 -> float decode: each of `nbytes` packed bytes gives two
 * outputs, low nibble first (element 2i), optionally scaled (scale_mode).
 * Replaces fp4x2_to_half_kernel (shaders/fp8_matmul.metal:251-261) plus the
 * scale and cast passes of fp4_dequantize (fp8_mps_native.py:162-179) and
 * ops.py:104-111.
 */
int fp8b200_decode_fp4(const void *src, int64_t nbytes, void *dst, int out_dtype,
                       const float *scale, int scale_mode, void *stream);

/*
 * Per-tensor dynamic quantisation to float8: amax = max|x|, scale =
 * 448/amax (57344/amax for e5m2; 1 if amax is 0 or NaN), dst = encode(x *
 * scale), scale_out[0] = scale, scale_out[1] = 1/scale (the value the
 * reference returns). `amax_scratch` is one caller-provided device uint32
 * used as the reduction accumulator; it is cleared by this call.
 * Replaces fp8_quantize (fp8_mps_native.py:101-120) without its .item() sync.
 */
int fp8b200_quantize_fp8(const void *src, int src_dtype, void *dst, int fp8_dtype,
                         int64_t n, float *scale_out, uint32_t *amax_scratch,
                         void *stream);

/*
 * Per-row (per-token) dynamic quantisation of a rows x cols matrix (row
 * strides ld_src / ld_dst in elements): for each row r, amax_r = max|x_r|,
 * scale_r = fmax/amax_r (1 if amax_r is 0 or NaN), dst_r = encode(x_r *
 * scale_r), inv_scale[r] = 1/scale_r. One launch, no scratch, no host sync;
 * inv_scale is the (M,1) scale_a of a rowwise fp8b200_scaled_mm.
 * Generalises fp8_quantize (fp8_mps_native.py:101-120) from one scale per
 * tensor to one scale per row.
 */
int fp8b200_quantize_rows_fp8(const void *src, int src_dtype, int64_t rows, int64_t cols,
                              int64_t ld_src, void *dst, int64_t ld_dst, int fp8_dtype,
                              float *inv_scale, void *stream);

/*
 * Fused SiLU-gate + per-row quantisation (no counterpart in the reference;
 * it feeds the rowwise fp8b200_scaled_mm of an FP8 MLP). gate_up is a
 * rows x (2f) bfloat16 matrix with row stride ld elements whose row r holds
 * [g_r | u_r]; for each row y_r = bf16(bf16(silu(g_r)) * u_r), rounded exactly
 * as PyTorch computes F.silu(g) * u in bfloat16, is quantised like
 * fp8b200_quantize_rows_fp8: dst_r = encode(y_r * scale_r) with scale_r =
 * fmax/amax(y_r), inv_scale[r] = 1/scale_r. dst has row stride ld_dst bytes.
 * Limits: f <= 102400 (the row of y is staged in shared memory).
 */
int fp8b200_silu_mul_quantize_rows_fp8(const void *gate_up, int64_t rows, int64_t f, int64_t ld,
                                       void *dst, int64_t ld_dst, int fp8_dtype,
                                       float *inv_scale, void *stream);

/*
 * Rotary position embedding of the q and k heads of a fused bf16 qkv
 * projection (no counterpart in the reference; it serves the FP8 inference
 * stack around fp8b200_scaled_mm). qkv: tokens x ld bf16, row t holds
 * n_q_heads then n_k_heads heads of head_dim values (position = t % seq).
 * cos_table / sin_table: seq x head_dim/2 bf16. Writes out_q (tokens x
 * n_q_heads x head_dim) and out_k (tokens x n_k_heads x head_dim), bf16,
 * contiguous: out[:h] = x1*cos - x2*sin, out[h:] = x2*cos + x1*sin with
 * PyTorch's bf16 roundings (each product, then the difference / sum).
 * head_dim a multiple of 16, ld a multiple of 8, 16-byte aligned tensors.
 */
int fp8b200_rope_bf16(const void *qkv, int64_t tokens, int64_t ld, int n_q_heads, int n_k_heads,
                      int head_dim, int seq, const void *cos_table, const void *sin_table,
                      void *out_q, void *out_k, void *stream);

/*
 * Allocation-free fp8b200_quantize_fp8 (no counterpart in the reference; the
 * reference has no device memory management of its own). Same inputs,
 * outputs and results, but no amax_scratch argument: the scratch is a fixed
 * 16 KiB array inside this library's device memory (4096 amax partials,
 * one per slice of 4096 to 65536 elements), so a caller that cannot
 * allocate device memory, such as a host runtime that only passes in the
 * tensors to read and write, needs nothing beyond src, dst and scale_out.
 * Limits: n <= FP8B200_NOALLOC_MAX_ELEMENTS, else FP8B200_EINVAL. The first
 * call on each device looks up the array's device address (make that first
 * call before any stream capture). Every call shares the array: calls that
 * overlap on the GPU (other streams or threads) race and must be serialised.
 * Each GPU that loads the library holds the array until the process exits.
 */
#define FP8B200_NOALLOC_MAX_ELEMENTS (4096LL * 65536LL)
int fp8b200_quantize_fp8_noalloc(const void *src, int src_dtype, void *dst, int fp8_dtype,
                                 int64_t n, float *scale_out, void *stream);

/*
 * float -> float4_e2m1fn_x2 encode of n (even) contiguous elements into n/2
 * packed bytes, element 2i in the low nibble, with the reference's
 * nearest-of-8 thresholds (not round-to-nearest-even at ties; NaN -> +6).
 * If `scale` is non-NULL each element is first multiplied by *scale.
 * Replaces float_to_fp4x2_kernel (shaders/fp8_matmul.metal:264-274, encoder
 * :88-102) launched by fp4_encode (fp8_mps_native.py:182-197).
 */
int fp8b200_encode_fp4(const void *src, int src_dtype, void *dst, int64_t n,
                       const float *scale, void *stream);

/*
 * Per-tensor FP4 quantisation: scale = 6/amax (1 if amax is 0 or NaN),
 * dst = encode_fp4(x * scale), scale_out = {scale, 1/scale}; `amax_scratch`
 * as for fp8b200_quantize_fp8.
 * Replaces fp4_quantize (fp8_mps_native.py:200-221) without its .item() sync.
 */
int fp8b200_quantize_fp4(const void *src, int src_dtype, void *dst, int64_t n,
                         float *scale_out, uint32_t *amax_scratch, void *stream);

/*
 * D = (A * scale_a) @ (B * scale_b)^T [+ bias] [* scale_result] -> out_dtype.
 * A: M x K codes, row-major with row stride lda (bytes).
 * B: N x K codes, row-major with row stride ldb (bytes): the bytes of
 *    torch._scaled_mm's column-major mat2 (K x N).
 * a_dtype / b_dtype: FP8B200_E4M3, FP8B200_E5M2 or FP8B200_E2M1, chosen per
 *    operand (mixed float4 x float8 is allowed). A float4 operand is packed
 *    (K/2 bytes per row, element 2i in the low nibble of byte i) and needs K
 *    a multiple of 128, a row stride that is a multiple of 32 bytes and a
 *    32-byte aligned base.
 * scale_a / scale_b: float32 device pointers, layout FP8B200_SCALE_TENSOR or
 *    FP8B200_SCALE_ROWWISE (M values for A, N values for B).
 * bias: N values of bias_dtype (F32/BF16/F16) or NULL; scale_result: one
 *    float32 or NULL. D: M x N of out_dtype (F32/BF16/F16/E4M3/E5M2), row
 *    stride ldd elements. K must be a positive multiple of 16; lda/ldb
 *    multiples of 16; A and B 16-byte aligned.
 * Accumulation is float32 on the tcgen05 tensor cores (kind::f8f6f4, which
 * takes e4m3, e5m2 and e2m1 operands at the same rate; e2m1 x e2m1 with K a
 * multiple of 256 on large shapes runs as kind::mxf4 with unit block scales,
 * at twice that rate and with the same result).
 * Replaces the reference's _scaled_mm override (ops.py:33-49) and the GEMM
 * kernels behind it: fp8_scaled_matmul_kernel (shaders/fp8_matmul.metal:
 * 145-180), fp8_scaled_vecmat_kernel (:183-226) and the decode+fp16-matmul
 * fast path (fp8_mps_native.py:129-159). The float4 operands extend it to the
 * reference's packed FP4 format (shaders/fp8_matmul.metal:77-102, produced by
 * fp4_quantize, fp8_mps_native.py:200-221), which the reference can only
 * decode, never multiply.
 */
int fp8b200_scaled_mm(const void *A, int a_dtype, int64_t lda,
                      const void *B, int b_dtype, int64_t ldb,
                      int64_t M, int64_t N, int64_t K,
                      const float *scale_a, int scale_a_layout,
                      const float *scale_b, int scale_b_layout,
                      const void *bias, int bias_dtype,
                      const float *scale_result,
                      void *D, int out_dtype, int64_t ldd,
                      void *stream);

/*
 * Linear layer with float8 weights dequantised on load:
 * D = x @ (w * w_scale)^T [+ bias] -> out_dtype (F32/BF16/F16).
 * x: M x K bf16 or f16 activations, row stride ldx elements (multiple of 8);
 * w: N x K float8 weight codes, row stride ldw bytes (multiple of 16); x and w
 * 16-byte aligned. w_scale: one float (FP8B200_SCALE_TENSOR) or N floats, one
 * per output channel (FP8B200_SCALE_ROWWISE); bias: N values or NULL.
 * The weights are converted to x's type (exact) and the products are
 * accumulated in float32 on the tensor cores; the scale and bias are applied
 * to the float32 sums. M <= 64 with K a multiple of 128: weights converted in
 * registers for warp-level m16n8k16 MMAs, K split over a cluster; otherwise
 * converted in shared memory for tcgen05 kind::f16 MMAs.
 * Replaces the reference's dequantise-then-matmul path: fp8_scaled_mm_fast
 * (fp8_mps_native.py:129-159), which decodes both operands to f16 and calls
 * an MPS f16 matmul, for the case where only the weights are float8.
 */
int fp8b200_linear_fp8w(const void *x, int x_dtype, int64_t ldx, const void *w, int w_dtype, int64_t ldw,
                        int64_t M, int64_t N, int64_t K, const float *w_scale, int w_scale_layout,
                        const void *bias, int bias_dtype, void *D, int out_dtype, int64_t ldd,
                        void *stream);

/*
 * 16-bit GEMM: D = A @ B^T * scale_b [+ bias] -> out_dtype (F32/BF16/F16),
 * A: M x K and B: N x K of the same type (FP8B200_BF16 or FP8B200_F16), row
 * strides lda / ldb elements (multiples of 8), 16-byte aligned; scale_b one
 * float or N floats (per output column); D 16-byte aligned rows.
 * The CTA-pair 256x512 tcgen05 kernel of fp8b200_scaled_mm with kind::f16
 * MMAs. It serves the large-M path of the float8-weight linear (weights
 * decoded once to the activation type, scale applied here); the reference
 * has no counterpart beyond its f16 matmul call (fp8_mps_native.py:150-155).
 */
int fp8b200_gemm_16bit(const void *A, const void *B, int dtype, int64_t lda, int64_t ldb,
                       int64_t M, int64_t N, int64_t K, const float *scale_b, int scale_b_layout,
                       const void *bias, int bias_dtype, void *D, int out_dtype, int64_t ldd,
                       void *stream);

/*
 * Device-side status of the scaled GEMM on the current device: 0 if no
 * bounded wait has timed out, else FP8B200_ETIMEOUT with *status_out holding
 * the site code of the last launch that timed out (that launch's output is
 * incomplete). A timeout affects only its own launch: later launches run to
 * completion. Synchronises the device. `reset` clears the word.
 * (Failure reporting for the GEMM's bounded waits; the reference has none.)
 */
int fp8b200_gemm_status(uint32_t *status_out, int reset);

/*
 * Test hook for the bounded waits of the GEMM kernels and of the few-row
 * fp8b200_linear_fp8w kernel: skip_first_load != 0 makes the producer never
 * fill the first pipeline stage, so the consumers' waits run out after
 * wait_timeout_ns (0 = the default of 2 s) and the kernel returns with the
 * status word set. Applies to launches from the calling host thread only.
 * Not for production use.
 */
int fp8b200_debug_gemm(int skip_first_load, unsigned long long wait_timeout_ns);

/*
 * Kernel choice for fp8b200_scaled_mm: 0 = by shape (M <= 256: the small-M
 * kernel, which puts 128 output columns on the MMA's rows and splits K over
 * a cluster of up to 8 CTAs; else, when N >= 256, a CTA pair per 256x512
 * output tile, or per 256x256 tile where the wider tiles would leave too many
 * SMs idle in the last wave; else the single-CTA kernel with 128x256 tiles),
 * 1 = always single-CTA, 2 = always CTA-pair 256x256, 3 = always small-M
 * (tiles of 256 rows of A when M > 256), 4 = always CTA-pair 256x512 (or
 * 256x480 where the shape picks it; 256x256 when the output rows are not
 * 16-byte aligned, since the 256x512 kernel stores through a tensor map).
 * Path 3 also sends fp8b200_linear_fp8w calls with M <= 64 to its tcgen05
 * small-M kernel instead of the warp-level MMA kernel.
 * Applies to launches from the calling host thread only; for tests and tuning.
 */
int fp8b200_gemm_set_path(int path);

/* Number of kernels this library launched since load (all devices). */
uint64_t fp8b200_launch_count(void);

#ifdef __cplusplus
}
#endif

#endif /* FP8_B200_H_ */
