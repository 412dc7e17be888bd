/*
 * CPU oracle for the int8 GEMM + DynamicQuantizeLinear path of onegpu.
 *
 * TEST INFRASTRUCTURE ONLY. Nothing in the product path (the CUDA library, its C ABI or the Python host mirror) may
 * link, load or call this code. Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / --impl reference
 * legs use it, as the checker or as the timed CPU baseline.
 *
 * Every function restates, in plain C, the CPU reference that the reference repository's own tests compare its GPU
 * kernels against (paths are relative to the reference repository root):
 *   og_oracle_bytes            tests/RecursiveAI.OneGpu.Kernels.Tests/Int8Tests.cs:36-47   (Bytes: seeded LCG bytes)
 *   og_oracle_random           tests/RecursiveAI.OneGpu.Kernels.Tests/Rig.cs:8-19          (Rig.Random: seeded uniform floats)
 *   og_oracle_dq_input         tests/RecursiveAI.OneGpu.Kernels.Tests/Int8Tests.cs:632-647 (the seven DQL input kinds)
 *   og_oracle_int8_gemm        tests/RecursiveAI.OneGpu.Kernels.Tests/Int8Tests.cs:52-82   (Reference: wrapping int32 sums)
 *   og_oracle_int8_gemm_tiled  src/RecursiveAI.OneGpu.Kernels/Shaders/Int8GemmKernel.hlsl:98-244 (the same sums
 *                              through the reference portable kernel's 64 x 64 x 16 blocking; the second CPU baseline)
 *   og_oracle_requant          tests/RecursiveAI.OneGpu.Kernels.Tests/Int8Tests.cs:84-97   (Requant: QLinearMatMul byte)
 *   og_oracle_float_epilogue   tests/RecursiveAI.OneGpu.Kernels.Tests/Int8Tests.cs:356-373 (float form, two roundings)
 *   og_oracle_dynamic_quantize tests/RecursiveAI.OneGpu.Kernels.Tests/Int8Tests.cs:577-615 (DynamicReference)
 *   og_oracle_dequantize       tests/RecursiveAI.OneGpu.Kernels.Tests/DequantizeTests.cs:57-68 (float(x - zp) * scale)
 *   og_oracle_quantize         tests/RecursiveAI.OneGpu.Kernels.Tests/DequantizeTests.cs:138-148 (QuantizeOne)
 *   og_oracle_conv_integer     tests/RecursiveAI.OneGpu.Kernels.Tests/ConvIntegerTests.cs:41-88 (Reference: direct
 *                              convolution, padded taps skipped, wrapping int32 sums)
 * with the IEEE binary16 conversions the C# (Half) casts perform (og_oracle_float_to_half: round to nearest even;
 * og_oracle_half_to_float: exact),
 * and two independent cross-checks of the oracle itself:
 *   og_oracle_int8_gemm_signed_domain  src/RecursiveAI.OneGpu.Kernels/Shaders/Int8GemmDot.hlsl:4-10,134-140,301
 *                                      (operands moved to the signed domain, zero points applied from byte sums)
 *   og_oracle_div_exact                src/RecursiveAI.OneGpu.Kernels/Shaders/DivExact.hlsli:4-99
 *                                      (correctly rounded division by integer long division)
 *
 * Float arithmetic follows C# single precision: every operation is rounded to binary32, no contraction (build with
 * -ffp-contract=off), round-half-to-even via nearbyintf under the default rounding mode (MathF.Round).
 */
#ifndef OG_ORACLE_H
#define OG_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* The shape of one batch of products; mirrors Int8GemmProblem (src/RecursiveAI.OneGpu.Kernels/Int8Gemm.cs:43-95).
 * Lda/Ldb of 0 mean dense. Offsets and strides are in bytes of A / B. */
typedef struct og_oracle_problem {
    int32_t m, n, k, batch;
    int32_t transpose_b;
    int32_t lda, ldb;
    int32_t offset_a, offset_b;
    int32_t stride_a, stride_b;
} og_oracle_problem;

void og_oracle_bytes(uint8_t* out, int64_t length, int32_t seed);
void og_oracle_random(float* out, int64_t n, int32_t seed, float lo, float hi);
void og_oracle_dq_input(float* out, int64_t count, int32_t seed, int32_t kind);

/* C[batch, m, n] = sum_k (A - za)(B - zb), wrapping modulo 2^32. za/zb may be NULL (zero point 0). Rows are split
 * over `threads` POSIX threads (the reference's Parallel.For over rows). `c` holds batch*m*n int32. */
void og_oracle_int8_gemm(const og_oracle_problem* p, const uint8_t* a, int32_t a_signed, const uint8_t* b,
                         int32_t b_signed, const uint8_t* za, int32_t za_vector, const uint8_t* zb, int32_t zb_vector,
                         int32_t* c, int32_t threads);
/* The same sums through the reference portable kernel's blocking (Int8GemmKernel.hlsl:98-244): 64 x 64 tiles over
 * `threads` threads, K in chunks of 16 accumulated in float and folded into int32 every 128 k. Bit-identical to
 * og_oracle_int8_gemm; timed as the second CPU baseline. */
void og_oracle_int8_gemm_tiled(const og_oracle_problem* p, const uint8_t* a, int32_t a_signed, const uint8_t* b,
                               int32_t b_signed, const uint8_t* za, int32_t za_vector, const uint8_t* zb,
                               int32_t zb_vector, int32_t* c, int32_t threads);

/* Same sums computed the packed-dot way: bytes xor 0x80 into the signed domain, byte sums, correction at the end. */
void og_oracle_int8_gemm_signed_domain(const og_oracle_problem* p, const uint8_t* a, int32_t a_signed,
                                       const uint8_t* b, int32_t b_signed, const uint8_t* za, int32_t za_vector,
                                       const uint8_t* zb, int32_t zb_vector, int32_t* c);

int32_t og_oracle_requant(int32_t acc, float mult, int32_t zero, int32_t is_unsigned);
float og_oracle_float_epilogue(int32_t acc, int32_t has_int_bias, int32_t int_bias, float scale, int32_t has_float_bias,
                               float float_bias);

void og_oracle_dynamic_quantize(const float* x, int64_t count, uint8_t* y, float* scale, uint8_t* zero_point);
float og_oracle_div_exact(float x, float s);

uint16_t og_oracle_float_to_half(float f);
float og_oracle_half_to_float(uint16_t h);

/* DequantizeLinear over `count` elements viewed as [outer, axis_len, inner]: kind 0 uint8, 1 int8, 2 int32 (x and
 * zero_point, which may be NULL); `out` receives float32 or, with half_out, binary16 bits. */
void og_oracle_dequantize(int32_t kind, const void* x, int64_t count, int32_t per_axis, int64_t axis_len, int64_t inner,
                          const float* scale, const void* zero_point, int32_t half_out, void* out);
/* QuantizeLinear: x float32 or, with half_in, binary16 bits; zero_point (uint8 / int8 by is_signed) may be NULL. */
void og_oracle_quantize(int32_t is_signed, int32_t half_in, const void* x, int64_t count, int32_t per_axis,
                        int64_t axis_len, int64_t inner, const float* scale, const uint8_t* zero_point, uint8_t* out);

/* ConvInteger over NCHW x and OIHW w (bytes; x_signed / w_signed give their types), zero point of x one value
 * (NULL: 0), of w one value or one per output channel (NULL: 0). `y` receives [batch, cout, oh, ow] int32. */
typedef struct og_oracle_conv {
    int32_t batch, cin, h, w, cout, kh, kw;
    int32_t stride_h, stride_w, dilation_h, dilation_w;
    int32_t pad_top, pad_left, pad_bottom, pad_right;
    int32_t groups;
    int32_t offset_x, offset_w;
} og_oracle_conv;
int32_t og_oracle_conv_out_extent(int32_t input, int32_t kernel, int32_t stride, int32_t dilation, int32_t pad_begin,
                                  int32_t pad_end);
void og_oracle_conv_integer(const og_oracle_conv* p, const uint8_t* x, int32_t x_signed, const uint8_t* w,
                            int32_t w_signed, const uint8_t* xz, const uint8_t* wz, int32_t wz_vector, int32_t* y,
                            int32_t threads);

#ifdef __cplusplus
}
#endif

#endif
