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
 *   og_oracle_requant          tests/RecursiveAI.OneGpu.Kernels.Tests/Int8Tests.cs:84-97   (Requant: QLinearMatMul byte)
 *   og_oracle_float_epilogue   tests/RecursiveAI.OneGpu.Kernels.Tests/Int8Tests.cs:356-373 (float form, two roundings)
 *   og_oracle_dynamic_quantize tests/RecursiveAI.OneGpu.Kernels.Tests/Int8Tests.cs:577-615 (DynamicReference)
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

/* Same sums computed the packed-dot way: bytes xor 0x80 into the signed domain, byte sums, correction at the end. */
void og_oracle_int8_gemm_signed_domain(const og_oracle_problem* p, const uint8_t* a, int32_t a_signed,
                                       const uint8_t* b, int32_t b_signed, const uint8_t* za, int32_t za_vector,
                                       const uint8_t* zb, int32_t zb_vector, int32_t* c);

int32_t og_oracle_requant(int32_t acc, float mult, int32_t zero, int32_t is_unsigned);
float og_oracle_float_epilogue(int32_t acc, int32_t has_int_bias, int32_t int_bias, float scale, int32_t has_float_bias,
                               float float_bias);

void og_oracle_dynamic_quantize(const float* x, int64_t count, uint8_t* y, float* scale, uint8_t* zero_point);
float og_oracle_div_exact(float x, float s);

#ifdef __cplusplus
}
#endif

#endif
