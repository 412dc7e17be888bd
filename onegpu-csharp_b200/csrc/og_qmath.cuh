// Quotient rounding shared by QuantizeLinear (og_quant.cu) and DynamicQuantizeLinear (og_dq.cu):
// round_half_even(x / s) with the division correctly rounded, and the saturation to a byte.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

namespace og {

// round_half_even(x / s), the quotient correctly rounded (IEEE division); kept out of line so that callers that
// reach it rarely do not pay for it inline.
static __device__ __noinline__ float rne_quotient_exact(float x, float s) { return rintf(__fdiv_rn(x, s)); }

// The same value when the scale is shared by many elements: with r = RN(1 / s) and m = RN(x * r),
// |m - x/s| <= |x/s| (2^-23 + 2^-48) and the correctly rounded quotient lies within |x/s| 2^-24 of x/s, so both round
// to the same integer unless a half-integer lies within about |m| 2^-22 of m. With q = rint(m), d = m - q is exact
// (|d| <= 1/2, a multiple of m's ulp) and 1/2 - |d| is m's distance to the nearest half-integer; m's rounding q is
// used when that distance exceeds |m| 2^-20 + 2^-20, tested as RN(|m| 2^-20 + |d|) < 1/2 - 2^-19 (the one rounding
// of the fused multiply-add is below 2^-25, inside the 2^-20 of slack). The test fails for |m| >= 2^22, NaN and
// infinities, and near ties: there the quotient itself is rounded. `r_ok` says r is finite and normal.
__device__ __forceinline__ float rne_quotient_r(float x, float s, float r, bool r_ok) {
    const float m = __fmul_rn(x, r);
    const float q = rintf(m);
    const float d = __fsub_rn(m, q);
    if (r_ok && __fmaf_rn(fabsf(m), 0x1p-20f, fabsf(d)) < 0.5f - 0x1p-19f) return q;
    return rne_quotient_exact(x, s);
}

// Clamps an integer-valued v (a rounded quotient plus a zero point) to the output type's range and returns its byte;
// NaN gives the lowest value (fmaxf returns the other operand for NaN). The clamped integer c lies in [-128, 255], so
// c + 1.5 * 2^23 is exact and lies in [2^23, 2^24), where the float's mantissa is c + 2^22: its low byte is c's two's
// complement byte, with no float-to-integer conversion.
template <bool SIGNED>
__device__ __forceinline__ uint32_t saturate_byte(float v) {
    const float lo = SIGNED ? -128.0f : 0.0f;
    const float hi = SIGNED ? 127.0f : 255.0f;
    v = fminf(fmaxf(v, lo), hi);
    return __float_as_uint(__fadd_rn(v, 12582912.0f)) & 0xFFu;
}

}  // namespace og
