// Shared definitions of the int8 product kernels: launch arguments and the per-element finishing step (zero-point
// correction, int/float bias, scale, requantization) that every product variant applies as it stores a sum.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace og {

enum OutKind : int { OUT_I32 = 0, OUT_F32 = 1, OUT_U8 = 2, OUT_S8 = 3 };

// What a product kernel needs to finish and store C[b, m, n]. Zero points: mode 0 absent, 1 one value, 2 one per row
// (A) or per column (B). The correction uses the byte sums of the other operand:
//   C = dot - zb[n] * rowsumA[b, m] - za[m] * colsumB[b, n] + K * za[m] * zb[n]   (all modulo 2^32)
// which equals sum_k (a - za)(b - zb) exactly in the integers, so also modulo 2^32.
struct Epilogue {
    int out_kind;
    void* c;              // output buffer (int32, float or bytes), already advanced by OffsetC
    int64_t ldc;          // N
    int64_t batch_stride_c;  // M * N
    int m, n, k;
    const uint8_t* za;    // zero point of A (already offset), or null
    int za_vector, za_signed;
    const uint8_t* zb;
    int zb_vector, zb_signed;
    const int32_t* row_sum_a;     // [batchA][M] byte sums of A, or null when no zero point of B is present
    int64_t row_sum_a_stride;     // M, or 0 when every batch shares A
    const int32_t* col_sum_b;     // [batchB][N] byte sums of B, or null when no zero point of A is present
    int64_t col_sum_b_stride;     // N, or 0 when every batch shares B
    const int32_t* int_bias;      // per column, or null
    const float* scale;           // float form: scale; requantized form: multiplier
    int scale_vector;
    const float* scale_a;         // dequantize form: one scale of A multiplied into every column's scale, or null
    const float* float_bias;      // per column, or null
    int zero_point_y;
    int vec_ok;                   // every output row starts on a 16-byte boundary
};

__device__ __forceinline__ int32_t zp_value(const uint8_t* z, int vector, int is_signed, int idx) {
    if (z == nullptr) return 0;
    const uint8_t v = __ldg(z + (vector ? idx : 0));
    return is_signed ? static_cast<int32_t>(static_cast<int8_t>(v)) : static_cast<int32_t>(v);
}

// Row-dependent part of the correction for row m of batch b: returns za[m] and the row's byte sum.
struct RowTerms {
    int32_t za;
    int32_t rsa;
};

__device__ __forceinline__ RowTerms row_terms(const Epilogue& e, int b, int m) {
    RowTerms t;
    t.za = zp_value(e.za, e.za_vector, e.za_signed, m);
    t.rsa = e.row_sum_a ? __ldg(e.row_sum_a + b * e.row_sum_a_stride + m) : 0;
    return t;
}

// The corrected int32 sum of one element (wrapping arithmetic in uint32).
__device__ __forceinline__ uint32_t corrected(const Epilogue& e, const RowTerms& rt, int b, int n, uint32_t dot) {
    uint32_t s = dot;
    if (e.zb != nullptr) {
        const int32_t zb = zp_value(e.zb, e.zb_vector, e.zb_signed, n);
        s -= static_cast<uint32_t>(zb) * static_cast<uint32_t>(rt.rsa);
        s += static_cast<uint32_t>(e.k) * static_cast<uint32_t>(rt.za) * static_cast<uint32_t>(zb);
    }
    if (e.za != nullptr) {
        const int32_t csb = __ldg(e.col_sum_b + b * e.col_sum_b_stride + n);
        s -= static_cast<uint32_t>(rt.za) * static_cast<uint32_t>(csb);
    }
    if (e.int_bias != nullptr) s += static_cast<uint32_t>(__ldg(e.int_bias + n));
    return s;
}

// The scale of column n: scale[n] (or the single scale), times the scale of A when one is given - one float32
// product, the same rounding as forming scaleA * scaleB[n] in a pass of its own.
__device__ __forceinline__ float col_scale(const Epilogue& e, int n) {
    const float s = __ldg(e.scale + (e.scale_vector ? n : 0));
    return e.scale_a != nullptr ? __fmul_rn(__ldg(e.scale_a), s) : s;
}

// float(sum) * scale, then + float bias: two separate roundings, never fused (Int8GemmEpilogue.hlsli semantics).
__device__ __forceinline__ float finish_float(const Epilogue& e, int n, uint32_t s) {
    const float sc = col_scale(e, n);
    float f = __fmul_rn(__int2float_rn(static_cast<int32_t>(s)), sc);
    if (e.float_bias != nullptr) f = __fadd_rn(f, __ldg(e.float_bias + n));
    return f;
}

// clamp(round_half_even(float(sum) * multiplier) + zeroPointY) to the output type, NaN to the smallest value
// (Int8Epilogue.hlsl Quantized semantics).
__device__ __forceinline__ uint8_t finish_byte(const Epilogue& e, int n, uint32_t s, bool out_unsigned) {
    const int lo = out_unsigned ? 0 : -128;
    const int hi = out_unsigned ? 255 : 127;
    const float mult = col_scale(e, n);
    const float v = __fmul_rn(__int2float_rn(static_cast<int32_t>(s)), mult);
    if (isnan(v)) return static_cast<uint8_t>(lo & 0xFF);
    float r = rintf(v);
    const float flo = static_cast<float>(lo - e.zero_point_y);
    const float fhi = static_cast<float>(hi - e.zero_point_y);
    r = r < flo ? flo : (r > fhi ? fhi : r);
    return static_cast<uint8_t>((static_cast<int>(r) + e.zero_point_y) & 0xFF);
}

// Error word shared by the kernels of one device: a kernel whose bounded wait gave up sets it.
struct DeviceStatus {
    int error;
};

}  // namespace og
