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
    int sum_splits;               // the sums are this many partial sums over K ranges, to be added up
    int64_t row_sum_split_stride; // batchA * M
    int64_t col_sum_split_stride; // batchB * N
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

// The byte sum of row m of A (batch b) and of column n of B: the partial sums of the K splits added up (wrapping).
__device__ __forceinline__ uint32_t row_sum_of(const Epilogue& e, int b, int m) {
    uint32_t s = 0;
    for (int i = 0; i < e.sum_splits; i++)
        s += static_cast<uint32_t>(__ldg(e.row_sum_a + i * e.row_sum_split_stride + b * e.row_sum_a_stride + m));
    return s;
}

__device__ __forceinline__ uint32_t col_sum_of(const Epilogue& e, int b, int n) {
    uint32_t s = 0;
    for (int i = 0; i < e.sum_splits; i++)
        s += static_cast<uint32_t>(__ldg(e.col_sum_b + i * e.col_sum_split_stride + b * e.col_sum_b_stride + n));
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
