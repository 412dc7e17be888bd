// DequantizeKernels (DequantizeKernels.cs:29-298): ONNX DequantizeLinear and QuantizeLinear, per tensor or per axis,
// with their argument checks and C ABI.
//
//   DequantizeLinear: y = float(x - zeroPoint) * scale   (Shaders/Dequantize.hlsl:42-57)
//     x uint8 / int8 / int32; the subtraction wraps in 32 bits, the conversion rounds to nearest even, then one float32
//     multiply; half output rounds that float32 to the nearest half (even on ties).
//   QuantizeLinear: y = saturate(round_half_even(x / scale) + zeroPoint)   (Shaders/Quantize.hlsl:54-81)
//     x float32 / half (widened exactly); the division is IEEE round-to-nearest, the zero point is added in float32,
//     NaN gives the output type's lowest value, then the result is clamped to uint8 / int8.
//
// The tensor is seen as [outer, axisLen, inner]; element j uses parameter (j / inner) % axisLen. Both kernels are
// HBM-bound streams: consecutive threads take consecutive aligned vectors of input and output (so every warp-wide
// load and store covers contiguous memory), four vectors in flight per thread, the parameter index walked without a
// division per element; the few elements before the first aligned vector and after the last go one by one. No two
// threads write the same byte.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "og_gemm.h"
#include "og_host.h"
#include "og_ptx.cuh"
#include "og_qmath.cuh"

namespace og {

constexpr int QTHREADS = 256;

struct QuantArgs {
    const void* x;        // first element
    int64_t count;
    const float* scale;   // first scale
    const void* zp;       // first zero point, or null
    int per_axis;
    uint32_t axis_len;
    uint32_t inner;
    void* out;            // first output element
    int64_t head;         // elements handled one by one before the first whole vector
    int64_t vectors;      // whole vectors of E elements after the head
    int64_t threads;      // threads the launch needs
    uint32_t inner_magic, axis_magic;  // j / inner and q / axis_len by div_magic
    int32_t inner_shift, axis_shift;
    int vec_params;       // DequantizeLinear: every vector's E parameters are consecutive and aligned (inner = 1)
    int keep_out;         // QuantizeLinear: store with the default cache policy (a consumer follows), not streaming
};

// Fills in the division constants of a's inner and axis_len.
static void set_param_magics(QuantArgs& a) {
    magic_for(a.inner, &a.inner_magic, &a.inner_shift);
    magic_for(a.axis_len, &a.axis_magic, &a.axis_shift);
}

// The parameter (scale / zero point) index of element j and its position inside the current run of `inner` elements;
// param_next steps both to element j + 1 without a division.
struct ParamCursor {
    uint32_t pi, r;
};

__device__ __forceinline__ ParamCursor param_at(const QuantArgs& a, int64_t j) {
    if (!a.per_axis) return {0u, 0u};
    const int32_t jj = static_cast<int32_t>(j);  // counts stay below 2^31
    const int32_t q = div_magic(jj, a.inner_magic, a.inner_shift);
    const int32_t pi = q - div_magic(q, a.axis_magic, a.axis_shift) * static_cast<int32_t>(a.axis_len);
    return {static_cast<uint32_t>(pi), static_cast<uint32_t>(jj - q * static_cast<int32_t>(a.inner))};
}

__device__ __forceinline__ void param_next(const QuantArgs& a, ParamCursor& c) {
    if (!a.per_axis) return;
    if (++c.r == a.inner) {
        c.r = 0;
        if (++c.pi == a.axis_len) c.pi = 0;
    }
}

template <int KIND>  // 0 uint8, 1 int8, 2 int32
__device__ __forceinline__ int32_t load_q(const void* p, int64_t i) {
    if constexpr (KIND == 0) return static_cast<int32_t>(__ldg(static_cast<const uint8_t*>(p) + i));
    else if constexpr (KIND == 1) return static_cast<int32_t>(static_cast<int8_t>(__ldg(static_cast<const uint8_t*>(p) + i)));
    else return __ldg(static_cast<const int32_t*>(p) + i);
}

// float(d) for |d| < 2^22, exactly as __int2float_rn(d): d added to the bits of 1.5 * 2^23 (whose unit in the last
// place is 1) gives 1.5 * 2^23 + d, and subtracting 1.5 * 2^23 is exact.
__device__ __forceinline__ float small_int_to_float(int32_t d) {
    return __fsub_rn(__int_as_float(d + 0x4B400000), 12582912.0f);
}

template <int KIND>
__device__ __forceinline__ float dequantize_one(const QuantArgs& a, int32_t q, const ParamCursor& c) {
    const int32_t zp = a.zp != nullptr ? load_q<KIND>(a.zp, c.pi) : 0;
    const int32_t d = static_cast<int32_t>(static_cast<uint32_t>(q) - static_cast<uint32_t>(zp));
    return __fmul_rn(__int2float_rn(d), __ldg(a.scale + c.pi));
}

template <bool HALF>
__device__ __forceinline__ float load_x(const void* p, int64_t i) {
    if constexpr (HALF) return __half2float(__ushort_as_half(__ldg(static_cast<const unsigned short*>(p) + i)));
    else return __ldg(static_cast<const float*>(p) + i);
}

// The scale and the zero point of one parameter index.
struct QParam {
    uint32_t pi;
    float s, zf;
};

template <bool SIGNED>
__device__ __forceinline__ void qparam_load(const QuantArgs& a, uint32_t pi, QParam& q) {
    q.pi = pi;
    q.s = __ldg(a.scale + pi);
    int32_t zp = 0;
    if (a.zp != nullptr) {
        const uint8_t z = __ldg(static_cast<const uint8_t*>(a.zp) + pi);
        zp = SIGNED ? static_cast<int32_t>(static_cast<int8_t>(z)) : static_cast<int32_t>(z);
    }
    q.zf = static_cast<float>(zp);
}

__device__ __forceinline__ float rne_quotient(float x, const QParam& p) { return rne_quotient_exact(x, p.s); }

template <bool SIGNED>
__device__ __forceinline__ uint32_t quantize_with(float xv, const QParam& p) {
    return saturate_byte<SIGNED>(__fadd_rn(rne_quotient(xv, p), p.zf));
}

template <bool SIGNED>
__device__ __forceinline__ uint32_t quantize_one(const QuantArgs& a, float xv, const ParamCursor& c) {
    QParam p;
    qparam_load<SIGNED>(a, c.pi, p);
    return quantize_with<SIGNED>(xv, p);
}

// Vector shapes: E elements per vector, an input vector and an output vector per thread and step.
//   DequantizeLinear: bytes -> float E = 4 (4 B -> 16 B), bytes -> half E = 8 (8 B -> 16 B),
//                     int32 -> float E = 4 (16 B -> 16 B), int32 -> half E = 4 (16 B -> 8 B);
//   QuantizeLinear:   float -> bytes E = 4 (16 B -> 4 B), half -> bytes E = 8 (16 B -> 8 B).
// Consecutive threads take consecutive vectors, so every warp-wide load and store covers contiguous memory. The
// elements before the output's first 16-byte boundary (`head`) and after the last whole vector go element by element.
template <int KIND, bool HALF>
struct DqShape {
    static constexpr int E = (KIND != 2 && HALF) ? 8 : 4;
};

constexpr int UNROLL = 4;  // vectors in flight per thread

template <int KIND, bool HALF>
__device__ __forceinline__ void dq_load(const QuantArgs& a, int64_t first, int32_t (&q)[DqShape<KIND, HALF>::E]) {
    constexpr int E = DqShape<KIND, HALF>::E;
    if constexpr (KIND == 2) {
        const int4 w = __ldcs(reinterpret_cast<const int4*>(static_cast<const int32_t*>(a.x) + first));
        q[0] = w.x;
        q[1] = w.y;
        q[2] = w.z;
        q[3] = w.w;
    } else if constexpr (E == 8) {
        const uint2 w = __ldcs(reinterpret_cast<const uint2*>(static_cast<const uint8_t*>(a.x) + first));
#pragma unroll
        for (int e = 0; e < 8; e++) {
            const uint32_t b = ((e < 4 ? w.x : w.y) >> (8 * (e & 3))) & 0xFFu;
            q[e] = KIND == 1 ? static_cast<int32_t>(static_cast<int8_t>(b)) : static_cast<int32_t>(b);
        }
    } else {
        const uint32_t w = __ldcs(reinterpret_cast<const unsigned int*>(static_cast<const uint8_t*>(a.x) + first));
#pragma unroll
        for (int e = 0; e < 4; e++) {
            const uint32_t b = (w >> (8 * e)) & 0xFFu;
            q[e] = KIND == 1 ? static_cast<int32_t>(static_cast<int8_t>(b)) : static_cast<int32_t>(b);
        }
    }
}

// The scales and zero points of E elements from parameter pi: E consecutive ones (vector loads; pi is a multiple of
// E and the parameter arrays are aligned) or pi's for all.
template <int KIND, int E>
__device__ __forceinline__ void dq_params(const QuantArgs& a, uint32_t pi, bool consecutive, float (&s)[E],
                                          int32_t (&z)[E]) {
    if (consecutive) {
#pragma unroll
        for (int h = 0; h < E / 4; h++) {
            const float4 sv = __ldg(reinterpret_cast<const float4*>(a.scale + pi) + h);
            s[4 * h] = sv.x;
            s[4 * h + 1] = sv.y;
            s[4 * h + 2] = sv.z;
            s[4 * h + 3] = sv.w;
        }
        if (a.zp != nullptr) {
#pragma unroll
            for (int h = 0; h < E / 4; h++) {
                const uint32_t w = __ldg(reinterpret_cast<const unsigned int*>(static_cast<const uint8_t*>(a.zp) + pi) + h);
#pragma unroll
                for (int e = 0; e < 4; e++) {
                    const uint32_t b = (w >> (8 * e)) & 0xFFu;
                    z[4 * h + e] = KIND == 1 ? static_cast<int32_t>(static_cast<int8_t>(b)) : static_cast<int32_t>(b);
                }
            }
        } else {
#pragma unroll
            for (int e = 0; e < E; e++) z[e] = 0;
        }
    } else {
        const float s0 = __ldg(a.scale + pi);
        const int32_t z0 = a.zp != nullptr ? load_q<KIND>(a.zp, pi) : 0;
#pragma unroll
        for (int e = 0; e < E; e++) {
            s[e] = s0;
            z[e] = z0;
        }
    }
}

template <int KIND, bool HALF>
__device__ __forceinline__ void dq_store(const QuantArgs& a, int64_t first, const float (&v)[DqShape<KIND, HALF>::E]) {
    constexpr int E = DqShape<KIND, HALF>::E;
    if constexpr (!HALF) {
        __stcs(reinterpret_cast<float4*>(static_cast<float*>(a.out) + first), make_float4(v[0], v[1], v[2], v[3]));
    } else {
        uint32_t w[E / 2];
#pragma unroll
        for (int e = 0; e < E / 2; e++)
            w[e] = static_cast<uint32_t>(__half_as_ushort(__float2half_rn(v[2 * e]))) |
                   (static_cast<uint32_t>(__half_as_ushort(__float2half_rn(v[2 * e + 1]))) << 16);
        if constexpr (E == 8)
            __stcs(reinterpret_cast<uint4*>(static_cast<__half*>(a.out) + first), make_uint4(w[0], w[1], w[2], w[3]));
        else
            __stcs(reinterpret_cast<uint2*>(static_cast<__half*>(a.out) + first), make_uint2(w[0], w[1]));
    }
}

template <int KIND, bool HALF>
__device__ __forceinline__ void dq_scalar(const QuantArgs& a, int64_t j) {
    const float v = dequantize_one<KIND>(a, load_q<KIND>(a.x, j), param_at(a, j));
    if constexpr (HALF)
        static_cast<__half*>(a.out)[j] = __float2half_rn(v);
    else
        static_cast<float*>(a.out)[j] = v;
}

template <int KIND, bool HALF>
__global__ void __launch_bounds__(QTHREADS) dequantize_kernel(const QuantArgs a) {
    pdl_trigger();
    pdl_wait();
    constexpr int E = DqShape<KIND, HALF>::E;
    const int64_t tid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const int64_t nthreads = static_cast<int64_t>(gridDim.x) * blockDim.x;
    const int64_t tail0 = a.head + a.vectors * E;
    if (tid < a.head) dq_scalar<KIND, HALF>(a, tid);
    if (tid < a.count - tail0) dq_scalar<KIND, HALF>(a, tail0 + tid);
    for (int64_t v0 = tid; v0 < a.vectors; v0 += nthreads * UNROLL) {
        int32_t q[UNROLL][E];
#pragma unroll
        for (int u = 0; u < UNROLL; u++)
            if (v0 + u * nthreads < a.vectors) dq_load<KIND, HALF>(a, a.head + (v0 + u * nthreads) * E, q[u]);
#pragma unroll
        for (int u = 0; u < UNROLL; u++) {
            const int64_t vi = v0 + u * nthreads;
            if (vi >= a.vectors) break;
            const int64_t first = a.head + vi * E;
            ParamCursor c = param_at(a, first);
            float v[E];
            if (KIND != 2 && (a.vec_params || !a.per_axis || c.r + E <= a.inner)) {
                // Byte inputs with the vector's parameters in one or E consecutive places: loaded once, d = q - zp
                // is at most 255 in size (converted exactly without the conversion unit).
                float s[E];
                int32_t z[E];
                dq_params<KIND, E>(a, c.pi, a.vec_params != 0, s, z);
#pragma unroll
                for (int e = 0; e < E; e++) v[e] = __fmul_rn(small_int_to_float(q[u][e] - z[e]), s[e]);
            } else {
#pragma unroll
                for (int e = 0; e < E; e++) {
                    v[e] = dequantize_one<KIND>(a, q[u][e], c);
                    param_next(a, c);
                }
            }
            dq_store<KIND, HALF>(a, first, v);
        }
    }
}

// The 16 inputs x[first .. first + 15] of one vector (four float or two half 16-byte loads).
template <bool HALF>
__device__ __forceinline__ void q_load16(const QuantArgs& a, int64_t first, float (&x)[16]) {
    if constexpr (HALF) {
        const uint4* p = reinterpret_cast<const uint4*>(static_cast<const __half*>(a.x) + first);
#pragma unroll
        for (int v = 0; v < 2; v++) {
            const uint4 w = __ldcs(p + v);
            const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
            for (int e = 0; e < 4; e++) {
                x[8 * v + 2 * e] = __half2float(__ushort_as_half(static_cast<unsigned short>(ws[e] & 0xFFFFu)));
                x[8 * v + 2 * e + 1] = __half2float(__ushort_as_half(static_cast<unsigned short>(ws[e] >> 16)));
            }
        }
    } else {
        const float4* p = reinterpret_cast<const float4*>(static_cast<const float*>(a.x) + first);
#pragma unroll
        for (int v = 0; v < 4; v++) {
            const float4 w = __ldcs(p + v);
            x[4 * v] = w.x;
            x[4 * v + 1] = w.y;
            x[4 * v + 2] = w.z;
            x[4 * v + 3] = w.w;
        }
    }
}

// Thread t owns output bytes [head + 16 t, +16): one 16-byte store, consecutive threads consecutive stores. When the
// 16 elements share one scale (per tensor, or a run of `inner` elements that covers them), the quotient is formed by
// the multiply-first rounding; otherwise each element divides by its own scale.
template <bool SIGNED, bool HALF>
__global__ void __launch_bounds__(QTHREADS) quantize_kernel(const QuantArgs a) {
    pdl_trigger();
    pdl_wait();
    constexpr int E = 16;
    const int64_t tid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    uint8_t* y = static_cast<uint8_t*>(a.out);
    const int64_t tail0 = a.head + a.vectors * E;
    if (tid < a.head) y[tid] = static_cast<uint8_t>(quantize_one<SIGNED>(a, load_x<HALF>(a.x, tid), param_at(a, tid)));
    if (tid < a.count - tail0) {
        const int64_t j = tail0 + tid;
        y[j] = static_cast<uint8_t>(quantize_one<SIGNED>(a, load_x<HALF>(a.x, j), param_at(a, j)));
    }
    if (tid >= a.vectors) return;
    const int64_t first = a.head + tid * E;
    float x[16];
    q_load16<HALF>(a, first, x);
    ParamCursor c = param_at(a, first);
    uint32_t w[4] = {0, 0, 0, 0};
    if (!a.per_axis || c.r + E <= a.inner) {
        QParam p;
        qparam_load<SIGNED>(a, c.pi, p);
        const float r = __frcp_rn(p.s);
        const bool r_ok = fabsf(r) >= 1.17549435e-38f && fabsf(r) <= 3.40282347e+38f;  // normal and finite
#pragma unroll
        for (int e = 0; e < E; e++)
            w[e >> 2] |= saturate_byte<SIGNED>(__fadd_rn(rne_quotient_r(x[e], p.s, r, r_ok), p.zf)) << (8 * (e & 3));
    } else {
        QParam p;
        qparam_load<SIGNED>(a, c.pi, p);
#pragma unroll
        for (int e = 0; e < E; e++) {
            if (c.pi != p.pi) qparam_load<SIGNED>(a, c.pi, p);
            w[e >> 2] |= quantize_with<SIGNED>(x[e], p) << (8 * (e & 3));
            param_next(a, c);
        }
    }
    if (a.keep_out)
        *reinterpret_cast<uint4*>(y + first) = make_uint4(w[0], w[1], w[2], w[3]);
    else
        __stcs(reinterpret_cast<uint4*>(y + first), make_uint4(w[0], w[1], w[2], w[3]));
}

// Splits the elements into a scalar head (up to the output's first boundary of `out_align` bytes), whole vectors of E
// elements whose input (in_esize bytes per element) and output both start aligned, and a scalar tail; when the input
// is not aligned where the output is, everything goes element by element.
static void split_vectors(QuantArgs& a, int e, int in_esize, int out_esize, int in_align, int out_align) {
    const uintptr_t o = reinterpret_cast<uintptr_t>(a.out);
    int64_t head = static_cast<int64_t>((out_align - (o % out_align)) % out_align) / out_esize;
    if (head > a.count) head = a.count;
    const uintptr_t xin = reinterpret_cast<uintptr_t>(a.x) + static_cast<uintptr_t>(head) * in_esize;
    a.head = head;
    a.vectors = (xin % in_align) == 0 ? (a.count - head) / e : 0;
    if (a.vectors == 0) a.head = 0;
    const int64_t scalar = a.count - a.vectors * e;  // head + tail elements, one thread each
    const int64_t want = (a.vectors + UNROLL - 1) / UNROLL;
    a.threads = want > scalar ? want : scalar;
}

static unsigned grid_of(const QuantArgs& a) {
    const int64_t blocks = (a.threads + QTHREADS - 1) / QTHREADS;
    return static_cast<unsigned>(blocks < 1 ? 1 : blocks);
}

static cudaError_t launch_dequantize(QuantArgs a, int kind, bool half, cudaStream_t s) {
    const int in_es = kind == 2 ? 4 : 1, out_es = half ? 2 : 4;
    const int e = (kind != 2 && half) ? 8 : 4;
    split_vectors(a, e, in_es, out_es, e * in_es, e * out_es);
    set_param_magics(a);
    // Parameters along the contiguous axis: vector v's E parameters start at (head + v E) % axis_len, a multiple of E
    // when head and axis_len are, and load as whole vectors when the arrays are aligned for them.
    a.vec_params = kind != 2 && a.per_axis && a.inner == 1 && a.axis_len % e == 0 && a.head % e == 0 &&
                   (reinterpret_cast<uintptr_t>(a.scale) & 15) == 0 &&
                   (a.zp == nullptr || (reinterpret_cast<uintptr_t>(a.zp) & 3) == 0);
    const unsigned blocks = grid_of(a);
    switch (kind * 2 + (half ? 1 : 0)) {
        case 0: return launch_pdl(dequantize_kernel<0, false>, dim3(blocks), dim3(QTHREADS), 0, s, a);
        case 1: return launch_pdl(dequantize_kernel<0, true>, dim3(blocks), dim3(QTHREADS), 0, s, a);
        case 2: return launch_pdl(dequantize_kernel<1, false>, dim3(blocks), dim3(QTHREADS), 0, s, a);
        case 3: return launch_pdl(dequantize_kernel<1, true>, dim3(blocks), dim3(QTHREADS), 0, s, a);
        case 4: return launch_pdl(dequantize_kernel<2, false>, dim3(blocks), dim3(QTHREADS), 0, s, a);
        default: return launch_pdl(dequantize_kernel<2, true>, dim3(blocks), dim3(QTHREADS), 0, s, a);
    }
}

static cudaError_t launch_quantize(QuantArgs a, bool is_signed, bool half, cudaStream_t s);

// DynamicQuantizeLinear's second pass is QuantizeLinear per tensor to uint8 with the scale and zero point the first
// pass stored on the device: clamp(round_half_even(x / scale) + zp, 0, 255), NaN to 0.
cudaError_t launch_quantize_u8_tensor(const float* x, int64_t count, uint8_t* y, const float* scale,
                                      const uint8_t* zero_point, cudaStream_t s) {
    QuantArgs a{};
    a.x = x;
    a.count = count;
    a.scale = scale;
    a.zp = zero_point;
    a.per_axis = 0;
    a.axis_len = 1;
    a.inner = 1;
    a.out = y;
    a.keep_out = 1;  // the product (and its byte sums) read the bytes next: leave them in L2
    return launch_quantize(a, false, false, s);
}

static cudaError_t launch_quantize(QuantArgs a, bool is_signed, bool half, cudaStream_t s) {
    split_vectors(a, 16, half ? 2 : 4, 1, 16, 16);
    set_param_magics(a);
    const int64_t scalar = a.count - a.vectors * 16;
    a.threads = a.vectors > scalar ? a.vectors : scalar;  // one vector per thread
    const unsigned blocks = grid_of(a);
    switch ((is_signed ? 2 : 0) + (half ? 1 : 0)) {
        case 0: return launch_pdl(quantize_kernel<false, false>, dim3(blocks), dim3(QTHREADS), 0, s, a);
        case 1: return launch_pdl(quantize_kernel<false, true>, dim3(blocks), dim3(QTHREADS), 0, s, a);
        case 2: return launch_pdl(quantize_kernel<true, false>, dim3(blocks), dim3(QTHREADS), 0, s, a);
        default: return launch_pdl(quantize_kernel<true, true>, dim3(blocks), dim3(QTHREADS), 0, s, a);
    }
}

}  // namespace og

// ---- argument checks and C ABI ------------------------------------------------------------------------------------

struct og_dequantize {
    og_device* device = nullptr;
};

namespace {

using namespace og_host;

const char* kDequant = "DequantizeLinear";
const char* kQuant = "QuantizeLinear";

// KernelTypes.IsHalf<T> (KernelSupport.cs:50-65, with KernelTypes.Of's message for types outside its list).
bool is_half(const char* op, int32_t t) {
    if (t == OG_F32) return false;
    if (t == OG_F16) return true;
    if (t == OG_I32 || t == OG_U32 || t == OG_I64)
        shape(op, "T", std::string("element type ") + type_name(t) + " is not supported; use float or Half");
    shape(op, "T", std::string("element type ") + type_name(t) +
                       " is not supported; use float, Half, int, long or uint as the operation allows");
}

struct Geometry {
    int64_t count = 0;
    int64_t axis_len = 1;
    int64_t inner = 1;
};

Geometry geometry(const char* op, const int32_t* dims, int32_t rank, int32_t axis, int32_t per_axis) {
    if (rank < 0) shape(op, "shape", "rank " + std::to_string(rank) + " is negative");
    if (rank > 0 && dims == nullptr) null_arg(op, "shape");
    Geometry g;
    g.count = product(op, "shape", dims, rank);
    if (per_axis) {
        const int32_t ax = axis_of(op, axis, rank);
        g.axis_len = dims[ax];
        for (int32_t i = ax + 1; i < rank; i++) g.inner *= dims[i];
    }
    return g;
}

void require_float_scale(const char* op, const og_buffer* scale) {
    if (scale->type != OG_F32)
        shape(op, "scale", std::string("element type ") + type_name(scale->type) + " is not supported; use float");
}

// DequantizeKernels.Encode's checks in the reference's order (DequantizeKernels.cs:64-130). Returns the input kind
// (0 uint8, 1 int8, 2 int32) and whether the output is half.
Geometry check_dequantize(const og_buffer* x, int32_t offset_x, const int32_t* dims, int32_t rank, int32_t axis,
                          int32_t per_axis, const og_buffer* scale, int32_t offset_scale, const og_buffer* zp,
                          int32_t offset_zp, const og_buffer* out, int32_t offset_out, int* kind, bool* half) {
    if (x == nullptr) null_arg(kDequant, "x");
    if (scale == nullptr) null_arg(kDequant, "scale");
    if (out == nullptr) null_arg(kDequant, "output");
    if (x->type == OG_U8) *kind = 0;
    else if (x->type == OG_S8) *kind = 1;
    else if (x->type == OG_I32) *kind = 2;
    else
        shape(kDequant, "TIn", std::string("element type ") + type_name(x->type) +
                                   " is not supported; use byte (uint8), sbyte (int8) or int");
    *half = is_half(kDequant, out->type);
    const Geometry g = geometry(kDequant, dims, rank, axis, per_axis);
    const int64_t params = per_axis ? g.axis_len : 1;
    require_float_scale(kDequant, scale);
    range(kDequant, "scale", scale->length, offset_scale, params);
    if (*kind == 2) range(kDequant, "x", x->length, offset_x, g.count);
    else range_bytes(kDequant, "x", x->length, offset_x, g.count);
    if (zp != nullptr) {
        if (zp->type != x->type)
            shape(kDequant, "zeroPoint", std::string("element type ") + type_name(zp->type) +
                                             " differs from the type of x, " + type_name(x->type));
        if (*kind == 2) range(kDequant, "zeroPoint", zp->length, offset_zp, params);
        else range_bytes(kDequant, "zeroPoint", zp->length, offset_zp, params);
    }
    if (*half) range_half(kDequant, "output", out->length, offset_out, g.count);
    else range(kDequant, "output", out->length, offset_out, g.count);
    return g;
}

// DequantizeKernels.EncodeQuantize's checks in the reference's order (DequantizeKernels.cs:184-240).
Geometry check_quantize(const og_buffer* x, int32_t offset_x, const int32_t* dims, int32_t rank, int32_t axis,
                        int32_t per_axis, const og_buffer* scale, int32_t offset_scale, const og_buffer* zp,
                        int32_t offset_zp, const og_buffer* out, int32_t offset_out, bool* is_signed, bool* half) {
    if (x == nullptr) null_arg(kQuant, "x");
    if (scale == nullptr) null_arg(kQuant, "scale");
    if (out == nullptr) null_arg(kQuant, "output");
    if (out->type == OG_U8) *is_signed = false;
    else if (out->type == OG_S8) *is_signed = true;
    else
        shape(kQuant, "TOut", std::string("element type ") + type_name(out->type) +
                                  " is not supported; use byte (uint8) or sbyte (int8)");
    *half = is_half(kQuant, x->type);
    const Geometry g = geometry(kQuant, dims, rank, axis, per_axis);
    const int64_t params = per_axis ? g.axis_len : 1;
    if (*half) range_half(kQuant, "x", x->length, offset_x, g.count);
    else range(kQuant, "x", x->length, offset_x, g.count);
    require_float_scale(kQuant, scale);
    range(kQuant, "scale", scale->length, offset_scale, params);
    if (zp != nullptr) {
        if (zp->type != out->type)
            shape(kQuant, "zeroPoint", std::string("element type ") + type_name(zp->type) +
                                           " differs from the output's, " + type_name(out->type));
        range_bytes(kQuant, "zeroPoint", zp->length, offset_zp, params);
    }
    range_bytes(kQuant, "output", out->length, offset_out, g.count);
    return g;
}

og::QuantArgs args_of(const Geometry& g, const og_buffer* x, int32_t offset_x, int x_esize, const og_buffer* scale,
                      int32_t offset_scale, const og_buffer* zp, int32_t offset_zp, int zp_esize, int32_t per_axis,
                      const og_buffer* out, int32_t offset_out, int out_esize) {
    og::QuantArgs a{};
    a.x = static_cast<const uint8_t*>(x->ptr) + static_cast<int64_t>(offset_x) * x_esize;
    a.count = g.count;
    a.scale = static_cast<const float*>(scale->ptr) + offset_scale;
    a.zp = zp != nullptr ? static_cast<const uint8_t*>(zp->ptr) + static_cast<int64_t>(offset_zp) * zp_esize : nullptr;
    a.per_axis = per_axis ? 1 : 0;
    a.axis_len = static_cast<uint32_t>(g.axis_len > 0 ? g.axis_len : 1);
    a.inner = static_cast<uint32_t>(g.inner > 0 ? g.inner : 1);
    a.out = static_cast<uint8_t*>(out->ptr) + static_cast<int64_t>(offset_out) * out_esize;
    return a;
}

}  // namespace

extern "C" {

OG_API og_status og_dequantize_create(og_device* d, og_dequantize** out) {
    return guard([&] {
        if (d == nullptr) null_arg(kDequant, "device");
        if (out == nullptr) null_arg(kDequant, "out");
        auto* k = new og_dequantize();
        k->device = d;
        *out = k;
    });
}

OG_API og_status og_dequantize_destroy(og_dequantize* k) {
    return guard([&] { delete k; });
}

OG_API og_status og_dequantize_check(const og_buffer* x, int32_t offset_x, const int32_t* shape_, int32_t rank,
                                     int32_t axis, int32_t per_axis, const og_buffer* scale, int32_t offset_scale,
                                     const og_buffer* zero_point, int32_t offset_zero_point, const og_buffer* output,
                                     int32_t offset_output) {
    return guard([&] {
        int kind;
        bool half;
        check_dequantize(x, offset_x, shape_, rank, axis, per_axis, scale, offset_scale, zero_point, offset_zero_point,
                         output, offset_output, &kind, &half);
    });
}

OG_API og_status og_dequantize_check_quantize(const og_buffer* x, int32_t offset_x, const int32_t* shape_,
                                              int32_t rank, int32_t axis, int32_t per_axis, const og_buffer* scale,
                                              int32_t offset_scale, const og_buffer* zero_point,
                                              int32_t offset_zero_point, const og_buffer* output,
                                              int32_t offset_output) {
    return guard([&] {
        bool is_signed, half;
        check_quantize(x, offset_x, shape_, rank, axis, per_axis, scale, offset_scale, zero_point, offset_zero_point,
                       output, offset_output, &is_signed, &half);
    });
}

OG_API og_status og_dequantize_encode(og_dequantize* k, og_encoder* enc, const og_buffer* x, int32_t offset_x,
                                      const int32_t* shape_, int32_t rank, int32_t axis, int32_t per_axis,
                                      const og_buffer* scale, int32_t offset_scale, const og_buffer* zero_point,
                                      int32_t offset_zero_point, const og_buffer* output, int32_t offset_output) {
    return guard([&] {
        if (k == nullptr) throw OgError{OG_ERROR_INVALID_HANDLE, kDequant, "kernels", "null handle", "", "", ""};
        if (enc == nullptr) null_arg(kDequant, "encoder");
        int kind;
        bool half;
        const Geometry g = check_dequantize(x, offset_x, shape_, rank, axis, per_axis, scale, offset_scale,
                                            zero_point, offset_zero_point, output, offset_output, &kind, &half);
        if (g.count == 0) return;
        const int xs = kind == 2 ? 4 : 1;
        const og::QuantArgs a = args_of(g, x, offset_x, xs, scale, offset_scale, zero_point, offset_zero_point, xs,
                                        per_axis, output, offset_output, half ? 2 : 4);
        enc->ops.push_back([=](cudaStream_t s) { return og::launch_dequantize(a, kind, half, s); });
        enc->dispatches += 1;
    });
}

OG_API og_status og_dequantize_encode_quantize(og_dequantize* k, og_encoder* enc, const og_buffer* x,
                                               int32_t offset_x, const int32_t* shape_, int32_t rank, int32_t axis,
                                               int32_t per_axis, const og_buffer* scale, int32_t offset_scale,
                                               const og_buffer* zero_point, int32_t offset_zero_point,
                                               const og_buffer* output, int32_t offset_output) {
    return guard([&] {
        if (k == nullptr) throw OgError{OG_ERROR_INVALID_HANDLE, kQuant, "kernels", "null handle", "", "", ""};
        if (enc == nullptr) null_arg(kQuant, "encoder");
        bool is_signed, half;
        const Geometry g = check_quantize(x, offset_x, shape_, rank, axis, per_axis, scale, offset_scale, zero_point,
                                          offset_zero_point, output, offset_output, &is_signed, &half);
        if (g.count == 0) return;
        const og::QuantArgs a = args_of(g, x, offset_x, half ? 2 : 4, scale, offset_scale, zero_point,
                                        offset_zero_point, 1, per_axis, output, offset_output, 1);
        enc->ops.push_back([=](cudaStream_t s) { return og::launch_quantize(a, is_signed, half, s); });
        enc->dispatches += 1;
    });
}

}  // extern "C"
