// DynamicQuantizeLinear (float32 -> uint8) in two kernels:
//  1. dq_range: every thread folds a grid-stride slice of x (16-byte loads where x is aligned) into a minimum and a
//     maximum, warps reduce with shuffles, blocks write one partial each; the last block to finish (ticket counter,
//     no spinning) combines the partials and derives scale and zero point, which it stores for the caller and for
//     pass 2.
//  2. QuantizeLinear per tensor to uint8 (og_quant.cu) with the scale and zero point pass 1 stored: the same
//     arithmetic, y = clamp(round_half_even(x / scale) + zero point, 0, 255), NaN to 0.
// The arithmetic is onemodel's (DynamicQuantizeKernels.cs:9-16): lo = min(0, min x), hi = max(0, max x),
// scale = (hi - lo) / 255, zero point = clamp(round_half_even(-(lo / scale)), 0, 255) when scale is finite and not 0,
// an all-zero range gives scale 1 and zero point 0, y = clamp(round_half_even(x / scale) + zero point, 0, 255) and
// NaN gives 0. The divisions are IEEE round-to-nearest (__fdiv_rn), rounding is rintf (half to even), and minimum and
// maximum do not depend on the order they are found in, so the bits equal the CPU's.
#include <cuda_runtime.h>

#include "og_gemm.h"
#include "og_ptx.cuh"

namespace og {

constexpr int DQ_MAX_BLOCKS = 1024;
constexpr int DQ_THREADS = 256;

struct DqScratch {
    float part_min[DQ_MAX_BLOCKS];
    float part_max[DQ_MAX_BLOCKS];
    unsigned int ticket;
    float scale;
    int zero_point;
};

size_t dq_scratch_bytes() { return sizeof(DqScratch); }

__device__ __forceinline__ void block_min_max(float& mn, float& mx, float* smin, float* smax) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        mn = fminf(mn, __shfl_xor_sync(0xFFFFFFFFu, mn, o));
        mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, o));
    }
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) {
        smin[warp] = mn;
        smax[warp] = mx;
    }
    __syncthreads();
    if (warp == 0) {
        const int nw = blockDim.x >> 5;
        mn = lane < nw ? smin[lane] : INFINITY;
        mx = lane < nw ? smax[lane] : -INFINITY;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            mn = fminf(mn, __shfl_xor_sync(0xFFFFFFFFu, mn, o));
            mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, o));
        }
    }
}

// fminf / fmaxf skip NaN exactly like the reference's `v < min` / `v > max` tests; they may order -0 and +0 either
// way, which cannot change scale or zero point (both give hi - lo and lo / scale of the same value).
__global__ void __launch_bounds__(DQ_THREADS)
    dq_range_kernel(const float* __restrict__ x, int64_t count, DqScratch* __restrict__ s, float* __restrict__ scale_out,
                    uint8_t* __restrict__ zp_out) {
    pdl_trigger();
    pdl_wait();
    __shared__ float smin[32], smax[32];
    __shared__ bool last;
    float mn = INFINITY, mx = -INFINITY;
    const int64_t tid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const int64_t nthreads = static_cast<int64_t>(gridDim.x) * blockDim.x;
    // Elements before the first 16-byte boundary, then float4 body, then the tail.
    int64_t head = static_cast<int64_t>(((16 - (reinterpret_cast<uintptr_t>(x) & 15)) & 15) >> 2);
    if (head > count) head = count;
    for (int64_t i = tid; i < head; i += nthreads) {
        const float v = __ldg(x + i);
        mn = fminf(mn, v);
        mx = fmaxf(mx, v);
    }
    const int64_t nvec = (count - head) / 4;
    const float4* xv = reinterpret_cast<const float4*>(x + head);
    constexpr int U = 4;  // loads in flight per thread
    for (int64_t i0 = tid; i0 < nvec; i0 += nthreads * U) {
        float4 v[U];
#pragma unroll
        for (int u = 0; u < U; u++) {
            const int64_t i = i0 + u * nthreads;
            v[u] = i < nvec ? __ldg(xv + i) : make_float4(NAN, NAN, NAN, NAN);  // NaN is skipped by fminf/fmaxf
        }
#pragma unroll
        for (int u = 0; u < U; u++) {
            mn = fminf(mn, fminf(fminf(v[u].x, v[u].y), fminf(v[u].z, v[u].w)));
            mx = fmaxf(mx, fmaxf(fmaxf(v[u].x, v[u].y), fmaxf(v[u].z, v[u].w)));
        }
    }
    for (int64_t i = head + nvec * 4 + tid; i < count; i += nthreads) {
        const float v = __ldg(x + i);
        mn = fminf(mn, v);
        mx = fmaxf(mx, v);
    }
    block_min_max(mn, mx, smin, smax);
    if (threadIdx.x == 0) {
        s->part_min[blockIdx.x] = mn;
        s->part_max[blockIdx.x] = mx;
        __threadfence();
        const unsigned t = atomicAdd(&s->ticket, 1u);
        last = (t == gridDim.x - 1);
    }
    __syncthreads();
    if (!last) return;
    __threadfence();
    mn = INFINITY;
    mx = -INFINITY;
    for (int i = threadIdx.x; i < static_cast<int>(gridDim.x); i += blockDim.x) {
        mn = fminf(mn, __ldcg(&s->part_min[i]));
        mx = fmaxf(mx, __ldcg(&s->part_max[i]));
    }
    __syncthreads();
    block_min_max(mn, mx, smin, smax);
    if (threadIdx.x == 0) {
        const float lo = mn < 0.0f ? mn : 0.0f;
        const float hi = mx > 0.0f ? mx : 0.0f;
        float scale = __fdiv_rn(__fsub_rn(hi, lo), 255.0f);
        int zp = 0;
        if (scale != 0.0f && isfinite(scale)) {
            const float z = rintf(__fsub_rn(0.0f, __fdiv_rn(lo, scale)));
            zp = z < 0.0f ? 0 : (z > 255.0f ? 255 : static_cast<int>(z));
        }
        if (scale == 0.0f) {
            scale = 1.0f;
            zp = 0;
        }
        s->scale = scale;
        s->zero_point = zp;
        s->ticket = 0;
        *scale_out = scale;
        *zp_out = static_cast<uint8_t>(zp);
    }
}

cudaError_t launch_dynamic_quantize(const float* x, int64_t count, uint8_t* y, float* scale_out, uint8_t* zp_out,
                                    DqScratch* scratch, int num_sms, cudaStream_t stream) {
    int64_t blocks = (count + DQ_THREADS * 16 - 1) / (DQ_THREADS * 16);
    const int64_t cap = 4 * static_cast<int64_t>(num_sms) < DQ_MAX_BLOCKS ? 4 * static_cast<int64_t>(num_sms)
                                                                          : DQ_MAX_BLOCKS;
    if (blocks > cap) blocks = cap;
    if (blocks < 1) blocks = 1;
    cudaError_t err = launch_pdl(dq_range_kernel, dim3(static_cast<unsigned>(blocks)), dim3(DQ_THREADS), 0, stream, x,
                                 count, scratch, scale_out, zp_out);
    if (err != cudaSuccess) return err;
    // Pass 2 is QuantizeLinear per tensor with the scale and zero point pass 1 stored for the caller.
    return launch_quantize_u8_tensor(x, count, y, scale_out, zp_out, stream);
}

}  // namespace og
