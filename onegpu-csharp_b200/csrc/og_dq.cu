// DynamicQuantizeLinear (float32 -> uint8). Tensors of 2^18 elements and more with aligned buffers take one
// cooperative kernel (dq_fused_kernel, below: x read from DRAM once, most of it kept on chip across a grid barrier);
// the others take two kernels:
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

#include <atomic>

#include "og_gemm.h"
#include "og_ptx.cuh"
#include "og_qmath.cuh"

namespace og {

constexpr int DQ_MAX_BLOCKS = 1024;
constexpr int DQ_THREADS = 256;

struct DqScratch {
    float part_min[DQ_MAX_BLOCKS];
    float part_max[DQ_MAX_BLOCKS];
    unsigned int ticket;
    float scale;
    int zero_point;
    // The single-kernel path's grid barrier: arrivals of all its launches so far (a multiple of the grid size between
    // launches, every CTA arriving once per launch); a launch's CTAs wait for the next multiple.
    unsigned long long arrivals;
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

// Scale and zero point of the range [mn, mx] (DynamicQuantizeKernels.cs:9-16).
__device__ __forceinline__ void dq_scale_zero_point(float mn, float mx, float& scale, int& zp) {
    const float lo = mn < 0.0f ? mn : 0.0f;
    const float hi = mx > 0.0f ? mx : 0.0f;
    scale = __fdiv_rn(__fsub_rn(hi, lo), 255.0f);
    zp = 0;
    if (scale != 0.0f && isfinite(scale)) {
        const float z = rintf(__fsub_rn(0.0f, __fdiv_rn(lo, scale)));
        zp = z < 0.0f ? 0 : (z > 255.0f ? 255 : static_cast<int>(z));
    }
    if (scale == 0.0f) {
        scale = 1.0f;
        zp = 0;
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
        float scale;
        int zp;
        dq_scale_zero_point(mn, mx, scale, zp);
        s->scale = scale;
        s->zero_point = zp;
        s->ticket = 0;
        *scale_out = scale;
        *zp_out = static_cast<uint8_t>(zp);
    }
}

// ---- one kernel: range, grid barrier, quantize from on-chip copies -----------------------------------------------
//
// For tensors of at least DQF_MIN_COUNT floats: one CTA per SM (a cooperative launch, so all are resident), each
// owning a contiguous slice of x. The first DQF_SMEM_VECS float4 of its slice arrive in shared memory by bulk copies,
// the next DQF_KEEP float4 per thread are loaded into registers and kept, and the rest is read for the range only.
// After the block's range is folded and published, the CTAs meet at a grid barrier (bounded wait), every CTA derives
// the same scale and zero point from all the partial ranges, and each quantizes its slice: the staged and kept parts
// from the chip, only the rest from memory again. x is read from DRAM once plus that rest, against twice for the
// two-kernel path.

constexpr int DQF_THREADS = 1024;
constexpr int DQF_SMEM_VECS = 14336;  // 224 KB of float4 per CTA
constexpr int DQF_SMEM_BYTES = DQF_SMEM_VECS * 16;
constexpr int DQF_KEEP = 4;           // float4 kept in registers per thread (64 KB per CTA)
constexpr int DQF_CHUNK = 16384;      // bytes per bulk copy
constexpr int64_t DQF_MIN_COUNT = int64_t(1) << 18;

__device__ __forceinline__ void fold4(const float4& v, float& mn, float& mx) {
    mn = fminf(mn, fminf(fminf(v.x, v.y), fminf(v.z, v.w)));
    mx = fmaxf(mx, fmaxf(fmaxf(v.x, v.y), fmaxf(v.z, v.w)));
}

// clamp(round_half_even(x / s) + zero point, 0, 255) with the quotient rule of rne_quotient_r, returned in the low
// byte. Where the rule accepts m = RN(x * r) (away from half-integers), t = RN(m + cz) with cz = zero point +
// 1.5 * 2^23 lies in [2^23, 2^24), where floats are the integers: t = cz + round(m) exactly, t - cz gives round(m) for
// the rule's test, and t's bits (0x4B400000 + round(m) + zero point, monotonic in t) are clamped to
// [0x4B400000, 0x4B4000FF] with integer min / max, leaving the byte in the low 8 bits. Elsewhere the quotient is
// divided exactly and clamped in floating point (NaN to 0). Here the scale is the tensor's own range over 255, so
// every finite x has |x / s| <= 255 and |m| <= 256: the rule's margin |m| 2^-20 + 2^-19 is then below 2^-11, and
// the test is |d| < 1/2 - 2^-11 (NaN, infinities and a non-normal reciprocal fail it and take the exact path).
struct DqQuant {
    float s, r, zf, cz;
    bool r_ok;
    __device__ __forceinline__ uint32_t one(float x) const {
        const float m = __fmul_rn(x, r);
        const float t = __fadd_rn(m, cz);
        const float d = __fsub_rn(m, __fsub_rn(t, cz));
        if (r_ok && fabsf(d) < 0.5f - 0x1p-11f) return min(max(__float_as_uint(t), 0x4B400000u), 0x4B4000FFu);
        return saturate_byte<false>(__fadd_rn(rne_quotient_exact(x, s), zf));
    }
    __device__ __forceinline__ uint32_t four(const float4& v) const {
        return __byte_perm(__byte_perm(one(v.x), one(v.y), 0x0040), __byte_perm(one(v.z), one(v.w), 0x0040), 0x5410);
    }
};

__global__ void __launch_bounds__(DQF_THREADS, 1)
    dq_fused_kernel(const float* __restrict__ x, int64_t count, uint8_t* __restrict__ y, DqScratch* __restrict__ s,
                    float* __restrict__ scale_out, uint8_t* __restrict__ zp_out, int* __restrict__ error_flag) {
    extern __shared__ __align__(128) uint8_t dqf_smem[];
    __shared__ uint64_t bar;
    __shared__ float smin[32], smax[32];
    __shared__ int failed;
    __shared__ float q_scale;
    __shared__ int q_zp;
    pdl_trigger();
    pdl_wait();
    const int T = DQF_THREADS, t = threadIdx.x;
    const int G = gridDim.x, b = blockIdx.x;
    const float4* xv = reinterpret_cast<const float4*>(x);
    const float4* sv = reinterpret_cast<const float4*>(dqf_smem);
    const int64_t nvec = count >> 2;
    const int64_t v0 = nvec * b / G, v1 = nvec * (b + 1) / G;
    const int n_s = static_cast<int>(v1 - v0 < DQF_SMEM_VECS ? v1 - v0 : DQF_SMEM_VECS);
    const int64_t r0 = v0 + n_s;  // the first vector not staged
    if (t == 0) {
        mbar_init(&bar, 1);
        fence_mbar_init();
        failed = 0;
    }
    __syncthreads();
    if (t == 0 && n_s > 0) {
        const uint32_t bytes = static_cast<uint32_t>(n_s) * 16u;
        mbar_arrive_expect_tx(&bar, bytes);
        for (uint32_t off = 0; off < bytes; off += DQF_CHUNK)
            bulk_load(dqf_smem + off, reinterpret_cast<const uint8_t*>(xv + v0) + off,
                      bytes - off < DQF_CHUNK ? bytes - off : DQF_CHUNK, &bar);
    }
    float mn = INFINITY, mx = -INFINITY;
    // Kept in registers: vectors r0 + j T + t.
    float4 keep[DQF_KEEP];
#pragma unroll
    for (int j = 0; j < DQF_KEEP; j++) {
        const int64_t i = r0 + int64_t(j) * T + t;
        keep[j] = i < v1 ? __ldg(xv + i) : make_float4(NAN, NAN, NAN, NAN);
        fold4(keep[j], mn, mx);
    }
    // Read for the range only: the rest of the slice, four loads in flight per thread.
    const int64_t rest0 = r0 + int64_t(DQF_KEEP) * T;
    for (int64_t i0 = rest0 + t; i0 < v1; i0 += 4 * int64_t(T)) {
        float4 v[4];
#pragma unroll
        for (int u = 0; u < 4; u++) {
            const int64_t i = i0 + int64_t(u) * T;
            v[u] = i < v1 ? __ldg(xv + i) : make_float4(NAN, NAN, NAN, NAN);
        }
#pragma unroll
        for (int u = 0; u < 4; u++) fold4(v[u], mn, mx);
    }
    if (b == G - 1)
        for (int64_t i = nvec * 4 + t; i < count; i += T) {
            const float v = __ldg(x + i);
            mn = fminf(mn, v);
            mx = fmaxf(mx, v);
        }
    // The staged part, once it has landed.
    if (n_s > 0 && !mbar_wait(&bar, 0, &failed)) failed = 1;
    __syncthreads();
    if (!failed)
        for (int i = t; i < n_s; i += T) fold4(sv[i], mn, mx);
    block_min_max(mn, mx, smin, smax);

    // Grid barrier: publish this CTA's range, arrive, wait (bounded) until every CTA of this launch has arrived.
    if (t == 0) {
        s->part_min[b] = mn;
        s->part_max[b] = mx;
        __threadfence();
        const unsigned long long before = atomicAdd(&s->arrivals, 1ull);
        const unsigned long long target = (before / static_cast<unsigned>(G) + 1ull) * static_cast<unsigned>(G);
        if (before + 1ull != target) {
            const uint64_t t0 = global_timer_ns();
            while (true) {
                unsigned long long now;
                asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(now) : "l"(&s->arrivals) : "memory");
                if (now >= target) break;
                if (global_timer_ns() - t0 > OG_WAIT_LIMIT_NS) {
                    failed = 1;
                    break;
                }
            }
        }
        __threadfence();
    }
    __syncthreads();
    if (failed) {
        if (t == 0) atomicExch(error_flag, 1);
        // No copy may still be landing when the CTA exits: a second bounded wait for the staged copies of this CTA's
        // own slice (they depend on no other CTA). If that one runs out too, the CTA exits anyway rather than wait
        // without a limit; the failure is already raised, and y is not defined after a failed launch.
        if (n_s > 0 && t == 0) {
            int unraised = 0;
            mbar_wait(&bar, 0, &unraised);
        }
        return;
    }
    // Every CTA forms the same scale and zero point from all the partial ranges.
    mn = INFINITY;
    mx = -INFINITY;
    for (int i = t; i < G; i += T) {
        mn = fminf(mn, __ldcg(&s->part_min[i]));
        mx = fmaxf(mx, __ldcg(&s->part_max[i]));
    }
    __syncthreads();  // smin / smax are reused
    block_min_max(mn, mx, smin, smax);
    if (t == 0) {
        float scale;
        int zp;
        dq_scale_zero_point(mn, mx, scale, zp);
        q_scale = scale;
        q_zp = zp;
        if (b == 0) {
            s->scale = scale;
            s->zero_point = zp;
            *scale_out = scale;
            *zp_out = static_cast<uint8_t>(zp);
        }
    }
    __syncthreads();
    DqQuant q;
    q.s = q_scale;
    q.zf = static_cast<float>(q_zp);
    q.r = __frcp_rn(q.s);
    q.r_ok = fabsf(q.r) >= 1.17549435e-38f && fabsf(q.r) <= 3.40282347e+38f;  // normal and finite
    q.cz = __fadd_rn(q.zf, 12582912.0f);  // exact: an integer below 2^24
    // This CTA's words of y (a slice holds fewer than 2^31 vectors); four independent vectors per thread and step.
    uint32_t* yb = reinterpret_cast<uint32_t*>(y) + v0;
    const float4* xb = xv + v0;
    const int n_all = static_cast<int>(v1 - v0);
    int i = t;
    for (; i + 3 * T < n_s; i += 4 * T) {
        float4 v[4];
#pragma unroll
        for (int u = 0; u < 4; u++) v[u] = sv[i + u * T];
#pragma unroll
        for (int u = 0; u < 4; u++) yb[i + u * T] = q.four(v[u]);
    }
    for (; i < n_s; i += T) yb[i] = q.four(sv[i]);
#pragma unroll
    for (int j = 0; j < DQF_KEEP; j++) {
        const int k = n_s + j * T + t;
        if (k < n_all) yb[k] = q.four(keep[j]);
    }
    for (int i0 = n_s + DQF_KEEP * T + t; i0 < n_all; i0 += 4 * T) {
        float4 v[4];
#pragma unroll
        for (int u = 0; u < 4; u++)
            if (i0 + u * T < n_all) v[u] = __ldcs(xb + i0 + u * T);
#pragma unroll
        for (int u = 0; u < 4; u++)
            if (i0 + u * T < n_all) yb[i0 + u * T] = q.four(v[u]);
    }
    if (b == G - 1)
        for (int64_t i = nvec * 4 + t; i < count; i += T) y[i] = static_cast<uint8_t>(q.one(__ldg(x + i)));
}

// True (once per device) when one dq_fused_kernel CTA fits on every SM.
static bool dq_fused_fits() {
    static std::atomic<uint64_t> known{0}, fits{0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return false;
    const uint64_t bit = uint64_t(1) << (dev & 63);
    if (!(known.load() & bit)) {
        bool ok = cudaFuncSetAttribute(dq_fused_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       DQF_SMEM_BYTES) == cudaSuccess;
        int per_sm = 0;
        ok = ok && cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, dq_fused_kernel, DQF_THREADS,
                                                                 DQF_SMEM_BYTES) == cudaSuccess && per_sm >= 1;
        if (!ok) cudaGetLastError();
        if (ok) fits.fetch_or(bit);
        known.fetch_or(bit);
    }
    return (fits.load() & bit) != 0;
}

bool dq_single_kernel(const float* x, int64_t count, const uint8_t* y) {
    return count >= DQF_MIN_COUNT && (reinterpret_cast<uintptr_t>(x) & 15) == 0 &&
           (reinterpret_cast<uintptr_t>(y) & 3) == 0 && dq_fused_fits();
}

cudaError_t launch_dynamic_quantize(const float* x, int64_t count, uint8_t* y, float* scale_out, uint8_t* zp_out,
                                    DqScratch* scratch, int num_sms, int* error_flag, cudaStream_t stream) {
    if (dq_single_kernel(x, count, y)) {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(static_cast<unsigned>(num_sms));
        cfg.blockDim = dim3(DQF_THREADS);
        cfg.dynamicSmemBytes = DQF_SMEM_BYTES;
        cfg.stream = stream;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeCooperative;  // every CTA resident at once: the grid barrier can complete
        attr[0].val.cooperative = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        const cudaError_t e = cudaLaunchKernelEx(&cfg, dq_fused_kernel, x, count, y, scratch, scale_out, zp_out,
                                                 error_flag);
        if (e != cudaErrorCooperativeLaunchTooLarge) return e;
        cudaGetLastError();  // refused before anything ran (the grid cannot be resident at once): two launches instead
    }
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
