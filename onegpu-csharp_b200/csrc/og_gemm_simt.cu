// The portable int8 product (SIMT, any alignment) and the byte-sum kernels that feed the tensor-core product's
// zero-point correction.
//
// The portable kernel computes the definition directly: bytes minus their zero points are staged as int16 in shared
// memory and multiplied with 32-bit integer multiply-adds in wrapping unsigned arithmetic, 64 x 64 outputs per block
// of 256 threads (4 x 4 each), K in steps of 32. It serves Int8GemmOptions.AllowPackedDot = false and every product
// whose operands the tensor-core path cannot load with TMA (rows or batches not on 16-byte boundaries, K = 0).
#include <cuda_runtime.h>

#include "og_gemm.h"
#include "og_kernels.cuh"

namespace og {

namespace simt {
constexpr int BM = 64;
constexpr int BN = 64;
constexpr int BK = 32;
constexpr int THREADS = 256;
}  // namespace simt

__device__ __forceinline__ int32_t byte_val(uint8_t v, int is_signed) {
    return is_signed ? static_cast<int32_t>(static_cast<int8_t>(v)) : static_cast<int32_t>(v);
}

template <int OUT>
__device__ __forceinline__ void simt_store(const Epilogue& e, int b, int m, int n, uint32_t sum) {
    if (e.int_bias != nullptr) sum += static_cast<uint32_t>(__ldg(e.int_bias + n));
    const int64_t idx = b * e.batch_stride_c + static_cast<int64_t>(m) * e.ldc + n;
    if constexpr (OUT == OUT_I32) {
        static_cast<int32_t*>(e.c)[idx] = static_cast<int32_t>(sum);
    } else if constexpr (OUT == OUT_F32) {
        static_cast<float*>(e.c)[idx] = finish_float(e, n, sum);
    } else {
        static_cast<uint8_t*>(e.c)[idx] = finish_byte(e, n, sum, OUT == OUT_U8);
    }
}

template <int OUT>
__global__ void __launch_bounds__(simt::THREADS)
    int8_gemm_simt_kernel(const GemmLaunch L, int tiles_m, int tiles_n) {
    __shared__ int16_t As[simt::BK][simt::BM + 8];
    __shared__ int16_t Bs[simt::BK][simt::BN + 8];
    const int64_t per_batch = static_cast<int64_t>(tiles_m) * tiles_n;
    const int64_t tile = blockIdx.x;
    const int b = static_cast<int>(tile / per_batch);
    const int64_t r = tile - b * per_batch;
    const int tm = static_cast<int>(r / tiles_n);
    const int tn = static_cast<int>(r - static_cast<int64_t>(tm) * tiles_n);
    const int tid = threadIdx.x;
    const int tx = tid & 15, ty = tid >> 4;
    const Epilogue& e = L.epi;
    const uint8_t* A = L.a + b * L.stride_a;
    const uint8_t* B = L.b + b * L.stride_b;

    uint32_t acc[4][4];
#pragma unroll
    for (int i = 0; i < 4; i++)
#pragma unroll
        for (int j = 0; j < 4; j++) acc[i][j] = 0;

    for (int k0 = 0; k0 < L.k; k0 += simt::BK) {
#pragma unroll
        for (int i = 0; i < (simt::BM * simt::BK) / simt::THREADS; i++) {
            const int el = tid + simt::THREADS * i;
            const int row = el >> 5, kk = el & 31;
            const int m = tm * simt::BM + row, k = k0 + kk;
            int32_t v = 0;
            if (m < L.m && k < L.k)
                v = byte_val(A[static_cast<int64_t>(m) * L.lda + k], L.a_signed) -
                    zp_value(e.za, e.za_vector, e.za_signed, m);
            As[kk][row] = static_cast<int16_t>(v);
        }
#pragma unroll
        for (int i = 0; i < (simt::BN * simt::BK) / simt::THREADS; i++) {
            const int el = tid + simt::THREADS * i;
            int kk, col;
            if (L.trans_b) {
                kk = el & 31;
                col = el >> 5;
            } else {
                kk = el >> 6;
                col = el & 63;
            }
            const int n = tn * simt::BN + col, k = k0 + kk;
            int32_t v = 0;
            if (n < L.n && k < L.k) {
                const int64_t off = L.trans_b ? static_cast<int64_t>(n) * L.ldb + k : static_cast<int64_t>(k) * L.ldb + n;
                v = byte_val(B[off], L.b_signed) - zp_value(e.zb, e.zb_vector, e.zb_signed, n);
            }
            Bs[kk][col] = static_cast<int16_t>(v);
        }
        __syncthreads();
#pragma unroll 8
        for (int kk = 0; kk < simt::BK; kk++) {
            int32_t av[4], bv[4];
#pragma unroll
            for (int i = 0; i < 4; i++) av[i] = As[kk][ty * 4 + i];
#pragma unroll
            for (int j = 0; j < 4; j++) bv[j] = Bs[kk][tx * 4 + j];
#pragma unroll
            for (int i = 0; i < 4; i++)
#pragma unroll
                for (int j = 0; j < 4; j++) acc[i][j] += static_cast<uint32_t>(av[i] * bv[j]);
        }
        __syncthreads();
    }

#pragma unroll
    for (int i = 0; i < 4; i++) {
        const int m = tm * simt::BM + ty * 4 + i;
        if (m >= L.m) continue;
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const int n = tn * simt::BN + tx * 4 + j;
            if (n < L.n) simt_store<OUT>(e, b, m, n, acc[i][j]);
        }
    }
}

cudaError_t launch_gemm_simt(const GemmLaunch& L, cudaStream_t stream) {
    const int tiles_m = (L.m + simt::BM - 1) / simt::BM;
    const int tiles_n = (L.n + simt::BN - 1) / simt::BN;
    const int64_t blocks = static_cast<int64_t>(tiles_m) * tiles_n * L.batch;
    if (blocks <= 0) return cudaSuccess;
    if (blocks > 0x7FFFFFFF) return cudaErrorInvalidConfiguration;
    const dim3 grid(static_cast<unsigned>(blocks));
    switch (L.epi.out_kind) {
        case OUT_I32: int8_gemm_simt_kernel<OUT_I32><<<grid, simt::THREADS, 0, stream>>>(L, tiles_m, tiles_n); break;
        case OUT_F32: int8_gemm_simt_kernel<OUT_F32><<<grid, simt::THREADS, 0, stream>>>(L, tiles_m, tiles_n); break;
        case OUT_U8: int8_gemm_simt_kernel<OUT_U8><<<grid, simt::THREADS, 0, stream>>>(L, tiles_m, tiles_n); break;
        default: int8_gemm_simt_kernel<OUT_S8><<<grid, simt::THREADS, 0, stream>>>(L, tiles_m, tiles_n); break;
    }
    return cudaGetLastError();
}

// ---- byte sums ---------------------------------------------------------------------------------------------------

// One warp per row: sum of `len` bytes of row r of batch bt at base + bt * bstride + r * ld. 16-byte loads and a
// packed dot with 0x01010101 when the row is aligned, bytes otherwise.
__global__ void row_sums_kernel(const uint8_t* __restrict__ base, int rows, int len, int64_t ld, int64_t bstride,
                                int batches, int is_signed, int32_t* __restrict__ out) {
    const int64_t warp_id = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (warp_id >= static_cast<int64_t>(rows) * batches) return;
    const int bt = static_cast<int>(warp_id / rows);
    const int r = static_cast<int>(warp_id - static_cast<int64_t>(bt) * rows);
    const uint8_t* row = base + bt * bstride + r * ld;
    int32_t s = 0;
    int start = 0;
    if ((reinterpret_cast<uintptr_t>(row) & 15) == 0) {
        const int vec = len >> 4;
        const uint4* v = reinterpret_cast<const uint4*>(row);
        for (int i = lane; i < vec; i += 32) {
            const uint4 w = __ldg(v + i);
            if (is_signed) {
                s = __dp4a(static_cast<int>(w.x), 0x01010101, s);
                s = __dp4a(static_cast<int>(w.y), 0x01010101, s);
                s = __dp4a(static_cast<int>(w.z), 0x01010101, s);
                s = __dp4a(static_cast<int>(w.w), 0x01010101, s);
            } else {
                unsigned u = static_cast<unsigned>(s);
                u = __dp4a(w.x, 0x01010101u, u);
                u = __dp4a(w.y, 0x01010101u, u);
                u = __dp4a(w.z, 0x01010101u, u);
                u = __dp4a(w.w, 0x01010101u, u);
                s = static_cast<int32_t>(u);
            }
        }
        start = vec << 4;
    }
    for (int i = start + lane; i < len; i += 32) s += byte_val(__ldg(row + i), is_signed);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xFFFFFFFFu, s, o);
    if (lane == 0) out[warp_id] = s;
}

// Column sums of a K x N row-major byte matrix (columns contiguous): each thread owns four adjacent columns of a
// slab of K rows; slabs add into the zeroed output with integer atomics (exact in any order).
__global__ void col_sums_kernel(const uint8_t* __restrict__ base, int n, int k, int64_t ld, int64_t bstride,
                                int is_signed, int rows_per_block, int32_t* __restrict__ out) {
    const int bt = blockIdx.z;
    const int c0 = (blockIdx.x * blockDim.x + threadIdx.x) * 4;
    if (c0 >= n) return;
    const int k_begin = blockIdx.y * rows_per_block;
    const int k_end = min(k, k_begin + rows_per_block);
    const uint8_t* mat = base + bt * bstride;
    int32_t s0 = 0, s1 = 0, s2 = 0, s3 = 0;
    const bool four = c0 + 4 <= n;
    const bool aligned = four && ((reinterpret_cast<uintptr_t>(mat + c0) | static_cast<uintptr_t>(ld)) & 3) == 0;
    for (int kk = k_begin; kk < k_end; kk++) {
        const uint8_t* p = mat + static_cast<int64_t>(kk) * ld + c0;
        if (aligned) {
            const uint32_t w = __ldg(reinterpret_cast<const uint32_t*>(p));
            s0 += byte_val(w & 0xFF, is_signed);
            s1 += byte_val((w >> 8) & 0xFF, is_signed);
            s2 += byte_val((w >> 16) & 0xFF, is_signed);
            s3 += byte_val(w >> 24, is_signed);
        } else {
            s0 += byte_val(__ldg(p), is_signed);
            if (c0 + 1 < n) s1 += byte_val(__ldg(p + 1), is_signed);
            if (c0 + 2 < n) s2 += byte_val(__ldg(p + 2), is_signed);
            if (c0 + 3 < n) s3 += byte_val(__ldg(p + 3), is_signed);
        }
    }
    int32_t* o = out + static_cast<int64_t>(bt) * n + c0;
    atomicAdd(o, s0);
    if (c0 + 1 < n) atomicAdd(o + 1, s1);
    if (c0 + 2 < n) atomicAdd(o + 2, s2);
    if (c0 + 3 < n) atomicAdd(o + 3, s3);
}

cudaError_t launch_byte_sums(const GemmLaunch& L, int32_t* row_sums, int32_t* col_sums, cudaStream_t stream) {
    const int ba = (L.batch > 1 && L.stride_a != 0) ? L.batch : 1;
    const int bb = (L.batch > 1 && L.stride_b != 0) ? L.batch : 1;
    if (row_sums != nullptr) {
        const int64_t warps = static_cast<int64_t>(L.m) * ba;
        const int64_t blocks = (warps * 32 + 255) / 256;
        row_sums_kernel<<<static_cast<unsigned>(blocks), 256, 0, stream>>>(L.a, L.m, L.k, L.lda, L.stride_a, ba,
                                                                             L.a_signed, row_sums);
        cudaError_t err = cudaGetLastError();
        if (err != cudaSuccess) return err;
    }
    if (col_sums != nullptr) {
        if (L.trans_b) {
            const int64_t warps = static_cast<int64_t>(L.n) * bb;
            const int64_t blocks = (warps * 32 + 255) / 256;
            row_sums_kernel<<<static_cast<unsigned>(blocks), 256, 0, stream>>>(L.b, L.n, L.k, L.ldb, L.stride_b, bb,
                                                                                 L.b_signed, col_sums);
        } else {
            cudaError_t err = cudaMemsetAsync(col_sums, 0, sizeof(int32_t) * static_cast<size_t>(L.n) * bb, stream);
            if (err != cudaSuccess) return err;
            const int col_blocks = (L.n + 1023) / 1024;
            // Enough slabs of K to give every SM a few blocks.
            int slabs = (4 * L.num_sms + col_blocks * bb - 1) / (col_blocks * bb);
            if (slabs < 1) slabs = 1;
            int rows_per_block = (L.k + slabs - 1) / slabs;
            if (rows_per_block < 16) rows_per_block = 16;
            slabs = (L.k + rows_per_block - 1) / rows_per_block;
            if (slabs > 65535) {
                slabs = 65535;
                rows_per_block = (L.k + slabs - 1) / slabs;
            }
            for (int b0 = 0; b0 < bb; b0 += 65535) {
                const int nb = bb - b0 < 65535 ? bb - b0 : 65535;
                const dim3 grid(col_blocks, slabs, nb);
                col_sums_kernel<<<grid, 256, 0, stream>>>(L.b + b0 * L.stride_b, L.n, L.k, L.ldb, L.stride_b,
                                                          L.b_signed, rows_per_block,
                                                          col_sums + static_cast<int64_t>(b0) * L.n);
            }
        }
        return cudaGetLastError();
    }
    return cudaSuccess;
}

}  // namespace og
