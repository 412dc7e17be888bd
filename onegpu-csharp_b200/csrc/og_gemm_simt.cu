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

__device__ __forceinline__ int32_t byte_sum16(const uint4& w, int is_signed, int32_t s) {
    if (is_signed) {
        s = __dp4a(static_cast<int>(w.x), 0x01010101, s);
        s = __dp4a(static_cast<int>(w.y), 0x01010101, s);
        s = __dp4a(static_cast<int>(w.z), 0x01010101, s);
        return __dp4a(static_cast<int>(w.w), 0x01010101, s);
    }
    unsigned u = static_cast<unsigned>(s);
    u = __dp4a(w.x, 0x01010101u, u);
    u = __dp4a(w.y, 0x01010101u, u);
    u = __dp4a(w.z, 0x01010101u, u);
    return static_cast<int32_t>(__dp4a(w.w, 0x01010101u, u));
}

// One warp per row: sum of `len` bytes of row r of batch bt at base + bt * bstride + r * ld. 16-byte loads, eight in
// flight per lane, and a packed dot with 0x01010101 when the row is aligned; bytes otherwise.
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
        constexpr int U = 8;
        for (int i0 = lane; i0 < vec; i0 += 32 * U) {
            uint4 w[U];
#pragma unroll
            for (int u = 0; u < U; u++) {
                const int i = i0 + 32 * u;
                w[u] = i < vec ? __ldg(v + i) : make_uint4(0, 0, 0, 0);
            }
#pragma unroll
            for (int u = 0; u < U; u++) s = byte_sum16(w[u], is_signed, s);
        }
        start = vec << 4;
    }
    for (int i = start + lane; i < len; i += 32) s += byte_val(__ldg(row + i), is_signed);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xFFFFFFFFu, s, o);
    if (lane == 0) out[warp_id] = s;
}

// Column sums of a K x N row-major byte matrix (columns contiguous). A block of 8 warps owns 512 adjacent columns
// (16 per lane, one 16-byte load per row) and a slab of rows that its warps share out; the warps' sums meet in
// shared memory and each block adds its 512 results into the zeroed output with integer atomics (exact in any
// order). Columns that are not 16-byte aligned take byte loads.
constexpr int COLS_PER_BLOCK = 512;

__global__ void __launch_bounds__(256) col_sums_kernel(const uint8_t* __restrict__ base, int n, int k, int64_t ld,
                                                       int64_t bstride, int is_signed, int rows_per_block,
                                                       int32_t* __restrict__ out) {
    __shared__ int32_t part[8][COLS_PER_BLOCK + 1];
    const int bt = blockIdx.z;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int c0 = blockIdx.x * COLS_PER_BLOCK + lane * 16;
    const int k_begin = blockIdx.y * rows_per_block;
    const int k_end = min(k, k_begin + rows_per_block);
    const uint8_t* mat = base + bt * bstride;
    int32_t s[16];
#pragma unroll
    for (int j = 0; j < 16; j++) s[j] = 0;
    const bool vec = c0 + 16 <= n && ((reinterpret_cast<uintptr_t>(mat + c0) | static_cast<uintptr_t>(ld)) & 15) == 0;
    if (vec) {
        constexpr int U = 4;
        for (int k0 = k_begin + warp; k0 < k_end; k0 += 8 * U) {
            uint4 w[U];
#pragma unroll
            for (int u = 0; u < U; u++) {
                const int kk = k0 + 8 * u;
                w[u] = kk < k_end ? __ldg(reinterpret_cast<const uint4*>(mat + static_cast<int64_t>(kk) * ld + c0))
                                  : make_uint4(0u, 0u, 0u, 0u);
            }
#pragma unroll
            for (int u = 0; u < U; u++) {
                const uint32_t ws[4] = {w[u].x, w[u].y, w[u].z, w[u].w};
#pragma unroll
                for (int q = 0; q < 4; q++)
#pragma unroll
                    for (int t = 0; t < 4; t++) s[4 * q + t] += byte_val((ws[q] >> (8 * t)) & 0xFF, is_signed);
            }
        }
    } else if (c0 < n) {
        for (int kk = k_begin + warp; kk < k_end; kk += 8) {
            const uint8_t* p = mat + static_cast<int64_t>(kk) * ld + c0;
#pragma unroll
            for (int j = 0; j < 16; j++)
                if (c0 + j < n) s[j] += byte_val(__ldg(p + j), is_signed);
        }
    }
#pragma unroll
    for (int j = 0; j < 16; j++) part[warp][lane * 16 + j] = s[j];
    __syncthreads();
    for (int j = threadIdx.x; j < COLS_PER_BLOCK; j += blockDim.x) {
        const int col = blockIdx.x * COLS_PER_BLOCK + j;
        if (col >= n) continue;
        int32_t t = 0;
#pragma unroll
        for (int w8 = 0; w8 < 8; w8++) t += part[w8][j];
        atomicAdd(out + static_cast<int64_t>(bt) * n + col, t);
    }
}

// The byte sums through the tensor cores (the few-rows kernel's sums-only mode: a block of ones times the matrix),
// which stream the operand at TMA speed and write each sum once; the SIMT kernels below are the path for operands
// TMA cannot load and for more than 65535 batches.
static bool sums_on_tensor_cores(const GemmLaunch& L) {
    const int ba = (L.batch > 1 && L.stride_a != 0) ? L.batch : 1;
    const int bb = (L.batch > 1 && L.stride_b != 0) ? L.batch : 1;
    return tc_eligible(L) && ba <= 65535 && bb <= 65535;
}

int byte_sum_splits(const GemmLaunch& L, int max_splits) {
    if (!sums_on_tensor_cores(L)) return 1;
    const int ba = (L.batch > 1 && L.stride_a != 0) ? L.batch : 1;
    const int bb = (L.batch > 1 && L.stride_b != 0) ? L.batch : 1;
    // Both operands' tiles run in one launch (two CTAs per SM): as many K splits as fit all of them in one round of
    // resident CTAs (a second, partial round would cost a whole CTA's time again), at most max_splits and one K block
    // per split. One count for both operands (they share K, so neither gets an empty split).
    const int64_t ta = L.epi.zb != nullptr ? int64_t((L.m + 127) / 128) * ba : 0;
    const int64_t tb = L.epi.za != nullptr ? int64_t((L.n + 127) / 128) * bb : 0;
    const int kb = (L.k + 127) / 128;
    int64_t s = ta + tb > 0 ? (2 * int64_t(L.num_sms)) / (ta + tb) : 1;
    s = s < 1 ? 1 : (s > max_splits ? max_splits : s);
    s = s > kb ? kb : s;
    const int per = static_cast<int>((kb + s - 1) / s);
    return (kb + per - 1) / per;
}

LaunchFn prepare_byte_sums(const GemmLaunch& L, int32_t* row_sums, int32_t* col_sums, int splits, cudaError_t* err) {
    *err = cudaSuccess;
    const int ba = (L.batch > 1 && L.stride_a != 0) ? L.batch : 1;
    const int bb = (L.batch > 1 && L.stride_b != 0) ? L.batch : 1;
    if (!sums_on_tensor_cores(L)) {
        if (splits != 1) {
            *err = cudaErrorInvalidValue;
            return nullptr;
        }
        return [L, row_sums, col_sums](cudaStream_t s) { return launch_byte_sums_simt(L, row_sums, col_sums, s); };
    }
    (void)ba;
    (void)bb;
    return prepare_byte_sums_pair_tc(L, row_sums, col_sums, splits, err);  // both operands in one launch
}

cudaError_t launch_byte_sums(const GemmLaunch& L, int32_t* row_sums, int32_t* col_sums, cudaStream_t stream) {
    cudaError_t err;
    LaunchFn fn = prepare_byte_sums(L, row_sums, col_sums, 1, &err);
    return fn ? fn(stream) : err;
}

cudaError_t launch_byte_sums_simt(const GemmLaunch& L, int32_t* row_sums, int32_t* col_sums, cudaStream_t stream) {
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
            const int col_blocks = (L.n + COLS_PER_BLOCK - 1) / COLS_PER_BLOCK;
            // Enough slabs of K to give every SM a few blocks, each slab at least 64 rows (8 per warp).
            int slabs = (4 * L.num_sms + col_blocks * bb - 1) / (col_blocks * bb);
            if (slabs < 1) slabs = 1;
            int rows_per_block = (L.k + slabs - 1) / slabs;
            if (rows_per_block < 64) rows_per_block = 64;
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
