// The int8 product for few rows (M <= 16 per batch: decode steps), bandwidth-bound on B.
//
// The roles of the operands are swapped so that B streams through the tensor cores exactly once: the MMA computes
// D[n, j] = sum_k B[k, n] * X[j, k] with tcgen05.mma.kind::i8, M = 128 columns of B per CTA, N = 32, where X's rows
// 0..15 are the rows of A (TMA zero-fills the rows past M) and rows 16..31 are all ones. D's columns 0..15 are then
// the dot products of the tile's 128 columns with the rows of A, and its columns 16..31 the column sums of B over K,
// which the zero point of A needs - so no separate pass over B (235 MB at the decode config) is made for them.
//
// One CTA per 128 columns (and batch), the whole of K per CTA, 5 stages of 16 KB of B + 4 KB of X; two CTAs fit on
// an SM, so every tile of the decode config (224) is resident at once and each pulls its share of HBM bandwidth
// until all finish together. Warp 0 loads (TMA, no multicast), warp 1 issues the MMAs into a 32-column TMEM
// accumulator, warps 2-5 compute the row sums of A while B streams (the zero point of B needs them), then drain TMEM:
// lane = column, 16 results per lane, stores coalesced along N.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include "og_gemm.h"
#include "og_kernels.cuh"
#include "og_ptx.cuh"

namespace og {

namespace rows {
constexpr int BN = 128;          // columns of B (rows of the MMA) per CTA
constexpr int BK = 128;
constexpr int MAXM = 16;
constexpr int XROWS = 32;        // rows of A (16) then ones (16)
constexpr int STAGES = 5;
constexpr int B_BYTES = BN * BK;          // 16 KB
constexpr int X_BYTES = XROWS * BK;       // 4 KB
constexpr int A_BYTES = MAXM * BK;        // 2 KB loaded by TMA into the first half of X
constexpr int THREADS = 192;
constexpr int TMEM_COLS = 32;
constexpr int SMEM_BYTES = STAGES * (B_BYTES + X_BYTES) + 1024 + 256;
}  // namespace rows

struct RowsParams {
    int m, n, k;
    int k_blocks;
    int a_batched, b_batched;
    int64_t lda, stride_a;  // for the row sums of A, read from global memory
    const uint8_t* a;
    Epilogue epi;
    int* error_flag;
};

template <int OUT>
__device__ __forceinline__ void store_one(const Epilogue& e, int b, int m, int n, uint32_t s) {
    const int64_t idx = b * e.batch_stride_c + static_cast<int64_t>(m) * e.ldc + n;
    if constexpr (OUT == OUT_I32) {
        __stcs(static_cast<int32_t*>(e.c) + idx, static_cast<int32_t>(s));
    } else if constexpr (OUT == OUT_F32) {
        __stcs(static_cast<float*>(e.c) + idx, finish_float(e, n, s));
    } else {
        static_cast<uint8_t*>(e.c)[idx] = finish_byte(e, n, s, OUT == OUT_U8);
    }
}

template <bool B_KMAJOR, int OUT>
__global__ void __launch_bounds__(rows::THREADS, 2)
    int8_gemm_rows_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                          const RowsParams p, uint32_t idesc) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sB = smem;                                   // [STAGES][128 columns x 128 k]
    uint8_t* sX = smem + rows::STAGES * rows::B_BYTES;    // [STAGES][32 rows x 128 k]
    uint64_t* bars = reinterpret_cast<uint64_t*>(sX + rows::STAGES * rows::X_BYTES);
    uint64_t* full = bars;
    uint64_t* empty = bars + rows::STAGES;
    uint64_t* tfull = bars + 2 * rows::STAGES;
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + 2 * rows::STAGES + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
    int32_t* row_sum = reinterpret_cast<int32_t*>(tmem_holder + 2);  // [16]

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int tile = blockIdx.x;
    const int b = blockIdx.y;

    // The ones of X (rows 16..31 of every stage); any swizzle of all-ones bytes is all ones.
    for (int i = threadIdx.x; i < rows::STAGES * (rows::X_BYTES - rows::A_BYTES) / 16; i += blockDim.x) {
        const int s = i / ((rows::X_BYTES - rows::A_BYTES) / 16);
        const int o = i % ((rows::X_BYTES - rows::A_BYTES) / 16);
        reinterpret_cast<uint4*>(sX + s * rows::X_BYTES + rows::A_BYTES)[o] =
            make_uint4(0x01010101u, 0x01010101u, 0x01010101u, 0x01010101u);
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // generic writes -> visible to the tensor cores
    if (threadIdx.x == 0) {
        for (int s = 0; s < rows::STAGES; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(tfull, 1);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 0 && lane == 0) {
        prefetch_tmap(&tmap_a);
        prefetch_tmap(&tmap_b);
    }
    if (warp == 1) {
        tmem_alloc(tmem_holder, rows::TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_holder;
    const int ba = p.a_batched ? b : 0;
    const int bb = p.b_batched ? b : 0;

    if (warp == 0) {
        for (int kb = 0; kb < p.k_blocks; kb++) {
            const int s = kb % rows::STAGES;
            const uint32_t ph = (kb / rows::STAGES) & 1;
            if (!mbar_wait(&empty[s], ph ^ 1, abort_flag)) goto done;
            if (lane == 0) {
                mbar_arrive_expect_tx(&full[s], rows::B_BYTES + rows::A_BYTES);
                if constexpr (B_KMAJOR)
                    tma_load_3d(sB + s * rows::B_BYTES, &tmap_b, &full[s], kb * rows::BK, tile * rows::BN, bb);
                else
                    tma_load_3d(sB + s * rows::B_BYTES, &tmap_b, &full[s], tile * rows::BN, kb * rows::BK, bb);
                tma_load_3d(sX + s * rows::X_BYTES, &tmap_a, &full[s], kb * rows::BK, 0, ba);
            }
            __syncwarp();
        }
    } else if (warp == 1) {
        for (int kb = 0; kb < p.k_blocks; kb++) {
            const int s = kb % rows::STAGES;
            const uint32_t ph = (kb / rows::STAGES) & 1;
            if (!mbar_wait(&full[s], ph, abort_flag)) goto done;
            tc_fence_after();
            if (lane == 0) {
                const uint32_t b_addr = smem_u32(sB + s * rows::B_BYTES);
                const uint32_t x_addr = smem_u32(sX + s * rows::X_BYTES);
#pragma unroll
                for (int kk = 0; kk < rows::BK / 32; kk++) {
                    const uint64_t adesc = B_KMAJOR ? smem_desc_sw128(b_addr + kk * 32, 16, 1024)
                                                    : smem_desc_sw128(b_addr + kk * 32 * 128, rows::B_BYTES, 1024);
                    const uint64_t bdesc = smem_desc_sw128(x_addr + kk * 32, 16, 1024);
                    mma_i8(tmem_base, adesc, bdesc, idesc, (kb | kk) != 0 ? 1u : 0u);
                }
                mma_commit(&empty[s]);
            }
            __syncwarp();
        }
        if (lane == 0) mma_commit(tfull);
        __syncwarp();
    } else {
        const int q = warp & 3;
        const Epilogue& e = p.epi;
        // Row sums of A over K while B streams (needed for the zero point of B): warp q sums rows q, q+4, ...
        if (e.zb != nullptr) {
            for (int r = q; r < rows::MAXM; r += 4) {
                int32_t sum = 0;
                if (r < p.m) {
                    const uint8_t* row = p.a + ba * p.stride_a + r * p.lda;
                    for (int kk = lane * 16; kk < p.k; kk += 32 * 16) {
                        if (kk + 16 <= p.k) {
                            const uint4 w = __ldg(reinterpret_cast<const uint4*>(row + kk));
                            if (e.za_signed) {
                                sum = __dp4a(static_cast<int>(w.x), 0x01010101, sum);
                                sum = __dp4a(static_cast<int>(w.y), 0x01010101, sum);
                                sum = __dp4a(static_cast<int>(w.z), 0x01010101, sum);
                                sum = __dp4a(static_cast<int>(w.w), 0x01010101, sum);
                            } else {
                                unsigned u = static_cast<unsigned>(sum);
                                u = __dp4a(w.x, 0x01010101u, u);
                                u = __dp4a(w.y, 0x01010101u, u);
                                u = __dp4a(w.z, 0x01010101u, u);
                                u = __dp4a(w.w, 0x01010101u, u);
                                sum = static_cast<int32_t>(u);
                            }
                        } else {
                            for (int t = kk; t < p.k; t++) {
                                const uint8_t v = __ldg(row + t);
                                sum += e.za_signed ? static_cast<int32_t>(static_cast<int8_t>(v)) : v;
                            }
                        }
                    }
#pragma unroll
                    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xFFFFFFFFu, sum, o);
                }
                if (lane == 0) row_sum[r] = sum;
            }
        }
        asm volatile("bar.sync 1, 128;" ::: "memory");  // the four epilogue warps
        if (!mbar_wait(tfull, 0, abort_flag)) goto done;
        tc_fence_after();
        uint32_t r[32];
        tmem_ld_32x32b_x32(tmem_base + (static_cast<uint32_t>(q * 32) << 16), r);
        tmem_ld_wait();
        const int n = tile * rows::BN + q * 32 + lane;
        if (n < p.n) {
            const uint32_t csb = r[16];  // sum over K of B[k, n]
            const int32_t zb = zp_value(e.zb, e.zb_vector, e.zb_signed, n);
            const uint32_t bias = e.int_bias ? static_cast<uint32_t>(__ldg(e.int_bias + n)) : 0u;
#pragma unroll
            for (int m = 0; m < rows::MAXM; m++) {
                if (m < p.m) {
                    const int32_t za = zp_value(e.za, e.za_vector, e.za_signed, m);
                    uint32_t s = r[m];
                    if (e.zb != nullptr)
                        s += static_cast<uint32_t>(p.k) * static_cast<uint32_t>(za) * static_cast<uint32_t>(zb) -
                             static_cast<uint32_t>(zb) * static_cast<uint32_t>(row_sum[m]);
                    if (e.za != nullptr) s -= static_cast<uint32_t>(za) * csb;
                    store_one<OUT>(e, b, m, n, s + bias);
                }
            }
        }
        tc_fence_before();
    }

done:
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, rows::TMEM_COLS);
    }
    if (threadIdx.x == 0 && *abort_flag) atomicExch(p.error_flag, 1);
}

// ---- host side ---------------------------------------------------------------------------------------------------

bool make_tensor_map_u8(CUtensorMap* map, const void* base, uint64_t x, uint64_t y, uint64_t z, uint64_t stride_y,
                        uint64_t stride_z, uint32_t box_x, uint32_t box_y);

bool rows_eligible(const GemmLaunch& L) { return L.m >= 1 && L.m <= rows::MAXM && tc_eligible(L); }

template <bool B_KMAJOR, int OUT>
static cudaError_t launch_rows_t(const RowsParams& p, const CUtensorMap& ma, const CUtensorMap& mb, dim3 grid,
                                 uint32_t idesc, cudaStream_t stream) {
    auto kern = int8_gemm_rows_kernel<B_KMAJOR, OUT>;
    static uint64_t configured = 0;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    const uint64_t bit = uint64_t(1) << (dev & 63);
    if (!(configured & bit)) {
        e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, rows::SMEM_BYTES);
        if (e != cudaSuccess) return e;
        configured |= bit;
    }
    kern<<<grid, rows::THREADS, rows::SMEM_BYTES, stream>>>(ma, mb, p, idesc);
    return cudaGetLastError();
}

cudaError_t launch_gemm_rows(const GemmLaunch& L, cudaStream_t stream) {
    const int ba = (L.batch > 1 && L.stride_a != 0) ? L.batch : 1;
    const int bb = (L.batch > 1 && L.stride_b != 0) ? L.batch : 1;
    CUtensorMap ma, mb;
    const uint64_t sa = ba > 1 ? uint64_t(L.stride_a) : (uint64_t(L.lda) * L.m + 15) & ~uint64_t(15);
    if (!make_tensor_map_u8(&ma, L.a, L.k, L.m, ba, L.lda, sa, rows::BK, rows::MAXM)) return cudaErrorInvalidValue;
    const uint64_t rows_b = L.trans_b ? L.n : L.k;
    const uint64_t sb = bb > 1 ? uint64_t(L.stride_b) : (uint64_t(L.ldb) * rows_b + 15) & ~uint64_t(15);
    const bool ok = L.trans_b ? make_tensor_map_u8(&mb, L.b, L.k, L.n, bb, L.ldb, sb, rows::BK, rows::BN)
                              : make_tensor_map_u8(&mb, L.b, L.n, L.k, bb, L.ldb, sb, rows::BN, rows::BK);
    if (!ok) return cudaErrorInvalidValue;
    RowsParams p;
    p.m = L.m;
    p.n = L.n;
    p.k = L.k;
    p.k_blocks = (L.k + rows::BK - 1) / rows::BK;
    p.a_batched = ba > 1;
    p.b_batched = bb > 1;
    p.lda = L.lda;
    p.stride_a = L.stride_a;
    p.a = L.a;
    p.epi = L.epi;
    p.error_flag = L.error_flag;
    // The MMA's A operand is B (its type, MN-major unless B is stored N x K); its B operand is A plus the ones.
    const uint32_t idesc = idesc_i8(L.b_signed, L.a_signed, !L.trans_b, false, rows::BN, rows::XROWS);
    const dim3 grid((L.n + rows::BN - 1) / rows::BN, L.batch);
    const bool km = L.trans_b != 0;
    switch (L.epi.out_kind) {
        case OUT_I32: return km ? launch_rows_t<true, OUT_I32>(p, ma, mb, grid, idesc, stream)
                                : launch_rows_t<false, OUT_I32>(p, ma, mb, grid, idesc, stream);
        case OUT_F32: return km ? launch_rows_t<true, OUT_F32>(p, ma, mb, grid, idesc, stream)
                                : launch_rows_t<false, OUT_F32>(p, ma, mb, grid, idesc, stream);
        case OUT_U8: return km ? launch_rows_t<true, OUT_U8>(p, ma, mb, grid, idesc, stream)
                               : launch_rows_t<false, OUT_U8>(p, ma, mb, grid, idesc, stream);
        default: return km ? launch_rows_t<true, OUT_S8>(p, ma, mb, grid, idesc, stream)
                           : launch_rows_t<false, OUT_S8>(p, ma, mb, grid, idesc, stream);
    }
}

}  // namespace og
