// The tensor-core int8 product for sm_100a: tcgen05.mma.kind::i8 with int32 accumulators in TMEM, operands staged by
// TMA into 128-byte-swizzled shared memory, warp-specialised and persistent.
//
// One CTA per SM walks the output tiles (BM x BN = 128 x 256 of one batch) in a grouped order so that concurrently
// running CTAs share A rows and B columns in L2. Warp 0 issues the TMA loads of a STAGES-deep ring of K blocks
// (BK = 128 bytes); warp 1 owns the TMEM allocation and issues the MMAs (four 128x256x32 instructions per K block)
// into one of two accumulators; warps 2-5 drain the other accumulator (tcgen05.ld), apply the zero-point
// correction and the epilogue and store C while the next tile is being multiplied.
//
// A is M x K row-major (K-major for the MMA). B is either K x N row-major (TransposeB = false; MN-major for the MMA,
// loaded as two 128-column boxes) or N x K (TransposeB = true; K-major). The MMA multiplies the operands' own
// types (u8 or s8); the zero points are applied afterwards from byte sums (og_kernels.cuh). Ragged M, N and K
// edges are zero-filled by TMA and never stored. No load uses cluster multicast, so the kernel is the same on any
// number of GPUs.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <cstdio>
#include <cstring>

#include "og_gemm.h"
#include "og_kernels.cuh"
#include "og_ptx.cuh"

namespace og {

namespace tc {
constexpr int BM = 128;
constexpr int BN = 256;
constexpr int BK = 128;  // bytes of K per stage = one 128-byte swizzle row
constexpr int STAGES = 4;
constexpr int A_BYTES = BM * BK;           // 16 KB
constexpr int B_BYTES = BN * BK;           // 32 KB
constexpr int B_HALF = 128 * BK;           // one 128-column box of an MN-major B
constexpr int NUM_ACC = 2;
constexpr int TMEM_COLS = NUM_ACC * BN;    // 512: all of TMEM
constexpr int THREADS = 192;               // producer, MMA, 4 epilogue warps
constexpr int GROUP_M = 8;                 // M tiles per raster group
constexpr int SMEM_BYTES = STAGES * (A_BYTES + B_BYTES) + 1024 /* alignment */ + 256 /* barriers */;
}  // namespace tc

struct TcParams {
    int m, n, k;
    int tiles_m, tiles_n;
    int batch;
    int a_batched, b_batched;
    int k_blocks;
    int total_tiles;
    Epilogue epi;
    int* error_flag;
};

__device__ __forceinline__ void tile_coords(const TcParams& p, int tile, int& b, int& tm, int& tn) {
    const int per_batch = p.tiles_m * p.tiles_n;
    b = tile / per_batch;
    const int r = tile - b * per_batch;
    const int group_span = tc::GROUP_M * p.tiles_n;
    const int group = r / group_span;
    const int first_m = group * tc::GROUP_M;
    const int gsize = min(p.tiles_m - first_m, tc::GROUP_M);
    const int in_group = r - group * group_span;
    tm = first_m + in_group % gsize;
    tn = in_group / gsize;
}

template <int OUT>
__device__ __forceinline__ void store_chunk(const Epilogue& e, const RowTerms& rt, int b, int m, int n0,
                                            const uint32_t (&r)[32]) {
    const bool full = e.vec_ok && (n0 + 32 <= e.n);
    if constexpr (OUT == OUT_I32) {
        int32_t* row = static_cast<int32_t*>(e.c) + b * e.batch_stride_c + static_cast<int64_t>(m) * e.ldc;
        if (full) {
            int4* dst = reinterpret_cast<int4*>(row + n0);
#pragma unroll
            for (int j = 0; j < 8; j++) {
                int4 v;
                v.x = static_cast<int32_t>(corrected(e, rt, b, n0 + 4 * j + 0, r[4 * j + 0]));
                v.y = static_cast<int32_t>(corrected(e, rt, b, n0 + 4 * j + 1, r[4 * j + 1]));
                v.z = static_cast<int32_t>(corrected(e, rt, b, n0 + 4 * j + 2, r[4 * j + 2]));
                v.w = static_cast<int32_t>(corrected(e, rt, b, n0 + 4 * j + 3, r[4 * j + 3]));
                __stcs(dst + j, v);
            }
        } else {
#pragma unroll
            for (int j = 0; j < 32; j++) {
                if (n0 + j < e.n) row[n0 + j] = static_cast<int32_t>(corrected(e, rt, b, n0 + j, r[j]));
            }
        }
    } else if constexpr (OUT == OUT_F32) {
        float* row = static_cast<float*>(e.c) + b * e.batch_stride_c + static_cast<int64_t>(m) * e.ldc;
        if (full) {
            float4* dst = reinterpret_cast<float4*>(row + n0);
#pragma unroll
            for (int j = 0; j < 8; j++) {
                float4 v;
                v.x = finish_float(e, n0 + 4 * j + 0, corrected(e, rt, b, n0 + 4 * j + 0, r[4 * j + 0]));
                v.y = finish_float(e, n0 + 4 * j + 1, corrected(e, rt, b, n0 + 4 * j + 1, r[4 * j + 1]));
                v.z = finish_float(e, n0 + 4 * j + 2, corrected(e, rt, b, n0 + 4 * j + 2, r[4 * j + 2]));
                v.w = finish_float(e, n0 + 4 * j + 3, corrected(e, rt, b, n0 + 4 * j + 3, r[4 * j + 3]));
                __stcs(dst + j, v);
            }
        } else {
#pragma unroll
            for (int j = 0; j < 32; j++) {
                if (n0 + j < e.n) row[n0 + j] = finish_float(e, n0 + j, corrected(e, rt, b, n0 + j, r[j]));
            }
        }
    } else {
        constexpr bool U = (OUT == OUT_U8);
        uint8_t* row = static_cast<uint8_t*>(e.c) + b * e.batch_stride_c + static_cast<int64_t>(m) * e.ldc;
        if (full) {
            uint32_t w[8];
#pragma unroll
            for (int j = 0; j < 8; j++) {
                uint32_t x = 0;
#pragma unroll
                for (int t = 0; t < 4; t++) {
                    const int n = n0 + 4 * j + t;
                    x |= static_cast<uint32_t>(finish_byte(e, n, corrected(e, rt, b, n, r[4 * j + t]), U)) << (8 * t);
                }
                w[j] = x;
            }
            uint4* dst = reinterpret_cast<uint4*>(row + n0);
            dst[0] = make_uint4(w[0], w[1], w[2], w[3]);
            dst[1] = make_uint4(w[4], w[5], w[6], w[7]);
        } else {
#pragma unroll
            for (int j = 0; j < 32; j++) {
                if (n0 + j < e.n) row[n0 + j] = finish_byte(e, n0 + j, corrected(e, rt, b, n0 + j, r[j]), U);
            }
        }
    }
}

template <bool B_MN, int OUT>
__global__ void __launch_bounds__(tc::THREADS, 1)
    int8_gemm_tc_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                        const TcParams p, uint32_t idesc) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sA = smem;
    uint8_t* sB = smem + tc::STAGES * tc::A_BYTES;
    uint64_t* bars = reinterpret_cast<uint64_t*>(sB + tc::STAGES * tc::B_BYTES);
    uint64_t* full = bars;
    uint64_t* empty = bars + tc::STAGES;
    uint64_t* tfull = bars + 2 * tc::STAGES;
    uint64_t* tempty = bars + 2 * tc::STAGES + tc::NUM_ACC;
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + 2 * tc::STAGES + 2 * tc::NUM_ACC);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < tc::STAGES; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int a = 0; a < tc::NUM_ACC; a++) {
            mbar_init(&tfull[a], 1);
            mbar_init(&tempty[a], 4);
        }
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 0 && lane == 0) {
        prefetch_tmap(&tmap_a);
        prefetch_tmap(&tmap_b);
    }
    if (warp == 1) {
        tmem_alloc(tmem_holder, tc::TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_holder;

    if (warp == 0) {
        // TMA producer: the whole warp walks the ring, lane 0 issues.
        uint32_t it = 0;
        for (int tile = blockIdx.x; tile < p.total_tiles; tile += gridDim.x) {
            int b, tm, tn;
            tile_coords(p, tile, b, tm, tn);
            const int ba = p.a_batched ? b : 0;
            const int bb = p.b_batched ? b : 0;
            const bool second_half = B_MN && (tn * tc::BN + 128 < p.n);
            const uint32_t bytes = tc::A_BYTES + (B_MN ? (second_half ? 2 : 1) * tc::B_HALF : tc::B_BYTES);
            for (int kb = 0; kb < p.k_blocks; kb++, it++) {
                const int s = it % tc::STAGES;
                const uint32_t ph = (it / tc::STAGES) & 1;
                if (!mbar_wait(&empty[s], ph ^ 1, abort_flag)) goto done;
                if (lane == 0) {
                    mbar_arrive_expect_tx(&full[s], bytes);
                    tma_load_3d(sA + s * tc::A_BYTES, &tmap_a, &full[s], kb * tc::BK, tm * tc::BM, ba);
                    if constexpr (B_MN) {
                        tma_load_3d(sB + s * tc::B_BYTES, &tmap_b, &full[s], tn * tc::BN, kb * tc::BK, bb);
                        if (second_half)
                            tma_load_3d(sB + s * tc::B_BYTES + tc::B_HALF, &tmap_b, &full[s], tn * tc::BN + 128,
                                        kb * tc::BK, bb);
                    } else {
                        tma_load_3d(sB + s * tc::B_BYTES, &tmap_b, &full[s], kb * tc::BK, tn * tc::BN, bb);
                    }
                }
                __syncwarp();
            }
        }
    } else if (warp == 1) {
        // MMA issuer: lane 0 issues four K=32 MMAs per stage into the accumulator of this tile.
        uint32_t it = 0;
        int lt = 0;
        for (int tile = blockIdx.x; tile < p.total_tiles; tile += gridDim.x, lt++) {
            const int acc = lt & 1;
            const uint32_t aph = (lt >> 1) & 1;
            if (!mbar_wait(&tempty[acc], aph ^ 1, abort_flag)) goto done;
            tc_fence_after();
            const uint32_t d_tmem = tmem_base + acc * tc::BN;
            for (int kb = 0; kb < p.k_blocks; kb++, it++) {
                const int s = it % tc::STAGES;
                const uint32_t ph = (it / tc::STAGES) & 1;
                if (!mbar_wait(&full[s], ph, abort_flag)) goto done;
                tc_fence_after();
                if (lane == 0) {
                    const uint32_t a_addr = smem_u32(sA + s * tc::A_BYTES);
                    const uint32_t b_addr = smem_u32(sB + s * tc::B_BYTES);
#pragma unroll
                    for (int kk = 0; kk < tc::BK / 32; kk++) {
                        const uint64_t adesc = smem_desc_sw128(a_addr + kk * 32, 16, 1024);
                        const uint64_t bdesc = B_MN ? smem_desc_sw128(b_addr + kk * 32 * 128, tc::B_HALF, 1024)
                                                    : smem_desc_sw128(b_addr + kk * 32, 16, 1024);
                        mma_i8(d_tmem, adesc, bdesc, idesc, (kb | kk) != 0 ? 1u : 0u);
                    }
                    mma_commit(&empty[s]);
                }
                __syncwarp();
            }
            if (lane == 0) mma_commit(&tfull[acc]);
            __syncwarp();
        }
    } else {
        // Epilogue: warp w reads TMEM lanes 32*(w%4) .. +31, i.e. rows 32*(w%4) + lane of the tile.
        const int q = warp & 3;
        int lt = 0;
        for (int tile = blockIdx.x; tile < p.total_tiles; tile += gridDim.x, lt++) {
            int b, tm, tn;
            tile_coords(p, tile, b, tm, tn);
            const int acc = lt & 1;
            const uint32_t aph = (lt >> 1) & 1;
            if (!mbar_wait(&tfull[acc], aph, abort_flag)) goto done;
            tc_fence_after();
            const int m = tm * tc::BM + q * 32 + lane;
            const bool row_ok = m < p.m;
            const RowTerms rt = row_ok ? row_terms(p.epi, b, m) : RowTerms{0, 0};
            const uint32_t t_row = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * tc::BN;
#pragma unroll 1
            for (int c = 0; c < tc::BN / 32; c++) {
                const int n0 = tn * tc::BN + c * 32;
                if (n0 >= p.n) break;
                uint32_t r[32];
                tmem_ld_32x32b_x32(t_row + c * 32, r);
                tmem_ld_wait();
                if (row_ok) store_chunk<OUT>(p.epi, rt, b, m, n0, r);
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&tempty[acc]);
        }
    }

done:
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, tc::TMEM_COLS);
    }
    if (threadIdx.x == 0 && *abort_flag) atomicExch(p.error_flag, 1);
}

// ---- host side ---------------------------------------------------------------------------------------------------

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (fn == nullptr) {
        cudaDriverEntryPointQueryResult q;
        void* f = nullptr;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
    }
    return fn;
}

// A 3-D byte tensor (x innermost) with 128-byte swizzled boxes of box_x x box_y.
static bool make_map(CUtensorMap* map, const void* base, uint64_t x, uint64_t y, uint64_t z, uint64_t stride_y,
                     uint64_t stride_z, uint32_t box_x, uint32_t box_y) {
    auto fn = encode_fn();
    if (fn == nullptr) return false;
    cuuint64_t dims[3] = {x, y, z};
    cuuint64_t strides[2] = {stride_y, stride_z};
    cuuint32_t box[3] = {box_x, box_y, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(base), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

static uint64_t round16(uint64_t v) { return (v + 15) & ~uint64_t(15); }

bool tc_eligible(const GemmLaunch& L) {
    if (L.k < 1 || L.m < 1 || L.n < 1) return false;
    auto al = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
    if (!al(L.a) || !al(L.b)) return false;
    if ((L.lda & 15) || (L.ldb & 15)) return false;
    if (L.batch > 1 && ((L.stride_a & 15) || (L.stride_b & 15))) return false;
    return true;
}

template <bool B_MN, int OUT>
static cudaError_t launch_tc_t(const GemmLaunch& L, const TcParams& p, const CUtensorMap& ma, const CUtensorMap& mb,
                               int grid, cudaStream_t stream) {
    auto kern = int8_gemm_tc_kernel<B_MN, OUT>;
    static uint64_t configured = 0;  // one bit per device ordinal: the attribute is per device
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    const uint64_t bit = uint64_t(1) << (dev & 63);
    if (!(configured & bit)) {
        e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, tc::SMEM_BYTES);
        if (e != cudaSuccess) return e;
        configured |= bit;
    }
    const uint32_t idesc = idesc_i8(L.a_signed, L.b_signed, false, B_MN, tc::BM, tc::BN);
    kern<<<grid, tc::THREADS, tc::SMEM_BYTES, stream>>>(ma, mb, p, idesc);
    return cudaGetLastError();
}

cudaError_t launch_gemm_tc(const GemmLaunch& L, cudaStream_t stream) {
    const int ba = (L.batch > 1 && L.stride_a != 0) ? L.batch : 1;
    const int bb = (L.batch > 1 && L.stride_b != 0) ? L.batch : 1;
    CUtensorMap ma, mb;
    if (!make_map(&ma, L.a, L.k, L.m, ba, L.lda, ba > 1 ? L.stride_a : round16(uint64_t(L.lda) * L.m), tc::BK,
                  tc::BM))
        return cudaErrorInvalidValue;
    const uint64_t rows_b = L.trans_b ? L.n : L.k;
    const uint64_t sb = bb > 1 ? uint64_t(L.stride_b) : round16(uint64_t(L.ldb) * rows_b);
    const bool ok = L.trans_b ? make_map(&mb, L.b, L.k, L.n, bb, L.ldb, sb, tc::BK, tc::BN)
                              : make_map(&mb, L.b, L.n, L.k, bb, L.ldb, sb, 128, tc::BK);
    if (!ok) return cudaErrorInvalidValue;

    TcParams p;
    p.m = L.m;
    p.n = L.n;
    p.k = L.k;
    p.tiles_m = (L.m + tc::BM - 1) / tc::BM;
    p.tiles_n = (L.n + tc::BN - 1) / tc::BN;
    p.batch = L.batch;
    p.a_batched = ba > 1;
    p.b_batched = bb > 1;
    p.k_blocks = (L.k + tc::BK - 1) / tc::BK;
    const int64_t total = int64_t(p.tiles_m) * p.tiles_n * L.batch;
    p.total_tiles = static_cast<int>(total);
    p.epi = L.epi;
    p.error_flag = L.error_flag;
    const int grid = static_cast<int>(total < L.num_sms ? total : L.num_sms);
    const bool bmn = !L.trans_b;
    switch (L.epi.out_kind) {
        case OUT_I32: return bmn ? launch_tc_t<true, OUT_I32>(L, p, ma, mb, grid, stream)
                                 : launch_tc_t<false, OUT_I32>(L, p, ma, mb, grid, stream);
        case OUT_F32: return bmn ? launch_tc_t<true, OUT_F32>(L, p, ma, mb, grid, stream)
                                 : launch_tc_t<false, OUT_F32>(L, p, ma, mb, grid, stream);
        case OUT_U8: return bmn ? launch_tc_t<true, OUT_U8>(L, p, ma, mb, grid, stream)
                                : launch_tc_t<false, OUT_U8>(L, p, ma, mb, grid, stream);
        default: return bmn ? launch_tc_t<true, OUT_S8>(L, p, ma, mb, grid, stream)
                            : launch_tc_t<false, OUT_S8>(L, p, ma, mb, grid, stream);
    }
}

}  // namespace og
