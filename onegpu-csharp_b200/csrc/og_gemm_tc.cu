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
constexpr int BN = 256;
constexpr int BK = 128;                    // bytes of K per stage = one 128-byte swizzle row
constexpr int NUM_ACC = 2;
constexpr int TMEM_COLS = NUM_ACC * BN;    // 512: all of TMEM
constexpr int THREADS = 192;               // producer, MMA, 4 epilogue warps
constexpr int GROUP_M = 8;                 // output tiles per raster group along M

// CG = 1: one CTA computes a 128 x 256 tile. CG = 2: a CTA pair computes a 256 x 256 tile with tcgen05.mma
// cta_group::2; each CTA stages its own 128 rows of A and its own 128 columns of B, so every SM pulls 32 KB per
// K block instead of 48 KB.
template <int CG>
struct Cfg {
    static constexpr int BM = 128 * CG;
    static constexpr int A_BYTES = 128 * BK;          // 16 KB per CTA
    static constexpr int B_COLS = BN / CG;            // columns of B staged by one CTA
    static constexpr int B_BYTES = B_COLS * BK;       // 32 KB or 16 KB per CTA
    static constexpr int B_BOX = 128 * BK;            // one 128-column box of an MN-major B
    static constexpr int STAGES = CG == 1 ? 4 : 6;
    static constexpr int TERMS_BYTES = 5 * 4 * BN;     // per-column epilogue terms
    static constexpr int BOX_BYTES = 32 * 128;          // one 32-row x 32-word store box
    static constexpr int STAGING_BYTES = 4 * BOX_BYTES; // one box per epilogue warp
    static constexpr int SMEM_BYTES =
        STAGES * (A_BYTES + B_BYTES) + STAGING_BYTES + 1024 /* alignment */ + 256 /* barriers */ + TERMS_BYTES;
};
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
    int tma_store;  // int32 / float results leave through shared memory and TMA stores (C rows 16-byte aligned)
};

template <int BM>
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

// Per-column terms of one output tile, staged in shared memory by the epilogue warps so that each element needs one
// multiply-add and broadcast shared-memory reads:
//   C = dot + zb[n] * (K * za[m] - rowsumA[m]) + c[n] - (za per row ? za[m] * colsumB[n] : 0)
// with c[n] = intBias[n] - za * colsumB[n] when A has one zero point (intBias[n] otherwise), all modulo 2^32.
struct ColTerms {
    int32_t zb[tc::BN];
    int32_t c[tc::BN];
    int32_t csb[tc::BN];
    float scale[tc::BN];
    float fbias[tc::BN];
};

__device__ __forceinline__ void fill_col_terms(ColTerms& t, const Epilogue& e, int b, int col0, int tid, int nthreads) {
    const bool za_scalar = e.za != nullptr && !e.za_vector;
    const int32_t zas = za_scalar ? zp_value(e.za, 0, e.za_signed, 0) : 0;
    for (int j = tid; j < tc::BN; j += nthreads) {
        const int n = col0 + j;
        const bool ok = n < e.n;
        const int32_t csb = (ok && e.za != nullptr) ? static_cast<int32_t>(col_sum_of(e, b, n)) : 0;
        const int32_t bias = (ok && e.int_bias != nullptr) ? __ldg(e.int_bias + n) : 0;
        t.zb[j] = ok ? zp_value(e.zb, e.zb_vector, e.zb_signed, n) : 0;
        t.csb[j] = csb;
        t.c[j] = static_cast<int32_t>(static_cast<uint32_t>(bias) - static_cast<uint32_t>(zas) * static_cast<uint32_t>(csb));
        t.scale[j] = (ok && e.scale != nullptr) ? col_scale(e, n) : 0.0f;
        t.fbias[j] = (ok && e.float_bias != nullptr) ? __ldg(e.float_bias + n) : 0.0f;
    }
}

// The corrected int32 sum of column j of the tile, for a row with zero point za and rt = K * za - rowsumA.
__device__ __forceinline__ uint32_t tile_sum(const ColTerms& t, bool za_per_row, uint32_t za, uint32_t rt, int j,
                                             uint32_t dot) {
    uint32_t s = dot + static_cast<uint32_t>(t.zb[j]) * rt + static_cast<uint32_t>(t.c[j]);
    if (za_per_row) s -= za * static_cast<uint32_t>(t.csb[j]);
    return s;
}

template <int OUT>
__device__ __forceinline__ uint32_t finish_word(const ColTerms& t, const Epilogue& e, bool terms, bool za_per_row,
                                                uint32_t za, uint32_t rt, int j, uint32_t dot) {
    if constexpr (OUT == OUT_I32) {
        return terms ? tile_sum(t, za_per_row, za, rt, j, dot) : dot;
    } else if constexpr (OUT == OUT_F32) {
        const uint32_t s = tile_sum(t, za_per_row, za, rt, j, dot);
        float f = __fmul_rn(__int2float_rn(static_cast<int32_t>(s)), t.scale[j]);
        if (e.float_bias != nullptr) f = __fadd_rn(f, t.fbias[j]);
        return __float_as_uint(f);
    } else {
        const uint32_t s = tile_sum(t, za_per_row, za, rt, j, dot);
        constexpr bool U = OUT == OUT_U8;
        const int lo = U ? 0 : -128, hi = U ? 255 : 127;
        const float v = __fmul_rn(__int2float_rn(static_cast<int32_t>(s)), t.scale[j]);
        if (isnan(v)) return static_cast<uint32_t>(lo & 0xFF);
        float r = rintf(v);
        const float flo = static_cast<float>(lo - e.zero_point_y), fhi = static_cast<float>(hi - e.zero_point_y);
        r = r < flo ? flo : (r > fhi ? fhi : r);
        return static_cast<uint32_t>((static_cast<int>(r) + e.zero_point_y) & 0xFF);
    }
}

// Finishes 32 consecutive int32 / float results of one row (tile columns j0..) and writes them as row `lane` of a
// 32 x 32-word box in 128-byte-swizzled shared memory: 16-byte chunk j of the row lands at chunk j ^ (lane % 8), so the
// eight lanes of each store phase hit eight different bank groups.
template <int OUT>
__device__ __forceinline__ void stage_chunk(const ColTerms& t, const Epilogue& e, bool terms, bool za_per_row,
                                            uint32_t za, uint32_t rt, int j0, const uint32_t (&r)[32], uint8_t* box,
                                            int lane) {
    uint32_t w[32];
#pragma unroll
    for (int q = 0; q < 32; q++) w[q] = finish_word<OUT>(t, e, terms, za_per_row, za, rt, j0 + q, r[q]);
    const uint32_t row = smem_u32(box) + lane * 128;
#pragma unroll
    for (int j = 0; j < 8; j++) {
        const uint32_t addr = row + ((j ^ (lane & 7)) << 4);
        asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(w[4 * j]), "r"(w[4 * j + 1]),
                     "r"(w[4 * j + 2]), "r"(w[4 * j + 3])
                     : "memory");
    }
}

// Stores 32 consecutive results of row m (columns n0.. of the output; j0 is n0's column within the tile).
template <int OUT>
__device__ __forceinline__ void store_chunk(const ColTerms& t, const Epilogue& e, bool terms, bool za_per_row,
                                            uint32_t za, uint32_t rt, int b, int m, int n0, int j0,
                                            const uint32_t (&r)[32]) {
    const bool full = e.vec_ok && (n0 + 32 <= e.n);
    if constexpr (OUT == OUT_I32 || OUT == OUT_F32) {
        uint32_t* row = static_cast<uint32_t*>(e.c) + b * e.batch_stride_c + static_cast<int64_t>(m) * e.ldc;
        if (full) {
            uint4* dst = reinterpret_cast<uint4*>(row + n0);
#pragma unroll
            for (int q = 0; q < 8; q++) {
                uint4 v;
                v.x = finish_word<OUT>(t, e, terms, za_per_row, za, rt, j0 + 4 * q + 0, r[4 * q + 0]);
                v.y = finish_word<OUT>(t, e, terms, za_per_row, za, rt, j0 + 4 * q + 1, r[4 * q + 1]);
                v.z = finish_word<OUT>(t, e, terms, za_per_row, za, rt, j0 + 4 * q + 2, r[4 * q + 2]);
                v.w = finish_word<OUT>(t, e, terms, za_per_row, za, rt, j0 + 4 * q + 3, r[4 * q + 3]);
                __stcs(dst + q, v);
            }
        } else {
#pragma unroll
            for (int q = 0; q < 32; q++) {
                if (n0 + q < e.n) row[n0 + q] = finish_word<OUT>(t, e, terms, za_per_row, za, rt, j0 + q, r[q]);
            }
        }
    } else {
        uint8_t* row = static_cast<uint8_t*>(e.c) + b * e.batch_stride_c + static_cast<int64_t>(m) * e.ldc;
        if (full) {
            uint32_t w[8];
#pragma unroll
            for (int q = 0; q < 8; q++) {
                uint32_t x = 0;
#pragma unroll
                for (int u = 0; u < 4; u++)
                    x |= finish_word<OUT>(t, e, terms, za_per_row, za, rt, j0 + 4 * q + u, r[4 * q + u]) << (8 * u);
                w[q] = x;
            }
            uint4* dst = reinterpret_cast<uint4*>(row + n0);
            dst[0] = make_uint4(w[0], w[1], w[2], w[3]);
            dst[1] = make_uint4(w[4], w[5], w[6], w[7]);
        } else {
#pragma unroll
            for (int q = 0; q < 32; q++) {
                if (n0 + q < e.n)
                    row[n0 + q] = static_cast<uint8_t>(finish_word<OUT>(t, e, terms, za_per_row, za, rt, j0 + q, r[q]));
            }
        }
    }
}

template <int CG, bool B_MN, int OUT>
__device__ __forceinline__ void gemm_tc_body(const CUtensorMap& tmap_a, const CUtensorMap& tmap_b,
                                             const CUtensorMap& tmap_c, const TcParams& p, uint32_t idesc) {
    using C = tc::Cfg<CG>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sA = smem;
    uint8_t* sB = smem + C::STAGES * C::A_BYTES;
    uint8_t* staging = sB + C::STAGES * C::B_BYTES;  // 1024-byte aligned store boxes of the epilogue warps
    uint64_t* bars = reinterpret_cast<uint64_t*>(staging + C::STAGING_BYTES);
    uint64_t* full = bars;
    uint64_t* empty = bars + C::STAGES;
    uint64_t* tfull = bars + 2 * C::STAGES;
    uint64_t* tempty = bars + 2 * C::STAGES + tc::NUM_ACC;
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + 2 * C::STAGES + 2 * tc::NUM_ACC);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t rank = CG == 2 ? cluster_ctarank() : 0;  // CTA of the pair: rank 0 issues the MMAs
    const bool leader = rank == 0;
    const int worker = CG == 2 ? static_cast<int>(blockIdx.x >> 1) : static_cast<int>(blockIdx.x);
    const int workers = CG == 2 ? static_cast<int>(gridDim.x >> 1) : static_cast<int>(gridDim.x);

    if (threadIdx.x == 0) {
        for (int s = 0; s < C::STAGES; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int a = 0; a < tc::NUM_ACC; a++) {
            mbar_init(&tfull[a], 1);
            mbar_init(&tempty[a], 4 * CG);  // one arrival per epilogue warp of every CTA of the pair
        }
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 0 && lane == 0) {
        prefetch_tmap(&tmap_a);
        prefetch_tmap(&tmap_b);
    }
    constexpr bool WORDS = OUT == OUT_I32 || OUT == OUT_F32;
    const bool tma_store = WORDS && p.tma_store;
    if (tma_store && warp == 2 && lane == 0) prefetch_tmap(&tmap_c);
    if (warp == 1) {
        if constexpr (CG == 2) {
            tmem_alloc_pair(tmem_holder, tc::TMEM_COLS);
            tmem_relinquish_pair();
        } else {
            tmem_alloc(tmem_holder, tc::TMEM_COLS);
            tmem_relinquish();
        }
    }
    tc_fence_before();
    __syncthreads();
    if constexpr (CG == 2) cluster_sync_all();  // the peer's barriers are initialised before any remote arrival
    tc_fence_after();
    const uint32_t tmem_base = *tmem_holder;

    if (warp == 0) {
        // TMA producer: the whole warp walks the ring, lane 0 issues.
        uint32_t it = 0;
        for (int tile = worker; tile < p.total_tiles; tile += workers) {
            int b, tm, tn;
            tile_coords<C::BM>(p, tile, b, tm, tn);
            const int ba = p.a_batched ? b : 0;
            const int bb = p.b_batched ? b : 0;
            const int row0 = tm * C::BM + static_cast<int>(rank) * 128;
            const int col0 = tn * tc::BN + static_cast<int>(rank) * C::B_COLS;
            // With one CTA, a second 128-column box wholly past N is skipped; a pair always loads full boxes
            // (TMA fills what lies outside the tensor with zeros) so the leader knows the byte count.
            const bool second_half = CG == 1 && B_MN && (col0 + 128 < p.n);
            const uint32_t bytes = CG == 2 ? 2u * (C::A_BYTES + C::B_BYTES)
                                           : C::A_BYTES + (B_MN ? (second_half ? 2 : 1) * C::B_BOX : C::B_BYTES);
            for (int kb = 0; kb < p.k_blocks; kb++, it++) {
                const int s = it % C::STAGES;
                const uint32_t ph = (it / C::STAGES) & 1;
                if (!mbar_wait(&empty[s], ph ^ 1, abort_flag)) goto done;
                if (lane == 0) {
                    if constexpr (CG == 2) {
                        const uint32_t bar = mapa_shared(smem_u32(&full[s]), 0);
                        if (leader) mbar_arrive_expect_tx(&full[s], bytes);
                        tma_load_3d_pair(sA + s * C::A_BYTES, &tmap_a, bar, kb * tc::BK, row0, ba);
                        if constexpr (B_MN)
                            tma_load_3d_pair(sB + s * C::B_BYTES, &tmap_b, bar, col0, kb * tc::BK, bb);
                        else
                            tma_load_3d_pair(sB + s * C::B_BYTES, &tmap_b, bar, kb * tc::BK, col0, bb);
                    } else {
                        mbar_arrive_expect_tx(&full[s], bytes);
                        tma_load_3d(sA + s * C::A_BYTES, &tmap_a, &full[s], kb * tc::BK, row0, ba);
                        if constexpr (B_MN) {
                            tma_load_3d(sB + s * C::B_BYTES, &tmap_b, &full[s], col0, kb * tc::BK, bb);
                            if (second_half)
                                tma_load_3d(sB + s * C::B_BYTES + C::B_BOX, &tmap_b, &full[s], col0 + 128,
                                            kb * tc::BK, bb);
                        } else {
                            tma_load_3d(sB + s * C::B_BYTES, &tmap_b, &full[s], kb * tc::BK, col0, bb);
                        }
                    }
                }
                __syncwarp();
            }
        }
    } else if (warp == 1) {
        // MMA issuer (the leader CTA of a pair issues for both): four K = 32 MMAs per stage.
        if (leader) {
            uint32_t it = 0;
            int lt = 0;
            for (int tile = worker; tile < p.total_tiles; tile += workers, lt++) {
                const int acc = lt & 1;
                const uint32_t aph = (lt >> 1) & 1;
                if (!mbar_wait(&tempty[acc], aph ^ 1, abort_flag)) goto done;
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + acc * tc::BN;
                for (int kb = 0; kb < p.k_blocks; kb++, it++) {
                    const int s = it % C::STAGES;
                    const uint32_t ph = (it / C::STAGES) & 1;
                    if (!mbar_wait(&full[s], ph, abort_flag)) goto done;
                    tc_fence_after();
                    if (lane == 0) {
                        const uint32_t a_addr = smem_u32(sA + s * C::A_BYTES);
                        const uint32_t b_addr = smem_u32(sB + s * C::B_BYTES);
#pragma unroll
                        for (int kk = 0; kk < tc::BK / 32; kk++) {
                            const uint64_t adesc = smem_desc_sw128(a_addr + kk * 32, 16, 1024);
                            const uint64_t bdesc = B_MN ? smem_desc_sw128(b_addr + kk * 32 * 128, C::B_BOX, 1024)
                                                        : smem_desc_sw128(b_addr + kk * 32, 16, 1024);
                            const uint32_t accum = (kb | kk) != 0 ? 1u : 0u;
                            if constexpr (CG == 2)
                                mma_i8_pair(d_tmem, adesc, bdesc, idesc, accum);
                            else
                                mma_i8(d_tmem, adesc, bdesc, idesc, accum);
                        }
                        if constexpr (CG == 2)
                            mma_commit_pair(&empty[s], 0x3);
                        else
                            mma_commit(&empty[s]);
                    }
                    __syncwarp();
                }
                if (lane == 0) {
                    if constexpr (CG == 2)
                        mma_commit_pair(&tfull[acc], 0x3);
                    else
                        mma_commit(&tfull[acc]);
                }
                __syncwarp();
            }
        }
    } else {
        // Epilogue: warp w reads TMEM lanes 32*(w%4) .. +31, i.e. rows 32*(w%4) + lane of this CTA's 128 rows.
        const int q = warp & 3;
        const uint32_t tempty_leader = CG == 2 ? mapa_shared(smem_u32(&tempty[0]), 0) : 0;
        const Epilogue& e = p.epi;
        ColTerms& terms_smem = *reinterpret_cast<ColTerms*>(reinterpret_cast<uint8_t*>(bars) + 256);
        // Column terms are needed unless the result is the raw int32 sum.
        const bool terms = OUT != OUT_I32 || e.za != nullptr || e.zb != nullptr || e.int_bias != nullptr;
        const bool za_per_row = e.za != nullptr && e.za_vector;
        int lt = 0;
        for (int tile = worker; tile < p.total_tiles; tile += workers, lt++) {
            int b, tm, tn;
            tile_coords<C::BM>(p, tile, b, tm, tn);
            const int acc = lt & 1;
            const uint32_t aph = (lt >> 1) & 1;
            if (!mbar_wait(&tfull[acc], aph, abort_flag)) goto done;
            tc_fence_after();
            if (terms) {
                asm volatile("bar.sync 1, 128;" ::: "memory");  // the previous tile's terms are no longer read
                fill_col_terms(terms_smem, e, b, tn * tc::BN, threadIdx.x - 64, 128);
                asm volatile("bar.sync 1, 128;" ::: "memory");
            }
            const int m = tm * C::BM + static_cast<int>(rank) * 128 + q * 32 + lane;
            const bool row_ok = m < p.m;
            uint32_t za = 0, rt = 0;  // zero point of A for this row, and K * za - rowsumA
            if (row_ok && terms) {
                za = static_cast<uint32_t>(zp_value(e.za, e.za_vector, e.za_signed, m));
                const uint32_t rsa = e.row_sum_a ? row_sum_of(e, b, m) : 0u;
                rt = static_cast<uint32_t>(p.k) * za - rsa;
            }
            const uint32_t t_row = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * tc::BN;
            if (tma_store) {
                // Each 32 x 32 chunk goes through this warp's box and leaves as one TMA store of full 128-byte row
                // segments; rows past M and columns past N are clipped by the tensor map.
                uint8_t* box = staging + q * C::BOX_BYTES;
                const int box_row = tm * C::BM + static_cast<int>(rank) * 128 + q * 32;
#pragma unroll 1
                for (int c = 0; c < tc::BN / 32; c++) {
                    const int n0 = tn * tc::BN + c * 32;
                    if (n0 >= p.n || box_row >= p.m) break;  // boxes start inside C
                    uint32_t r[32];
                    tmem_ld_32x32b_x32(t_row + c * 32, r);
                    tmem_ld_wait();
                    if (lane == 0) bulk_wait_group_read<0>();  // the previous store has read the box
                    __syncwarp();
                    stage_chunk<OUT>(terms_smem, e, terms, za_per_row, za, rt, c * 32, r, box, lane);
                    fence_proxy_async_smem();
                    __syncwarp();
                    if (lane == 0) {
                        tma_store_3d(&tmap_c, box, n0, box_row, b);
                        bulk_commit_group();
                    }
                }
            } else {
#pragma unroll 1
                for (int c = 0; c < tc::BN / 32; c++) {
                    const int n0 = tn * tc::BN + c * 32;
                    if (n0 >= p.n) break;
                    uint32_t r[32];
                    tmem_ld_32x32b_x32(t_row + c * 32, r);
                    tmem_ld_wait();
                    if (row_ok) store_chunk<OUT>(terms_smem, e, terms, za_per_row, za, rt, b, m, n0, c * 32, r);
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                if constexpr (CG == 2)
                    mbar_arrive_cluster(tempty_leader + acc * sizeof(uint64_t));
                else
                    mbar_arrive(&tempty[acc]);
            }
        }
    }

done:
    if (tma_store && warp >= 2 && lane == 0) bulk_wait_group_all();  // stores finished before shared memory goes
    __syncthreads();
    if constexpr (CG == 2) cluster_sync_all();  // neither CTA frees the pair's TMEM while the other still reads it
    if (warp == 1) {
        tc_fence_after();
        if constexpr (CG == 2)
            tmem_dealloc_pair(tmem_base, tc::TMEM_COLS);
        else
            tmem_dealloc(tmem_base, tc::TMEM_COLS);
    }
    if (threadIdx.x == 0 && *abort_flag) atomicExch(p.error_flag, 1);
}

template <bool B_MN, int OUT>
__global__ void __launch_bounds__(tc::THREADS, 1)
    int8_gemm_tc_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                        const __grid_constant__ CUtensorMap tmap_c, const TcParams p, uint32_t idesc) {
    gemm_tc_body<1, B_MN, OUT>(tmap_a, tmap_b, tmap_c, p, idesc);
}

template <bool B_MN, int OUT>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(tc::THREADS, 1)
    int8_gemm_tc2_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                         const __grid_constant__ CUtensorMap tmap_c, const TcParams p, uint32_t idesc) {
    gemm_tc_body<2, B_MN, OUT>(tmap_a, tmap_b, tmap_c, p, idesc);
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

// The output C as a 3-D tensor of 4-byte words (columns innermost) stored in 32 x 32-word boxes from 128-byte-swizzled
// shared memory.
static bool make_store_map(CUtensorMap* map, void* base, uint64_t n, uint64_t m, uint64_t batch, uint64_t row_bytes,
                           uint64_t batch_bytes) {
    auto fn = encode_fn();
    if (fn == nullptr) return false;
    cuuint64_t dims[3] = {n, m, batch};
    cuuint64_t strides[2] = {row_bytes, batch_bytes};
    cuuint32_t box[3] = {32, 32, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_INT32, 3, base, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

bool make_tensor_map_u8(CUtensorMap* map, const void* base, uint64_t x, uint64_t y, uint64_t z, uint64_t stride_y,
                        uint64_t stride_z, uint32_t box_x, uint32_t box_y) {
    return make_map(map, base, x, y, z, stride_y, stride_z, box_x, box_y);
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

// Sets the kernel's dynamic shared-memory limit once per device (the attribute is per device).
template <class K>
static cudaError_t configure(K kern, int smem, uint64_t& configured) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    const uint64_t bit = uint64_t(1) << (dev & 63);
    if (!(configured & bit)) {
        e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return e;
        configured |= bit;
    }
    return cudaSuccess;
}

// Binds the kernel and its arguments; the returned function only sets the shared-memory limit (first time per
// device) and launches.
template <int CG, bool B_MN, int OUT>
static LaunchFn bind_tc_t(const GemmLaunch& L, const TcParams& p, const CUtensorMap& ma, const CUtensorMap& mb,
                          const CUtensorMap& mc, int grid) {
    using C = tc::Cfg<CG>;
    const uint32_t idesc = idesc_i8(L.a_signed, L.b_signed, false, B_MN, C::BM, tc::BN);
    return [=](cudaStream_t stream) -> cudaError_t {
        static uint64_t configured = 0;
        if constexpr (CG == 2) {
            auto kern = int8_gemm_tc2_kernel<B_MN, OUT>;
            cudaError_t e = configure(kern, C::SMEM_BYTES, configured);
            if (e != cudaSuccess) return e;
            kern<<<grid, tc::THREADS, C::SMEM_BYTES, stream>>>(ma, mb, mc, p, idesc);
        } else {
            auto kern = int8_gemm_tc_kernel<B_MN, OUT>;
            cudaError_t e = configure(kern, C::SMEM_BYTES, configured);
            if (e != cudaSuccess) return e;
            kern<<<grid, tc::THREADS, C::SMEM_BYTES, stream>>>(ma, mb, mc, p, idesc);
        }
        return cudaGetLastError();
    };
}

template <int CG>
static LaunchFn prepare_cg(const GemmLaunch& L, cudaError_t* err) {
    using C = tc::Cfg<CG>;
    *err = cudaSuccess;
    const int ba = (L.batch > 1 && L.stride_a != 0) ? L.batch : 1;
    const int bb = (L.batch > 1 && L.stride_b != 0) ? L.batch : 1;
    CUtensorMap ma, mb;
    if (!make_map(&ma, L.a, L.k, L.m, ba, L.lda, ba > 1 ? L.stride_a : round16(uint64_t(L.lda) * L.m), tc::BK, 128)) {
        *err = cudaErrorInvalidValue;
        return nullptr;
    }
    const uint64_t rows_b = L.trans_b ? L.n : L.k;
    const uint64_t sb = bb > 1 ? uint64_t(L.stride_b) : round16(uint64_t(L.ldb) * rows_b);
    const bool ok = L.trans_b ? make_map(&mb, L.b, L.k, L.n, bb, L.ldb, sb, tc::BK, C::B_COLS)
                              : make_map(&mb, L.b, L.n, L.k, bb, L.ldb, sb, 128, tc::BK);
    if (!ok) {
        *err = cudaErrorInvalidValue;
        return nullptr;
    }

    TcParams p;
    p.m = L.m;
    p.n = L.n;
    p.k = L.k;
    p.tiles_m = (L.m + C::BM - 1) / C::BM;
    p.tiles_n = (L.n + tc::BN - 1) / tc::BN;
    p.batch = L.batch;
    p.a_batched = ba > 1;
    p.b_batched = bb > 1;
    p.k_blocks = (L.k + tc::BK - 1) / tc::BK;
    const int64_t total = int64_t(p.tiles_m) * p.tiles_n * L.batch;
    p.total_tiles = static_cast<int>(total);
    p.epi = L.epi;
    p.error_flag = L.error_flag;
    // int32 / float results go out through TMA stores when C's rows (and batches) start on 16-byte boundaries.
    CUtensorMap mc;
    std::memset(&mc, 0, sizeof(mc));
    const bool words = L.epi.out_kind == OUT_I32 || L.epi.out_kind == OUT_F32;
    const bool c_aligned = (reinterpret_cast<uintptr_t>(L.epi.c) & 15) == 0 && (L.epi.ldc & 3) == 0 &&
                           (L.batch == 1 || (L.epi.batch_stride_c & 3) == 0);
    p.tma_store = words && c_aligned &&
                  make_store_map(&mc, L.epi.c, L.n, L.m, L.batch, uint64_t(L.epi.ldc) * 4,
                                 L.batch > 1 ? uint64_t(L.epi.batch_stride_c) * 4 : round16(uint64_t(L.epi.ldc) * 4 * L.m));
    const int64_t workers = L.num_sms / CG;
    const int grid = static_cast<int>((total < workers ? total : workers) * CG);
    const bool bmn = !L.trans_b;
    switch (L.epi.out_kind) {
        case OUT_I32: return bmn ? bind_tc_t<CG, true, OUT_I32>(L, p, ma, mb, mc, grid)
                                 : bind_tc_t<CG, false, OUT_I32>(L, p, ma, mb, mc, grid);
        case OUT_F32: return bmn ? bind_tc_t<CG, true, OUT_F32>(L, p, ma, mb, mc, grid)
                                 : bind_tc_t<CG, false, OUT_F32>(L, p, ma, mb, mc, grid);
        case OUT_U8: return bmn ? bind_tc_t<CG, true, OUT_U8>(L, p, ma, mb, mc, grid)
                                : bind_tc_t<CG, false, OUT_U8>(L, p, ma, mb, mc, grid);
        default: return bmn ? bind_tc_t<CG, true, OUT_S8>(L, p, ma, mb, mc, grid)
                            : bind_tc_t<CG, false, OUT_S8>(L, p, ma, mb, mc, grid);
    }
}

int tc_cta_group(const GemmLaunch& L) {
    if (L.tile == 128) return 1;
    if (L.tile == 256) return 2;
    // The pair tile halves the operand bytes each SM pulls from L2 per MMA; use it once there are enough 256-row
    // tiles to give most SM pairs work.
    const int64_t pair_tiles = int64_t((L.m + 255) / 256) * ((L.n + 255) / 256) * L.batch;
    return (L.m > 128 && pair_tiles * 4 >= int64_t(L.num_sms / 2) * 3) ? 2 : 1;
}

LaunchFn prepare_gemm_tc(const GemmLaunch& L, cudaError_t* err) {
    return tc_cta_group(L) == 2 ? prepare_cg<2>(L, err) : prepare_cg<1>(L, err);
}

cudaError_t launch_gemm_tc(const GemmLaunch& L, cudaStream_t stream) {
    cudaError_t err;
    LaunchFn fn = prepare_gemm_tc(L, &err);
    return fn ? fn(stream) : err;
}

}  // namespace og
