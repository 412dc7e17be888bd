// The tensor-core int8 product for sm_100a: tcgen05.mma.kind::i8 with int32 accumulators in TMEM, operands staged by
// TMA into 128-byte-swizzled shared memory, warp-specialised and persistent.
//
// One CTA per SM (or a CTA pair with cta_group::2, 256 x 256 tiles) walks the output tiles (BM x BN = 128 x 256 of
// one batch per CTA) in a grouped order so that concurrently running CTAs share A rows and B columns in L2. Warp 0
// issues the TMA loads of a STAGES-deep ring of K blocks (BK = 128 bytes); warp 1 owns the TMEM allocation and
// issues the MMAs (four K = 32 instructions per K block) into one of two accumulators; warps 2-9 drain the other
// accumulator (tcgen05.ld; two warps per TMEM lane quadrant, each half of the columns), apply the zero-point
// correction and the epilogue and store C (through one shared-memory box per warp and TMA stores) while the next
// tile is being multiplied.
//
// A is M x K row-major (K-major for the MMA). B is either K x N row-major (TransposeB = false; MN-major for the MMA,
// loaded as two 128-column boxes) or N x K (TransposeB = true; K-major). The MMA multiplies the operands' own
// types (u8 or s8); the zero points are applied afterwards from byte sums (og_kernels.cuh). Ragged M, N and K
// edges are zero-filled by TMA and never stored. No load uses cluster multicast, so the kernel is the same on any
// number of GPUs.
//
// Every kernel is compiled twice, on SPLIT: with the stream-K and split-tail schedules, for the launches that use
// them, and without, for launches of whole tiles only (most of them), whose loops then carry none of that code
// (8192 x 1024 x 8192 took 57.3 us with it and 55.2 us without).
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>

#include <cstdio>
#include <cstdlib>
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
constexpr int EPI_WARPS = 8;               // two per TMEM lane quadrant, each taking half of the tile's columns
constexpr int EPI_THREADS = 32 * EPI_WARPS;
constexpr int THREADS = 64 + EPI_THREADS;  // producer, MMA, epilogue warps
// Output tiles per raster group along M: 16 when there are at least 32 tile rows, 8 otherwise. A group walks its
// rows of A against every column tile of B, so taller groups read B fewer times. Measured on B200, 8192^3 took
// 319.4-320.4 us with 16 against 323.6 us with 8 (12, 20, 24 and 32 were 1-16 us slower than 16), while 4096^3
// with the dequantize epilogue (both operands fit in L2) was ~0.9 us slower with 16, and the shard shapes did not
// change.
constexpr int GROUP_M = 8;
constexpr int GROUP_M_TALL = 16;

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
    static constexpr int BOX_BYTES = 32 * 64;          // one 32-row x 16-word store box (64-byte rows)
    static constexpr int BOXES = 1;                    // store boxes per epilogue warp
    static constexpr int STAGING_BYTES = EPI_WARPS * BOXES * BOX_BYTES;
    static constexpr int SMEM_BYTES =
        STAGES * (A_BYTES + B_BYTES) + STAGING_BYTES + 1024 /* alignment */ + 256 /* barriers */ + TERMS_BYTES;
};
}  // namespace tc

struct TcParams {
    int m, n, k;
    int tiles_m, tiles_n;
    int group_m;  // output tiles per raster group along M
    int batch;
    int a_batched, b_batched;
    int k_blocks;
    int total_tiles;
    Epilogue epi;
    int* error_flag;
    int tma_store;  // int32 / float results leave through shared memory and TMA stores (C rows 16-byte aligned)
    // Stream-K: the workers split the total_tiles * k_blocks (tile, K block) units into equal contiguous ranges. A
    // tile cut by a range boundary is finished by the worker holding its K-block-0 segment (the end of its range),
    // after the next worker has handed over the sums of the later segment (the start of its range) through
    // sk_part[next worker] and set sk_flag[next worker] to this launch's generation. The generation lives after the
    // flags (with a ticket counter): every CTA reads it when it starts and the last CTA to finish advances it, so no
    // flag needs clearing between launches, replays of a captured graph included.
    int stream_k;
    int64_t units;
    int32_t* sk_part;       // [slots][CG][8 chunks][8 quads][128 rows][4] int32
    unsigned int* sk_flag;  // [slots] flags, then the generation and the ticket
    int sk_slots;
    // Split tail (int32 results): tiles [0, dp_tiles) are whole tiles dealt round-robin to the workers; each
    // remaining tile is cut into tail_parts equal K ranges, and the tail_units = tail tiles x tail_parts pieces,
    // ordered part by part (piece u is part u / tail tiles of tail tile u % tail tiles), are dealt in equal
    // contiguous ranges to the first tail_workers workers, each worker taking its range before its whole tiles. The
    // workers busy with tail pieces at any moment read the same K range of neighbouring tiles, so they share operands
    // in L2 as a wave of whole tiles does. The tail tiles are put together in C itself: every CTA first clears its
    // share of them (the epilogue warps, while the first MMAs run) and counts itself in tail_zeroed; then every piece
    // adds its sums with TMA reductions, after that count is complete, the piece holding K block 0 of its tile adding
    // the zero-point terms and bias too. The last CTA to finish sets the count back to zero, with the stream-K
    // generation and ticket that follow sk_flag's slots.
    int tail_split;
    int tail_first;  // a worker takes its tail range before (1) or after (0) its whole tiles
    int dp_tiles;
    int tail_parts;
    int64_t tail_units;
    int tail_workers;
    unsigned int* tail_zeroed;
};

// One piece of a worker's work: K blocks [kb0, kb1) of a tile.
struct WorkItem {
    int tile, kb0, kb1;
};

struct WorkCursor {
    int64_t u, u1;  // stream-K, or the split tail: the worker's remaining units
    int tile;       // whole tiles: the next tile
};

template <bool SPLIT>
__device__ __forceinline__ void work_begin(const TcParams& p, int worker, int workers, WorkCursor& c) {
    if (!SPLIT) {
        c.u = c.u1 = 0;
    } else if (p.stream_k) {
        c.u = p.units * worker / workers;
        c.u1 = p.units * (worker + 1) / workers;
    } else if (p.tail_split && worker < p.tail_workers) {
        c.u = p.tail_units * worker / p.tail_workers;
        c.u1 = p.tail_units * (worker + 1) / p.tail_workers;
    } else {
        c.u = c.u1 = 0;
    }
    c.tile = worker;
}

// A worker of the split tail takes its range of tail units before its whole tiles (tail_first; after them
// otherwise): the reductions of its tail segments then overlap the MMAs of its whole tiles, and every worker ends on
// a whole tile whose epilogue is a plain store.
template <bool SPLIT>
__device__ __forceinline__ bool work_next(const TcParams& p, int workers, WorkCursor& c, WorkItem& w) {
    if (!SPLIT) {  // whole tiles only
        if (c.tile >= p.total_tiles) return false;
        w.tile = c.tile;
        w.kb0 = 0;
        w.kb1 = p.k_blocks;
        c.tile += workers;
        return true;
    }
    if (!p.stream_k && !p.tail_first && c.tile < p.dp_tiles) {
        w.tile = c.tile;
        w.kb0 = 0;
        w.kb1 = p.k_blocks;
        c.tile += workers;
        return true;
    }
    if (c.u < c.u1 && !p.stream_k) {
        const int tail_tiles = p.total_tiles - p.dp_tiles;
        const int part = static_cast<int>(c.u / tail_tiles);
        w.tile = p.dp_tiles + static_cast<int>(c.u - static_cast<int64_t>(part) * tail_tiles);
        w.kb0 = static_cast<int>(static_cast<int64_t>(part) * p.k_blocks / p.tail_parts);
        w.kb1 = static_cast<int>(static_cast<int64_t>(part + 1) * p.k_blocks / p.tail_parts);
        c.u += 1;
        return true;
    }
    if (c.u < c.u1) {
        const int t = static_cast<int>(c.u / p.k_blocks);
        w.kb0 = static_cast<int>(c.u - static_cast<int64_t>(t) * p.k_blocks);
        const int64_t end = static_cast<int64_t>(w.kb0) + (c.u1 - c.u);
        w.kb1 = end < p.k_blocks ? static_cast<int>(end) : p.k_blocks;
        w.tile = t;
        c.u += w.kb1 - w.kb0;
        return true;
    }
    if (p.stream_k || c.tile >= p.dp_tiles) return false;
    w.tile = c.tile;
    w.kb0 = 0;
    w.kb1 = p.k_blocks;
    c.tile += workers;
    return true;
}

constexpr int SK_SLOT_INTS = 8 * 8 * 128 * 4;  // one CTA's 128 x 256 int32 sums
constexpr uint32_t SK_SLOT_BYTES = SK_SLOT_INTS * 4;

// The raw sums of the later segment of a split tile, written where the finishing worker reads them: quad v of chunk c
// of row `row` at ((c * 8 + v) * 128 + row) * 4, so that every warp-wide 16-byte store covers 512 contiguous bytes.
__device__ __forceinline__ void sk_put(int32_t* slot, int c, int row, const uint32_t (&r)[32]) {
#pragma unroll
    for (int v = 0; v < 8; v++)
        __stcg(reinterpret_cast<int4*>(slot + ((c * 8 + v) * 128 + row) * 4),
               make_int4(int(r[4 * v]), int(r[4 * v + 1]), int(r[4 * v + 2]), int(r[4 * v + 3])));
}

// Waits (bounded, like every wait here) until another CTA of the grid has set *flag to `want`; false when the wait
// gave up or another role of this CTA raised the abort flag.
__device__ __forceinline__ bool flag_wait(const unsigned int* flag, unsigned int want, volatile int* abort) {
    const uint64_t t0 = global_timer_ns();
    while (true) {
        unsigned int v;
        asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(flag) : "memory");
        if (v == want) return true;
        if (*abort) return false;
        if (global_timer_ns() - t0 > OG_WAIT_LIMIT_NS) {
            *abort = 1;
            return false;
        }
    }
}

// Waits (bounded) until *word has reached `count`; false when the wait gave up or another role of this CTA raised the
// abort flag.
__device__ __forceinline__ bool count_wait(const unsigned int* word, unsigned int count, volatile int* abort) {
    const uint64_t t0 = global_timer_ns();
    while (true) {
        unsigned int v;
        asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(word) : "memory");
        if (v >= count) return true;
        if (*abort) return false;
        if (global_timer_ns() - t0 > OG_WAIT_LIMIT_NS) {
            *abort = 1;
            return false;
        }
        __nanosleep(64);
    }
}

// Adds the handed-over sums (already copied into this CTA's shared memory, same layout) to chunk c of a row.
__device__ __forceinline__ void sk_add(const int32_t* slot_smem, int c, int row, uint32_t (&r)[32]) {
#pragma unroll
    for (int v = 0; v < 8; v++) {
        const int4 x = *reinterpret_cast<const int4*>(slot_smem + ((c * 8 + v) * 128 + row) * 4);
        r[4 * v] += uint32_t(x.x);
        r[4 * v + 1] += uint32_t(x.y);
        r[4 * v + 2] += uint32_t(x.z);
        r[4 * v + 3] += uint32_t(x.w);
    }
}

template <int BM>
__device__ __forceinline__ void tile_coords(const TcParams& p, int tile, int& b, int& tm, int& tn) {
    const int per_batch = p.tiles_m * p.tiles_n;
    b = tile / per_batch;
    const int r = tile - b * per_batch;
    const int group_span = p.group_m * p.tiles_n;
    const int group = r / group_span;
    const int first_m = group * p.group_m;
    const int gsize = min(p.tiles_m - first_m, p.group_m);
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

// Finishes 16 consecutive int32 / float results of one row (tile columns j0..) and writes them as row `lane` of a
// 32 x 16-word box in 64-byte-swizzled shared memory: 16-byte chunk j of the row lands at chunk j ^ ((lane / 2) % 4),
// so the eight lanes of each store phase hit eight different 16-byte bank groups. The column terms are read four
// columns per 16-byte shared load.
template <int OUT>
__device__ __forceinline__ void stage_half(const ColTerms& t, const Epilogue& e, bool terms, bool za_per_row,
                                           uint32_t za, uint32_t rt, int j0, const uint32_t* r, uint8_t* box,
                                           int lane) {
    uint32_t w[16];
    if (OUT == OUT_I32 && !terms) {
#pragma unroll
        for (int q = 0; q < 16; q++) w[q] = r[q];
    } else {
#pragma unroll
        for (int v = 0; v < 4; v++) {
            const int4 zb = *reinterpret_cast<const int4*>(&t.zb[j0 + 4 * v]);
            const int4 cc = *reinterpret_cast<const int4*>(&t.c[j0 + 4 * v]);
            const uint32_t zbv[4] = {uint32_t(zb.x), uint32_t(zb.y), uint32_t(zb.z), uint32_t(zb.w)};
            const uint32_t ccv[4] = {uint32_t(cc.x), uint32_t(cc.y), uint32_t(cc.z), uint32_t(cc.w)};
            uint32_t s4[4];
#pragma unroll
            for (int u = 0; u < 4; u++) s4[u] = r[4 * v + u] + zbv[u] * rt + ccv[u];
            if (za_per_row) {
                const int4 cs = *reinterpret_cast<const int4*>(&t.csb[j0 + 4 * v]);
                s4[0] -= za * uint32_t(cs.x);
                s4[1] -= za * uint32_t(cs.y);
                s4[2] -= za * uint32_t(cs.z);
                s4[3] -= za * uint32_t(cs.w);
            }
            if constexpr (OUT == OUT_F32) {
                const float4 sc = *reinterpret_cast<const float4*>(&t.scale[j0 + 4 * v]);
                const float scv[4] = {sc.x, sc.y, sc.z, sc.w};
                float f[4];
#pragma unroll
                for (int u = 0; u < 4; u++) f[u] = __fmul_rn(__int2float_rn(static_cast<int32_t>(s4[u])), scv[u]);
                if (e.float_bias != nullptr) {
                    const float4 fb = *reinterpret_cast<const float4*>(&t.fbias[j0 + 4 * v]);
                    f[0] = __fadd_rn(f[0], fb.x);
                    f[1] = __fadd_rn(f[1], fb.y);
                    f[2] = __fadd_rn(f[2], fb.z);
                    f[3] = __fadd_rn(f[3], fb.w);
                }
#pragma unroll
                for (int u = 0; u < 4; u++) w[4 * v + u] = __float_as_uint(f[u]);
            } else {
#pragma unroll
                for (int u = 0; u < 4; u++) w[4 * v + u] = s4[u];
            }
        }
    }
    const uint32_t row = smem_u32(box) + lane * 64;
    const uint32_t sw = (lane >> 1) & 3;
#pragma unroll
    for (int j = 0; j < 4; j++) {
        const uint32_t addr = row + ((j ^ sw) << 4);
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

template <int CG, bool B_MN, int OUT, bool SPLIT>
__device__ __forceinline__ void gemm_tc_body(const CUtensorMap& tmap_a, const CUtensorMap& tmap_b,
                                             const CUtensorMap& tmap_c, const TcParams& p, uint32_t idesc) {
    using C = tc::Cfg<CG>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sA = smem;
    uint8_t* sB = smem + C::STAGES * C::A_BYTES;
    uint8_t* staging = sB + C::STAGES * C::B_BYTES;  // 1024-byte aligned store boxes of the epilogue warps (2 each)
    uint64_t* bars = reinterpret_cast<uint64_t*>(staging + C::STAGING_BYTES);
    uint64_t* full = bars;
    uint64_t* empty = bars + C::STAGES;
    uint64_t* tfull = bars + 2 * C::STAGES;
    uint64_t* tempty = bars + 2 * C::STAGES + tc::NUM_ACC;
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + 2 * C::STAGES + 2 * tc::NUM_ACC);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
    volatile int* epi_go = reinterpret_cast<volatile int*>(tmem_holder + 2);  // [2]: per tile parity
    volatile unsigned int* sk_gen = reinterpret_cast<volatile unsigned int*>(tmem_holder + 4);
    uint64_t* sk_bar = bars + 24;  // byte 192 of the barrier block: the hand-over copy

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t rank = CG == 2 ? cluster_ctarank() : 0;  // CTA of the pair: rank 0 issues the MMAs
    const bool leader = rank == 0;
    const int worker = CG == 2 ? static_cast<int>(blockIdx.x >> 1) : static_cast<int>(blockIdx.x);
    const int workers = CG == 2 ? static_cast<int>(gridDim.x >> 1) : static_cast<int>(gridDim.x);
    const bool stream_k = SPLIT && p.stream_k;
    const bool tail_split = SPLIT && p.tail_split;

    pdl_trigger();
    if (threadIdx.x == 0) {
        for (int s = 0; s < C::STAGES; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int a = 0; a < tc::NUM_ACC; a++) {
            mbar_init(&tfull[a], 1);
            mbar_init(&tempty[a], tc::EPI_WARPS * CG);  // one arrival per epilogue warp of every CTA of the pair
        }
        mbar_init(sk_bar, 1);
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
    pdl_wait();  // the preceding grid is done: its outputs are readable and its TMEM is free
    // This launch's stream-K generation: flags set to it belong to this launch.
    if (threadIdx.x == 0) *sk_gen = (stream_k || tail_split) ? __ldcg(p.sk_flag + p.sk_slots) + 1u : 0u;
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
        WorkCursor cur;
        work_begin<SPLIT>(p, worker, workers, cur);
        WorkItem wi;
        while (work_next<SPLIT>(p, workers, cur, wi)) {
            int b, tm, tn;
            tile_coords<C::BM>(p, wi.tile, b, tm, tn);
            const int ba = p.a_batched ? b : 0;
            const int bb = p.b_batched ? b : 0;
            const int row0 = tm * C::BM + static_cast<int>(rank) * 128;
            const int col0 = tn * tc::BN + static_cast<int>(rank) * C::B_COLS;
            // With one CTA, a second 128-column box wholly past N is skipped; a pair always loads full boxes
            // (TMA fills what lies outside the tensor with zeros) so the leader knows the byte count.
            const bool second_half = CG == 1 && B_MN && (col0 + 128 < p.n);
            const uint32_t bytes = CG == 2 ? 2u * (C::A_BYTES + C::B_BYTES)
                                           : C::A_BYTES + (B_MN ? (second_half ? 2 : 1) * C::B_BOX : C::B_BYTES);
            for (int kb = wi.kb0; kb < wi.kb1; kb++, it++) {
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
            WorkCursor cur;
            work_begin<SPLIT>(p, worker, workers, cur);
            WorkItem wi;
            for (int lt = 0; work_next<SPLIT>(p, workers, cur, wi); lt++) {
                const int acc = lt & 1;
                const uint32_t aph = (lt >> 1) & 1;
                if (!mbar_wait(&tempty[acc], aph ^ 1, abort_flag)) goto done;
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + acc * tc::BN;
                for (int kb = wi.kb0; kb < wi.kb1; kb++, it++) {
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
                            const uint32_t accum = (kb != wi.kb0 || kk != 0) ? 1u : 0u;
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
        // Epilogue: warp w reads TMEM lanes 32*(w%4) .. +31, i.e. rows 32*(w%4) + lane of this CTA's 128 rows; warps
        // 2-5 take the tile's first 128 columns (chunks 0-3 of 32), warps 6-9 the other 128.
        const int q = warp & 3;
        const int ew = warp - 2;
        const int c_first = (ew >> 2) * (tc::BN / 64), c_end = c_first + tc::BN / 64;
        const uint32_t tempty_leader = CG == 2 ? mapa_shared(smem_u32(&tempty[0]), 0) : 0;
        const Epilogue& e = p.epi;
        ColTerms& terms_smem = *reinterpret_cast<ColTerms*>(reinterpret_cast<uint8_t*>(bars) + 256);
        // Column terms are needed unless the result is the raw int32 sum.
        const bool terms = OUT != OUT_I32 || e.za != nullptr || e.zb != nullptr || e.int_bias != nullptr;
        const bool za_per_row = e.za != nullptr && e.za_vector;
        if (tail_split) {
            // Clear this CTA's share of the tail tiles (rows of 256 columns, dealt to the epilogue warps of the grid in
            // turn) while the first MMAs run, then count the CTA in the launch's tally. C's rows start on 16-byte
            // boundaries and N is a multiple of 4 (the TMA-store condition), so whole 16-byte stores stay inside C.
            const int64_t rows_total = static_cast<int64_t>(p.total_tiles - p.dp_tiles) * C::BM;
            for (int64_t r = static_cast<int64_t>(blockIdx.x) * tc::EPI_WARPS + ew; r < rows_total;
                 r += static_cast<int64_t>(gridDim.x) * tc::EPI_WARPS) {
                int zb_, ztm, ztn;
                tile_coords<C::BM>(p, p.dp_tiles + static_cast<int>(r / C::BM), zb_, ztm, ztn);
                const int zm = ztm * C::BM + static_cast<int>(r % C::BM);
                if (zm >= p.m) continue;
                uint32_t* zrow = static_cast<uint32_t*>(e.c) + zb_ * e.batch_stride_c + static_cast<int64_t>(zm) * e.ldc;
#pragma unroll
                for (int h = 0; h < 2; h++) {
                    const int zn = ztn * tc::BN + h * 128 + lane * 4;
                    if (zn < p.n) *reinterpret_cast<uint4*>(zrow + zn) = make_uint4(0u, 0u, 0u, 0u);
                }
            }
            __threadfence();
            fence_proxy_async_global();
            asm volatile("bar.sync 1, %0;" ::"n"(tc::EPI_THREADS) : "memory");
            if (threadIdx.x == 64) atomicAdd(p.tail_zeroed, 1u);
        }
        bool tail_ready = false;  // thread 64: the whole grid has cleared the tail
        WorkCursor cur;
        work_begin<SPLIT>(p, worker, workers, cur);
        WorkItem wi;
        for (int lt = 0; work_next<SPLIT>(p, workers, cur, wi); lt++) {
            int b, tm, tn;
            tile_coords<C::BM>(p, wi.tile, b, tm, tn);
            const int acc = lt & 1;
            const uint32_t aph = (lt >> 1) & 1;
            // Stream-K: the K-block-0 segment of a split tile (the end of this worker's range) also waits for the
            // next worker's sums of the later segment. Split tail: a segment of a tail tile adds to C, once every CTA
            // has cleared its share of the tail. One thread does every wait and publishes the outcome, so the
            // epilogue warps always leave or continue together (the named barriers below cannot time out).
            const bool sk_wait = stream_k && wi.kb0 == 0 && wi.kb1 < p.k_blocks;
            const bool tail_item = tail_split && wi.tile >= p.dp_tiles;
            const int sk_slot = (worker + 1) * CG + static_cast<int>(rank);
            if (threadIdx.x == 64) {
                bool ok = mbar_wait(&tfull[acc], aph, abort_flag);
                if (ok && tail_item && !tail_ready) {
                    ok = count_wait(p.tail_zeroed, gridDim.x, abort_flag);
                    tail_ready = ok;
                }
                if (ok && sk_wait) {
                    // This is the worker's last item: its MMAs are complete, so the operand ring is idle and takes
                    // the handed-over sums in one bulk copy.
                    ok = flag_wait(p.sk_flag + sk_slot, *sk_gen, abort_flag);
                    if (ok) {
                        mbar_arrive_expect_tx(sk_bar, SK_SLOT_BYTES);
                        bulk_load(sA, p.sk_part + static_cast<int64_t>(sk_slot) * SK_SLOT_INTS, SK_SLOT_BYTES, sk_bar);
                        ok = mbar_wait(sk_bar, 0, abort_flag);
                    }
                }
                epi_go[lt & 1] = ok ? 1 : 0;
            }
            asm volatile("bar.sync 1, %0;" ::"n"(tc::EPI_THREADS) : "memory");
            if (!epi_go[lt & 1]) goto done;
            const bool reduce = tail_item;
            if (reduce && lane == 0) fence_proxy_async_global();  // the reductions follow the cleared tail
            tc_fence_after();
            const int row_in_cta = q * 32 + lane;
            const uint32_t t_row = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * tc::BN;
            if (stream_k && wi.kb0 > 0) {
                // The later segment of a split tile (the start of this worker's range): hand its raw sums to the
                // worker that holds K block 0 (the previous one), then flag them.
                int32_t* slot = p.sk_part + static_cast<int64_t>(worker * CG + static_cast<int>(rank)) * SK_SLOT_INTS;
#pragma unroll 1
                for (int c = c_first; c < c_end; c++) {
                    uint32_t r[32];
                    tmem_ld_32x32b_x32(t_row + c * 32, r);
                    tmem_ld_wait();
                    sk_put(slot, c, row_in_cta, r);
                }
                __threadfence();
                asm volatile("bar.sync 1, %0;" ::"n"(tc::EPI_THREADS) : "memory");
                if (threadIdx.x == 64) {
                    unsigned int* flag = p.sk_flag + worker * CG + static_cast<int>(rank);
                    asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(flag), "r"(*sk_gen) : "memory");
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) {
                    if constexpr (CG == 2)
                        mbar_arrive_cluster(tempty_leader + acc * sizeof(uint64_t));
                    else
                        mbar_arrive(&tempty[acc]);
                }
                continue;
            }
            const int32_t* sk_in = sk_wait ? reinterpret_cast<const int32_t*>(sA) : nullptr;
            // The zero-point terms and the bias enter C once: with the K-block-0 piece of a tail tile.
            const bool with_terms = terms && (!reduce || wi.kb0 == 0);
            if (with_terms) {  // every warp has left the previous tile (the barrier above), so its terms are free
                fill_col_terms(terms_smem, e, b, tn * tc::BN, threadIdx.x - 64, tc::EPI_THREADS);
                asm volatile("bar.sync 1, %0;" ::"n"(tc::EPI_THREADS) : "memory");
            }
            const int m = tm * C::BM + static_cast<int>(rank) * 128 + q * 32 + lane;
            const bool row_ok = m < p.m;
            uint32_t za = 0, rt = 0;  // zero point of A for this row, and K * za - rowsumA
            if (row_ok && terms) {
                za = static_cast<uint32_t>(zp_value(e.za, e.za_vector, e.za_signed, m));
                const uint32_t rsa = e.row_sum_a ? row_sum_of(e, b, m) : 0u;
                rt = static_cast<uint32_t>(p.k) * za - rsa;
            }
            if (tma_store) {
                // Each 32 x 32 chunk leaves as two TMA stores of 32 x 16 words (64-byte row segments) through this
                // warp's boxes in turn (with two boxes, staging one half never waits for the store just issued);
                // rows past M and columns past N are clipped by the tensor map.
                const int box_row = tm * C::BM + static_cast<int>(rank) * 128 + q * 32;
#pragma unroll 1
                for (int c = c_first; c < c_end; c++) {
                    const int n0 = tn * tc::BN + c * 32;
                    if (n0 >= p.n || box_row >= p.m) break;  // boxes start inside C
                    uint32_t r[32];
                    tmem_ld_32x32b_x32(t_row + c * 32, r);
                    tmem_ld_wait();
                    if (sk_in != nullptr) sk_add(sk_in, c, row_in_cta, r);
#pragma unroll
                    for (int h = 0; h < 2; h++) {
                        if (n0 + 16 * h >= p.n) break;
                        // Alternate boxes: the box about to be written was last stored BOXES boxes ago.
                        uint8_t* box = staging + (ew * C::BOXES + h % C::BOXES) * C::BOX_BYTES;
                        if (lane == 0) bulk_wait_group_read<C::BOXES - 1>();
                        __syncwarp();
                        stage_half<OUT>(terms_smem, e, with_terms, za_per_row, za, rt, c * 32 + 16 * h, r + 16 * h,
                                        box, lane);
                        fence_proxy_async_smem();
                        __syncwarp();
                        if (lane == 0) {
                            if (reduce)
                                tma_reduce_add_3d(&tmap_c, box, n0 + 16 * h, box_row, b);
                            else
                                tma_store_3d(&tmap_c, box, n0 + 16 * h, box_row, b);
                            bulk_commit_group();
                        }
                    }
                }
            } else {
#pragma unroll 1
                for (int c = c_first; c < c_end; c++) {
                    const int n0 = tn * tc::BN + c * 32;
                    if (n0 >= p.n) break;
                    uint32_t r[32];
                    tmem_ld_32x32b_x32(t_row + c * 32, r);
                    tmem_ld_wait();
                    if (sk_in != nullptr) sk_add(sk_in, c, row_in_cta, r);
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
    // The stores have read their boxes before shared memory goes (their global writes complete with the grid).
    if (tma_store && warp >= 2 && lane == 0) bulk_wait_group_read<0>();
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
    if ((stream_k || tail_split) && threadIdx.x == 0) {
        // The last CTA to finish advances the generation (every CTA read it when it started) and resets the ticket.
        unsigned int* gen = p.sk_flag + p.sk_slots;
        __threadfence();
        if (atomicAdd(gen + 1, 1u) == gridDim.x - 1) {
            atomicExch(gen + 1, 0u);
            if (tail_split) atomicExch(p.tail_zeroed, 0u);  // every CTA has left its waits on the count
            atomicAdd(gen, 1u);
        }
    }
}

template <bool B_MN, int OUT, bool SPLIT>
__global__ void __launch_bounds__(tc::THREADS, 1)
    int8_gemm_tc_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                        const __grid_constant__ CUtensorMap tmap_c, const TcParams p, uint32_t idesc) {
    gemm_tc_body<1, B_MN, OUT, SPLIT>(tmap_a, tmap_b, tmap_c, p, idesc);
}

template <bool B_MN, int OUT, bool SPLIT>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(tc::THREADS, 1)
    int8_gemm_tc2_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                         const __grid_constant__ CUtensorMap tmap_c, const TcParams p, uint32_t idesc) {
    gemm_tc_body<2, B_MN, OUT, SPLIT>(tmap_a, tmap_b, tmap_c, p, idesc);
}

// ---- host side ---------------------------------------------------------------------------------------------------

bool pdl_enabled() {
    static const bool on = [] {
        const char* v = std::getenv("ONEGPU_PDL");
        return v == nullptr || std::strcmp(v, "0") != 0;
    }();
    return on;
}

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

// The output C as a 3-D tensor of 4-byte words (columns innermost) stored in 32-row x 16-word boxes from 64-byte-swizzled
// shared memory.
static bool make_store_map(CUtensorMap* map, void* base, uint64_t n, uint64_t m, uint64_t batch, uint64_t row_bytes,
                           uint64_t batch_bytes) {
    auto fn = encode_fn();
    if (fn == nullptr) return false;
    cuuint64_t dims[3] = {n, m, batch};
    cuuint64_t strides[2] = {row_bytes, batch_bytes};
    cuuint32_t box[3] = {16, 32, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_INT32, 3, base, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
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
static cudaError_t configure(K kern, int smem, std::atomic<uint64_t>& configured) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    const uint64_t bit = uint64_t(1) << (dev & 63);
    if (!(configured.load() & bit)) {
        e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return e;
        configured.fetch_or(bit);
    }
    return cudaSuccess;
}

// Binds the kernel and its arguments; the returned function only sets the shared-memory limit (first time per
// device) and launches.
template <int CG, bool B_MN, int OUT, bool SPLIT>
static LaunchFn bind_tc_t(const GemmLaunch& L, const TcParams& p, const CUtensorMap& ma, const CUtensorMap& mb,
                          const CUtensorMap& mc, int grid) {
    using C = tc::Cfg<CG>;
    const uint32_t idesc = idesc_i8(L.a_signed, L.b_signed, false, B_MN, C::BM, tc::BN);
    return [=](cudaStream_t stream) -> cudaError_t {
        static std::atomic<uint64_t> configured{0};  // devices whose attribute is set
        if constexpr (CG == 2) {
            auto kern = int8_gemm_tc2_kernel<B_MN, OUT, SPLIT>;
            cudaError_t e = configure(kern, C::SMEM_BYTES, configured);
            if (e != cudaSuccess) return e;
            return launch_pdl(kern, dim3(grid), dim3(tc::THREADS), C::SMEM_BYTES, stream, ma, mb, mc, p, idesc);
        } else {
            auto kern = int8_gemm_tc_kernel<B_MN, OUT, SPLIT>;
            cudaError_t e = configure(kern, C::SMEM_BYTES, configured);
            if (e != cudaSuccess) return e;
            return launch_pdl(kern, dim3(grid), dim3(tc::THREADS), C::SMEM_BYTES, stream, ma, mb, mc, p, idesc);
        }
    };
}

// The kernel without the stream-K and split-tail paths when neither is in use (whole tiles only).
template <int CG, bool B_MN, int OUT>
static LaunchFn bind_tc_s(const GemmLaunch& L, const TcParams& p, const CUtensorMap& ma, const CUtensorMap& mb,
                          const CUtensorMap& mc, int grid) {
    return (p.stream_k || p.tail_split) ? bind_tc_t<CG, B_MN, OUT, true>(L, p, ma, mb, mc, grid)
                                        : bind_tc_t<CG, B_MN, OUT, false>(L, p, ma, mb, mc, grid);
}

// The split tail of an int32 product: the tiles beyond the last full wave of whole tiles are cut into P equal K
// ranges and the pieces dealt, part by part, over the workers. A worker then spends ceil(tail tiles x P / workers)
// pieces of 1/P tile on the tail instead of one whole tile; P (2..8, each piece at least TAIL_MIN_BLOCKS K blocks)
// minimises that fraction, and the tail is split only when it is at most TAIL_MAX_FRACTION of a tile. Every piece
// costs an epilogue and a TMA reduction of a whole tile's sums into C (L2 read-modify-write traffic that competes
// with the operand loads), so a split must at least halve the tail. Measured on B200 with zero points (the byte-sums pass included):
// 8192 x 2048 x 8192 111.8 us in halves against 119.8 us whole, 4096^3 68.6 against 70.7 us, while quarters of
// 8192 x 1024 x 8192 (54 tail tiles, three quarters per pair) took 80.9 us against 74.9 us whole and thirds of the
// batched 8 x 2048 x 12288 x 4096 558 against 547 us. Without zero points the same shard took 63.4 us in quarters and
// 77.8 us in eighths against 55.2 us whole: each piece's reduction of a whole tile into C takes longer than its share
// of the MMAs. The cut tiles are put together in C with TMA reductions, so C's rows must allow TMA stores.
constexpr int TAIL_MIN_BLOCKS = 8;
constexpr double TAIL_MAX_FRACTION = 0.5;

struct TailPlan {
    int dp_tiles = 0, workers = 0, parts = 0;
    int64_t units = 0;
};

static TailPlan tail_plan(int64_t tiles, int64_t k_blocks, int64_t workers) {
    TailPlan t;
    t.dp_tiles = static_cast<int>(tiles);
    const int64_t rem = tiles % workers;
    if (rem == 0) return t;
    double best = 2.0;
    for (int parts = 2; parts <= 8 && k_blocks / parts >= TAIL_MIN_BLOCKS; parts++) {
        const int64_t units = rem * parts;
        const double fraction = static_cast<double>((units + workers - 1) / workers) / parts;
        if (fraction <= TAIL_MAX_FRACTION + 1e-9 && fraction < best - 1e-9) {
            best = fraction;
            t.parts = parts;
            t.units = units;
        }
    }
    if (t.parts == 0) return t;
    t.dp_tiles = static_cast<int>(tiles - rem);
    t.workers = static_cast<int>(std::min<int64_t>(workers, t.units));
    return t;
}

static bool tail_eligible(const GemmLaunch& L) {
    if (L.stream_k != 0 || L.epi.out_kind != OUT_I32) return false;
    const bool c_aligned = (reinterpret_cast<uintptr_t>(L.epi.c) & 15) == 0 && (L.epi.ldc & 3) == 0 &&
                           (L.batch == 1 || (L.epi.batch_stride_c & 3) == 0);
    return c_aligned;
}

// Stream-K runs only when asked for (mode 2) and when every worker gets at least one tile's worth of K blocks, so
// that a tile is split between two workers at most. It is not chosen by size: measured on B200 the int8 product's
// K-block rate is capped by operand delivery to the SMs rather than by how many SM pairs are busy, so the partial last
// wave of the data-parallel schedule costs less than the hand-over does (4096^3: 53.2 vs 57.6 us; 8192 x 1024 x 8192:
// 52.0 vs 60.9 us).
static bool sk_worthwhile(int64_t tiles, int64_t workers, int mode) {
    if (mode != 2 || tiles < workers) return false;
    return tiles % workers != 0;
}

int tc_split_mode(const GemmLaunch& L) {
    const int cg = tc_cta_group(L);
    const int64_t bm = 128 * cg;
    const int64_t tiles = ((L.m + bm - 1) / bm) * ((L.n + tc::BN - 1) / tc::BN) * int64_t(L.batch);
    if (sk_worthwhile(tiles, L.num_sms / cg, L.stream_k)) return 2;
    return tail_eligible(L) && tail_plan(tiles, (L.k + tc::BK - 1) / tc::BK, L.num_sms / cg).workers > 0 ? 1 : 0;
}

bool sk_wanted(const GemmLaunch& L) { return tc_split_mode(L) != 0; }

// Hand-over slots: one per CTA of the grid plus one pair (slot (worker + 1) * CG + rank is the largest read).
static int64_t sk_slots(int num_sms) { return int64_t(num_sms) + 2; }

// Split tail: the count of CTAs that have cleared their share of the tail, after the generation and the ticket.
constexpr int64_t TAIL_WORDS = 1;

int64_t sk_bytes_needed(int num_sms) {
    return sk_slots(num_sms) * (SK_SLOT_INTS * int64_t(sizeof(int32_t)) + int64_t(sizeof(unsigned int))) +
           2 * int64_t(sizeof(unsigned int)) +  // the generation and the ticket
           TAIL_WORDS * int64_t(sizeof(unsigned int));
}

void sk_bind(GemmLaunch& L, void* buffer, int64_t bytes) {
    if (buffer == nullptr || bytes < sk_bytes_needed(L.num_sms)) {
        L.sk_part = nullptr;
        L.sk_flag = nullptr;
        L.sk_bytes = 0;
        return;
    }
    L.sk_part = static_cast<int32_t*>(buffer);
    L.sk_flag = reinterpret_cast<unsigned int*>(static_cast<uint8_t*>(buffer) +
                                                sk_slots(L.num_sms) * SK_SLOT_INTS * int64_t(sizeof(int32_t)));
    L.sk_bytes = bytes;
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
    p.group_m = p.tiles_m >= 32 ? tc::GROUP_M_TALL : tc::GROUP_M;
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
    int grid = static_cast<int>((total < workers ? total : workers) * CG);
    // Stream-K when it pays (sk_worthwhile) and the caller gave the hand-over buffers.
    p.units = total * p.k_blocks;
    p.sk_part = L.sk_part;
    p.sk_flag = L.sk_flag;
    p.sk_slots = static_cast<int>(sk_slots(L.num_sms));
    const bool buffers = L.sk_part != nullptr && sk_bytes_needed(L.num_sms) <= L.sk_bytes;
    p.stream_k = buffers && sk_worthwhile(total, workers, L.stream_k);
    // Otherwise the split tail, for int32 results stored through TMA.
    p.tail_split = 0;
    p.tail_first = 1;
    p.dp_tiles = static_cast<int>(total);
    p.tail_parts = 0;
    p.tail_units = 0;
    p.tail_workers = 0;
    p.tail_zeroed = nullptr;
    if (!p.stream_k && buffers && p.tma_store && tail_eligible(L)) {
        const TailPlan t = tail_plan(total, p.k_blocks, workers);
        if (t.workers > 0) {
            p.tail_split = 1;
            p.dp_tiles = t.dp_tiles;
            p.tail_parts = t.parts;
            p.tail_units = t.units;
            p.tail_workers = t.workers;
            p.tail_zeroed = L.sk_flag + p.sk_slots + 2;
            grid = static_cast<int>(std::max<int64_t>(grid / CG, t.workers) * CG);
        }
    }
    const bool bmn = !L.trans_b;
    switch (L.epi.out_kind) {
        case OUT_I32: return bmn ? bind_tc_s<CG, true, OUT_I32>(L, p, ma, mb, mc, grid)
                                 : bind_tc_s<CG, false, OUT_I32>(L, p, ma, mb, mc, grid);
        case OUT_F32: return bmn ? bind_tc_s<CG, true, OUT_F32>(L, p, ma, mb, mc, grid)
                                 : bind_tc_s<CG, false, OUT_F32>(L, p, ma, mb, mc, grid);
        case OUT_U8: return bmn ? bind_tc_s<CG, true, OUT_U8>(L, p, ma, mb, mc, grid)
                                : bind_tc_s<CG, false, OUT_U8>(L, p, ma, mb, mc, grid);
        default: return bmn ? bind_tc_s<CG, true, OUT_S8>(L, p, ma, mb, mc, grid)
                            : bind_tc_s<CG, false, OUT_S8>(L, p, ma, mb, mc, grid);
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
