// The int8 product for few rows (M <= 16 per batch: decode steps), bandwidth-bound on B.
//
// The roles of the operands are swapped so that B streams through the tensor cores exactly once: the MMA computes
// D[n, j] = sum_k B[k, n] * A[j, k] with tcgen05.mma.kind::i8, M = 128 columns of B per CTA, N = 16 rows of A (TMA
// zero-fills the rows past M). When A has a zero point, a second N = 16 MMA multiplies the same B tile with a block
// of ones kept once in shared memory, so TMEM columns 16..31 hold the column sums of B over K - no separate pass over
// B (235 MB at the decode config) is made for them.
//
// One CTA per 128 columns (and batch), the whole of K per CTA, 6 stages of 16 KB of B + 2 KB of A; two CTAs fit on
// an SM, so every tile of the decode config (224) is resident at once, all CTAs walking K together (so the rows of B
// they read at any moment are the same few DRAM pages). There 76 SMs hold two tiles and 72 one, which sets the time.
// Warp 0 loads (TMA, no multicast), warp 1 issues the MMAs into a 32-column TMEM accumulator, warps 2-5 compute the
// row sums of A while B streams (the zero point of B needs them), then drain TMEM: lane = column, 16 results per
// lane, stores coalesced along N. Products with too few column tiles to occupy the SMs split K evenly instead
// (int8_gemm_rows_stream_kernel below).
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <atomic>

#include "og_gemm.h"
#include "og_kernels.cuh"
#include "og_ptx.cuh"

namespace og {

namespace rows {
constexpr int BN = 128;          // columns of B (rows of the MMA) per CTA
constexpr int BK = 128;
constexpr int MAXM = 16;         // rows of A = N of the MMA
// Stages of B in flight per CTA. Measured on B200, the decode config runs faster with 4 than with 6 (45.1 against
// 48.0 us at 16 x 28672 x 8192): fewer rows of B open at once keep the CTAs' DRAM reads closer together.
constexpr int STAGES = 4;
constexpr int SUMS_STAGES = 6;  // the byte-sums kernel's ring
constexpr int B_BYTES = BN * BK;          // 16 KB
constexpr int A_BYTES = MAXM * BK;        // 2 KB
constexpr int ONES_BYTES = MAXM * BK;     // 16 rows of ones, shared by every stage
constexpr int THREADS = 192;
// Four accumulators, one per K = 32 step of a K block: consecutive MMAs of a block write different accumulators, so
// they do not wait for one another (an N = 16 MMA is short next to the latency of the accumulation it depends on; a
// single accumulator held one CTA to ~29 GB/s of B however many stages were in flight). The epilogue adds them up.
constexpr int ACCS = 4;
constexpr int ACC_COLS = 32;                   // per accumulator: columns 0..15 dot products, 16..31 column sums of B
constexpr int TMEM_COLS = ACCS * ACC_COLS;     // 128
constexpr int SMEM_BYTES = STAGES * (B_BYTES + A_BYTES) + ONES_BYTES + 1024 + 256;
}  // namespace rows

constexpr int SUMS_SMEM_BYTES = rows::SUMS_STAGES * rows::B_BYTES + rows::ONES_BYTES + 1024 + 256;
// The split kernel holds two 128-column TMEM accumulators per CTA: at most two CTAs per SM (4 x 256 = 512 columns),
// which a request of more than a third of an SM's shared memory guarantees.
constexpr int STREAM_SMEM_BYTES = rows::SMEM_BYTES > 80 * 1024 ? rows::SMEM_BYTES : 80 * 1024;

struct RowsParams {
    int m, n, k;
    int k_blocks;
    int a_batched, b_batched;
    int64_t lda, stride_a;  // for the row sums of A, read from global memory
    const uint8_t* a;
    Epilogue epi;
    int* error_flag;
    // Sums-only mode: no product; the column sums of B over K go to sums_out[b * sums_stride + n].
    int32_t* sums_out;
    int64_t sums_stride;
    int64_t sums_split_stride;  // between the partial sums of consecutive K splits (blockIdx.z)
    int k_blocks_total;         // K blocks of the whole product; p.k_blocks is the share of one split
    // Stream mode (int8_gemm_rows_stream_kernel): the (column tile, K block) units of all batches, split evenly.
    int64_t units;
    int tiles;                  // column tiles of one batch
    int32_t* split_part;        // [workers][2][PART_INTS]: a worker's first and last segments, when partial
    unsigned int* split_ticket; // [batch * tiles]: K blocks of the tile finished so far (back to 0 when complete)
};

// One partial record: the 16 x 128 dot products, the 128 column sums of B, the 16 row sums of A of a K range.
constexpr int PART_INTS = 17 * rows::BN + rows::MAXM;

// The 32 columns of this thread's TMEM lane summed over the accumulators (addition modulo 2^32). A product of
// fewer than ACCS K steps leaves the later accumulators unwritten, so only those written are read (every K block
// holds ACCS steps, so any K block count writes all of them).
__device__ __forceinline__ void tmem_ld_sum(uint32_t taddr, int k_blocks, uint32_t (&r)[32]) {
    tmem_ld_32x32b_x32(taddr, r);
    tmem_ld_wait();
    if (k_blocks < 1) return;
#pragma unroll 1
    for (int a = 1; a < rows::ACCS; a++) {
        uint32_t t[32];
        tmem_ld_32x32b_x32(taddr + a * rows::ACC_COLS, t);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 32; i++) r[i] += t[i];
    }
}

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
    uint8_t* sX = smem + rows::STAGES * rows::B_BYTES;    // [STAGES][16 rows of A x 128 k]
    uint8_t* sOnes = sX + rows::STAGES * rows::A_BYTES;   // [16 rows x 128 k] of ones
    uint64_t* bars = reinterpret_cast<uint64_t*>(sOnes + rows::ONES_BYTES);
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
    const int kb_begin = blockIdx.z * p.k_blocks;  // K split of this CTA (one split outside the sums-only mode)
    const int kb_count = min(p.k_blocks, p.k_blocks_total - kb_begin);
    const bool sums_only = p.sums_out != nullptr;
    const bool need_col_sums = sums_only || p.epi.za != nullptr;  // za * colsum(B)
    pdl_trigger();

    // The block of ones (any swizzle of all-ones bytes is all ones).
    for (int i = threadIdx.x; i < rows::ONES_BYTES / 16; i += blockDim.x)
        reinterpret_cast<uint4*>(sOnes)[i] = make_uint4(0x01010101u, 0x01010101u, 0x01010101u, 0x01010101u);
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
    pdl_wait();  // the preceding grid is done: its outputs are readable and its TMEM is free
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
        for (int kb = 0; kb < kb_count; kb++) {
            const int s = kb % rows::STAGES;
            const uint32_t ph = (kb / rows::STAGES) & 1;
            const int kc = (kb_begin + kb) * rows::BK;
            if (!mbar_wait(&empty[s], ph ^ 1, abort_flag)) goto done;
            if (lane == 0) {
                mbar_arrive_expect_tx(&full[s], rows::B_BYTES + (sums_only ? 0 : rows::A_BYTES));
                if constexpr (B_KMAJOR)
                    tma_load_3d(sB + s * rows::B_BYTES, &tmap_b, &full[s], kc, tile * rows::BN, bb);
                else
                    tma_load_3d(sB + s * rows::B_BYTES, &tmap_b, &full[s], tile * rows::BN, kc, bb);
                if (!sums_only) tma_load_3d(sX + s * rows::A_BYTES, &tmap_a, &full[s], kc, 0, ba);
            }
            __syncwarp();
        }
    } else if (warp == 1) {
        for (int kb = 0; kb < kb_count; kb++) {
            const int s = kb % rows::STAGES;
            const uint32_t ph = (kb / rows::STAGES) & 1;
            if (!mbar_wait(&full[s], ph, abort_flag)) goto done;
            tc_fence_after();
            if (lane == 0) {
                const uint32_t b_addr = smem_u32(sB + s * rows::B_BYTES);
                const uint32_t x_addr = smem_u32(sX + s * rows::A_BYTES);
                const uint32_t o_addr = smem_u32(sOnes);
#pragma unroll
                for (int kk = 0; kk < rows::BK / 32; kk++) {
                    const uint64_t adesc = B_KMAJOR ? smem_desc_sw128(b_addr + kk * 32, 16, 1024)
                                                    : smem_desc_sw128(b_addr + kk * 32 * 128, rows::B_BYTES, 1024);
                    const uint32_t acc = kb != 0 ? 1u : 0u;
                    const uint32_t d = tmem_base + kk * rows::ACC_COLS;
                    if (!sums_only) mma_i8(d, adesc, smem_desc_sw128(x_addr + kk * 32, 16, 1024), idesc, acc);
                    if (need_col_sums)
                        mma_i8(d + rows::MAXM, adesc, smem_desc_sw128(o_addr + kk * 32, 16, 1024), idesc, acc);
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
        // Row sums of A over K while B streams (needed for the zero point of B). Eight consecutive threads own a row
        // (16 rows x 8 = the 128 epilogue threads) and read it in 16-byte chunks, 16 loads in flight per thread.
        if (!sums_only && e.zb != nullptr) {
            const int t = threadIdx.x - 64;  // 0..127
            const int r = t >> 3, part = t & 7;
            int32_t sum = 0;
            if (r < p.m) {
                const uint8_t* row = p.a + ba * p.stride_a + r * p.lda;
                const int chunks = p.k >> 4;
                constexpr int U = 16;
                for (int c0 = part; c0 < chunks; c0 += 8 * U) {
                    uint4 w[U];
#pragma unroll
                    for (int u = 0; u < U; u++) {
                        const int c = c0 + 8 * u;
                        w[u] = c < chunks ? __ldg(reinterpret_cast<const uint4*>(row) + c) : make_uint4(0, 0, 0, 0);
                    }
#pragma unroll
                    for (int u = 0; u < U; u++) {
                        if (e.za_signed) {
                            sum = __dp4a(static_cast<int>(w[u].x), 0x01010101, sum);
                            sum = __dp4a(static_cast<int>(w[u].y), 0x01010101, sum);
                            sum = __dp4a(static_cast<int>(w[u].z), 0x01010101, sum);
                            sum = __dp4a(static_cast<int>(w[u].w), 0x01010101, sum);
                        } else {
                            unsigned s = static_cast<unsigned>(sum);
                            s = __dp4a(w[u].x, 0x01010101u, s);
                            s = __dp4a(w[u].y, 0x01010101u, s);
                            s = __dp4a(w[u].z, 0x01010101u, s);
                            s = __dp4a(w[u].w, 0x01010101u, s);
                            sum = static_cast<int32_t>(s);
                        }
                    }
                }
                for (int kk = (chunks << 4) + part; kk < p.k; kk += 8) {  // the last k % 16 bytes
                    const uint8_t v = __ldg(row + kk);
                    sum += e.za_signed ? static_cast<int32_t>(static_cast<int8_t>(v)) : v;
                }
            }
            sum += __shfl_xor_sync(0xFFFFFFFFu, sum, 1);
            sum += __shfl_xor_sync(0xFFFFFFFFu, sum, 2);
            sum += __shfl_xor_sync(0xFFFFFFFFu, sum, 4);
            if (part == 0) row_sum[r] = sum;
        }
        asm volatile("bar.sync 1, 128;" ::: "memory");  // the four epilogue warps
        if (!mbar_wait(tfull, 0, abort_flag)) goto done;
        tc_fence_after();
        uint32_t r[32];
        tmem_ld_sum(tmem_base + (static_cast<uint32_t>(q * 32) << 16), kb_count, r);
        const int n = tile * rows::BN + q * 32 + lane;
        if (sums_only) {
            if (n < p.n) p.sums_out[blockIdx.z * p.sums_split_stride + b * p.sums_stride + n] = static_cast<int32_t>(r[16]);
        } else if (n < p.n) {
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

// ---- few rows, K split evenly across the SMs ------------------------------------------------------------------------
//
// When there are too few column tiles to occupy the SMs (N of a few thousand), persistent workers (two per SM) take
// equal contiguous ranges of the (column tile, K block) units, stream-K style.
// A worker's range covers whole tiles and at most two partial ones (its first and last segments). A whole tile is
// finished directly; a partial segment leaves its sums (dot products, column sums of B, row sums of A over its K
// range) in the worker's record and adds its K blocks to the tile's ticket: the worker completing the tile's K
// blocks adds the other segments' records and finishes the tile. Nothing waits on another CTA. Two TMEM
// accumulators let a worker's next segment start while its last one is read out.

// The worker whose range holds unit u (ranges [floor(U i / W), floor(U (i + 1) / W))).
__device__ __forceinline__ int rows_owner(int64_t u, int64_t units, int workers) {
    return static_cast<int>(((u + 1) * workers - 1) / units);
}

template <bool B_KMAJOR, int OUT>
__global__ void __launch_bounds__(rows::THREADS, 2)
    int8_gemm_rows_stream_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                                 const RowsParams p, uint32_t idesc) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sB = smem;                                   // [STAGES][128 columns x 128 k]
    uint8_t* sX = smem + rows::STAGES * rows::B_BYTES;    // [STAGES][16 rows of A x 128 k]
    uint8_t* sOnes = sX + rows::STAGES * rows::A_BYTES;   // [16 rows x 128 k] of ones
    uint64_t* bars = reinterpret_cast<uint64_t*>(sOnes + rows::ONES_BYTES);
    uint64_t* full = bars;
    uint64_t* empty = bars + rows::STAGES;
    uint64_t* tfull = bars + 2 * rows::STAGES;       // [2]
    uint64_t* tempty = bars + 2 * rows::STAGES + 2;  // [2]
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + 2 * rows::STAGES + 4);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
    volatile int* go = reinterpret_cast<volatile int*>(tmem_holder + 2);  // [2]: a segment's wait outcome, its ticket
    int32_t* row_sum = reinterpret_cast<int32_t*>(tmem_holder + 4);        // [16]

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int worker = blockIdx.x;
    const int workers = gridDim.x;
    const int kbt = p.k_blocks_total;
    const int64_t u0 = p.units * worker / workers;
    const int64_t u1 = p.units * (worker + 1) / workers;
    const bool need_col_sums = p.epi.za != nullptr;  // za * colsum(B)
    pdl_trigger();

    for (int i = threadIdx.x; i < rows::ONES_BYTES / 16; i += blockDim.x)
        reinterpret_cast<uint4*>(sOnes)[i] = make_uint4(0x01010101u, 0x01010101u, 0x01010101u, 0x01010101u);
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // generic writes -> visible to the tensor cores
    if (threadIdx.x == 0) {
        for (int st = 0; st < rows::STAGES; st++) {
            mbar_init(&full[st], 1);
            mbar_init(&empty[st], 1);
        }
        for (int a = 0; a < 2; a++) {
            mbar_init(&tfull[a], 1);
            mbar_init(&tempty[a], 4);  // the four epilogue warps
        }
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 0 && lane == 0) {
        prefetch_tmap(&tmap_a);
        prefetch_tmap(&tmap_b);
    }
    pdl_wait();  // the preceding grid is done: its outputs are readable and its TMEM is free
    if (warp == 1) {
        tmem_alloc(tmem_holder, 2 * rows::TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_holder;

    if (warp == 0) {
        for (int64_t u = u0; u < u1; u++) {
            const int it = static_cast<int>(u - u0);
            const int st = it % rows::STAGES;
            const uint32_t ph = (it / rows::STAGES) & 1;
            const int t = static_cast<int>(u / kbt);
            const int kc = static_cast<int>(u - static_cast<int64_t>(t) * kbt) * rows::BK;
            const int tile = t % p.tiles, b = t / p.tiles;
            const int ba = p.a_batched ? b : 0, bb = p.b_batched ? b : 0;
            if (!mbar_wait(&empty[st], ph ^ 1, abort_flag)) break;
            if (lane == 0) {
                mbar_arrive_expect_tx(&full[st], rows::B_BYTES + rows::A_BYTES);
                if constexpr (B_KMAJOR)
                    tma_load_3d(sB + st * rows::B_BYTES, &tmap_b, &full[st], kc, tile * rows::BN, bb);
                else
                    tma_load_3d(sB + st * rows::B_BYTES, &tmap_b, &full[st], tile * rows::BN, kc, bb);
                tma_load_3d(sX + st * rows::A_BYTES, &tmap_a, &full[st], kc, 0, ba);
            }
            __syncwarp();
        }
    } else if (warp == 1) {
        int seg = 0;
        for (int64_t u = u0; u < u1; u++) {
            const int it = static_cast<int>(u - u0);
            const int st = it % rows::STAGES;
            const uint32_t ph = (it / rows::STAGES) & 1;
            const int kb = static_cast<int>(u % kbt);
            const bool first = u == u0 || kb == 0;
            const bool last = u == u1 - 1 || kb == kbt - 1;
            const int acc = seg & 1;
            if (first && !mbar_wait(&tempty[acc], ((seg >> 1) & 1) ^ 1, abort_flag)) break;
            if (!mbar_wait(&full[st], ph, abort_flag)) break;
            tc_fence_after();
            if (lane == 0) {
                const uint32_t b_addr = smem_u32(sB + st * rows::B_BYTES);
                const uint32_t x_addr = smem_u32(sX + st * rows::A_BYTES);
                const uint32_t o_addr = smem_u32(sOnes);
#pragma unroll
                for (int kk = 0; kk < rows::BK / 32; kk++) {
                    const uint32_t d = tmem_base + acc * rows::TMEM_COLS + kk * rows::ACC_COLS;
                    const uint64_t adesc = B_KMAJOR ? smem_desc_sw128(b_addr + kk * 32, 16, 1024)
                                                    : smem_desc_sw128(b_addr + kk * 32 * 128, rows::B_BYTES, 1024);
                    const uint32_t accum = first ? 0u : 1u;
                    mma_i8(d, adesc, smem_desc_sw128(x_addr + kk * 32, 16, 1024), idesc, accum);
                    if (need_col_sums)
                        mma_i8(d + rows::MAXM, adesc, smem_desc_sw128(o_addr + kk * 32, 16, 1024), idesc, accum);
                }
                mma_commit(&empty[st]);
                if (last) mma_commit(&tfull[acc]);
            }
            __syncwarp();
            seg += last ? 1 : 0;
        }
    } else {
        const int t128 = threadIdx.x - 64;
        const int col = (warp & 3) * 32 + lane;  // this thread's TMEM lane: column of the tile
        const Epilogue& e = p.epi;
        int seg = 0;
        for (int64_t u = u0; u < u1;) {
            const int t = static_cast<int>(u / kbt);
            const int kb0 = static_cast<int>(u - static_cast<int64_t>(t) * kbt);
            const int kb1 = static_cast<int>(kb0 + (u1 - u) < kbt ? kb0 + (u1 - u) : kbt);
            const int tile = t % p.tiles, b = t / p.tiles;
            const int ba = p.a_batched ? b : 0;
            const int acc = seg & 1;
            asm volatile("bar.sync 1, 128;" ::: "memory");  // the previous segment is done with row_sum and go
            if (e.zb != nullptr) {
                // Row sums of A over this segment's K range, while its MMAs run: eight threads per row.
                const int r = t128 >> 3, part = t128 & 7;
                int32_t sum = 0;
                if (r < p.m) {
                    const uint8_t* row = p.a + ba * p.stride_a + r * p.lda;
                    const int k_end = min(p.k, kb1 * rows::BK);
                    const int chunks = k_end >> 4;
                    for (int c = kb0 * (rows::BK / 16) + part; c < chunks; c += 8) {
                        const uint4 w = __ldg(reinterpret_cast<const uint4*>(row) + c);
                        if (e.za_signed) {
                            sum = __dp4a(static_cast<int>(w.x), 0x01010101, sum);
                            sum = __dp4a(static_cast<int>(w.y), 0x01010101, sum);
                            sum = __dp4a(static_cast<int>(w.z), 0x01010101, sum);
                            sum = __dp4a(static_cast<int>(w.w), 0x01010101, sum);
                        } else {
                            unsigned su = static_cast<unsigned>(sum);
                            su = __dp4a(w.x, 0x01010101u, su);
                            su = __dp4a(w.y, 0x01010101u, su);
                            su = __dp4a(w.z, 0x01010101u, su);
                            su = __dp4a(w.w, 0x01010101u, su);
                            sum = static_cast<int32_t>(su);
                        }
                    }
                    for (int kk = (chunks << 4) + part; kk < k_end; kk += 8) {  // the last k % 16 bytes
                        const uint8_t v = __ldg(row + kk);
                        sum += e.za_signed ? static_cast<int32_t>(static_cast<int8_t>(v)) : v;
                    }
                }
                sum += __shfl_xor_sync(0xFFFFFFFFu, sum, 1);
                sum += __shfl_xor_sync(0xFFFFFFFFu, sum, 2);
                sum += __shfl_xor_sync(0xFFFFFFFFu, sum, 4);
                if (part == 0) row_sum[r] = sum;
            }
            if (threadIdx.x == 64) go[0] = mbar_wait(&tfull[acc], (seg >> 1) & 1, abort_flag) ? 1 : 0;
            asm volatile("bar.sync 1, 128;" ::: "memory");
            const bool ok = go[0] != 0;
            uint32_t r[32];
            if (ok) {
                tc_fence_after();
                tmem_ld_sum(tmem_base + acc * rows::TMEM_COLS + (static_cast<uint32_t>((warp & 3) * 32) << 16),
                            kb1 - kb0, r);
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&tempty[acc]);
            bool finish = ok;
            if (kb0 != 0 || kb1 != kbt) {
                // A partial segment: leave its record, add its K blocks to the tile's ticket (also after a failed
                // wait, so that the tickets stay balanced); the segment completing the tile finishes it.
                const int slot = u == u0 ? 0 : 1;
                int32_t* mine = p.split_part + (static_cast<int64_t>(worker) * 2 + slot) * PART_INTS;
                if (ok) {
#pragma unroll
                    for (int v = 0; v < 17; v++) __stcg(mine + v * rows::BN + col, static_cast<int32_t>(r[v]));
                    if (t128 < rows::MAXM) __stcg(mine + 17 * rows::BN + t128, row_sum[t128]);
                }
                __threadfence();
                asm volatile("bar.sync 1, 128;" ::: "memory");
                if (threadIdx.x == 64) {
                    unsigned int* ticket = p.split_ticket + t;
                    const unsigned int add = static_cast<unsigned int>(kb1 - kb0);
                    const unsigned int old = atomicAdd(ticket, add);
                    const bool complete = old + add == static_cast<unsigned int>(kbt);
                    if (complete) atomicExch(ticket, 0u);
                    go[1] = complete ? 1 : 0;
                }
                asm volatile("bar.sync 1, 128;" ::: "memory");
                finish = ok && go[1] != 0;
                if (finish) {
                    __threadfence();
                    const int64_t tu0 = static_cast<int64_t>(t) * kbt;
                    const int w_first = rows_owner(tu0, p.units, workers);
                    const int w_last = rows_owner(tu0 + kbt - 1, p.units, workers);
                    // The other segments' records, four at a time: all their loads are in flight together.
                    int32_t rs = 0;
                    for (int w0 = w_first; w0 <= w_last; w0 += 4) {
                        uint32_t vals[4][17];
                        int32_t rsv[4];
#pragma unroll
                        for (int j = 0; j < 4; j++) {
                            const int w = w0 + j;
                            const bool use = w <= w_last && w != worker;
                            const int wslot = p.units * w / workers >= tu0 ? 0 : 1;  // its first segment, or its last
                            const int32_t* rec = p.split_part + (static_cast<int64_t>(use ? w : worker) * 2 + wslot) *
                                                                    PART_INTS;
#pragma unroll
                            for (int v = 0; v < 17; v++)
                                vals[j][v] = use ? static_cast<uint32_t>(__ldcg(rec + v * rows::BN + col)) : 0u;
                            rsv[j] = (use && t128 < rows::MAXM) ? __ldcg(rec + 17 * rows::BN + t128) : 0;
                        }
#pragma unroll
                        for (int j = 0; j < 4; j++) {
#pragma unroll
                            for (int v = 0; v < 17; v++) r[v] += vals[j][v];
                            rs += rsv[j];
                        }
                    }
                    if (t128 < rows::MAXM) row_sum[t128] += rs;
                    asm volatile("bar.sync 1, 128;" ::: "memory");
                }
            }
            if (finish) {
                const int n = tile * rows::BN + col;
                if (n < p.n) {
                    const uint32_t csb = r[16];  // sum over K of B[k, n]
                    const int32_t zb = zp_value(e.zb, e.zb_vector, e.zb_signed, n);
                    const uint32_t bias = e.int_bias ? static_cast<uint32_t>(__ldg(e.int_bias + n)) : 0u;
#pragma unroll
                    for (int m = 0; m < rows::MAXM; m++) {
                        if (m < p.m) {
                            const int32_t za = zp_value(e.za, e.za_vector, e.za_signed, m);
                            uint32_t sm = r[m];
                            if (e.zb != nullptr)
                                sm += static_cast<uint32_t>(p.k) * static_cast<uint32_t>(za) * static_cast<uint32_t>(zb) -
                                      static_cast<uint32_t>(zb) * static_cast<uint32_t>(row_sum[m]);
                            if (e.za != nullptr) sm -= static_cast<uint32_t>(za) * csb;
                            store_one<OUT>(e, b, m, n, sm + bias);
                        }
                    }
                }
            }
            seg++;
            u = static_cast<int64_t>(t) * kbt + kb1;
        }
    }

    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, 2 * rows::TMEM_COLS);
    }
    if (threadIdx.x == 0 && *abort_flag) atomicExch(p.error_flag, 1);
}

// ---- byte sums of two matrices in one launch ------------------------------------------------------------------------
//
// The zero-point correction needs the byte sums over K of A's rows and of B's columns. Each is a stream of the
// operand through the tensor cores against a block of ones: D[c, j] = sum_k T[c, k] * 1 with 128 rows or columns c
// of the operand as the MMA's M side and N = 16. One launch covers both operands: the first job's CTAs come first in
// the grid, then the second's; the layout (K-major rows, or MN-major columns) and the tensor map are the job's.

struct SumsJob {
    int32_t* out;  // [splits][batches][cols]
    int cols, tiles, batches, splits;
    int k_blocks_total, k_blocks;  // K blocks of the whole operand, and of one split
    int kmajor;                    // cols x K with K contiguous (1), or K x cols with columns contiguous (0)
    int batched;
    uint32_t idesc;
    int ctas;  // tiles * batches * splits
};

struct SumsParams {
    SumsJob job[2];
    int* error_flag;
};

__global__ void __launch_bounds__(rows::THREADS, 2)
    int8_byte_sums_kernel(const __grid_constant__ CUtensorMap tmap0, const __grid_constant__ CUtensorMap tmap1,
                          const __grid_constant__ SumsParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sB = smem;                                   // [STAGES][128 rows or columns x 128 k]
    uint8_t* sOnes = sB + rows::SUMS_STAGES * rows::B_BYTES;   // [16 rows x 128 k] of ones
    uint64_t* bars = reinterpret_cast<uint64_t*>(sOnes + rows::ONES_BYTES);
    uint64_t* full = bars;
    uint64_t* empty = bars + rows::SUMS_STAGES;
    uint64_t* tfull = bars + 2 * rows::SUMS_STAGES;
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + 2 * rows::SUMS_STAGES + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int j = static_cast<int>(blockIdx.x) < p.job[0].ctas ? 0 : 1;
    const SumsJob& job = p.job[j];
    const CUtensorMap* tmap = j == 0 ? &tmap0 : &tmap1;
    const int local = static_cast<int>(blockIdx.x) - (j == 0 ? 0 : p.job[0].ctas);
    const int tile = local % job.tiles;
    const int rest = local / job.tiles;
    const int b = rest % job.batches;
    const int split = rest / job.batches;
    const int kb_begin = split * job.k_blocks;
    const int kb_count = min(job.k_blocks, job.k_blocks_total - kb_begin);
    pdl_trigger();

    for (int i = threadIdx.x; i < rows::ONES_BYTES / 16; i += blockDim.x)
        reinterpret_cast<uint4*>(sOnes)[i] = make_uint4(0x01010101u, 0x01010101u, 0x01010101u, 0x01010101u);
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // generic writes -> visible to the tensor cores
    if (threadIdx.x == 0) {
        for (int s = 0; s < rows::SUMS_STAGES; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(tfull, 1);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 0 && lane == 0) prefetch_tmap(tmap);
    pdl_wait();  // the preceding grid is done: the operands are written and its TMEM is free
    if (warp == 1) {
        tmem_alloc(tmem_holder, rows::TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_holder;
    const int bz = job.batched ? b : 0;

    if (warp == 0) {
        for (int kb = 0; kb < kb_count; kb++) {
            const int s = kb % rows::SUMS_STAGES;
            const uint32_t ph = (kb / rows::SUMS_STAGES) & 1;
            const int kc = (kb_begin + kb) * rows::BK;
            if (!mbar_wait(&empty[s], ph ^ 1, abort_flag)) goto done;
            if (lane == 0) {
                mbar_arrive_expect_tx(&full[s], rows::B_BYTES);
                if (job.kmajor)
                    tma_load_3d(sB + s * rows::B_BYTES, tmap, &full[s], kc, tile * rows::BN, bz);
                else
                    tma_load_3d(sB + s * rows::B_BYTES, tmap, &full[s], tile * rows::BN, kc, bz);
            }
            __syncwarp();
        }
    } else if (warp == 1) {
        for (int kb = 0; kb < kb_count; kb++) {
            const int s = kb % rows::SUMS_STAGES;
            const uint32_t ph = (kb / rows::SUMS_STAGES) & 1;
            if (!mbar_wait(&full[s], ph, abort_flag)) goto done;
            tc_fence_after();
            if (lane == 0) {
                const uint32_t t_addr = smem_u32(sB + s * rows::B_BYTES);
                const uint32_t o_addr = smem_u32(sOnes);
#pragma unroll
                for (int kk = 0; kk < rows::BK / 32; kk++) {
                    const uint64_t tdesc = job.kmajor ? smem_desc_sw128(t_addr + kk * 32, 16, 1024)
                                                      : smem_desc_sw128(t_addr + kk * 32 * 128, rows::B_BYTES, 1024);
                    mma_i8(tmem_base + kk * rows::MAXM, tdesc, smem_desc_sw128(o_addr + kk * 32, 16, 1024), job.idesc,
                           kb != 0 ? 1u : 0u);
                }
                mma_commit(&empty[s]);
            }
            __syncwarp();
        }
        if (lane == 0) mma_commit(tfull);
        __syncwarp();
    } else {
        const int q = warp & 3;
        if (!mbar_wait(tfull, 0, abort_flag)) goto done;
        tc_fence_after();
        // Accumulator kk (one per K = 32 step of a block) holds its sum in all 16 of its columns kk*16 .. +15.
        uint32_t r[32], t[32];
        tmem_ld_32x32b_x32(tmem_base + (static_cast<uint32_t>(q * 32) << 16), r);
        tmem_ld_32x32b_x32(tmem_base + (static_cast<uint32_t>(q * 32) << 16) + 32, t);
        tmem_ld_wait();
        const uint32_t sum = r[0] + r[16] + t[0] + t[16];
        const int c = tile * rows::BN + q * 32 + lane;
        if (c < job.cols)
            job.out[(static_cast<int64_t>(split) * job.batches + b) * job.cols + c] = static_cast<int32_t>(sum);
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

bool rows_eligible(const GemmLaunch& L) {
    return L.m >= 1 && L.m <= rows::MAXM && L.batch <= 65535 && tc_eligible(L);
}

// Binds the kernel and its arguments; the returned function sets the shared-memory limit (first time per device)
// and launches.
template <bool B_KMAJOR, int OUT>
static LaunchFn bind_rows_t(const RowsParams& p, const CUtensorMap& ma, const CUtensorMap& mb, dim3 grid,
                            uint32_t idesc) {
    return [=](cudaStream_t stream) -> cudaError_t {
        auto kern = int8_gemm_rows_kernel<B_KMAJOR, OUT>;
        static std::atomic<uint64_t> configured{0};  // devices whose attribute is set
        int dev = 0;
        cudaError_t e = cudaGetDevice(&dev);
        if (e != cudaSuccess) return e;
        const uint64_t bit = uint64_t(1) << (dev & 63);
        if (!(configured.load() & bit)) {
            e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, rows::SMEM_BYTES);
            if (e != cudaSuccess) return e;
            configured.fetch_or(bit);
        }
        return launch_pdl(kern, grid, dim3(rows::THREADS), rows::SMEM_BYTES, stream, ma, mb, p, idesc);
    };
}

template <bool B_KMAJOR, int OUT>
static LaunchFn bind_rows_stream_t(const RowsParams& p, const CUtensorMap& ma, const CUtensorMap& mb, dim3 grid,
                                   uint32_t idesc) {
    return [=](cudaStream_t stream) -> cudaError_t {
        auto kern = int8_gemm_rows_stream_kernel<B_KMAJOR, OUT>;
        static std::atomic<uint64_t> configured{0};  // devices whose attribute is set
        int dev = 0;
        cudaError_t e = cudaGetDevice(&dev);
        if (e != cudaSuccess) return e;
        const uint64_t bit = uint64_t(1) << (dev & 63);
        if (!(configured.load() & bit)) {
            e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, STREAM_SMEM_BYTES);
            if (e != cudaSuccess) return e;
            configured.fetch_or(bit);
        }
        return launch_pdl(kern, grid, dim3(rows::THREADS), STREAM_SMEM_BYTES, stream, ma, mb, p, idesc);
    };
}

// The split pays when one CTA per column tile would leave SMs idle. Measured on B200 with the decode shapes
// (K = 8192), the best split gives each tile's K blocks to S workers in equal, aligned parts (every worker one
// segment of one tile) with about one and a half workers per SM: 16 x 14336 34.7 us with 2 parts per tile against
// 38.9 us unsplit, 16 x 7168 24.7 us with 4 parts, 16 x 3584 22.6 us with 8 parts, against 38.9 us for both unsplit
// (more workers, or parts not aligned to the tiles, ran slower); 16 x 28672, with 224 tiles, runs unsplit.
int rows_workers(const GemmLaunch& L) {
    const int64_t tiles = static_cast<int64_t>((L.n + rows::BN - 1) / rows::BN) * L.batch;
    const int64_t kb = (L.k + rows::BK - 1) / rows::BK;
    const int64_t target = 3 * int64_t(L.num_sms) / 2;
    if (kb < 8 || L.num_sms < 1 || 10 * tiles >= 9 * target) return 0;
    int64_t parts = (target + tiles / 2) / tiles;       // the nearest whole number of parts per tile
    if (parts > kb / 4) parts = kb / 4;                  // segments of at least 4 K blocks
    const int64_t w = tiles * parts;
    return (parts < 2 || w > 2 * int64_t(L.num_sms)) ? 0 : static_cast<int>(w);
}

int64_t rows_part_ints(const GemmLaunch&, int workers) { return static_cast<int64_t>(workers) * 2 * PART_INTS; }

int64_t rows_tickets(const GemmLaunch& L) { return static_cast<int64_t>((L.n + rows::BN - 1) / rows::BN) * L.batch; }

LaunchFn prepare_gemm_rows(const GemmLaunch& L, cudaError_t* err) {
    *err = cudaErrorInvalidValue;
    const int ba = (L.batch > 1 && L.stride_a != 0) ? L.batch : 1;
    const int bb = (L.batch > 1 && L.stride_b != 0) ? L.batch : 1;
    CUtensorMap ma, mb;
    const uint64_t sa = ba > 1 ? uint64_t(L.stride_a) : (uint64_t(L.lda) * L.m + 15) & ~uint64_t(15);
    if (!make_tensor_map_u8(&ma, L.a, L.k, L.m, ba, L.lda, sa, rows::BK, rows::MAXM)) return nullptr;
    const uint64_t rows_b = L.trans_b ? L.n : L.k;
    const uint64_t sb = bb > 1 ? uint64_t(L.stride_b) : (uint64_t(L.ldb) * rows_b + 15) & ~uint64_t(15);
    const bool ok = L.trans_b ? make_tensor_map_u8(&mb, L.b, L.k, L.n, bb, L.ldb, sb, rows::BK, rows::BN)
                              : make_tensor_map_u8(&mb, L.b, L.n, L.k, bb, L.ldb, sb, rows::BN, rows::BK);
    if (!ok) return nullptr;
    *err = cudaSuccess;
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
    p.sums_out = nullptr;
    p.sums_stride = 0;
    p.sums_split_stride = 0;
    p.k_blocks_total = p.k_blocks;
    p.tiles = (L.n + rows::BN - 1) / rows::BN;
    p.units = static_cast<int64_t>(p.tiles) * L.batch * p.k_blocks;
    p.split_part = L.rows_part;
    p.split_ticket = L.rows_ticket;
    // The MMA's A operand is B (its type, MN-major unless B is stored N x K); its B operand is A (or the ones).
    const uint32_t idesc = idesc_i8(L.b_signed, L.a_signed, !L.trans_b, false, rows::BN, rows::MAXM);
    const bool km = L.trans_b != 0;
    if (L.rows_part != nullptr && L.rows_ticket != nullptr && L.rows_workers > 0) {
        const dim3 grid(static_cast<unsigned>(L.rows_workers));
        switch (L.epi.out_kind) {
            case OUT_I32: return km ? bind_rows_stream_t<true, OUT_I32>(p, ma, mb, grid, idesc)
                                    : bind_rows_stream_t<false, OUT_I32>(p, ma, mb, grid, idesc);
            case OUT_F32: return km ? bind_rows_stream_t<true, OUT_F32>(p, ma, mb, grid, idesc)
                                    : bind_rows_stream_t<false, OUT_F32>(p, ma, mb, grid, idesc);
            case OUT_U8: return km ? bind_rows_stream_t<true, OUT_U8>(p, ma, mb, grid, idesc)
                                   : bind_rows_stream_t<false, OUT_U8>(p, ma, mb, grid, idesc);
            default: return km ? bind_rows_stream_t<true, OUT_S8>(p, ma, mb, grid, idesc)
                               : bind_rows_stream_t<false, OUT_S8>(p, ma, mb, grid, idesc);
        }
    }
    const dim3 grid((L.n + rows::BN - 1) / rows::BN, L.batch);
    switch (L.epi.out_kind) {
        case OUT_I32: return km ? bind_rows_t<true, OUT_I32>(p, ma, mb, grid, idesc)
                                : bind_rows_t<false, OUT_I32>(p, ma, mb, grid, idesc);
        case OUT_F32: return km ? bind_rows_t<true, OUT_F32>(p, ma, mb, grid, idesc)
                                : bind_rows_t<false, OUT_F32>(p, ma, mb, grid, idesc);
        case OUT_U8: return km ? bind_rows_t<true, OUT_U8>(p, ma, mb, grid, idesc)
                               : bind_rows_t<false, OUT_U8>(p, ma, mb, grid, idesc);
        default: return km ? bind_rows_t<true, OUT_S8>(p, ma, mb, grid, idesc)
                           : bind_rows_t<false, OUT_S8>(p, ma, mb, grid, idesc);
    }
}

// Byte sums over K of every column of a matrix, with the few-rows kernel in its sums-only mode (the block of ones
// times the matrix): `mat` is K x cols with columns contiguous (k_major = false; B) or cols x K with K contiguous
// (k_major = true; the rows of A, or a B stored N x K). One result per column and batch, written (no accumulation).
LaunchFn prepare_byte_sums_tc(const uint8_t* mat, int cols, int k, int64_t ld, int64_t bstride, int batches,
                              bool k_major, bool is_signed, int32_t* out, int splits, int* error_flag, cudaError_t* err) {
    *err = cudaErrorInvalidValue;
    CUtensorMap mb;
    const uint64_t rows_stored = k_major ? cols : k;
    const uint64_t sb = batches > 1 ? uint64_t(bstride) : (uint64_t(ld) * rows_stored + 15) & ~uint64_t(15);
    const bool ok = k_major ? make_tensor_map_u8(&mb, mat, k, cols, batches, ld, sb, rows::BK, rows::BN)
                            : make_tensor_map_u8(&mb, mat, cols, k, batches, ld, sb, rows::BN, rows::BK);
    if (!ok) return nullptr;
    *err = cudaSuccess;
    RowsParams p = {};
    p.m = 0;
    p.n = cols;
    p.k = k;
    p.k_blocks_total = (k + rows::BK - 1) / rows::BK;
    p.k_blocks = (p.k_blocks_total + splits - 1) / splits;  // every split gets at least one K block (see byte_sum_splits)
    p.a_batched = 0;
    p.b_batched = batches > 1;
    p.error_flag = error_flag;
    p.sums_out = out;
    p.sums_stride = cols;
    p.sums_split_stride = int64_t(batches) * cols;
    const uint32_t idesc = idesc_i8(is_signed, false, !k_major, false, rows::BN, rows::MAXM);
    const dim3 grid((cols + rows::BN - 1) / rows::BN, batches, splits);
    return k_major ? bind_rows_t<true, OUT_I32>(p, mb, mb, grid, idesc)
                   : bind_rows_t<false, OUT_I32>(p, mb, mb, grid, idesc);
}

// One sums job: `mat` is cols x K with K contiguous (k_major) or K x cols with columns contiguous.
static bool sums_job(SumsJob& j, CUtensorMap& map, const uint8_t* mat, int cols, int k, int64_t ld, int64_t bstride,
                     int batches, bool k_major, bool is_signed, int32_t* out, int splits) {
    const uint64_t rows_stored = k_major ? cols : k;
    const uint64_t sb = batches > 1 ? uint64_t(bstride) : (uint64_t(ld) * rows_stored + 15) & ~uint64_t(15);
    const bool ok = k_major ? make_tensor_map_u8(&map, mat, k, cols, batches, ld, sb, rows::BK, rows::BN)
                            : make_tensor_map_u8(&map, mat, cols, k, batches, ld, sb, rows::BN, rows::BK);
    if (!ok) return false;
    j.out = out;
    j.cols = cols;
    j.tiles = (cols + rows::BN - 1) / rows::BN;
    j.batches = batches;
    j.splits = splits;
    j.k_blocks_total = (k + rows::BK - 1) / rows::BK;
    j.k_blocks = (j.k_blocks_total + splits - 1) / splits;  // every split gets at least one K block (byte_sum_splits)
    j.kmajor = k_major ? 1 : 0;
    j.batched = batches > 1;
    j.idesc = idesc_i8(is_signed, false, !k_major, false, rows::BN, rows::MAXM);
    j.ctas = j.tiles * batches * splits;
    return true;
}

// The byte sums of A's rows (row_sums, when non-null) and of B's columns (col_sums) in one launch, each as `splits`
// partial sums over K ([splits][batches][rows or columns]).
LaunchFn prepare_byte_sums_pair_tc(const GemmLaunch& L, int32_t* row_sums, int32_t* col_sums, int splits,
                                   cudaError_t* err) {
    *err = cudaErrorInvalidValue;
    const int ba = (L.batch > 1 && L.stride_a != 0) ? L.batch : 1;
    const int bb = (L.batch > 1 && L.stride_b != 0) ? L.batch : 1;
    SumsParams p = {};
    CUtensorMap maps[2];
    int jobs = 0;
    if (row_sums != nullptr) {
        if (!sums_job(p.job[jobs], maps[jobs], L.a, L.m, L.k, L.lda, L.stride_a, ba, true, L.a_signed, row_sums, splits))
            return nullptr;
        jobs++;
    }
    if (col_sums != nullptr) {
        if (!sums_job(p.job[jobs], maps[jobs], L.b, L.n, L.k, L.ldb, L.stride_b, bb, L.trans_b != 0, L.b_signed,
                      col_sums, splits))
            return nullptr;
        jobs++;
    }
    if (jobs == 0) {
        *err = cudaSuccess;
        return [](cudaStream_t) { return cudaSuccess; };
    }
    if (jobs == 1) {
        p.job[1] = p.job[0];
        p.job[1].ctas = 0;
        maps[1] = maps[0];
    }
    p.error_flag = L.error_flag;
    const int64_t ctas = int64_t(p.job[0].ctas) + p.job[1].ctas;
    if (ctas > 0x7FFFFFFF) return nullptr;
    *err = cudaSuccess;
    const CUtensorMap m0 = maps[0], m1 = maps[1];
    const dim3 grid(static_cast<unsigned>(ctas));
    return [=](cudaStream_t stream) -> cudaError_t {
        static std::atomic<uint64_t> configured{0};  // devices whose attribute is set
        int dev = 0;
        cudaError_t e = cudaGetDevice(&dev);
        if (e != cudaSuccess) return e;
        const uint64_t bit = uint64_t(1) << (dev & 63);
        if (!(configured.load() & bit)) {
            e = cudaFuncSetAttribute(int8_byte_sums_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     SUMS_SMEM_BYTES);
            if (e != cudaSuccess) return e;
            configured.fetch_or(bit);
        }
        return launch_pdl(int8_byte_sums_kernel, grid, dim3(rows::THREADS), SUMS_SMEM_BYTES, stream, m0, m1, p);
    };
}

cudaError_t launch_gemm_rows(const GemmLaunch& L, cudaStream_t stream) {
    cudaError_t err;
    LaunchFn fn = prepare_gemm_rows(L, &err);
    return fn ? fn(stream) : err;
}

}  // namespace og
