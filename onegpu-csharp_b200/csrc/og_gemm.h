// Internal launch descriptions shared by the host layer (og_capi.cu) and the kernel files.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <functional>

#include "og_kernels.cuh"

namespace og {

// One validated product, pointers resolved: a and b point at the first byte of batch 0 (OffsetA/OffsetB applied),
// the epilogue's output pointer at element OffsetC.
struct GemmLaunch {
    const uint8_t* a;
    const uint8_t* b;
    int m, n, k, batch;
    int trans_b;
    int64_t lda, ldb;        // bytes
    int64_t stride_a, stride_b;
    int a_signed, b_signed;
    Epilogue epi;
    int num_sms;
    int* error_flag;
    int tile;  // tensor-core tile rows: 0 chooses by size, 128 one CTA per tile, 256 a CTA pair (cta_group::2)
    // 0: whole tiles, and for int32 results the tiles past the last full wave split in K (the split tail);
    // 1: whole tiles only; 2: split the (tile, K block) work evenly across the workers (stream-K)
    int stream_k = 0;
    // Stream-K hand-over buffers of the tensor-core product (one device buffer of sk_bytes_needed(num_sms) bytes,
    // split by sk_bind); null leaves every worker whole tiles.
    int32_t* sk_part = nullptr;
    unsigned int* sk_flag = nullptr;
    int64_t sk_bytes = 0;
    // The few-rows kernel with its (column tile, K block) units split evenly across rows_workers persistent CTAs:
    // partial segments meet through rows_part (rows_part_ints) and one ticket per (batch, column tile) in rows_ticket
    // (rows_tickets, zero between launches). Null: one CTA per column tile.
    int32_t* rows_part = nullptr;
    unsigned int* rows_ticket = nullptr;
    int rows_workers = 0;
};

// Bytes of the stream-K hand-over buffer for a device with num_sms SMs, and the split of one such buffer.
int64_t sk_bytes_needed(int num_sms);
void sk_bind(GemmLaunch& L, void* buffer, int64_t bytes);
// How the tensor-core product of L would split tiles between workers given the hand-over buffer: 0 not at all
// (whole tiles), 1 the split tail (int32 results: the tiles past the last full wave split in K, put together in C by
// TMA reductions), 2 stream-K (option 2). sk_wanted: the mode is not 0, so the launch needs the buffer.
int tc_split_mode(const GemmLaunch& L);
bool sk_wanted(const GemmLaunch& L);

// A launch whose host-side preparation (tensor maps, parameters) is already done: calling it only launches.
using LaunchFn = std::function<cudaError_t(cudaStream_t)>;

// Whether launches may overlap the preceding grid (environment ONEGPU_PDL=0 turns it off; read once).
bool pdl_enabled();

// Launches a kernel that may overlap the tail of the preceding grid in the stream (programmatic dependent launch);
// the kernel must call pdl_wait() before it touches global memory or allocates TMEM.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                       Args... args) {
    if (!pdl_enabled()) {
        kernel<<<grid, block, smem, stream>>>(args...);
        return cudaGetLastError();
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, args...);
}

// tcgen05 product (og_gemm_tc.cu). Eligible when K >= 1 and both operands' rows and batches start on 16-byte
// boundaries (the TMA requirement). prepare_* builds the tensor maps at record time (null + *err on failure).
bool tc_eligible(const GemmLaunch& L);
int tc_cta_group(const GemmLaunch& L);  // 1 or 2: the tile launch_gemm_tc will use
LaunchFn prepare_gemm_tc(const GemmLaunch& L, cudaError_t* err);
cudaError_t launch_gemm_tc(const GemmLaunch& L, cudaStream_t stream);

// Few-rows product (og_gemm_rows.cu): M <= 16 per batch, TMA-loadable operands; streams B once and takes the column
// sums of B from the same MMA, so it needs no byte-sum pass and no scratch.
bool rows_eligible(const GemmLaunch& L);
LaunchFn prepare_gemm_rows(const GemmLaunch& L, cudaError_t* err);
// Persistent workers that spread the few-rows product evenly over the SMs (0: one CTA per column tile serves), and
// the int32 partials and tickets such a launch of L needs.
int rows_workers(const GemmLaunch& L);
int64_t rows_part_ints(const GemmLaunch& L, int workers);
int64_t rows_tickets(const GemmLaunch& L);
cudaError_t launch_gemm_rows(const GemmLaunch& L, cudaStream_t stream);

// A 3-D byte tensor map (x innermost) with 128-byte swizzled box_x x box_y boxes (og_gemm_tc.cu).
bool make_tensor_map_u8(CUtensorMap* map, const void* base, uint64_t x, uint64_t y, uint64_t z, uint64_t stride_y,
                        uint64_t stride_z, uint32_t box_x, uint32_t box_y);

// Portable SIMT product (og_gemm_simt.cu): any alignment, subtracts the zero points while staging, so it needs no
// byte sums; its epilogue ignores row_sum_a / col_sum_b.
cudaError_t launch_gemm_simt(const GemmLaunch& L, cudaStream_t stream);

// Byte sums for the zero-point correction (og_gemm_simt.cu): row sums of A ([batchA][M], batchA = batch when A has
// its own stride, else 1) when `row_sums` is set, column sums of B ([batchB][N]) when `col_sums` is set.
// With the tensor-core sums the K range may be split (at most `splits` ways, see byte_sum_splits): each split writes
// its partial sums, [split][batch][M] and [split][batch][N], and the product's epilogue adds them up
// (Epilogue::sum_splits). The scratch then holds splits * (batchA * M + batchB * N) int32.
int byte_sum_splits(const GemmLaunch& L, int max_splits);
LaunchFn prepare_byte_sums(const GemmLaunch& L, int32_t* row_sums, int32_t* col_sums, int splits, cudaError_t* err);
cudaError_t launch_byte_sums(const GemmLaunch& L, int32_t* row_sums, int32_t* col_sums, cudaStream_t stream);
cudaError_t launch_byte_sums_simt(const GemmLaunch& L, int32_t* row_sums, int32_t* col_sums, cudaStream_t stream);
// The byte sums of A's rows and B's columns (either may be null) in one launch of the tensor-core sums kernel.
LaunchFn prepare_byte_sums_pair_tc(const GemmLaunch& L, int32_t* row_sums, int32_t* col_sums, int splits,
                                   cudaError_t* err);
// Sums over K of every column of a K x cols (k_major = false) or cols x K (k_major = true) byte matrix, through the
// tensor cores (og_gemm_rows.cu), K split `splits` ways (partials at out + split * batches * cols).
LaunchFn prepare_byte_sums_tc(const uint8_t* mat, int cols, int k, int64_t ld, int64_t bstride, int batches,
                              bool k_major, bool is_signed, int32_t* out, int splits, int* error_flag,
                              cudaError_t* err);

// DynamicQuantizeLinear (og_dq.cu).
struct DqScratch;
// QuantizeLinear per tensor to uint8 (og_quant.cu): clamp(round_half_even(x / *scale) + *zero_point, 0, 255), NaN
// to 0 - the second pass of DynamicQuantizeLinear.
cudaError_t launch_quantize_u8_tensor(const float* x, int64_t count, uint8_t* y, const float* scale,
                                      const uint8_t* zero_point, cudaStream_t s);
size_t dq_scratch_bytes();
// Whether launch_dynamic_quantize runs as one kernel (range, grid barrier, quantize from on-chip copies of x) rather
// than the range and quantize passes: large tensors, x 16-byte and y 4-byte aligned, one 1024-thread CTA with 224 KB
// of shared memory fitting on every SM.
bool dq_single_kernel(const float* x, int64_t count, const uint8_t* y);
cudaError_t launch_dynamic_quantize(const float* x, int64_t count, uint8_t* y, float* scale_out, uint8_t* zp_out,
                                    DqScratch* scratch, int num_sms, int* error_flag, cudaStream_t stream);

}  // namespace og
