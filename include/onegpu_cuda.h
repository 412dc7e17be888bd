/*
 * onegpu_cuda.h - C ABI of libonegpu_cuda.so, the B200 (sm_100a) backend of onegpu's quantized-matmul path.
 *
 * The reference (recursive-ai-oss/onegpu-csharp) has no FFI of its own: its boundary is the shipped C# API of
 * RecursiveAI.OneGpu.Kernels (PublicAPI.Shipped.txt) written against the GpuDevice abstraction. Each entry point below
 * is what a `RecursiveAI.OneGpu.Cuda` backend binds through [LibraryImport] to keep that API drop-in; the comment on
 * each names the reference member it replaces (paths relative to the reference repository root).
 *
 * Conventions
 *  - Every function returns og_status. On failure, og_last_error() (per calling thread) holds the typed error the C#
 *    side turns into its exception: operation / argument / message for GpuKernelShapeException and
 *    ArgumentNullException, capability / expected / actual for GpuUnsupportedException.
 *  - Argument checks run synchronously, before anything is recorded, in the reference's order and with the
 *    reference's argument names (src/RecursiveAI.OneGpu.Kernels/Int8Gemm.cs:393-501,
 *    src/RecursiveAI.OneGpu.Kernels/DynamicQuantizeKernels.cs:59-75, KernelSupport.cs:75-91).
 *  - Buffers are plain device pointers with an element count and element type (og_buffer): the caller owns them.
 *  - Encoders record; nothing runs until og_device_submit, which replays the recorded work in order on the device's
 *    stream (src/RecursiveAI.OneGpu/GpuDevice.cs:155-167).
 *  - Objects are not thread-safe, like the reference's (Int8Gemm.cs:122, DynamicQuantizeKernels.cs:18).
 * No C++ exception crosses this boundary.
 */
#ifndef ONEGPU_CUDA_H
#define ONEGPU_CUDA_H

#include <stdint.h>

#if defined(__GNUC__)
#define OG_API __attribute__((visibility("default")))
#else
#define OG_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status and errors --------------------------------------------------------------------------------------- */

typedef enum og_status {
    OG_OK = 0,
    OG_ERROR_SHAPE = 1,           /* GpuKernelShapeException (GpuKernelShapeException.cs:7-25) */
    OG_ERROR_UNSUPPORTED = 2,     /* GpuUnsupportedException (src/RecursiveAI.OneGpu/GpuDevice.cs:283-312) */
    OG_ERROR_ARGUMENT_NULL = 3,   /* ArgumentNullException */
    OG_ERROR_ARGUMENT_RANGE = 4,  /* ArgumentOutOfRangeException (Int8Gemm.cs:541-542) */
    OG_ERROR_OUT_OF_MEMORY = 5,   /* GpuOutOfMemoryException */
    OG_ERROR_DEVICE_LOST = 6,     /* GpuDeviceLostException (GpuDevice.cs:377): a sticky CUDA error */
    OG_ERROR_COMMAND_FAILED = 7,  /* GpuCommandFailedException (GpuDevice.cs:337-374): a kernel reported a failure */
    OG_ERROR_CUDA = 8,            /* any other CUDA runtime error */
    OG_ERROR_INVALID_HANDLE = 9
} og_status;

typedef struct og_error_info {
    int32_t status;
    char operation[64];   /* "Int8Gemm", "DynamicQuantizeLinear", ... */
    char argument[64];    /* "M", "OffsetA", "zpA", "scratch", ... (GpuKernelShapeException.Argument) */
    char message[512];
    char capability[64];  /* GpuUnsupportedException.Capability */
    char expected[128];
    char actual[128];
} og_error_info;

/* The last error raised on the calling thread. */
OG_API og_status og_last_error(og_error_info* out);

/* ---- element types and buffer views ---------------------------------------------------------------------------- */

typedef enum og_element_type {
    OG_U8 = 0,  /* byte */
    OG_S8 = 1,  /* sbyte */
    OG_I32 = 2, /* int */
    OG_F32 = 3, /* float */
    OG_F16 = 4, /* Half */
    OG_U32 = 5, /* uint */
    OG_U16 = 6, /* ushort: no kernel takes it; named so that a caller's type is reported, not guessed */
    OG_I16 = 7, /* short: likewise */
    OG_I64 = 8  /* long: likewise */
} og_element_type;

/* A GpuBuffer<T> (src/RecursiveAI.OneGpu/GpuBufferOfT.cs:11): device pointer of element 0, element count, type. */
typedef struct og_buffer {
    void* ptr;
    int64_t length;
    int32_t type;
} og_buffer;

/* Int8Operand<T> (Int8Gemm.cs:28): a zero point, scale or bias - buffer, element offset, one value or a vector. */
typedef struct og_operand {
    og_buffer buffer;
    int32_t offset;
    int32_t is_vector;
} og_operand;

/* ---- device (compute subset of GpuDevice, src/RecursiveAI.OneGpu/GpuDevice.cs:27-228) ------------------------- */

typedef struct og_device og_device;
typedef struct og_encoder og_encoder;
typedef struct og_timestamps og_timestamps;

typedef struct og_device_info {
    char name[256];          /* GpuAdapterInfo.Name */
    int32_t ordinal;
    int32_t sm_count;
    int32_t cc_major, cc_minor;
    int64_t total_memory;    /* bytes */
    int32_t max_shared_memory_per_block;
    int32_t tensor_core_i8;  /* 1 when the tcgen05 int8 product runs here */
} og_device_info;

OG_API og_status og_device_count(int32_t* count);
/* GpuBackends.CreateDevice (src/RecursiveAI.OneGpu.Backends/GpuBackends.cs:69-72) for the CUDA backend. */
OG_API og_status og_device_create(int32_t ordinal, og_device** out);
/* GpuDevice.Dispose: waits for the device's work, then releases it. */
OG_API og_status og_device_destroy(og_device* device);
OG_API og_status og_device_info_get(og_device* device, og_device_info* out);
/* GpuDevice.WaitIdle. Also reports (once) a failure a kernel recorded since the last check. */
OG_API og_status og_device_wait_idle(og_device* device);
/* Watchdog self-test (no counterpart in the reference, whose device-lost and watchdog failures come from the
 * driver: GpuDevice.cs:337-377). Queues on the device's stream a kernel whose bounded wait on an mbarrier, the same
 * wait every pipeline stage of the product kernels uses, runs out after limit_us microseconds (1 .. 2,000,000)
 * because nothing ever arrives. The kernel then raises the device's failure word and returns, exactly as a product
 * kernel whose pipeline stalled would; the next og_device_wait_idle or readback reports OG_ERROR_COMMAND_FAILED
 * (GpuCommandFailedException, reason Watchdog), clears the word, and the device stays usable. */
OG_API og_status og_device_watchdog_selftest(og_device* device, uint32_t limit_us);
/* The cudaStream_t submissions run on; og_device_set_stream binds an external one (e.g. a framework's). */
OG_API og_status og_device_stream(og_device* device, void** stream);
OG_API og_status og_device_set_stream(og_device* device, void* stream);

/* GpuDevice.CreateBuffer<T> / GpuBuffer.Dispose: device memory. Free is stream-ordered: it happens once the work
 * submitted before it has finished (GpuBufferOfT.cs:77-78). */
OG_API og_status og_buffer_alloc(og_device* device, uint64_t bytes, void** ptr);
OG_API og_status og_buffer_free(og_device* device, void* ptr);
/* GpuDevice.WriteBuffer: the upload runs before any later submission (GpuDevice.cs:163-167). */
OG_API og_status og_buffer_write(og_device* device, void* dst, const void* host_src, uint64_t bytes);
/* GpuBuffer<T>.ReadAsync (GpuBufferOfT.cs:63-75) completed synchronously: returns after all prior work and the copy. */
OG_API og_status og_buffer_read(og_device* device, void* host_dst, const void* src, uint64_t bytes);
/* Asynchronous transfers on the device's copy engines (no counterpart in the reference's API beyond
 * GpuBuffer<T>.ReadAsync being asynchronous, GpuBufferOfT.cs:63-75), so that uploads, products and readbacks of
 * consecutive steps overlap.
 * og_buffer_write_async: the copy runs on the upload stream as soon as possible, possibly while work submitted
 * earlier still runs - the caller guarantees that no submitted work still reads or writes `dst`; work submitted
 * afterwards waits for the copy. `host_src` should be page-locked (og_host_alloc) for the copy to be asynchronous. */
typedef struct og_readback og_readback;
OG_API og_status og_buffer_write_async(og_device* device, void* dst, const void* host_src, uint64_t bytes);
/* og_buffer_read_async: queues, on the readback stream, the copy of `bytes` from `src` to page-locked host memory
 * after all work submitted so far, without blocking the caller or later submissions; og_readback_wait blocks until
 * that copy has finished (reporting OG_ERROR_COMMAND_FAILED if a kernel before it gave up a bounded wait) and
 * releases the ticket. */
OG_API og_status og_buffer_read_async(og_device* device, void* host_dst, const void* src, uint64_t bytes,
                                      og_readback** ticket);
OG_API og_status og_readback_wait(og_readback* ticket);
/* Fills bytes of a buffer with a value, in stream order. */
OG_API og_status og_buffer_fill(og_device* device, void* dst, int32_t value, uint64_t bytes);
/* Page-locked host memory for fast uploads and readbacks. */
OG_API og_status og_host_alloc(uint64_t bytes, void** ptr);
OG_API og_status og_host_free(void* ptr);

/* ---- encoders and timestamps (GpuCommandEncoder, Resources.cs:148-243; GpuTimestampSet, GpuDevice.cs:103-109) ---- */

/* GpuDevice.BeginCommands. */
OG_API og_status og_encoder_begin(og_device* device, og_encoder** out);
/* GpuDevice.Submit (GpuDevice.cs:161): replays the recorded work in order on the device stream; consumes the
 * encoder whatever the outcome. */
OG_API og_status og_device_submit(og_device* device, og_encoder* encoder);
OG_API og_status og_encoder_discard(og_encoder* encoder);
/* Number of kernel launches the encoder holds (GpuCommandEncoder.DispatchCount), as planned when the work was
 * recorded: a DynamicQuantizeLinear counted as its one cooperative kernel runs as two kernels instead if the device
 * refuses the cooperative launch when the encoder is submitted (fewer SMs available than at recording). */
OG_API og_status og_encoder_dispatch_count(og_encoder* encoder, int64_t* count);

OG_API og_status og_timestamps_create(og_device* device, uint32_t count, og_timestamps** out);
OG_API og_status og_timestamps_destroy(og_timestamps* set);
/* Records timestamp `index` at this point of the encoder (between recorded operations). */
OG_API og_status og_encoder_timestamp(og_encoder* encoder, og_timestamps* set, uint32_t index);
/* Records timestamp `index` on the device stream now (outside any encoder), e.g. around uploads and readbacks. */
OG_API og_status og_device_timestamp(og_device* device, og_timestamps* set, uint32_t index);
/* GpuDevice.TryReadTimestamps: nanoseconds of each timestamp relative to timestamp `first`; waits for them. */
OG_API og_status og_timestamps_read(og_timestamps* set, uint32_t first, uint32_t count, double* ns);

/* ---- CUDA graphs of submitted work (no counterpart in the reference, whose encoders are re-submitted) ------------
 * Launch-bound work such as a decode step is recorded once and replayed as one graph launch. Between
 * og_device_capture_begin and og_device_capture_end the device stream is captured (relaxed mode): work submitted to
 * the device then (og_device_submit, og_device_timestamp, og_buffer_fill) is recorded, not run. Encode and submit
 * the same work once before capturing it: a kernel instance's first encoding of a shape may allocate and clear its
 * scratch, which a capture would refuse. Calls that wait for the device (og_device_wait_idle, the blocking
 * transfers) fail while a capture is open. A graph reads and writes the buffers it was recorded with, as
 * they are when it is launched; it must not outlive them or the kernel instances (Int8Gemm, ...) that recorded it. */
typedef struct og_graph og_graph;
OG_API og_status og_device_capture_begin(og_device* device);
OG_API og_status og_device_capture_end(og_device* device, og_graph** out);
/* Replays the graph on its device's stream, in stream order with other submitted work. */
OG_API og_status og_graph_launch(og_graph* graph);
OG_API og_status og_graph_destroy(og_graph* graph);

/* ---- Int8Gemm (src/RecursiveAI.OneGpu.Kernels/Int8Gemm.cs:124-683) --------------------------------------------- */

typedef struct og_int8_gemm og_int8_gemm;

/* Int8GemmProblem (Int8Gemm.cs:43-95). Lda/Ldb 0 = dense. OffsetA/OffsetB/StrideA/StrideB in bytes, OffsetC in
 * elements of the output. */
typedef struct og_int8_gemm_problem {
    int32_t m, n, k, batch;
    int32_t transpose_b;
    int32_t lda, ldb;
    int32_t offset_a, offset_b, offset_c;
    int32_t stride_a, stride_b;
} og_int8_gemm_problem;

/* Kernel choice for og_int8_gemm_options.kernel (a test hook like Int8GemmOptions.Tile, Int8Gemm.cs:15-19). */
typedef enum og_int8_kernel {
    OG_KERNEL_AUTO = 0,         /* tensor cores when the operands allow, else the portable kernel */
    OG_KERNEL_TENSOR_CORE = 1,  /* tcgen05 only; OG_ERROR_UNSUPPORTED when the operands do not allow it */
    OG_KERNEL_PORTABLE = 2      /* the SIMT kernel */
} og_int8_kernel;

/* Int8GemmOptions (Int8Gemm.cs:7-21). allow_packed_dot = 0 forces the portable variant, as in the reference.
 * tile is the test hook of Int8GemmOptions.Tile: 0 chooses by size, 128 forces the one-SM 128 x 256 tile, 256 the
 * two-SM (CTA pair) 256 x 256 tile of the tensor-core kernel. */
typedef struct og_int8_gemm_options {
    int32_t allow_packed_dot;
    int32_t kernel;
    int32_t tile;
    int32_t stream_k;  /* test hook: 0 and 1 give every SM pair whole tiles; 2 splits the (tile, K block) work evenly
                        * across the SM pairs (stream-K) whenever the shape allows */
} og_int8_gemm_options;

/* new Int8Gemm(device, options) (Int8Gemm.cs:153-177). options may be NULL (defaults). */
OG_API og_status og_int8_gemm_create(og_device* device, const og_int8_gemm_options* options, og_int8_gemm** out);
/* Int8Gemm.Dispose (Int8Gemm.cs:378-391): waits for the device, releases the instance's scratch. */
OG_API og_status og_int8_gemm_destroy(og_int8_gemm* gemm);
/* Int8Gemm.Variant (Int8Gemm.cs:215). */
OG_API og_status og_int8_gemm_variant(og_int8_gemm* gemm, char* buffer, uint64_t capacity);
/* The kernel the last encode call recorded: "tensor-core-2sm" or "tensor-core-1sm" (with "-stream-k" when the
 * product's (tile, K block) work was split evenly across the SMs), "tensor-core-rows", "portable" or "none". */
OG_API og_status og_int8_gemm_last_kernel(og_int8_gemm* gemm, char* buffer, uint64_t capacity);
/* Int8Gemm.ScratchElements (Int8Gemm.cs:531). */
OG_API int64_t og_int8_gemm_scratch_elements(const og_int8_gemm_problem* problem);
/* Int8Gemm.ReserveScratch (Int8Gemm.cs:539-549): OG_ERROR_ARGUMENT_RANGE when negative or above int.MaxValue. */
OG_API og_status og_int8_gemm_reserve_scratch(og_int8_gemm* gemm, int64_t elements);
/* Int8Gemm.BindGroupsCreated (Int8Gemm.cs:366): always 0 on CUDA, where kernel arguments are passed by value. */
OG_API og_status og_int8_gemm_bind_groups_created(og_int8_gemm* gemm, int32_t* count);

/* Int8Gemm.EncodeInt32<TA,TB> (Int8Gemm.cs:230-253). zero_point_a / zero_point_b / bias may be NULL. */
OG_API og_status og_int8_gemm_encode_int32(og_int8_gemm* gemm, og_encoder* encoder, const og_int8_gemm_problem* problem,
                                           const og_buffer* a, const og_buffer* b, const og_buffer* c,
                                           const og_operand* zero_point_a, const og_operand* zero_point_b,
                                           const og_operand* bias);
/* Int8Gemm.EncodeFloat<TA,TB> (Int8Gemm.cs:270-314). */
OG_API og_status og_int8_gemm_encode_float(og_int8_gemm* gemm, og_encoder* encoder, const og_int8_gemm_problem* problem,
                                           const og_buffer* a, const og_buffer* b, const og_buffer* c,
                                           const og_operand* scale, const og_operand* zero_point_a,
                                           const og_operand* zero_point_b, const og_operand* float_bias,
                                           const og_operand* int_bias);
/* MatMulIntegerToFloat in one call: float(sum + intBias) * (aScale * bScale[n]) (+ floatBias[n]), the scale product
 * formed in the epilogue with the same float32 rounding as the reference's chain, which forms it in a pass of its own
 * (ElementwiseKernels.EncodeBinary(Mul), tests/RecursiveAI.OneGpu.Kernels.Tests/Int8Tests.cs:733-739) and hands it to
 * EncodeFloat (Int8Gemm.cs:270-314). aScale is one float (e.g. the scale DynamicQuantizeLinear wrote on the device);
 * bScale is one value or one per column. Checks as EncodeFloat, argument names "aScale" and "bScale". */
OG_API og_status og_int8_gemm_encode_dequantize(og_int8_gemm* gemm, og_encoder* encoder,
                                                const og_int8_gemm_problem* problem, const og_buffer* a,
                                                const og_buffer* b, const og_buffer* c, const og_operand* a_scale,
                                                const og_operand* b_scale, const og_operand* zero_point_a,
                                                const og_operand* zero_point_b, const og_operand* float_bias,
                                                const og_operand* int_bias);
/* Int8Gemm.EncodeRequantized<TA,TB,TY> (Int8Gemm.cs:336-363). scratch (Int8Scratch, Int8Gemm.cs:37) may be NULL; its
 * buffer is an int32 buffer and its offset an element offset. */
OG_API og_status og_int8_gemm_encode_requantized(og_int8_gemm* gemm, og_encoder* encoder,
                                                 const og_int8_gemm_problem* problem, const og_buffer* a,
                                                 const og_buffer* b, const og_buffer* y, const og_operand* multiplier,
                                                 int32_t zero_point_y, const og_operand* zero_point_a,
                                                 const og_operand* zero_point_b, const og_operand* int_bias,
                                                 const og_operand* scratch);

/* EncodeInt32 for callers that cannot allocate device memory. No counterpart in the reference.
 * Some callers cannot call cudaMalloc while they run products: serving hosts that reserve all of a GPU's memory for
 * their own pool at start-up, engines whose execution step only hands a kernel pre-sized workspaces and forbids
 * allocating inside it, and latency-bound loops (a decode step) that cannot afford cudaMalloc's implicit device
 * synchronisation. Int8Gemm allocates the scratch of the zero-point byte sums on demand; this entry point allocates
 * nothing (no cudaMalloc, no cudaFree, no allocating library call) and keeps those sums in a fixed array of the
 * library instead: at most 1,048,576 int32 (4 MiB, held on every GPU that loads the library until exit), i.e.
 * batchA * M (when B has a zero point) + batchB * N (when A has one); a product needing more is refused with
 * OG_ERROR_UNSUPPORTED (capability "NoAllocScratch"). It runs the product on `stream` (a cudaStream_t, NULL for the
 * default stream) of the current device, after the same checks as og_int8_gemm_encode_int32 and with the same
 * kernels, and returns once the work is queued; a kernel whose bounded wait gave up is reported by
 * og_int8_gemm_noalloc_status. The first call on a device (of this entry point or of the two below) looks up the
 * array's device address (cudaGetSymbolAddress, checked) and the SM count: make that first call before any stream
 * capture. The first product of each kernel kind on a device also sets that kernel's shared-memory limit. All calls
 * share the array and it keeps the last call's contents (what must start at zero is cleared on the stream before
 * use); calls whose work overlaps on the GPU (unordered streams) race on it. */
OG_API og_status og_int8_gemm_int32_noalloc(void* stream, const og_int8_gemm_problem* problem, const og_buffer* a,
                                            const og_buffer* b, const og_buffer* c, const og_operand* zero_point_a,
                                            const og_operand* zero_point_b, const og_operand* bias);
/* The failure word of the allocation-free products on the current device (companion of og_int8_gemm_int32_noalloc,
 * no counterpart in the reference): waits for `stream`, then returns OG_ERROR_COMMAND_FAILED (capability "Watchdog")
 * if a kernel of such a product gave up a bounded wait and skipped its work since the last check, clearing the word;
 * OG_OK otherwise. Allocates nothing. */
OG_API og_status og_int8_gemm_noalloc_status(void* stream);
/* Queues on `stream` a kernel whose bounded wait (limit_us, 1 .. 2000000) runs out and raises the allocation-free
 * products' failure word, the way a stalled product kernel does (no fault, nothing left in flight): tests use it to
 * check that og_int8_gemm_noalloc_status reports such a failure. No counterpart in the reference. */
OG_API og_status og_int8_gemm_noalloc_watchdog_selftest(void* stream, uint32_t limit_us);

/* The argument checks of the three forms alone (no device needed): the same checks, in the same order, that the
 * encode functions run before recording (Int8Gemm.cs:230-253, 270-314, 336-363, 419-501). */
OG_API og_status og_int8_gemm_check_int32(const og_int8_gemm_problem* problem, const og_buffer* a, const og_buffer* b,
                                          const og_buffer* c, const og_operand* zero_point_a,
                                          const og_operand* zero_point_b, const og_operand* bias);
OG_API og_status og_int8_gemm_check_float(const og_int8_gemm_problem* problem, const og_buffer* a, const og_buffer* b,
                                          const og_buffer* c, const og_operand* scale, const og_operand* zero_point_a,
                                          const og_operand* zero_point_b, const og_operand* float_bias,
                                          const og_operand* int_bias);
OG_API og_status og_int8_gemm_check_dequantize(const og_int8_gemm_problem* problem, const og_buffer* a,
                                               const og_buffer* b, const og_buffer* c, const og_operand* a_scale,
                                               const og_operand* b_scale, const og_operand* zero_point_a,
                                               const og_operand* zero_point_b, const og_operand* float_bias,
                                               const og_operand* int_bias);
OG_API og_status og_int8_gemm_check_requantized(const og_int8_gemm_problem* problem, const og_buffer* a,
                                                const og_buffer* b, const og_buffer* y, const og_operand* multiplier,
                                                int32_t zero_point_y, const og_operand* zero_point_a,
                                                const og_operand* zero_point_b, const og_operand* int_bias,
                                                const og_operand* scratch);

/* ---- DynamicQuantizeKernels (src/RecursiveAI.OneGpu.Kernels/DynamicQuantizeKernels.cs:20-110) ------------------- */

typedef struct og_dynamic_quantize og_dynamic_quantize;

/* new DynamicQuantizeKernels(device) (DynamicQuantizeKernels.cs:36-45): keeps a small partials buffer. */
OG_API og_status og_dynamic_quantize_create(og_device* device, og_dynamic_quantize** out);
OG_API og_status og_dynamic_quantize_destroy(og_dynamic_quantize* dq);
/* DynamicQuantizeKernels.Encode (DynamicQuantizeKernels.cs:59-90): x float32, y uint8, scale float32, zeroPoint
 * uint8 (only the byte at offset_zero_point is written). */
OG_API og_status og_dynamic_quantize_encode(og_dynamic_quantize* dq, og_encoder* encoder, const og_buffer* x,
                                            int32_t offset_x, int32_t count, const og_buffer* y, int32_t offset_y,
                                            const og_buffer* scale, int32_t offset_scale, const og_buffer* zero_point,
                                            int32_t offset_zero_point);
/* The checks of Encode alone (DynamicQuantizeKernels.cs:61-75). */
OG_API og_status og_dynamic_quantize_check(const og_buffer* x, int32_t offset_x, int32_t count, const og_buffer* y,
                                           int32_t offset_y, const og_buffer* scale, int32_t offset_scale,
                                           const og_buffer* zero_point, int32_t offset_zero_point);

/* ---- DequantizeKernels (src/RecursiveAI.OneGpu.Kernels/DequantizeKernels.cs:29-298) ------------------------------ */

typedef struct og_dequantize og_dequantize;

/* new DequantizeKernels(device) (DequantizeKernels.cs:46-51). */
OG_API og_status og_dequantize_create(og_device* device, og_dequantize** out);
OG_API og_status og_dequantize_destroy(og_dequantize* kernels);
/* DequantizeKernels.Encode<TIn, TOut> (DequantizeKernels.cs:69-130), ONNX DequantizeLinear:
 * output = float(x - zeroPoint) * scale. x is uint8, int8 or int32 (TIn); output float32 or half (TOut); scale float32;
 * zero_point (nullable) has x's type. shape has `rank` dimensions; with per_axis the scale and zero point hold one
 * value per index of `axis` (in [-rank, rank)), otherwise one value. Offsets are in elements. */
OG_API og_status og_dequantize_encode(og_dequantize* kernels, og_encoder* encoder, const og_buffer* x, int32_t offset_x,
                                      const int32_t* shape, int32_t rank, int32_t axis, int32_t per_axis,
                                      const og_buffer* scale, int32_t offset_scale, const og_buffer* zero_point,
                                      int32_t offset_zero_point, const og_buffer* output, int32_t offset_output);
/* DequantizeKernels.EncodeQuantize<TIn, TOut> (DequantizeKernels.cs:184-240), ONNX QuantizeLinear:
 * output = saturate(round_half_even(x / scale) + zeroPoint), NaN to the lowest value. x float32 or half (TIn); output
 * uint8 or int8 (TOut); zero_point (nullable) has the output's type. */
OG_API og_status og_dequantize_encode_quantize(og_dequantize* kernels, og_encoder* encoder, const og_buffer* x,
                                               int32_t offset_x, const int32_t* shape, int32_t rank, int32_t axis,
                                               int32_t per_axis, const og_buffer* scale, int32_t offset_scale,
                                               const og_buffer* zero_point, int32_t offset_zero_point,
                                               const og_buffer* output, int32_t offset_output);
/* The checks of DequantizeKernels.Encode / EncodeQuantize alone, in the reference's order. */
OG_API og_status og_dequantize_check(const og_buffer* x, int32_t offset_x, const int32_t* shape, int32_t rank,
                                     int32_t axis, int32_t per_axis, const og_buffer* scale, int32_t offset_scale,
                                     const og_buffer* zero_point, int32_t offset_zero_point, const og_buffer* output,
                                     int32_t offset_output);
OG_API og_status og_dequantize_check_quantize(const og_buffer* x, int32_t offset_x, const int32_t* shape,
                                              int32_t rank, int32_t axis, int32_t per_axis, const og_buffer* scale,
                                              int32_t offset_scale, const og_buffer* zero_point,
                                              int32_t offset_zero_point, const og_buffer* output,
                                              int32_t offset_output);

/* ---- ConvIntegerKernels (src/RecursiveAI.OneGpu.Kernels/ConvIntegerKernels.cs:25-351) --------------------------- */

/* ConvProblem (src/RecursiveAI.OneGpu.Kernels/ConvProblem.cs): NCHW input, OIHW weights, strides, dilations,
 * asymmetric padding, groups; offsets in elements. activation must be 0; offset_bias / offset_residual are unused. A
 * 1-D convolution is height 1 (ConvProblem.Conv1D). */
typedef struct og_conv_problem {
    int32_t batch, in_channels, height, width, out_channels, kernel_height, kernel_width;
    int32_t stride_height, stride_width, dilation_height, dilation_width;
    int32_t pad_top, pad_left, pad_bottom, pad_right;
    int32_t groups;
    int32_t activation;
    int32_t offset_x, offset_w, offset_bias, offset_residual, offset_y;
} og_conv_problem;

typedef struct og_conv_integer og_conv_integer;

/* new ConvIntegerKernels(device, options) (ConvIntegerKernels.cs:46-63): options of the underlying Int8Gemm, NULL for
 * the defaults. */
OG_API og_status og_conv_integer_create(og_device* device, const og_int8_gemm_options* options, og_conv_integer** out);
OG_API og_status og_conv_integer_destroy(og_conv_integer* conv);
/* ConvIntegerKernels.Variant (ConvIntegerKernels.cs:66): the underlying product's variant. */
OG_API og_status og_conv_integer_variant(og_conv_integer* conv, char* buffer, uint64_t capacity);
/* ConvIntegerKernels.BindGroupsCreated (ConvIntegerKernels.cs:69): the product's count plus the device buffers the
 * instance allocated; a warm call with a problem already seen adds nothing. */
OG_API og_status og_conv_integer_bind_groups_created(og_conv_integer* conv, int32_t* count);
/* ConvIntegerKernels.ScratchBytesPerImage (ConvIntegerKernels.cs:79-83): Groups * K * ceil(OH * OW / 4) * 4. Scratch
 * of this size per image runs the problem; a buffer that also holds the 16-byte-padded rows
 * (Groups * K * ceil(OH * OW / 16) * 16 per image) keeps the product on the tensor cores. */
OG_API og_status og_conv_integer_scratch_bytes_per_image(const og_conv_problem* problem, int64_t* bytes);
/* ConvIntegerKernels.Encode<TX, TW> (ConvIntegerKernels.cs:104-264): x and w uint8 / int8 in any mix, y int32;
 * x_zero_point one value of x's type, w_zero_point one value or one per output channel of w's type (either NULL for
 * 0); scratch (NULL: the instance's own) has x's type and scratch_offset is a non-negative multiple of 4. */
OG_API og_status og_conv_integer_encode(og_conv_integer* conv, og_encoder* encoder, const og_conv_problem* problem,
                                        const og_buffer* x, const og_buffer* w, const og_buffer* y,
                                        const og_operand* x_zero_point, const og_operand* w_zero_point,
                                        const og_buffer* scratch, int32_t scratch_offset);
/* The checks of Encode alone, in the reference's order. */
OG_API og_status og_conv_integer_check(const og_conv_problem* problem, const og_buffer* x, const og_buffer* w,
                                       const og_buffer* y, const og_operand* x_zero_point,
                                       const og_operand* w_zero_point, const og_buffer* scratch,
                                       int32_t scratch_offset);

/* ---- Several GPUs of one node: NCCL over NVLink (no counterpart in the reference, whose devices never exchange
 * data: MultiDeviceTests.cs:6-107) -------------------------------------------------------------------------------
 * The product shards with no reduction (by batch, or by column slabs of B), so no collective runs inside it. These
 * calls move what surrounds it: the column shards of a result gathered onto the one device that needs the whole
 * result, and an operand that every rank uploaded one part of replicated onto all ranks. One og_comm per device
 * (one process or thread per GPU); every call is queued on that device's stream, in order with submitted work, and
 * every rank makes the same calls in the same order. NCCL (libnccl.so.2) is loaded at the first call; without it the
 * calls fail with OG_ERROR_UNSUPPORTED (capability "NCCL"). */
#define OG_COMM_ID_BYTES 128
typedef struct og_comm og_comm;
/* A new communicator id (NCCL's unique id): made by one rank and handed to all the others by the host. */
OG_API og_status og_comm_unique_id(uint8_t* id /* OG_COMM_ID_BYTES */);
/* Joins rank `rank` of `nranks` on `device`; every rank calls it with the same id, concurrently. */
OG_API og_status og_comm_create(og_device* device, int32_t nranks, int32_t rank, const uint8_t* id, og_comm** out);
/* Waits for the device's stream, then releases the communicator and its staging memory. */
OG_API og_status og_comm_destroy(og_comm* comm);
/* Gathers the column shards of a dense result [batch][m][N] (N = the sum of widths[0 .. nranks-1]) onto `root`:
 * rank r passes its shard [batch][m][widths[r]] (columns [widths[0] + ... + widths[r-1], + widths[r]) of the result)
 * as `shard`, elements of elem_bytes bytes (1, 2, 4 or 8); root also passes the whole result `out`. The other ranks'
 * shards arrive over NVLink into a staging buffer of the communicator and are put in place by one kernel. */
OG_API og_status og_comm_gather_columns(og_comm* comm, const void* shard, int32_t elem_bytes, int32_t batch, int32_t m,
                                        const int32_t* widths, void* out, int32_t root);
/* ncclAllGather: recv (nranks * bytes) receives every rank's `bytes` of send, in rank order. */
OG_API og_status og_comm_all_gather(og_comm* comm, const void* send, uint64_t bytes, void* recv);

#ifdef __cplusplus
}
#endif

#endif /* ONEGPU_CUDA_H */
