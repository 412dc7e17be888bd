// P/Invoke declarations of libonegpu_cuda.so (include/onegpu_cuda.h): one [LibraryImport] per exported entry point,
// and the structs the entry points take, laid out as in the header. The project needs AllowUnsafeBlocks=true and
// runtime marshalling disabled (as the reference's Vulkan loader does), since every argument is a plain pointer or
// value.
using System.Runtime.CompilerServices;
using System.Runtime.InteropServices;

[assembly: DisableRuntimeMarshalling]

namespace RecursiveAI.OneGpu.Cuda;

[StructLayout(LayoutKind.Sequential)]
internal struct OgBuffer { public nint Ptr; public long Length; public int Type; }              // og_buffer

[StructLayout(LayoutKind.Sequential)]
internal struct OgOperand { public OgBuffer Buffer; public int Offset; public int IsVector; }   // og_operand

[StructLayout(LayoutKind.Sequential)]
internal struct OgProblem                                                                      // og_int8_gemm_problem
{
    public int M, N, K, Batch, TransposeB, Lda, Ldb, OffsetA, OffsetB, OffsetC, StrideA, StrideB;
}

[StructLayout(LayoutKind.Sequential)]
internal struct OgOptions { public int AllowPackedDot, Kernel, Tile, StreamK; }                // og_int8_gemm_options

[StructLayout(LayoutKind.Sequential)]
internal struct OgConvProblem                                                                  // og_conv_problem
{
    public int Batch, InChannels, Height, Width, OutChannels, KernelHeight, KernelWidth;
    public int StrideHeight, StrideWidth, DilationHeight, DilationWidth, PadTop, PadLeft, PadBottom, PadRight;
    public int Groups, Activation, OffsetX, OffsetW, OffsetBias, OffsetResidual, OffsetY;
}

[StructLayout(LayoutKind.Sequential)]
internal unsafe struct OgErrorInfo                                                             // og_error_info
{
    public int Status;
    public fixed byte Operation[64], Argument[64], Message[512], Capability[64], Expected[128], Actual[128];
}

[StructLayout(LayoutKind.Sequential)]
internal unsafe struct OgDeviceInfo                                                            // og_device_info
{
    public fixed byte Name[256];
    public int Ordinal, SmCount, CcMajor, CcMinor;
    public long TotalMemory;
    public int MaxSharedMemoryPerBlock, TensorCoreI8;
}

internal static unsafe partial class Native
{
    const string Lib = "onegpu_cuda";   // libonegpu_cuda.so next to the assembly

    [LibraryImport(Lib)] internal static partial int og_last_error(OgErrorInfo* info);
    [LibraryImport(Lib)] internal static partial int og_device_count(int* count);
    [LibraryImport(Lib)] internal static partial int og_device_create(int ordinal, nint* device);
    [LibraryImport(Lib)] internal static partial int og_device_destroy(nint device);
    [LibraryImport(Lib)] internal static partial int og_device_wait_idle(nint device);
    [LibraryImport(Lib)] internal static partial int og_device_info_get(nint device, OgDeviceInfo* info);
    [LibraryImport(Lib)] internal static partial int og_device_stream(nint device, nint* stream);
    [LibraryImport(Lib)] internal static partial int og_device_set_stream(nint device, nint stream);
    [LibraryImport(Lib)] internal static partial int og_device_watchdog_selftest(nint device, uint limitUs);
    [LibraryImport(Lib)] internal static partial int og_buffer_alloc(nint device, ulong bytes, nint* ptr);
    [LibraryImport(Lib)] internal static partial int og_buffer_free(nint device, nint ptr);
    [LibraryImport(Lib)] internal static partial int og_buffer_write(nint device, nint dst, void* src, ulong bytes);
    [LibraryImport(Lib)] internal static partial int og_buffer_read(nint device, void* dst, nint src, ulong bytes);
    [LibraryImport(Lib)] internal static partial int og_buffer_fill(nint device, nint dst, int value, ulong bytes);
    [LibraryImport(Lib)] internal static partial int og_host_alloc(ulong bytes, void** ptr);
    [LibraryImport(Lib)] internal static partial int og_host_free(void* ptr);
    [LibraryImport(Lib)] internal static partial int og_buffer_write_async(nint device, nint dst, void* src,
        ulong bytes);
    [LibraryImport(Lib)] internal static partial int og_buffer_read_async(nint device, void* dst, nint src,
        ulong bytes, nint* ticket);
    [LibraryImport(Lib)] internal static partial int og_readback_wait(nint ticket);
    [LibraryImport(Lib)] internal static partial int og_device_capture_begin(nint device);
    [LibraryImport(Lib)] internal static partial int og_device_capture_end(nint device, nint* graph);
    [LibraryImport(Lib)] internal static partial int og_graph_launch(nint graph);
    [LibraryImport(Lib)] internal static partial int og_graph_destroy(nint graph);
    [LibraryImport(Lib)] internal static partial int og_encoder_begin(nint device, nint* encoder);
    [LibraryImport(Lib)] internal static partial int og_device_submit(nint device, nint encoder);
    [LibraryImport(Lib)] internal static partial int og_encoder_discard(nint encoder);
    [LibraryImport(Lib)] internal static partial int og_encoder_dispatch_count(nint encoder, long* count);
    [LibraryImport(Lib)] internal static partial int og_timestamps_create(nint device, uint count, nint* set);
    [LibraryImport(Lib)] internal static partial int og_encoder_timestamp(nint encoder, nint set, uint index);
    [LibraryImport(Lib)] internal static partial int og_timestamps_read(nint set, uint first, uint count, double* ns);
    [LibraryImport(Lib)] internal static partial int og_device_timestamp(nint device, nint set, uint index);
    [LibraryImport(Lib)] internal static partial int og_timestamps_destroy(nint set);

    [LibraryImport(Lib)] internal static partial int og_int8_gemm_create(nint device, OgOptions* options, nint* gemm);
    [LibraryImport(Lib)] internal static partial int og_int8_gemm_destroy(nint gemm);
    [LibraryImport(Lib)] internal static partial int og_int8_gemm_variant(nint gemm, byte* buffer, ulong capacity);
    [LibraryImport(Lib)] internal static partial int og_int8_gemm_last_kernel(nint gemm, byte* buffer, ulong capacity);
    [LibraryImport(Lib)] internal static partial int og_int8_gemm_bind_groups_created(nint gemm, int* count);
    [LibraryImport(Lib)] internal static partial long og_int8_gemm_scratch_elements(OgProblem* problem);
    [LibraryImport(Lib)] internal static partial int og_int8_gemm_reserve_scratch(nint gemm, long elements);
    [LibraryImport(Lib)] internal static partial int og_int8_gemm_encode_int32(nint gemm, nint encoder, OgProblem* p,
        OgBuffer* a, OgBuffer* b, OgBuffer* c, OgOperand* zpA, OgOperand* zpB, OgOperand* bias);
    [LibraryImport(Lib)] internal static partial int og_int8_gemm_encode_float(nint gemm, nint encoder, OgProblem* p,
        OgBuffer* a, OgBuffer* b, OgBuffer* c, OgOperand* scale, OgOperand* zpA, OgOperand* zpB,
        OgOperand* floatBias, OgOperand* intBias);
    [LibraryImport(Lib)] internal static partial int og_int8_gemm_encode_requantized(nint gemm, nint encoder,
        OgProblem* p, OgBuffer* a, OgBuffer* b, OgBuffer* y, OgOperand* multiplier, int zeroPointY,
        OgOperand* zpA, OgOperand* zpB, OgOperand* intBias, OgOperand* scratch);
    [LibraryImport(Lib)] internal static partial int og_int8_gemm_encode_dequantize(nint gemm, nint encoder,
        OgProblem* p, OgBuffer* a, OgBuffer* b, OgBuffer* c, OgOperand* aScale, OgOperand* bScale, OgOperand* zpA,
        OgOperand* zpB, OgOperand* floatBias, OgOperand* intBias);
    // EncodeInt32 queued straight onto a stream, using only memory the library reserved when it was loaded.
    [LibraryImport(Lib)] internal static partial int og_int8_gemm_int32_noalloc(nint stream, OgProblem* p,
        OgBuffer* a, OgBuffer* b, OgBuffer* c, OgOperand* zpA, OgOperand* zpB, OgOperand* bias);
    // Its failure word (a kernel that gave up a bounded wait), read back and cleared on the caller's stream.
    [LibraryImport(Lib)] internal static partial int og_int8_gemm_noalloc_status(nint stream);
    [LibraryImport(Lib)] internal static partial int og_int8_gemm_noalloc_watchdog_selftest(nint stream, uint limitUs);
    // The argument checks alone (no device), in the order the encode calls run them.
    [LibraryImport(Lib)] internal static partial int og_int8_gemm_check_int32(OgProblem* p, OgBuffer* a, OgBuffer* b,
        OgBuffer* c, OgOperand* zpA, OgOperand* zpB, OgOperand* bias);
    [LibraryImport(Lib)] internal static partial int og_int8_gemm_check_float(OgProblem* p, OgBuffer* a, OgBuffer* b,
        OgBuffer* c, OgOperand* scale, OgOperand* zpA, OgOperand* zpB, OgOperand* floatBias, OgOperand* intBias);
    [LibraryImport(Lib)] internal static partial int og_int8_gemm_check_dequantize(OgProblem* p, OgBuffer* a,
        OgBuffer* b, OgBuffer* c, OgOperand* aScale, OgOperand* bScale, OgOperand* zpA, OgOperand* zpB,
        OgOperand* floatBias, OgOperand* intBias);
    [LibraryImport(Lib)] internal static partial int og_int8_gemm_check_requantized(OgProblem* p, OgBuffer* a,
        OgBuffer* b, OgBuffer* y, OgOperand* multiplier, int zeroPointY, OgOperand* zpA, OgOperand* zpB,
        OgOperand* intBias, OgOperand* scratch);

    [LibraryImport(Lib)] internal static partial int og_dynamic_quantize_create(nint device, nint* dq);
    [LibraryImport(Lib)] internal static partial int og_dynamic_quantize_destroy(nint dq);
    [LibraryImport(Lib)] internal static partial int og_dynamic_quantize_encode(nint dq, nint encoder, OgBuffer* x,
        int offsetX, int count, OgBuffer* y, int offsetY, OgBuffer* scale, int offsetScale, OgBuffer* zeroPoint,
        int offsetZeroPoint);
    [LibraryImport(Lib)] internal static partial int og_dynamic_quantize_check(OgBuffer* x, int offsetX, int count,
        OgBuffer* y, int offsetY, OgBuffer* scale, int offsetScale, OgBuffer* zeroPoint, int offsetZeroPoint);

    [LibraryImport(Lib)] internal static partial int og_dequantize_create(nint device, nint* kernels);
    [LibraryImport(Lib)] internal static partial int og_dequantize_destroy(nint kernels);
    [LibraryImport(Lib)] internal static partial int og_dequantize_encode(nint kernels, nint encoder, OgBuffer* x,
        int offsetX, int* shape, int rank, int axis, int perAxis, OgBuffer* scale, int offsetScale,
        OgBuffer* zeroPoint, int offsetZeroPoint, OgBuffer* output, int offsetOutput);
    [LibraryImport(Lib)] internal static partial int og_dequantize_encode_quantize(nint kernels, nint encoder,
        OgBuffer* x, int offsetX, int* shape, int rank, int axis, int perAxis, OgBuffer* scale, int offsetScale,
        OgBuffer* zeroPoint, int offsetZeroPoint, OgBuffer* output, int offsetOutput);
    [LibraryImport(Lib)] internal static partial int og_dequantize_check(OgBuffer* x, int offsetX, int* shape,
        int rank, int axis, int perAxis, OgBuffer* scale, int offsetScale, OgBuffer* zeroPoint, int offsetZeroPoint,
        OgBuffer* output, int offsetOutput);
    [LibraryImport(Lib)] internal static partial int og_dequantize_check_quantize(OgBuffer* x, int offsetX,
        int* shape, int rank, int axis, int perAxis, OgBuffer* scale, int offsetScale, OgBuffer* zeroPoint,
        int offsetZeroPoint, OgBuffer* output, int offsetOutput);

    [LibraryImport(Lib)] internal static partial int og_conv_integer_create(nint device, OgOptions* options, nint* conv);
    [LibraryImport(Lib)] internal static partial int og_conv_integer_destroy(nint conv);
    [LibraryImport(Lib)] internal static partial int og_conv_integer_variant(nint conv, byte* buffer, ulong capacity);
    [LibraryImport(Lib)] internal static partial int og_conv_integer_bind_groups_created(nint conv, int* count);
    [LibraryImport(Lib)] internal static partial int og_conv_integer_scratch_bytes_per_image(OgConvProblem* p,
        long* bytes);
    [LibraryImport(Lib)] internal static partial int og_conv_integer_encode(nint conv, nint encoder, OgConvProblem* p,
        OgBuffer* x, OgBuffer* w, OgBuffer* y, OgOperand* xZeroPoint, OgOperand* wZeroPoint, OgBuffer* scratch,
        int scratchOffset);
    [LibraryImport(Lib)] internal static partial int og_conv_integer_check(OgConvProblem* p, OgBuffer* x, OgBuffer* w,
        OgBuffer* y, OgOperand* xZeroPoint, OgOperand* wZeroPoint, OgBuffer* scratch, int scratchOffset);

    // Several GPUs of one node (NCCL over NVLink): gathering column shards of a result, replicating an operand.
    [LibraryImport(Lib)] internal static partial int og_comm_unique_id(byte* id);
    [LibraryImport(Lib)] internal static partial int og_comm_create(nint device, int nranks, int rank, byte* id,
        nint* comm);
    [LibraryImport(Lib)] internal static partial int og_comm_destroy(nint comm);
    [LibraryImport(Lib)] internal static partial int og_comm_gather_columns(nint comm, nint shard, int elemBytes,
        int batch, int m, int* widths, nint output, int root);
    [LibraryImport(Lib)] internal static partial int og_comm_all_gather(nint comm, nint send, ulong bytes, nint recv);
}
