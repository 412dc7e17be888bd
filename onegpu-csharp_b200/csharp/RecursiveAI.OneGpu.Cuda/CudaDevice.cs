// The compute subset of GpuDevice on CUDA (src/RecursiveAI.OneGpu/GpuDevice.cs:27-228): buffers are device
// allocations of libonegpu_cuda.so, uploads and readbacks are ordered on the device's stream, encoders record library
// operations that Submit replays in order, and timestamps are CUDA events. Graphics members (textures, samplers,
// shaders, pipelines, swapchains) throw GpuUnsupportedException: the kernels of this backend are the library's own,
// not shaders. GpuBackend.Cuda is the one public API addition (an unshipped entry of src/RecursiveAI.OneGpu/Enums.cs).
using System.Runtime.InteropServices;

namespace RecursiveAI.OneGpu.Cuda;

/// <summary>Creates CUDA devices (one og_device per GPU; one thread uses a device at a time, as GpuDevice.cs:6
/// says of every backend).</summary>
public static unsafe class CudaGpu
{
    /// <summary>Number of CUDA devices visible to this process (0 without a driver).</summary>
    public static int DeviceCount
    {
        get
        {
            int n;
            NativeCheck.Check(Native.og_device_count(&n));
            return n;
        }
    }

    /// <summary>Opens CUDA device <paramref name="ordinal"/>; GpuUnsupportedException when there is none.</summary>
    public static GpuDevice CreateDevice(int ordinal = 0, GpuDeviceOptions? options = null)
    {
        nint handle;
        NativeCheck.Check(Native.og_device_create(ordinal, &handle));
        return new CudaDevice(handle);
    }
}

internal sealed unsafe class CudaDevice : GpuDevice
{
    internal nint Handle { get; private set; }
    readonly GpuAdapterInfo _adapter;
    readonly GpuCapabilities _caps;

    internal CudaDevice(nint handle)
    {
        Handle = handle;
        OgDeviceInfo info;
        NativeCheck.Check(Native.og_device_info_get(handle, &info));
        var name = Marshal.PtrToStringUTF8((nint)info.Name) ?? "CUDA device";
        _adapter = new GpuAdapterInfo(name, AdapterKind.Discrete, 0x10DE, 0, $"CUDA sm_{info.CcMajor}{info.CcMinor}");
        _caps = new GpuCapabilities(Timestamps: true, MultiDrawIndirect: false, IndirectFirstInstance: false,
                                    DepthClamp: false, DepthBiasClamp: false, NonUniformArrayIndexing: false,
                                    MaxSampleCount: 1, MaxTextureSize: 0, MaxTextureSize3D: 0, MaxArrayLayers: 0,
                                    MaxResourceArrayCount: 0) { PushConstants = false };
    }

    public override GpuAdapterInfo Adapter => _adapter;
    public override GpuBackend Backend => GpuBackend.Cuda;
    public override GpuCapabilities Capabilities => _caps;

    /// <summary>The cudaStream_t the device replays submitted work on.</summary>
    public nint Stream
    {
        get
        {
            nint s;
            NativeCheck.Check(Native.og_device_stream(Handle, &s));
            return s;
        }
    }

    public override GpuBuffer CreateBuffer(in BufferDesc desc)
    {
        nint ptr;
        NativeCheck.Check(Native.og_buffer_alloc(Handle, desc.Size, &ptr));
        return new CudaBuffer(this, ptr, desc.Size, desc.Usage, desc.Label);
    }

    public override GpuTimestampSet CreateTimestampSet(uint count)
    {
        nint set;
        NativeCheck.Check(Native.og_timestamps_create(Handle, count, &set));
        return new CudaTimestampSet(set, count);
    }

    public override bool TryReadTimestamps(GpuTimestampSet timestamps, uint first, Span<ulong> nanoseconds)
    {
        var set = (CudaTimestampSet)timestamps;
        var ns = new double[nanoseconds.Length];
        fixed (double* p = ns)
        {
            if (Native.og_timestamps_read(set.Handle, first, (uint)ns.Length, p) != NativeCheck.Ok) return false;
        }
        for (int i = 0; i < ns.Length; i++) nanoseconds[i] = (ulong)Math.Max(0.0, ns[i]);
        return true;
    }

    public override GpuCommandEncoder BeginCommands()
    {
        nint enc;
        NativeCheck.Check(Native.og_encoder_begin(Handle, &enc));
        return new CudaCommandEncoder(this, enc);
    }

    public override void Submit(GpuCommandEncoder commands)
    {
        var enc = (CudaCommandEncoder)commands;
        NativeCheck.Check(Native.og_device_submit(Handle, enc.TakeHandle()));
    }

    public override void WriteBuffer(GpuBuffer buffer, ulong offset, ReadOnlySpan<byte> data)
    {
        var b = (CudaBuffer)buffer;
        fixed (byte* p = data) NativeCheck.Check(Native.og_buffer_write(Handle, b.Pointer + (nint)offset, p, (ulong)data.Length));
    }

    public override void ReadBuffer(GpuBuffer buffer, ulong offset, Span<byte> destination)
    {
        var b = (CudaBuffer)buffer;
        fixed (byte* p = destination) NativeCheck.Check(Native.og_buffer_read(Handle, p, b.Pointer + (nint)offset, (ulong)destination.Length));
    }

    /// <summary>GpuBufferOfT.ReadAsync (GpuBufferOfT.cs:71-75): the copy is queued on the library's readback stream
    /// behind all work submitted so far, into page-locked staging, and the task completes on the thread pool once it
    /// has landed, so the caller can keep submitting meanwhile.</summary>
    public override ValueTask ReadBufferAsync(GpuBuffer buffer, ulong offset, Memory<byte> destination)
    {
        var b = (CudaBuffer)buffer;
        ulong bytes = (ulong)destination.Length;
        void* staging;
        NativeCheck.Check(Native.og_host_alloc(bytes, &staging));
        nint ticket;
        int st = Native.og_buffer_read_async(Handle, staging, b.Pointer + (nint)offset, bytes, &ticket);
        if (st != NativeCheck.Ok)
        {
            Native.og_host_free(staging);
            NativeCheck.Check(st);
        }
        nint stagingPtr = (nint)staging;
        return new ValueTask(Task.Run(() =>
        {
            try
            {
                NativeCheck.Check(Native.og_readback_wait(ticket));
                new ReadOnlySpan<byte>((void*)stagingPtr, (int)bytes).CopyTo(destination.Span);
            }
            finally
            {
                Native.og_host_free((void*)stagingPtr);
            }
        }));
    }

    public override void WaitIdle() => NativeCheck.Check(Native.og_device_wait_idle(Handle));

    public override string[] TakeValidationMessages() => [];

    public override void Dispose()
    {
        if (Handle == 0) return;
        Native.og_device_destroy(Handle);
        Handle = 0;
    }

    // ---- graphics members: not part of a compute backend -------------------------------------------------------

    static GpuUnsupportedException NoGraphics(string what) =>
        new($"the CUDA backend has no {what}: it runs the library's compute kernels only", "Graphics",
            "a graphics backend (Vulkan, Metal, WebGPU)", "CUDA");

    public override GpuTexture CreateTexture(in TextureDesc desc) => throw NoGraphics("textures");
    public override GpuSampler CreateSampler(in SamplerDesc desc) => throw NoGraphics("samplers");
    public override GpuShader CreateShader(ShaderStage stage, ReadOnlySpan<byte> spirv, string entryPoint) =>
        throw NoGraphics("shaders");
    public override GpuPipelineLayout CreatePipelineLayout(ReadOnlySpan<ResourceBinding> bindings) =>
        throw NoGraphics("pipeline layouts");
    public override GpuPipelineLayout CreatePipelineLayout(ReadOnlySpan<ResourceBinding> bindings,
                                                           in PushConstantRange pushConstants) =>
        throw NoGraphics("pipeline layouts");
    public override GpuBindGroup CreateBindGroup(GpuPipelineLayout layout, uint setIndex,
                                                 ReadOnlySpan<BindGroupEntry> entries) =>
        throw NoGraphics("bind groups");
    public override GpuGraphicsPipeline CreateGraphicsPipeline(GraphicsPipelineDesc desc) =>
        throw NoGraphics("graphics pipelines");
    public override GpuComputePipeline CreateComputePipeline(ComputePipelineDesc desc) =>
        throw NoGraphics("shader compute pipelines");
    public override GpuSwapchain CreateSwapchain(in SurfaceSource surface, in SwapchainDesc desc) =>
        throw NoGraphics("swapchains");
    public override void WriteTexture(GpuTexture texture, uint mipLevel, uint layer, ReadOnlySpan<byte> data) =>
        throw NoGraphics("textures");
    public override void WriteTexture(GpuTexture texture, in TextureRegion region, ReadOnlySpan<byte> data) =>
        throw NoGraphics("textures");
    public override void ReadTexture(GpuTexture texture, uint mipLevel, uint layer, Span<byte> destination) =>
        throw NoGraphics("textures");
}

/// <summary>A device allocation (og_buffer_alloc). Dispose frees it in stream order, once the GPU has finished with
/// it (GpuBufferOfT.cs:77-78).</summary>
internal sealed class CudaBuffer : GpuBuffer
{
    readonly CudaDevice _device;
    internal nint Pointer { get; private set; }

    internal CudaBuffer(CudaDevice device, nint pointer, ulong size, BufferUsage usage, string? label)
    {
        _device = device;
        Pointer = pointer;
        Size = size;
        Usage = usage;
        Label = label;
    }

    public override void Dispose()
    {
        if (Pointer == 0) return;
        Native.og_buffer_free(_device.Handle, Pointer);
        Pointer = 0;
    }
}

/// <summary>GpuTimestampSet on CUDA events (og_timestamps).</summary>
internal sealed class CudaTimestampSet : GpuTimestampSet
{
    internal nint Handle { get; private set; }

    internal CudaTimestampSet(nint handle, uint count)
    {
        Handle = handle;
        Count = count;
    }

    public override void Dispose()
    {
        if (Handle == 0) return;
        Native.og_timestamps_destroy(Handle);
        Handle = 0;
    }
}

/// <summary>An og_encoder: the library operations recorded on it (Int8Gemm.EncodeInt32, DynamicQuantizeKernels.
/// Encode, ...) run in order when the device submits it. Pass timing records CUDA events between operations.</summary>
internal sealed unsafe class CudaCommandEncoder : GpuCommandEncoder
{
    readonly CudaDevice _device;
    nint _handle;
    PassTiming? _timing;
    uint _passes;

    internal CudaCommandEncoder(CudaDevice device, nint handle)
    {
        _device = device;
        _handle = handle;
    }

    internal CudaDevice Device => _device;

    /// <summary>The og_encoder the kernel families record into.</summary>
    internal nint Handle => _handle != 0 ? _handle : throw new ObjectDisposedException(nameof(CudaCommandEncoder));

    internal nint TakeHandle()
    {
        var h = Handle;
        _handle = 0;
        return h;
    }

    /// <summary>Kernel launches recorded so far (og_encoder_dispatch_count).</summary>
    internal long LibraryDispatches
    {
        get
        {
            long n;
            NativeCheck.Check(Native.og_encoder_dispatch_count(Handle, &n));
            return n;
        }
    }

    public override void BeginPassTiming(in PassTiming timing)
    {
        _timing = timing;
        _passes = 0;
        NativeCheck.Check(Native.og_encoder_timestamp(Handle, ((CudaTimestampSet)timing.Set).Handle, timing.First));
    }

    public override uint EndPassTiming()
    {
        if (_timing is not { } t) return 0;
        NativeCheck.Check(Native.og_encoder_timestamp(Handle, ((CudaTimestampSet)t.Set).Handle, t.First + 1));
        _timing = null;
        return ++_passes;
    }

    static GpuUnsupportedException NoGraphics(string what) =>
        new($"the CUDA backend records library operations, not {what}", "Graphics",
            "a graphics backend (Vulkan, Metal, WebGPU)", "CUDA");

    public override GpuRenderPass BeginRenderPass(ReadOnlySpan<ColorAttachment> colors, DepthAttachment? depth) =>
        throw NoGraphics("render passes");
    public override GpuComputePass BeginComputePass() => throw NoGraphics("shader compute passes");
    public override void CopyBuffer(GpuBuffer source, ulong sourceOffset, GpuBuffer destination,
                                    ulong destinationOffset, ulong size) =>
        throw NoGraphics("buffer copies inside an encoder (use GpuDevice.WriteBuffer / ReadBuffer)");
    public override void CopyTextureToBuffer(GpuTexture source, uint mipLevel, uint layer, GpuBuffer destination,
                                             ulong destinationOffset) => throw NoGraphics("textures");
    public override void CopyBufferToTexture(GpuBuffer source, ulong sourceOffset, GpuTexture destination,
                                             uint mipLevel, uint layer) => throw NoGraphics("textures");
    public override void CopyTexture(GpuTexture source, GpuTexture destination) => throw NoGraphics("textures");
    public override void GenerateMips(GpuTexture texture) => throw NoGraphics("textures");
}
