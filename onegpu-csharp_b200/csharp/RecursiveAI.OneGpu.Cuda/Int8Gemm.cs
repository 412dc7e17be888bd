// Int8Gemm with its shipped signatures (src/RecursiveAI.OneGpu.Kernels/PublicAPI.Shipped.txt:491-548) on the CUDA
// library: every Encode* builds the C structures from its arguments and records the product on the encoder through
// the C ABI, which runs the reference's argument checks (Int8Gemm.cs:393-501) in its order and with its argument
// names before anything is recorded. The problem, operand, scratch and options types keep the reference's members.
using System.Runtime.InteropServices;
using RecursiveAI.OneGpu.Cuda;

namespace RecursiveAI.OneGpu.Kernels;

/// <summary>Int8GemmOptions (Int8Gemm.cs:7-21). AllowPackedDot = false runs the portable (CUDA-core) kernel.</summary>
public sealed class Int8GemmOptions
{
    public bool AllowPackedDot { get; init; } = true;

    /// <summary>Test hook like the reference's internal Tile: 0 chooses by size, 128 the one-SM tensor-core tile,
    /// 256 the CTA-pair tile.</summary>
    internal int Tile { get; init; }
}

/// <summary>Int8GemmProblem (Int8Gemm.cs:43-95): A is M x K, B is K x N (N x K with TransposeB), row-major; C is
/// dense [Batch, M, N]. Offsets and strides of A and B are in bytes, OffsetC in elements; 0 for Lda / Ldb means
/// dense rows, 0 for StrideA / StrideB means every batch shares the operand.</summary>
public struct Int8GemmProblem
{
    public Int8GemmProblem() => Batch = 1;

    public Int8GemmProblem(int m, int n, int k)
    {
        M = m;
        N = n;
        K = k;
        Batch = 1;
    }

    public int M { get; set; }
    public int N { get; set; }
    public int K { get; set; }
    public int Batch { get; set; }
    public bool TransposeB { get; set; }
    public int Lda { get; set; }
    public int Ldb { get; set; }
    public int OffsetA { get; set; }
    public int OffsetB { get; set; }
    public int OffsetC { get; set; }
    public int StrideA { get; set; }
    public int StrideB { get; set; }

    /// <summary>2 * Batch * M * N * K multiply-add operations.</summary>
    public readonly double Ops => 2.0 * Batch * M * N * (double)K;

    internal readonly OgProblem Native() => new()
    {
        M = M, N = N, K = K, Batch = Batch, TransposeB = TransposeB ? 1 : 0, Lda = Lda, Ldb = Ldb,
        OffsetA = OffsetA, OffsetB = OffsetB, OffsetC = OffsetC, StrideA = StrideA, StrideB = StrideB,
    };
}

/// <summary>Int8Operand&lt;T&gt; (Int8Gemm.cs:28): a zero point, scale or bias in a buffer, one value at Offset or, with
/// IsVector, one per row of A (its zero point) or per column (zero point of B, scale, bias).</summary>
public readonly record struct Int8Operand<T>(GpuBuffer<T> Buffer, int Offset, bool IsVector = false) where T : unmanaged;

/// <summary>Int8Scratch (Int8Gemm.cs:37): caller-placed int32 scratch of EncodeRequantized.</summary>
public readonly record struct Int8Scratch(GpuBuffer<int> Buffer, int Offset = 0);

/// <summary>The int8 product family on CUDA: tcgen05 tensor-core kernels (CTA pairs, TMEM accumulators, TMA-staged
/// tiles), the few-rows decode kernel, and the portable kernel. Not thread-safe (Int8Gemm.cs:122).</summary>
public sealed unsafe class Int8Gemm : IDisposable
{
    nint _handle;
    readonly GpuDevice _device;

    public Int8Gemm(GpuDevice device, Int8GemmOptions? options = null, int maxCachedBindGroups = 1024)
    {
        ArgumentNullException.ThrowIfNull(device);
        ArgumentOutOfRangeException.ThrowIfLessThan(maxCachedBindGroups, 1);
        if (device is not CudaDevice cuda)
            throw new GpuUnsupportedException("Int8Gemm of the CUDA backend needs a CUDA device", "Backend", "CUDA",
                                              device.Backend.ToString());
        var o = options ?? new Int8GemmOptions();
        var opts = new OgOptions { AllowPackedDot = o.AllowPackedDot ? 1 : 0, Kernel = 0, Tile = o.Tile, StreamK = 0 };
        nint h;
        NativeCheck.Check(Cuda.Native.og_int8_gemm_create(cuda.Handle, &opts, &h));
        _handle = h;
        _device = device;
    }

    nint Handle => _handle != 0 ? _handle : throw new ObjectDisposedException(nameof(Int8Gemm));

    /// <summary>The kernels this instance runs, e.g. "tcgen05-i8-2sm-tile256x256x128+1sm-tile128x256x128".</summary>
    public string Variant => NativeCheck.ReadString((p, n) => Cuda.Native.og_int8_gemm_variant(Handle, (byte*)p, n));

    /// <summary>0: CUDA kernels take their arguments by value, there are no bind groups.</summary>
    public int BindGroupsCreated
    {
        get
        {
            int n;
            NativeCheck.Check(Cuda.Native.og_int8_gemm_bind_groups_created(Handle, &n));
            return n;
        }
    }

    /// <summary>Int32 elements of scratch EncodeRequantized needs for a problem (Int8Gemm.cs:531).</summary>
    public static long ScratchElements(in Int8GemmProblem problem)
    {
        var p = problem.Native();
        return Cuda.Native.og_int8_gemm_scratch_elements(&p);
    }

    /// <summary>Int8Gemm.ReserveScratch (Int8Gemm.cs:539-549).</summary>
    public void ReserveScratch(long elements) => NativeCheck.Check(Cuda.Native.og_int8_gemm_reserve_scratch(Handle, elements));

    /// <summary>Nothing to release: no bind groups are cached.</summary>
    public void ReleaseBindings() { }

    static nint Encoder(GpuCommandEncoder encoder)
    {
        ArgumentNullException.ThrowIfNull(encoder);
        return encoder is CudaCommandEncoder e
            ? e.Handle
            : throw new GpuUnsupportedException("the encoder belongs to another backend", "Backend", "CUDA", null);
    }

    /// <summary>EncodeInt32 (Int8Gemm.cs:230-253): C = sum_k (A - zpA)(B - zpB) (+ bias[n]), int32 wrapping.</summary>
    public void EncodeInt32<TA, TB>(GpuCommandEncoder encoder, in Int8GemmProblem problem, GpuBuffer<TA> a,
                                    GpuBuffer<TB> b, GpuBuffer<int> c, Int8Operand<TA>? zeroPointA = null,
                                    Int8Operand<TB>? zeroPointB = null, Int8Operand<int>? bias = null)
        where TA : unmanaged
        where TB : unmanaged
    {
        ArgumentNullException.ThrowIfNull(a);
        ArgumentNullException.ThrowIfNull(b);
        ArgumentNullException.ThrowIfNull(c);
        var p = problem.Native();
        OgBuffer va = NativeCheck.View(a), vb = NativeCheck.View(b), vc = NativeCheck.View(c);
        OgOperand za = NativeCheck.Operand(zeroPointA), zb = NativeCheck.Operand(zeroPointB);
        OgOperand ib = NativeCheck.Operand(bias);
        NativeCheck.Check(Cuda.Native.og_int8_gemm_encode_int32(Handle, Encoder(encoder), &p, &va, &vb, &vc,
                                                                 zeroPointA is null ? null : &za,
                                                                 zeroPointB is null ? null : &zb,
                                                                 bias is null ? null : &ib));
    }

    /// <summary>EncodeFloat (Int8Gemm.cs:270-314): float(sum + intBias) * scale (+ floatBias), two roundings.</summary>
    public void EncodeFloat<TA, TB>(GpuCommandEncoder encoder, in Int8GemmProblem problem, GpuBuffer<TA> a,
                                    GpuBuffer<TB> b, GpuBuffer<float> c, Int8Operand<float> scale,
                                    Int8Operand<TA>? zeroPointA = null, Int8Operand<TB>? zeroPointB = null,
                                    Int8Operand<float>? floatBias = null, Int8Operand<int>? intBias = null)
        where TA : unmanaged
        where TB : unmanaged
    {
        ArgumentNullException.ThrowIfNull(a);
        ArgumentNullException.ThrowIfNull(b);
        ArgumentNullException.ThrowIfNull(c);
        var p = problem.Native();
        OgBuffer va = NativeCheck.View(a), vb = NativeCheck.View(b), vc = NativeCheck.View(c);
        OgOperand sc = NativeCheck.Operand<float>(scale);
        OgOperand za = NativeCheck.Operand(zeroPointA), zb = NativeCheck.Operand(zeroPointB);
        OgOperand fb = NativeCheck.Operand(floatBias), ib = NativeCheck.Operand(intBias);
        NativeCheck.Check(Cuda.Native.og_int8_gemm_encode_float(Handle, Encoder(encoder), &p, &va, &vb, &vc, &sc,
                                                                 zeroPointA is null ? null : &za,
                                                                 zeroPointB is null ? null : &zb,
                                                                 floatBias is null ? null : &fb,
                                                                 intBias is null ? null : &ib));
    }

    /// <summary>EncodeRequantized (Int8Gemm.cs:336-363): clamp(round_half_even(float(sum + intBias) * multiplier) +
    /// zeroPointY) as uint8 or int8 (NaN to the lowest value), written by the product's epilogue.</summary>
    public void EncodeRequantized<TA, TB, TY>(GpuCommandEncoder encoder, in Int8GemmProblem problem, GpuBuffer<TA> a,
                                              GpuBuffer<TB> b, GpuBuffer<TY> y, Int8Operand<float> multiplier,
                                              int zeroPointY, Int8Operand<TA>? zeroPointA = null,
                                              Int8Operand<TB>? zeroPointB = null, Int8Operand<int>? intBias = null,
                                              Int8Scratch? scratch = null)
        where TA : unmanaged
        where TB : unmanaged
        where TY : unmanaged
    {
        ArgumentNullException.ThrowIfNull(a);
        ArgumentNullException.ThrowIfNull(b);
        ArgumentNullException.ThrowIfNull(y);
        var p = problem.Native();
        OgBuffer va = NativeCheck.View(a), vb = NativeCheck.View(b), vy = NativeCheck.View(y);
        OgOperand mu = NativeCheck.Operand<float>(multiplier);
        OgOperand za = NativeCheck.Operand(zeroPointA), zb = NativeCheck.Operand(zeroPointB);
        OgOperand ib = NativeCheck.Operand(intBias);
        OgOperand sc = scratch is { } s
            ? new OgOperand { Buffer = NativeCheck.View(s.Buffer), Offset = s.Offset, IsVector = 0 }
            : default;
        NativeCheck.Check(Cuda.Native.og_int8_gemm_encode_requantized(Handle, Encoder(encoder), &p, &va, &vb, &vy, &mu,
                                                                       zeroPointY,
                                                                       zeroPointA is null ? null : &za,
                                                                       zeroPointB is null ? null : &zb,
                                                                       intBias is null ? null : &ib,
                                                                       scratch is null ? null : &sc));
    }

    /// <summary>The float form with the scale formed in the epilogue as aScale * bScale[n] (a float32 product), as
    /// the DynamicQuantizeLinear chain needs it (Int8Tests.cs:733-745) without an elementwise pass. No counterpart
    /// in the reference's shipped API.</summary>
    public void EncodeDequantize<TA, TB>(GpuCommandEncoder encoder, in Int8GemmProblem problem, GpuBuffer<TA> a,
                                         GpuBuffer<TB> b, GpuBuffer<float> c, Int8Operand<float> aScale,
                                         Int8Operand<float> bScale, Int8Operand<TA>? zeroPointA = null,
                                         Int8Operand<TB>? zeroPointB = null, Int8Operand<float>? floatBias = null,
                                         Int8Operand<int>? intBias = null)
        where TA : unmanaged
        where TB : unmanaged
    {
        var p = problem.Native();
        OgBuffer va = NativeCheck.View(a), vb = NativeCheck.View(b), vc = NativeCheck.View(c);
        OgOperand sa = NativeCheck.Operand<float>(aScale), sb = NativeCheck.Operand<float>(bScale);
        OgOperand za = NativeCheck.Operand(zeroPointA), zb = NativeCheck.Operand(zeroPointB);
        OgOperand fb = NativeCheck.Operand(floatBias), ib = NativeCheck.Operand(intBias);
        NativeCheck.Check(Cuda.Native.og_int8_gemm_encode_dequantize(Handle, Encoder(encoder), &p, &va, &vb, &vc, &sa,
                                                                      &sb, zeroPointA is null ? null : &za,
                                                                      zeroPointB is null ? null : &zb,
                                                                      floatBias is null ? null : &fb,
                                                                      intBias is null ? null : &ib));
    }

    /// <summary>Waits for the device, then releases the instance's scratch (Int8Gemm.cs:378-391).</summary>
    public void Dispose()
    {
        if (_handle == 0) return;
        Cuda.Native.og_int8_gemm_destroy(_handle);
        _handle = 0;
    }
}

/// <summary>DynamicQuantizeKernels (DynamicQuantizeKernels.cs:20-110): y = clamp(round_half_even(x / scale) +
/// zeroPoint, 0, 255) with scale = (max(0, max x) - min(0, min x)) / 255 over the whole range, on CUDA as one
/// cooperative kernel for large tensors (x read from DRAM once). Not thread-safe.</summary>
public sealed unsafe class DynamicQuantizeKernels : IDisposable
{
    nint _handle;

    public DynamicQuantizeKernels(GpuDevice device, int maxCachedBindGroups = 1024)
    {
        ArgumentNullException.ThrowIfNull(device);
        ArgumentOutOfRangeException.ThrowIfLessThan(maxCachedBindGroups, 1);
        if (device is not CudaDevice cuda)
            throw new GpuUnsupportedException("DynamicQuantizeKernels of the CUDA backend needs a CUDA device", "Backend",
                                              "CUDA", device.Backend.ToString());
        nint h;
        NativeCheck.Check(Cuda.Native.og_dynamic_quantize_create(cuda.Handle, &h));
        _handle = h;
    }

    nint Handle => _handle != 0 ? _handle : throw new ObjectDisposedException(nameof(DynamicQuantizeKernels));

    public int BindGroupsCreated => 0;

    public void ReleaseBindings() { }

    /// <summary>DynamicQuantizeKernels.Encode (DynamicQuantizeKernels.cs:59-90).</summary>
    public void Encode(GpuCommandEncoder encoder, GpuBuffer<float> x, int offsetX, int count, GpuBuffer<byte> y,
                       int offsetY, GpuBuffer<float> scale, int offsetScale, GpuBuffer<byte> zeroPoint,
                       int offsetZeroPoint)
    {
        ArgumentNullException.ThrowIfNull(encoder);
        var enc = encoder as CudaCommandEncoder
                  ?? throw new GpuUnsupportedException("the encoder belongs to another backend", "Backend", "CUDA", null);
        OgBuffer vx = NativeCheck.View(x), vy = NativeCheck.View(y), vs = NativeCheck.View(scale);
        OgBuffer vz = NativeCheck.View(zeroPoint);
        NativeCheck.Check(Cuda.Native.og_dynamic_quantize_encode(Handle, enc.Handle, x is null ? null : &vx, offsetX, count,
                                                                 y is null ? null : &vy, offsetY,
                                                                 scale is null ? null : &vs, offsetScale,
                                                                 zeroPoint is null ? null : &vz, offsetZeroPoint));
    }

    public void Dispose()
    {
        if (_handle == 0) return;
        Cuda.Native.og_dynamic_quantize_destroy(_handle);
        _handle = 0;
    }
}
