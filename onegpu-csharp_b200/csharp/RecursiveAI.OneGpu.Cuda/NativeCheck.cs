// Turns the og_status of an entry point into the reference's exceptions, with the operation, argument and
// capability the library reported through og_last_error (read on the calling thread, right after the call).
using System.Runtime.InteropServices;
using RecursiveAI.OneGpu.Kernels;

namespace RecursiveAI.OneGpu.Cuda;

internal static unsafe class NativeCheck
{
    public const int Ok = 0;

    static string Text(byte* p) => Marshal.PtrToStringUTF8((nint)p) ?? "";

    public static void Check(int status)
    {
        if (status == Ok) return;
        OgErrorInfo e;
        Native.og_last_error(&e);
        string op = Text(e.Operation), arg = Text(e.Argument), msg = Text(e.Message);
        string cap = Text(e.Capability), exp = Text(e.Expected), act = Text(e.Actual);
        throw status switch
        {
            1 => new GpuKernelShapeException(op, arg, msg),
            2 => new GpuUnsupportedException($"{op}: {msg}", cap, exp, act.Length == 0 ? null : act),
            3 => new ArgumentNullException(arg),
            4 => new ArgumentOutOfRangeException(arg, msg),
            5 => new GpuOutOfMemoryException($"{op}: {msg}"),
            6 => new GpuDeviceLostException($"{op}: {msg}"),
            7 => new GpuCommandFailedException($"{op}: {msg}",
                                               cap == "Watchdog" ? GpuCommandFailure.Watchdog : GpuCommandFailure.Unknown),
            _ => new GpuException($"{op}: {msg}"),
        };
    }

    /// <summary>The library's element type code of <typeparamref name="T"/> (og_type); -1 for a type it has none for,
    /// which its checks then report under the caller's argument name.</summary>
    public static int TypeCode<T>() where T : unmanaged
    {
        if (typeof(T) == typeof(byte)) return 0;
        if (typeof(T) == typeof(sbyte)) return 1;
        if (typeof(T) == typeof(int)) return 2;
        if (typeof(T) == typeof(float)) return 3;
        if (typeof(T) == typeof(Half)) return 4;
        if (typeof(T) == typeof(uint)) return 5;
        if (typeof(T) == typeof(ushort)) return 6;
        if (typeof(T) == typeof(short)) return 7;
        if (typeof(T) == typeof(long)) return 8;
        return -1;
    }

    /// <summary>The og_buffer view of a typed buffer of this backend.</summary>
    public static OgBuffer View<T>(GpuBuffer<T>? b) where T : unmanaged
    {
        if (b is null) return default;
        if (b.Buffer is not CudaBuffer cb)
            throw new GpuUnsupportedException("the buffer belongs to another backend", "Backend", "a CUDA buffer",
                                              b.Device.Backend.ToString());
        return new OgBuffer { Ptr = cb.Pointer, Length = b.Length, Type = TypeCode<T>() };
    }

    public static OgOperand Operand<T>(Int8Operand<T>? o) where T : unmanaged =>
        o is { } v ? new OgOperand { Buffer = View(v.Buffer), Offset = v.Offset, IsVector = v.IsVector ? 1 : 0 } : default;

    public static string ReadString(Func<nint, ulong, int> call)
    {
        var buf = new byte[256];
        fixed (byte* p = buf)
        {
            Check(call((nint)p, (ulong)buf.Length));
            return Text(p);
        }
    }
}
