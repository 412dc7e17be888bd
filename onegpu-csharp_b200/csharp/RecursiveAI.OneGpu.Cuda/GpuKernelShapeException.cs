// The kernel families' argument error (src/RecursiveAI.OneGpu.Kernels/GpuKernelShapeException.cs): an
// ArgumentException carrying the operation ("Int8Gemm", "DynamicQuantizeLinear", ...) and the argument's name, which
// the library's checks report in the reference's order.
namespace RecursiveAI.OneGpu.Kernels;

public sealed class GpuKernelShapeException : ArgumentException
{
    public GpuKernelShapeException(string operation, string argument, string message)
        : base($"{operation}: {argument}: {message}", argument)
    {
        Operation = operation;
        Argument = argument;
    }

    public string Operation { get; }

    public string Argument { get; }
}
