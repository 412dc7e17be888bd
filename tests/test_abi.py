"""The C ABI without a GPU: the library loads, exports every entry point of include/onegpu_cuda.h, and its argument
checks reject what the reference rejects, in the reference's order and with its argument names
(Int8Tests.BadArgumentsAreRejected, Int8Tests.cs:549-574; Int8ScratchTests.ScratchThatIsTooSmallIsRefused,
Int8ScratchTests.cs:68-89; DynamicQuantizeKernels.Encode, DynamicQuantizeKernels.cs:59-75)."""
import ctypes
import os
import re

import numpy as np
import pytest

import onegpu_cuda as og

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include", "onegpu_cuda.h")


def declared_symbols():
    text = open(HEADER, encoding="utf-8").read()
    return sorted(set(re.findall(r"OG_API\s+[\w\s\*]+?\b(og_\w+)\s*\(", text)))


def test_every_declared_entry_point_is_exported():
    names = declared_symbols()
    assert len(names) >= 40
    lib = ctypes.CDLL(og.LIBRARY_PATH)
    missing = [n for n in names if not hasattr(lib, n)]
    assert missing == []
    # The Python mirror binds every one of them.
    assert sorted(og.EXPORTS) == names


CSHARP = os.path.join(os.path.dirname(HEADER), "..", "onegpu-csharp_b200", "csharp", "RecursiveAI.OneGpu.Cuda")


def test_every_entry_point_has_a_csharp_binding():
    """The C# P/Invoke declarations (Native.cs) bind each entry point the header declares, and nothing else."""
    src = open(os.path.join(CSHARP, "Native.cs"), encoding="utf-8").read()
    bound = sorted(set(re.findall(r"\[LibraryImport\(Lib\)\][^;]*?\b(og_\w+)\s*\(", src)))
    assert bound == declared_symbols()


# The members of Int8Gemm and DynamicQuantizeKernels in the reference's shipped API
# (src/RecursiveAI.OneGpu.Kernels/PublicAPI.Shipped.txt:491-548), with the entry point each C# body must call.
SHIPPED_MEMBERS = {
    "Int8Gemm.cs": [
        ("public Int8Gemm(GpuDevice device, Int8GemmOptions? options = null, int maxCachedBindGroups = 1024)",
         "og_int8_gemm_create"),
        ("public string Variant", "og_int8_gemm_variant"),
        ("public int BindGroupsCreated", "og_int8_gemm_bind_groups_created"),
        ("public void ReserveScratch(long elements)", "og_int8_gemm_reserve_scratch"),
        ("public void ReleaseBindings()", None),
        ("public void EncodeInt32<TA, TB>(", "og_int8_gemm_encode_int32"),
        ("public void EncodeFloat<TA, TB>(", "og_int8_gemm_encode_float"),
        ("public void EncodeRequantized<TA, TB, TY>(", "og_int8_gemm_encode_requantized"),
        ("public void Dispose()", "og_int8_gemm_destroy"),
        ("public DynamicQuantizeKernels(GpuDevice device, int maxCachedBindGroups = 1024)",
         "og_dynamic_quantize_create"),
        ("public void Encode(GpuCommandEncoder encoder, GpuBuffer<float> x, int offsetX, int count, GpuBuffer<byte> y,",
         "og_dynamic_quantize_encode"),
    ],
}


def test_csharp_drop_in_classes_keep_the_shipped_members():
    """The C# Int8Gemm / DynamicQuantizeKernels of the CUDA backend declare every shipped public member, and each
    body calls the C entry point it maps to (declared in the header and bound in Native.cs)."""
    declared = set(declared_symbols())
    for fname, members in SHIPPED_MEMBERS.items():
        src = open(os.path.join(CSHARP, fname), encoding="utf-8").read()
        for signature, entry in members:
            at = src.find(signature)
            assert at >= 0, signature
            if entry is not None:
                assert entry in declared
                body = src[at:at + 4000]
                assert f"Native.{entry}(" in body, (signature, entry)
    for t in ("public struct Int8GemmProblem", "public readonly record struct Int8Operand<T>(GpuBuffer<T> Buffer, int "
              "Offset, bool IsVector = false)", "public readonly record struct Int8Scratch(GpuBuffer<int> Buffer, int "
              "Offset = 0)", "public sealed class Int8GemmOptions", "public bool AllowPackedDot { get; init; } = true;",
              "public readonly double Ops"):
        assert t in open(os.path.join(CSHARP, "Int8Gemm.cs"), encoding="utf-8").read(), t


def test_no_device_here_is_reported_not_crashed():
    if og.device_count() > 0:
        pytest.skip("a CUDA device is visible")
    with pytest.raises(og.GpuUnsupportedException):
        og.GpuDevice(0)


U8, S8, I32, F32 = np.uint8, np.int8, np.int32, np.float32
spec = og.buffer_spec
P = og.Int8GemmProblem
Op = og.Int8Operand


def argument_of(fn, *args, **kw):
    with pytest.raises(og.GpuException) as e:
        fn(*args, **kw)
    return type(e.value), getattr(e.value, "argument", None)


def test_bad_arguments_are_rejected():
    """Int8Tests.cs:555-571, replayed through the device-free checks."""
    a = spec(U8, 64)
    b = spec(S8, 64)
    c = spec(I32, 64)
    f = spec(F32, 64)
    fl = spec(F32, 1)
    shape = og.GpuKernelShapeException
    assert argument_of(og.check_int32, P(9, 9, 9), a, b, c) == (shape, "OffsetA")
    assert argument_of(og.check_int32, P(-1, 2, 2), a, b, c) == (shape, "M")
    assert argument_of(og.check_int32, P(2, 2, 2, batch=0), a, b, c) == (shape, "Batch")
    assert argument_of(og.check_int32, P(2, 2, 2, lda=1), a, b, c) == (shape, "Lda")
    assert argument_of(og.check_int32, P(2, 2, 2, offset_c=62), a, b, c) == (shape, "c")
    assert argument_of(og.check_int32, P(8, 8, 8, offset_a=1), a, b, c) == (shape, "OffsetA")
    assert argument_of(og.check_int32, P(2, 2, 2), a, b, c, Op(a, 63, True)) == (shape, "zpA")
    assert argument_of(og.check_int32, P(2, 2, 2), f, b, c) == (shape, "a")
    assert argument_of(og.check_float, P(2, 8, 2), a, b, f, Op(fl, 0, True)) == (shape, "scale")
    assert argument_of(og.check_requantized, P(2, 2, 2), a, b, a, Op(fl, 0), 300) == (shape, "zeroPointY")
    assert argument_of(og.check_requantized, P(2, 2, 2), a, b, b, Op(fl, 0), 128) == (shape, "zeroPointY")
    # A bias is one value per column whatever its IsVector says (Int8Gemm.cs:242,296,656): a one-value buffer is
    # refused for N > 1, as a float bias is (the kernels read one per column).
    ib1, ib8 = spec(I32, 1), spec(I32, 8)
    assert argument_of(og.check_int32, P(2, 8, 2), a, b, c, None, None, Op(ib1, 0, False)) == (shape, "bias")
    og.check_int32(P(2, 8, 2), a, b, c, None, None, Op(ib8, 0, False))
    assert argument_of(og.check_float, P(2, 8, 2), a, b, f, Op(fl, 0), None, None, Op(fl, 0, False)) == \
        (shape, "floatBias")
    assert argument_of(og.check_float, P(2, 8, 2), a, b, f, Op(fl, 0), None, None, None, Op(ib1, 0, False)) == \
        (shape, "intBias")
    # The valid calls pass.
    og.check_int32(P(2, 2, 2), a, b, c)
    og.check_float(P(2, 8, 2), a, b, f, Op(fl, 0))
    og.check_requantized(P(2, 2, 2), a, b, a, Op(fl, 0), 255)
    og.check_requantized(P(2, 2, 2), a, b, b, Op(fl, 0), -128)


def test_more_checks_in_the_reference_order():
    a, b, c = spec(U8, 64), spec(S8, 64), spec(I32, 64)
    shape = og.GpuKernelShapeException
    for field in ("n", "k", "offset_a", "offset_b", "offset_c", "stride_a", "stride_b", "lda", "ldb"):
        name = {"n": "N", "k": "K", "offset_a": "OffsetA", "offset_b": "OffsetB", "offset_c": "OffsetC",
                "stride_a": "StrideA", "stride_b": "StrideB", "lda": "Lda", "ldb": "Ldb"}[field]
        fields = dict(m=2, n=2, k=2)
        fields[field] = -1
        assert argument_of(og.check_int32, P(**fields), a, b, c) == (shape, name)
    assert argument_of(og.check_int32, P(2, 4, 2, transpose_b=True, ldb=1), a, b, c) == (shape, "Ldb")
    assert argument_of(og.check_int32, P(2, 4, 2, ldb=3), a, b, c) == (shape, "Ldb")
    assert argument_of(og.check_int32, P(4, 4, 4, batch=5, stride_b=16), a, b, c) == (shape, "OffsetB")
    assert argument_of(og.check_int32, P(2, 2, 2), a, b, c, None, Op(b, 63, True)) == (shape, "zpB")
    assert argument_of(og.check_int32, P(2, 2, 2), a, b, c, Op(a, -1)) == (shape, "zpAOffset")
    assert argument_of(og.check_int32, P(2, 2, 2), a, b, c, None, None, Op(c, 63, True)) == (shape, "bias")
    assert argument_of(og.check_int32, P(2, 2, 2), a, b, c, Op(b, 0)) == (shape, "zpA")  # zero point of A's type
    assert argument_of(og.check_int32, P(2, 2, 2), a, b, spec(F32, 64)) == (shape, "c")
    assert argument_of(og.check_int32, P(65536, 65536, 1), a, b, c) == (shape, "Batch")
    assert argument_of(og.check_int32, P(2, 2, 2), spec(U8, 64, null=True), b, c) == (og.ArgumentNullException,
                                                                                     "a")
    assert argument_of(og.check_int32, P(2, 2, 2), a, b, None) == (og.ArgumentNullException, "c")
    # K = 0 skips the operand ranges (nothing is read), M = 0 records nothing but checks C.
    og.check_int32(P(2, 2, 0), spec(U8, 1), spec(S8, 1), c)
    og.check_int32(P(0, 2, 9), spec(U8, 1), spec(S8, 1), c)


def test_float_form_checks_int_bias_only_when_there_is_work():
    """EncodeFloat checks intBias after its early return for an empty product (Int8Gemm.cs:285-300)."""
    a, b, f, fl = spec(U8, 64), spec(S8, 64), spec(F32, 64), spec(F32, 64)
    bad_bias = Op(spec(I32, 1), 0, True)
    og.check_float(P(0, 8, 2), a, b, f, Op(fl, 0), int_bias=bad_bias)
    assert argument_of(og.check_float, P(2, 8, 2), a, b, f, Op(fl, 0), int_bias=bad_bias) == (
        og.GpuKernelShapeException, "intBias")
    assert argument_of(og.check_float, P(2, 8, 2), a, b, f, Op(fl, 0), float_bias=Op(fl, 60, True)) == (
        og.GpuKernelShapeException, "floatBias")


def test_dequantize_form_checks():
    """The fused MatMulIntegerToFloat form: EncodeFloat's checks plus a single-valued aScale."""
    a, b, f = spec(U8, 64), spec(S8, 64), spec(F32, 64)
    sa, sb = spec(F32, 1), spec(F32, 8)
    og.check_dequantize(P(2, 8, 2), a, b, f, Op(sa, 0), Op(sb, 0, True))
    shape = og.GpuKernelShapeException
    assert argument_of(og.check_dequantize, P(2, 8, 2), a, b, f, Op(sa, 0, True), Op(sb, 0, True)) == (shape, "aScale")
    assert argument_of(og.check_dequantize, P(2, 9, 2), a, b, f, Op(sa, 0), Op(sb, 0, True)) == (shape, "bScale")
    assert argument_of(og.check_dequantize, P(2, 8, 2), a, b, f, Op(spec(I32, 1), 0), Op(sb, 0, True)) == (
        shape, "aScale")
    assert argument_of(og.check_dequantize, P(2, 8, 2), a, b, f, None, Op(sb, 0, True)) == (og.ArgumentNullException,
                                                                                          "aScale")


def test_scratch_that_is_too_small_is_refused():
    """Int8ScratchTests.cs:68-89."""
    a = spec(U8, 64 * 8 + 4)
    b = spec(S8, 64 * 8 + 4)
    y = spec(U8, 64 * 64 + 4)
    mult = spec(F32, 1)
    small = og.Int8Scratch(spec(I32, 100))
    assert argument_of(og.check_requantized, P(64, 64, 8), a, b, y, Op(mult, 0), 0, scratch=small) == (
        og.GpuKernelShapeException, "scratch")
    og.check_requantized(P(64, 64, 8), a, b, y, Op(mult, 0), 0, scratch=og.Int8Scratch(spec(I32, 4096)))
    assert og.Int8Gemm.scratch_elements(P(160, 96, 64)) == 160 * 96
    assert og.Int8Gemm.scratch_elements(P(0, 96, 64)) == 0


def test_dynamic_quantize_checks():
    x, y, s, z = spec(F32, 16), spec(U8, 16), spec(F32, 2), spec(U8, 2)
    shape = og.GpuKernelShapeException
    og.check_dynamic_quantize(x, 0, 16, y, 0, s, 1, z, 1)
    assert argument_of(og.check_dynamic_quantize, x, 0, 0, y, 0, s, 0, z, 0) == (shape, "count")
    assert argument_of(og.check_dynamic_quantize, x, 1, 16, y, 0, s, 0, z, 0) == (shape, "x")
    assert argument_of(og.check_dynamic_quantize, x, -1, 4, y, 0, s, 0, z, 0) == (shape, "xOffset")
    assert argument_of(og.check_dynamic_quantize, x, 0, 16, y, 1, s, 0, z, 0) == (shape, "y")
    assert argument_of(og.check_dynamic_quantize, x, 0, 4, y, 0, s, 2, z, 0) == (shape, "scale")
    assert argument_of(og.check_dynamic_quantize, x, 0, 4, y, 0, s, 0, z, 2) == (shape, "zeroPoint")
    assert argument_of(og.check_dynamic_quantize, spec(I32, 16), 0, 4, y, 0, s, 0, z, 0) == (shape, "x")
    assert argument_of(og.check_dynamic_quantize, x, 0, 4, spec(U8, 4, null=True), 0, s, 0, z, 0) == (
        og.ArgumentNullException, "y")


def _shape_arg(fn, *args):
    with pytest.raises(og.GpuKernelShapeException) as info:
        fn(*args)
    return info.value.argument


def test_dequantize_linear_checks():
    """DequantizeTests.BadArgumentsAreRejected (DequantizeTests.cs:113-133) on the argument checks alone."""
    spec = og.buffer_spec
    x, s, o = spec(np.uint8, 16), spec(np.float32, 4), spec(np.float32, 16)
    big, ox = spec(np.uint32, 16), spec(np.uint16, 16)
    chk = og.check_dequantize_linear
    chk(x, 0, [4, 4], 1, True, s, 0, None, 0, o, 0)
    assert _shape_arg(chk, x, 0, [4, 4], 1, True, s, 1, None, 0, o, 0) == "scale"
    assert _shape_arg(chk, x, 0, [4, 4], 5, True, s, 0, None, 0, o, 0) == "axis"
    assert _shape_arg(chk, x, 8, [4, 4], 0, False, s, 0, None, 0, o, 0) == "x"
    assert _shape_arg(chk, big, 0, [4], 0, False, s, 0, None, 0, o, 0) == "TIn"
    assert _shape_arg(chk, x, 0, [4], 0, False, s, 0, None, 0, ox, 0) == "T"
    # Byte tensors end on a 32-bit word; half outputs too (Check.RangeBytes / Check.Range with half).
    assert _shape_arg(chk, spec(np.uint8, 6), 0, [5], 0, False, s, 0, None, 0, o, 0) == "x"
    assert _shape_arg(chk, x, 0, [3], 0, False, s, 0, None, 0, spec(np.float16, 3), 0) == "output"
    chk(x, 0, [3], 0, False, s, 0, None, 0, spec(np.float16, 4), 0)
    assert _shape_arg(chk, x, 0, [-1, 4], 0, False, s, 0, None, 0, o, 0) == "shape[0]"
    assert _shape_arg(chk, x, 0, [4], 0, False, s, 0, spec(np.int8, 4), 0, o, 0) == "zeroPoint"
    assert _shape_arg(chk, x, 0, [4, 4], -3, True, s, 0, None, 0, o, 0) == "axis"
    chk(spec(np.int32, 16), 0, [16], 0, False, s, 0, spec(np.int32, 1), 0, o, 0)  # int32: plain ranges
    with pytest.raises(og.ArgumentNullException):
        chk(x, 0, [4], 0, False, None, 0, None, 0, o, 0)


def test_quantize_linear_checks():
    """DequantizeTests.QuantizeRejectsBadArguments (DequantizeTests.cs:289-310) on the argument checks alone."""
    spec = og.buffer_spec
    x, s, o = spec(np.float32, 16), spec(np.float32, 4), spec(np.uint8, 16)
    chk = og.check_quantize_linear
    chk(x, 0, [4, 4], 1, True, s, 0, None, 0, o, 0)
    assert _shape_arg(chk, x, 0, [4, 4], 1, True, s, 1, None, 0, o, 0) == "scale"
    assert _shape_arg(chk, x, 0, [4, 4], 5, True, s, 0, None, 0, o, 0) == "axis"
    assert _shape_arg(chk, x, 8, [4, 4], 0, False, s, 0, None, 0, o, 0) == "x"
    assert _shape_arg(chk, x, 0, [4, 4], 0, False, s, 0, None, 0, o, 3) == "output"
    assert _shape_arg(chk, x, 0, [4], 0, False, s, 0, None, 0, spec(np.int16, 16), 0) == "TOut"
    assert _shape_arg(chk, spec(np.int32, 16), 0, [4], 0, False, s, 0, None, 0, o, 0) == "T"
    assert _shape_arg(chk, x, 0, [4], 0, False, s, 0, spec(np.int8, 4), 0, o, 0) == "zeroPoint"
    chk(spec(np.float16, 16), 0, [4, 4], 0, True, s, 0, spec(np.uint8, 4), 0, o, 0)


def test_conv_integer_checks():
    """ConvIntegerTests.BadShapesThrowTypedErrors (ConvIntegerTests.cs:299-323) and the scratch size rule."""
    spec = og.buffer_spec
    x, w, y, f = spec(np.uint8, 64), spec(np.int8, 64), spec(np.int32, 64), spec(np.float32, 64)
    P = og.ConvProblem
    chk = og.check_conv_integer
    assert _shape_arg(chk, P(1, 3, 4, 4, 4, 3, 3, groups=2), x, w, y) == "Groups"
    assert _shape_arg(chk, P(1, 3, 2, 2, 4, 3, 3), x, w, y) == "height"
    assert _shape_arg(chk, P(1, 3, 8, 8, 4, 3, 3), x, w, y) == "x"
    assert _shape_arg(chk, P(1, 1, 4, 4, 1, 1, 1), x, w, y, None, og.Int8Operand(w, 64, True)) == "wZeroPoint"
    assert _shape_arg(chk, P(1, 1, 4, 4, 1, 1, 1), f, w, y) == "x"
    assert _shape_arg(chk, P(1, 1, 4, 4, 1, 1, 1), x, w, y, None, None, x, 2) == "scratchOffset"
    chk(P(1, 1, 4, 4, 1, 1, 1), x, w, y, og.Int8Operand(x, 0), og.Int8Operand(w, 0), x, 4)
    assert _shape_arg(chk, P(1, 1, 4, 4, 1, 1, 1), x, w, y, og.Int8Operand(x, 0, True)) == "xZeroPoint"
    assert _shape_arg(chk, P(1, 1, 4, 4, 1, 1, 1, activation=1), x, w, y) == "Activation"
    assert _shape_arg(chk, P(0, 1, 4, 4, 1, 1, 1), x, w, y) == "Batch"
    assert _shape_arg(chk, P(1, 1, 4, 4, 1, 1, 1, stride_width=0), x, w, y) == "width stride"
    assert _shape_arg(chk, P(1, 1, 4, 4, 1, 1, 1, pad_top=-1), x, w, y) == "height padding"
    assert _shape_arg(chk, P(1, 1, 4, 4, 1, 1, 1), x, w, spec(np.float32, 64)) == "y"
    # One image's columns: Groups * K * ceil(OH * OW / 4) * 4 bytes.
    assert og.conv_scratch_bytes_per_image(P(2, 4, 9, 11, 5, 3, 3, stride_height=2, stride_width=2, pad_top=1,
                                                pad_left=1, pad_bottom=1, pad_right=1)) == 36 * 32
    assert og.conv_scratch_bytes_per_image(P(1, 4, 8, 8, 6, 3, 3, groups=2, pad_top=1, pad_left=1, pad_bottom=1,
                                                pad_right=1)) == 2 * 18 * 64
    small = P(3, 3, 8, 8, 4, 3, 3, pad_top=1, pad_left=1, pad_bottom=1, pad_right=1)
    one = og.conv_scratch_bytes_per_image(small)
    assert _shape_arg(chk, small, spec(np.uint8, 600), spec(np.int8, 200), spec(np.int32, 800), None, None,
                      spec(np.uint8, one + 7), 8) == "scratch"
