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
