"""ctypes binding of the CPU oracle (oracle/og_oracle.c).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and bench.py's CPU-baseline legs, as the
checker or as the timed CPU restatement. The product (onegpu-csharp_b200/) never imports it.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_lib", "libog_oracle.so")


def build() -> str:
    """Compiles the oracle with its Makefile (gcc, -ffp-contract=off) when the library is missing or stale."""
    src = os.path.join(HERE, "og_oracle.c")
    if not os.path.exists(LIB_PATH) or os.path.getmtime(LIB_PATH) < os.path.getmtime(src):
        subprocess.run(["make", "-C", HERE], check=True, capture_output=True)
    return LIB_PATH


class Problem(ctypes.Structure):
    _fields_ = [(name, ctypes.c_int32) for name in
                ("m", "n", "k", "batch", "transpose_b", "lda", "ldb", "offset_a", "offset_b", "stride_a",
                 "stride_b")]


class Conv(ctypes.Structure):
    _fields_ = [(name, ctypes.c_int32) for name in
                ("batch", "cin", "h", "w", "cout", "kh", "kw", "stride_h", "stride_w", "dilation_h", "dilation_w",
                 "pad_top", "pad_left", "pad_bottom", "pad_right", "groups", "offset_x", "offset_w")]


_lib = None


def lib():
    global _lib
    if _lib is None:
        _lib = ctypes.CDLL(build())
        u8p = ctypes.POINTER(ctypes.c_uint8)
        i32p = ctypes.POINTER(ctypes.c_int32)
        f32p = ctypes.POINTER(ctypes.c_float)
        _lib.og_oracle_bytes.argtypes = [u8p, ctypes.c_int64, ctypes.c_int32]
        _lib.og_oracle_random.argtypes = [f32p, ctypes.c_int64, ctypes.c_int32, ctypes.c_float, ctypes.c_float]
        _lib.og_oracle_dq_input.argtypes = [f32p, ctypes.c_int64, ctypes.c_int32, ctypes.c_int32]
        gemm_args = [ctypes.POINTER(Problem), u8p, ctypes.c_int32, u8p, ctypes.c_int32, u8p, ctypes.c_int32, u8p,
                     ctypes.c_int32, i32p]
        _lib.og_oracle_int8_gemm.argtypes = gemm_args + [ctypes.c_int32]
        _lib.og_oracle_int8_gemm_tiled.argtypes = gemm_args + [ctypes.c_int32]
        _lib.og_oracle_int8_gemm_signed_domain.argtypes = gemm_args
        _lib.og_oracle_requant.argtypes = [ctypes.c_int32, ctypes.c_float, ctypes.c_int32, ctypes.c_int32]
        _lib.og_oracle_requant.restype = ctypes.c_int32
        _lib.og_oracle_float_epilogue.argtypes = [ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_float,
                                                  ctypes.c_int32, ctypes.c_float]
        _lib.og_oracle_float_epilogue.restype = ctypes.c_float
        _lib.og_oracle_dynamic_quantize.argtypes = [f32p, ctypes.c_int64, u8p, f32p, u8p]
        _lib.og_oracle_div_exact.argtypes = [ctypes.c_float, ctypes.c_float]
        _lib.og_oracle_div_exact.restype = ctypes.c_float
        _lib.og_oracle_float_to_half.argtypes = [ctypes.c_float]
        _lib.og_oracle_float_to_half.restype = ctypes.c_uint16
        _lib.og_oracle_half_to_float.argtypes = [ctypes.c_uint16]
        _lib.og_oracle_half_to_float.restype = ctypes.c_float
        vp = ctypes.c_void_p
        _lib.og_oracle_dequantize.argtypes = [ctypes.c_int32, vp, ctypes.c_int64, ctypes.c_int32, ctypes.c_int64,
                                              ctypes.c_int64, f32p, vp, ctypes.c_int32, vp]
        _lib.og_oracle_quantize.argtypes = [ctypes.c_int32, ctypes.c_int32, vp, ctypes.c_int64, ctypes.c_int32,
                                            ctypes.c_int64, ctypes.c_int64, f32p, u8p, u8p]
        _lib.og_oracle_conv_out_extent.argtypes = [ctypes.c_int32] * 6
        _lib.og_oracle_conv_out_extent.restype = ctypes.c_int32
        _lib.og_oracle_conv_integer.argtypes = [ctypes.POINTER(Conv), u8p, ctypes.c_int32, u8p, ctypes.c_int32, u8p,
                                                u8p, ctypes.c_int32, i32p, ctypes.c_int32]
    return _lib


def _p(a: np.ndarray, t):
    return a.ctypes.data_as(ctypes.POINTER(t)) if a is not None else None


def bytes_(length: int, seed: int) -> np.ndarray:
    """Int8Tests.Bytes (Int8Tests.cs:36-47)."""
    out = np.empty(max(length, 0), dtype=np.uint8)
    lib().og_oracle_bytes(_p(out, ctypes.c_uint8), out.size, seed)
    return out


def random(n: int, seed: int, lo: float, hi: float) -> np.ndarray:
    """Rig.Random (Rig.cs:8-19)."""
    out = np.empty(n, dtype=np.float32)
    lib().og_oracle_random(_p(out, ctypes.c_float), n, seed, lo, hi)
    return out


def dq_input(count: int, seed: int, kind: int) -> np.ndarray:
    """The DynamicQuantizeIsBitExact inputs (Int8Tests.cs:632-647)."""
    out = np.empty(count, dtype=np.float32)
    lib().og_oracle_dq_input(_p(out, ctypes.c_float), count, seed, kind)
    return out


def _problem(m, n, k, batch=1, transpose_b=False, lda=0, ldb=0, offset_a=0, offset_b=0, stride_a=0, stride_b=0):
    return Problem(m, n, k, batch, int(bool(transpose_b)), lda, ldb, offset_a, offset_b, stride_a, stride_b)


def int8_gemm(a: np.ndarray, a_signed: bool, b: np.ndarray, b_signed: bool, za=None, za_vector=False, zb=None,
              zb_vector=False, threads: int = 0, signed_domain: bool = False, tiled: bool = False,
              **shape) -> np.ndarray:
    """Int8Tests.Reference (Int8Tests.cs:52-82): int32 sums (wrapping) of sum_k (A - za)(B - zb); returns
    [batch*m*n]. Bytes are passed as uint8 whatever their signedness."""
    p = _problem(**shape)
    out = np.zeros(max(p.batch * p.m * p.n, 1), dtype=np.int32)
    a = np.ascontiguousarray(a, dtype=np.uint8)
    b = np.ascontiguousarray(b, dtype=np.uint8)
    za = None if za is None else np.ascontiguousarray(za, dtype=np.uint8)
    zb = None if zb is None else np.ascontiguousarray(zb, dtype=np.uint8)
    u8 = ctypes.c_uint8
    args = [ctypes.byref(p), _p(a, u8), int(a_signed), _p(b, u8), int(b_signed), _p(za, u8), int(za_vector),
            _p(zb, u8), int(zb_vector), _p(out, ctypes.c_int32)]
    if signed_domain:
        lib().og_oracle_int8_gemm_signed_domain(*args)
    elif tiled:  # Int8GemmKernel.hlsl's blocking: the same sums, the second CPU baseline
        lib().og_oracle_int8_gemm_tiled(*args, threads if threads > 0 else (os.cpu_count() or 1))
    else:
        lib().og_oracle_int8_gemm(*args, threads if threads > 0 else (os.cpu_count() or 1))
    return out[: p.batch * p.m * p.n]


def requant(acc: int, mult: float, zero: int, unsigned: bool) -> int:
    """Int8Tests.Requant (Int8Tests.cs:84-97)."""
    return int(lib().og_oracle_requant(int(np.int32(acc)), float(np.float32(mult)), zero, int(unsigned)))


def requant_array(acc: np.ndarray, mult: np.ndarray, zero: int, unsigned: bool) -> np.ndarray:
    out = np.empty(acc.size, dtype=np.uint8)
    f = lib().og_oracle_requant
    for i, (s, m) in enumerate(zip(acc.tolist(), mult.tolist())):
        out[i] = f(s, m, zero, int(unsigned)) & 0xFF
    return out


def float_epilogue(acc: np.ndarray, scale: np.ndarray, int_bias=None, float_bias=None) -> np.ndarray:
    """The float form (Int8Tests.cs:356-373), vectorised: float32 rounding of each step, no fused multiply-add."""
    s = acc.astype(np.int64)
    if int_bias is not None:
        s = s + int_bias.astype(np.int64)
    s = ((s + 2 ** 31) % 2 ** 32 - 2 ** 31).astype(np.int32)
    f = (s.astype(np.float32) * scale.astype(np.float32)).astype(np.float32)
    if float_bias is not None:
        f = (f + float_bias.astype(np.float32)).astype(np.float32)
    return f


def float_epilogue_scalar(acc: int, scale: float, int_bias=None, float_bias=None) -> float:
    return float(lib().og_oracle_float_epilogue(int(acc), int(int_bias is not None),
                                                int(int_bias) if int_bias is not None else 0, float(scale),
                                                int(float_bias is not None),
                                                float(float_bias) if float_bias is not None else 0.0))


def dynamic_quantize(x: np.ndarray):
    """Int8Tests.DynamicReference (Int8Tests.cs:577-615): (y, scale, zero_point)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty(x.size, dtype=np.uint8)
    s = np.zeros(1, dtype=np.float32)
    z = np.zeros(1, dtype=np.uint8)
    lib().og_oracle_dynamic_quantize(_p(x, ctypes.c_float), x.size, _p(y, ctypes.c_uint8), _p(s, ctypes.c_float),
                                     _p(z, ctypes.c_uint8))
    return y, np.float32(s[0]), int(z[0])


def div_exact(x: float, s: float) -> float:
    """DivExact (DivExact.hlsli:28-99)."""
    return float(lib().og_oracle_div_exact(float(np.float32(x)), float(np.float32(s))))


def float_to_half(f: float) -> int:
    """The C# (Half) cast: binary16 bits, round to nearest even."""
    return int(lib().og_oracle_float_to_half(float(np.float32(f))))


def half_to_float(h: int) -> float:
    return float(lib().og_oracle_half_to_float(int(h)))


def _params(shape, axis, per_axis):
    count = int(np.prod(shape)) if len(shape) else 1
    if not per_axis:
        return count, 1, 1
    ax = axis + len(shape) if axis < 0 else axis
    inner = int(np.prod(shape[ax + 1:])) if ax + 1 < len(shape) else 1
    return count, int(shape[ax]), inner


def dequantize(x: np.ndarray, shape, axis: int, per_axis: bool, scale: np.ndarray, zero_point=None,
               half_out: bool = False) -> np.ndarray:
    """DequantizeTests.cs:57-68 over x (uint8, int8 or int32 elements, already offset): float32 values, or binary16
    bits as uint16 with half_out."""
    kind = {np.dtype(np.uint8): 0, np.dtype(np.int8): 1, np.dtype(np.int32): 2}[np.dtype(x.dtype)]
    count, axis_len, inner = _params(shape, axis, per_axis)
    x = np.ascontiguousarray(x[:count])
    scale = np.ascontiguousarray(scale, dtype=np.float32)
    zp = None if zero_point is None else np.ascontiguousarray(zero_point, dtype=x.dtype)
    out = np.empty(count, dtype=np.uint16 if half_out else np.float32)
    lib().og_oracle_dequantize(kind, x.ctypes.data, count, int(bool(per_axis)), axis_len, inner,
                               _p(scale, ctypes.c_float), None if zp is None else zp.ctypes.data, int(bool(half_out)),
                               out.ctypes.data)
    return out


def quantize(x: np.ndarray, shape, axis: int, per_axis: bool, scale: np.ndarray, zero_point=None,
             signed: bool = False) -> np.ndarray:
    """DequantizeTests.cs:138-148 over x (float32, or float16 taken as its binary16 bits): uint8 bytes of the
    uint8 / int8 results."""
    half_in = np.dtype(x.dtype) == np.dtype(np.float16)
    count, axis_len, inner = _params(shape, axis, per_axis)
    x = np.ascontiguousarray(x[:count])
    scale = np.ascontiguousarray(scale, dtype=np.float32)
    zp = None if zero_point is None else np.ascontiguousarray(zero_point).view(np.uint8)
    out = np.empty(count, dtype=np.uint8)
    lib().og_oracle_quantize(int(bool(signed)), int(half_in), x.ctypes.data, count, int(bool(per_axis)), axis_len,
                             inner, _p(scale, ctypes.c_float), _p(zp, ctypes.c_uint8), _p(out, ctypes.c_uint8))
    return out


def conv_out_extent(input_, kernel, stride, dilation, pad_begin, pad_end) -> int:
    return int(lib().og_oracle_conv_out_extent(input_, kernel, stride, dilation, pad_begin, pad_end))


def conv_integer(p: dict, x: np.ndarray, x_signed: bool, w: np.ndarray, w_signed: bool, xz=None, wz=None,
                 wz_vector: bool = False, threads: int = 0) -> np.ndarray:
    """ConvIntegerTests.cs:41-88 (Reference): y [batch, cout, oh, ow] int32. `p` holds the fields of Conv (missing
    ones default: strides and dilations 1, paddings and offsets 0, groups 1)."""
    d = dict(stride_h=1, stride_w=1, dilation_h=1, dilation_w=1, pad_top=0, pad_left=0, pad_bottom=0, pad_right=0,
             groups=1, offset_x=0, offset_w=0)
    d.update(p)
    c = Conv(**{k: int(d[k]) for k, _ in Conv._fields_})
    oh = conv_out_extent(c.h, c.kh, c.stride_h, c.dilation_h, c.pad_top, c.pad_bottom)
    ow = conv_out_extent(c.w, c.kw, c.stride_w, c.dilation_w, c.pad_left, c.pad_right)
    y = np.zeros(max(c.batch * c.cout * oh * ow, 1), dtype=np.int32)
    x = np.ascontiguousarray(x).view(np.uint8)
    w = np.ascontiguousarray(w).view(np.uint8)
    xz = None if xz is None else np.ascontiguousarray(xz).view(np.uint8)
    wz = None if wz is None else np.ascontiguousarray(wz).view(np.uint8)
    lib().og_oracle_conv_integer(ctypes.byref(c), _p(x, ctypes.c_uint8), int(bool(x_signed)), _p(w, ctypes.c_uint8),
                                 int(bool(w_signed)), _p(xz, ctypes.c_uint8), _p(wz, ctypes.c_uint8),
                                 int(bool(wz_vector)), _p(y, ctypes.c_int32),
                                 threads if threads > 0 else (os.cpu_count() or 1))
    return y[: c.batch * c.cout * oh * ow].reshape(c.batch, c.cout, oh, ow)
