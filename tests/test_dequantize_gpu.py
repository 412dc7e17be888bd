"""DequantizeLinear and QuantizeLinear on the GPU against the oracle, bit for bit (DequantizeTests.cs:99-111,
252-287): every case of the reference's table, per tensor and per axis, with and without a zero point, float32 and
half, odd offsets, sentinel values around every output."""
import numpy as np
import pytest

import og_oracle as oracle
import onegpu_cuda as og
from cases import axis_params, golden, quantize_input, quantized

TABLE = golden()["dequantize"]
OFF = TABLE["offsets"]
OFFX, OFFS, OFFZ, OFFO = OFF["OffX"], OFF["OffS"], OFF["OffZ"], OFF["OffO"]
NP = {"u8": np.uint8, "s8": np.int8, "i32": np.int32}


def _dequantize_case(device, k, kind, shape, axis, per_axis, with_zero, half, seed):
    count, axis_len, _ = axis_params(shape, axis, per_axis)
    x = quantized(kind, count + OFFX, seed)
    scale = oracle.random(axis_len + OFFS, seed + 1, 0.001, 2.0).astype(np.float32)
    zeros = quantized(kind, axis_len + OFFZ, seed + 2)
    out_len = count + OFFO + 1
    out_len += out_len % 2 if half else 0
    sentinel = np.full(out_len, -77.0, np.float16 if half else np.float32)
    bufs = [device.create_buffer(NP[kind], x), device.create_buffer(np.float32, scale),
            device.create_buffer(NP[kind], zeros), device.create_buffer(sentinel.dtype, sentinel)]
    bx, bs, bz, bo = bufs
    try:
        enc = device.begin_commands()
        k.encode(enc, bx, OFFX, shape, axis, per_axis, bs, OFFS, bz if with_zero else None, OFFZ, bo, OFFO)
        device.submit(enc)
        got = bo.read()
    finally:
        for b in bufs:
            b.dispose()
    want = oracle.dequantize(x[OFFX:], shape, axis, per_axis, scale[OFFS:], zeros[OFFZ:] if with_zero else None, half)
    bits = np.uint16 if half else np.uint32
    bad = int(np.count_nonzero(got[OFFO:OFFO + count].view(bits) != want.view(bits)))
    guard = np.concatenate([got[:OFFO], got[OFFO + count:]]).view(bits)
    return bad + int(np.count_nonzero(guard != sentinel[:guard.size].view(bits)))


@pytest.mark.gpu
@pytest.mark.parametrize("kind,seed0", [("u8", 1), ("s8", 100), ("i32", 200)])
def test_dequantize_is_exact(device, kind, seed0):
    k = og.DequantizeKernels(device)
    try:
        bad, runs, seed = 0, 0, seed0
        for shape, axis, per_axis in TABLE["cases"]:
            for with_zero in (True, False):
                for half in (False, True):
                    bad += _dequantize_case(device, k, kind, shape, axis, per_axis, with_zero, half, seed)
                    seed += 1
                    runs += 1
        assert runs == 4 * len(TABLE["cases"])
        assert bad == 0
    finally:
        k.dispose()


def _quantize_case(device, k, shape, axis, per_axis, with_zero, signed, half_in, scales, seed):
    count, axis_len, _ = axis_params(shape, axis, per_axis)
    x = quantize_input(count + OFFX, seed)
    if half_in:  # Rig.ToHalf: padded to a whole 32-bit word
        with np.errstate(over="ignore"):
            x = np.concatenate([x, np.zeros(x.size % 2, np.float32)]).astype(np.float16)
    scale = np.array([scales[i % len(scales)] for i in range(axis_len + OFFS)], np.float32)
    zeros = quantized("s8" if signed else "u8", axis_len + OFFZ, seed + 2)
    out_len = count + OFFO + 3
    out_len += (-out_len) % 4
    fill = np.full(out_len, 177, np.uint8) if not signed else np.full(out_len, -77, np.int8)
    out_t = np.int8 if signed else np.uint8
    bufs = [device.create_buffer(x.dtype, x), device.create_buffer(np.float32, scale),
            device.create_buffer(out_t, zeros.view(out_t)), device.create_buffer(out_t, fill)]
    bx, bs, bz, bo = bufs
    try:
        enc = device.begin_commands()
        k.encode_quantize(enc, bx, OFFX, shape, axis, per_axis, bs, OFFS, bz if with_zero else None, OFFZ, bo, OFFO)
        device.submit(enc)
        got = bo.read().view(np.uint8)
    finally:
        for b in bufs:
            b.dispose()
    want = oracle.quantize(x[OFFX:], shape, axis, per_axis, scale[OFFS:], zeros[OFFZ:] if with_zero else None, signed)
    bad = int(np.count_nonzero(got[OFFO:OFFO + count] != want))
    guard = np.concatenate([got[:OFFO], got[OFFO + count:]])
    return bad + int(np.count_nonzero(guard != fill.view(np.uint8)[:guard.size]))


@pytest.mark.gpu
def test_quantize_is_exact(device):
    k = og.DequantizeKernels(device)
    try:
        sets = TABLE["scale_sets"]
        bad, count, seed = 0, 0, 1
        for shape, axis, per_axis in TABLE["cases"]:
            for with_zero in (True, False):
                scales = sets[count % len(sets)]
                for signed, half_in in ((False, False), (True, False), (False, True), (True, True)):
                    bad += _quantize_case(device, k, shape, axis, per_axis, with_zero, signed, half_in, scales, seed)
                    seed += 1
                count += 4
        assert count == 8 * len(TABLE["cases"])
        assert bad == 0
    finally:
        k.dispose()


@pytest.mark.gpu
def test_large_tensors_per_axis(device):
    """A 64 Mi-element tensor each way (per-axis over the middle axis, odd offsets), against the oracle."""
    k = og.DequantizeKernels(device)
    shape, axis = [64, 1025, 1024], 1
    count, axis_len, _ = axis_params(shape, axis, True)
    rng = np.random.default_rng(5)
    try:
        # Byte tensors end on a whole 32-bit word (GpuKernelBuffers.PaddedBoolLength).
        x = rng.integers(-128, 128, size=count + 4, dtype=np.int16).astype(np.int8)
        scale = rng.uniform(0.001, 2.0, size=axis_len).astype(np.float32)
        zp = rng.integers(-128, 128, size=axis_len + 3, dtype=np.int16).astype(np.int8)
        bx, bs, bz = device.create_buffer(np.int8, x), device.create_buffer(np.float32, scale), \
            device.create_buffer(np.int8, zp)
        bo = device.create_buffer(np.float16, count + 2)
        enc = device.begin_commands()
        k.encode(enc, bx, 3, shape, axis, True, bs, 0, bz, 0, bo, 1)
        device.submit(enc)
        got = bo.read()[1:1 + count].view(np.uint16)
        want = oracle.dequantize(x[3:], shape, axis, True, scale, zp[:axis_len], True)
        assert np.array_equal(got, want)
        for b in (bx, bo):
            b.dispose()

        xf = (rng.standard_normal(count + 5).astype(np.float32) * np.float32(30.0))
        bx, by = device.create_buffer(np.float32, xf), device.create_buffer(np.int8, count + 8)
        enc = device.begin_commands()
        k.encode_quantize(enc, bx, 5, shape, axis, True, bs, 0, bz, 0, by, 7)
        device.submit(enc)
        got = by.read().view(np.uint8)[7:7 + count]
        want = oracle.quantize(xf[5:], shape, axis, True, scale, zp[:axis_len], True)
        assert np.array_equal(got, want)
        for b in (bx, by, bs, bz):
            b.dispose()
    finally:
        k.dispose()


def _near_ties(scale: np.float32, n: int, rng) -> np.ndarray:
    """Values within a few ulps of (k + 1/2) * scale, where the quotient's rounding is decided by its last bits."""
    k = rng.integers(-300, 300, size=n).astype(np.float64)
    base = ((k + 0.5) * np.float64(scale)).astype(np.float32)
    return (base.view(np.int32) + rng.integers(-4, 5, size=n).astype(np.int32)).view(np.float32)


@pytest.mark.gpu
def test_quantize_near_ties(device):
    """The uniform-scale quotient (multiply by the rounded reciprocal, divide where that could round differently) on
    inputs crowded around half-integer quotients, plus NaN, infinities, zeros, subnormals and huge values, per tensor
    and per axis (long runs of one scale), against the oracle's division."""
    k = og.DequantizeKernels(device)
    rng = np.random.default_rng(11)
    specials = np.array([np.nan, np.inf, -np.inf, 0.0, -0.0, 1e-42, -1e-42, 3e38, -3e38, 1e-30, 7e6, -7e6],
                        np.float32)
    try:
        for scale in (np.float32(0.1), np.float32(0.0234), np.float32(3.0), np.float32(1e-3), np.float32(7.5e-6),
                      np.float32(1e30), np.float32(1e-38)):
            count = 1 << 16
            x = np.concatenate([_near_ties(scale, count - specials.size, rng), specials])
            for signed in (False, True):
                for per_axis in (False, True):
                    shape, axis = ([4, 4, count // 16], 1) if per_axis else ([count], 0)
                    axis_len = 4 if per_axis else 1
                    scales = np.full(axis_len, scale, np.float32)
                    zp = rng.integers(-20, 20, size=axis_len + 3, dtype=np.int16).astype(np.int8)
                    zp = zp if signed else zp.view(np.uint8)
                    out_t = np.int8 if signed else np.uint8
                    bx, bs = device.create_buffer(np.float32, x), device.create_buffer(np.float32, scales)
                    bz, by = device.create_buffer(out_t, zp.view(out_t)), device.create_buffer(out_t, count)
                    enc = device.begin_commands()
                    k.encode_quantize(enc, bx, 0, shape, axis, per_axis, bs, 0, bz, 0, by, 0)
                    device.submit(enc)
                    got = by.read().view(np.uint8)
                    want = oracle.quantize(x, shape, axis, per_axis, scales, zp[:axis_len], signed)
                    for b in (bx, bs, bz, by):
                        b.dispose()
                    assert np.array_equal(got, want), f"scale {scale} signed {signed} per_axis {per_axis}"
    finally:
        k.dispose()


@pytest.mark.gpu
def test_dequantize_parameters_along_the_contiguous_axis(device):
    """Per-axis parameters on the last axis with aligned buffers, where each vector's scales and zero points are
    consecutive and load as whole vectors; sizes with and without whole vectors, both byte kinds, both outputs."""
    k = og.DequantizeKernels(device)
    rng = np.random.default_rng(21)
    try:
        for shape in ([3, 64], [5, 1000], [2, 3, 1024], [7, 8], [4, 12]):
            axis = len(shape) - 1
            count, axis_len, _ = axis_params(shape, axis, True)
            for kind in ("u8", "s8"):
                for half in (False, True):
                    for with_zero in (True, False):
                        for off_x, off_o in ((0, 0), (4, 8), (3, 0)):
                            x = quantized(kind, count + off_x + 4, int(rng.integers(1 << 30)))
                            scale = rng.uniform(0.001, 2.0, size=axis_len).astype(np.float32)
                            zeros = quantized(kind, axis_len + 4, int(rng.integers(1 << 30)))
                            out_len = count + off_o + 8
                            bx, bs = device.create_buffer(NP[kind], x), device.create_buffer(np.float32, scale)
                            bz = device.create_buffer(NP[kind], zeros)
                            bo = device.create_buffer(np.float16 if half else np.float32, out_len)
                            enc = device.begin_commands()
                            k.encode(enc, bx, off_x, shape, axis, True, bs, 0, bz if with_zero else None, 0, bo, off_o)
                            device.submit(enc)
                            got = bo.read()[off_o:off_o + count]
                            for b in (bx, bs, bz, bo):
                                b.dispose()
                            want = oracle.dequantize(x[off_x:], shape, axis, True, scale,
                                                     zeros[:axis_len] if with_zero else None, half)
                            bits = np.uint16 if half else np.uint32
                            assert np.array_equal(got.view(bits), want.view(bits)), \
                                f"{shape} {kind} half={half} zero={with_zero} offsets {off_x}, {off_o}"
    finally:
        k.dispose()
