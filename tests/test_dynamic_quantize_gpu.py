"""DynamicQuantizeKernels on the GPU through the C ABI, bit for bit against the oracle (Int8Tests.cs:617-751)."""
import numpy as np
import pytest

import og_oracle as oracle
import onegpu_cuda as og
from cases import golden, oracle_shape, problem

pytestmark = pytest.mark.gpu


def test_dynamic_quantize_is_bit_exact(device):
    """DynamicQuantizeIsBitExact: 15 counts x 7 distributions, odd offsets, sentinel bytes around every output."""
    t = golden()["tables"]["dq_counts"]
    off_x, off_y, off_s, off_z = 1, 3, 2, 5
    with og.DynamicQuantizeKernels(device) as dq:
        seed = 1
        bad = 0
        for count in t["counts"]:
            for kind in t["kinds"]:
                x = oracle.dq_input(count, seed, kind)
                wy, ws, wz = oracle.dynamic_quantize(x)
                xs = np.concatenate([np.zeros(off_x, np.float32), x])
                y_init = np.full(((off_y + count + 3) & ~3) + 4, 0x3C, np.uint8)
                z_init = np.full(8, 0xEE, np.uint8)
                bx = device.create_buffer(np.float32, xs)
                by = device.create_buffer(np.uint8, y_init)
                bs = device.create_buffer(np.float32, np.zeros(4, np.float32))
                bz = device.create_buffer(np.uint8, z_init)
                enc = device.begin_commands()
                dq.encode(enc, bx, off_x, count, by, off_y, bs, off_s, bz, off_z)
                device.submit(enc)
                y, s, z = by.read(), bs.read(), bz.read()
                here = int(np.count_nonzero(y[off_y:off_y + count] != wy))
                here += int(s[off_s].view(np.uint32) != np.float32(ws).view(np.uint32))
                here += int(z[off_z] != wz)
                here += int(np.count_nonzero(y[:off_y] != 0x3C)) + int(np.count_nonzero(y[off_y + count:] != 0x3C))
                here += int(np.count_nonzero(np.delete(z, off_z) != 0xEE))
                assert here == 0, f"count {count} kind {kind}: scale {s[off_s]!r} want {ws!r}, zero {z[off_z]} want {wz}"
                bad += here
                for v in (bx, by, bs, bz):
                    v.dispose()
                seed += 1
        assert bad == 0


@pytest.mark.parametrize("count", [4096 * 4096, 8 * 2048 * 4096 + 5])
def test_dynamic_quantize_full_size(device, count):
    """The configs' sizes (16.8 M and 67 M elements) against the oracle, aligned and misaligned offsets."""
    rng = np.random.default_rng(count)
    x = rng.standard_normal(count).astype(np.float32) * np.float32(0.5)
    wy, ws, wz = oracle.dynamic_quantize(x)
    with og.DynamicQuantizeKernels(device) as dq:
        for off in (0, 1):
            bx = device.create_buffer(np.float32, np.concatenate([np.zeros(off, np.float32), x]))
            by = device.create_buffer(np.uint8, count + off)
            bs = device.create_buffer(np.float32, 1)
            bz = device.create_buffer(np.uint8, 1)
            enc = device.begin_commands()
            dq.encode(enc, bx, off, count, by, off, bs, 0, bz, 0)
            device.submit(enc)
            assert np.array_equal(by.read()[off:], wy)
            assert bs.read()[0].view(np.uint32) == np.float32(ws).view(np.uint32)
            assert int(bz.read()[0]) == wz
            for v in (bx, by, bs, bz):
                v.dispose()


@pytest.mark.parametrize("m,n,k,trans_b,options", [
    (128, 384, 384, True, og.Int8GemmOptions()),
    (128, 384, 384, True, og.Int8GemmOptions(allow_packed_dot=False)),
    (16, 384, 384, False, og.Int8GemmOptions()),           # the few-rows kernel
])
def test_dynamic_quantize_then_fused_dequantize_product(device, m, n, k, trans_b, options):
    """The DynamicQuantizeLinear -> MatMulIntegerToFloat chain with the scale product formed in the epilogue:
    expected (float)sum * (a_scale * b_scale[n]) with a per-column zero point of the weights."""
    rng = np.random.default_rng(m + n + k)
    x = rng.standard_normal(m * k).astype(np.float32)
    wy, wscale, wzero = oracle.dynamic_quantize(x)
    w = rng.integers(-127, 128, size=n * k).astype(np.int8)
    zw = rng.integers(-8, 9, size=n).astype(np.int8)
    bscale = rng.uniform(0.001, 0.02, size=n).astype(np.float32)
    rows = np.arange(m)
    p = problem(m, n, k, trans_b=trans_b)
    sums = oracle.int8_gemm(wy.reshape(m, k)[rows].reshape(-1), False, w.view(np.uint8), True,
                            np.array([wzero], np.uint8), False, zw.view(np.uint8), True,
                            **dict(oracle_shape(p), m=len(rows)))
    scale_vec = (np.float32(wscale) * bscale).astype(np.float32)
    want = (sums.astype(np.float32) * np.tile(scale_vec, len(rows))).astype(np.float32)
    with og.DynamicQuantizeKernels(device) as dq, og.Int8Gemm(device, options) as gemm:
        bx = device.create_buffer(np.float32, x)
        by = device.create_buffer(np.uint8, m * k)
        bs = device.create_buffer(np.float32, 1)
        bz = device.create_buffer(np.uint8, 1)
        bw = device.create_buffer(np.int8, w)
        bzw = device.create_buffer(np.int8, zw)
        bbs = device.create_buffer(np.float32, bscale)
        bc = device.create_buffer(np.float32, m * n)
        enc = device.begin_commands()
        dq.encode(enc, bx, 0, m * k, by, 0, bs, 0, bz, 0)
        gemm.encode_dequantize(enc, og.Int8GemmProblem(**p), by, bw, bc, og.Int8Operand(bs, 0),
                               og.Int8Operand(bbs, 0, True), og.Int8Operand(bz, 0), og.Int8Operand(bzw, 0, True))
        device.submit(enc)
        got = bc.read().reshape(m, n)[rows].reshape(-1)
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), gemm.last_kernel
        for v in (bx, by, bs, bz, bw, bzw, bbs, bc):
            v.dispose()


def test_dynamic_quantize_feeds_the_product_without_leaving_the_device(device):
    """DynamicQuantizeFeedsTheProductWithoutLeavingTheDevice (Int8Tests.cs:705-751): quantize, then the float form
    with the activation's zero point read from the device; expected (float)sum * (a_scale * w_scale[n])."""
    M, N, K = 128, 384, 384
    x = oracle.random(M * K, 3, -3.0, 5.0)
    wy, wscale, wzero = oracle.dynamic_quantize(x)
    w = oracle.bytes_(N * K, 4)
    wscales = (np.float32(0.002) + (np.arange(N) % 17).astype(np.float32) * np.float32(1e-4)).astype(np.float32)
    p = problem(M, N, K, trans_b=True)
    sums = oracle.int8_gemm(wy, False, w, True, np.array([wzero], np.uint8), False, **oracle_shape(p))
    scale_vec = (np.float32(wscale) * wscales).astype(np.float32)  # the elementwise Mul of the chain, in float32
    want = (sums.astype(np.float32) * np.tile(scale_vec, M)).astype(np.float32)
    with og.DynamicQuantizeKernels(device) as dq, og.Int8Gemm(device) as gemm:
        bx = device.create_buffer(np.float32, x)
        by = device.create_buffer(np.uint8, M * K)
        bs = device.create_buffer(np.float32, 1)
        bz = device.create_buffer(np.uint8, 1)
        bw = device.create_buffer(np.int8, w.view(np.int8))
        bscale = device.create_buffer(np.float32, scale_vec)
        bc = device.create_buffer(np.float32, M * N)
        enc = device.begin_commands()
        dq.encode(enc, bx, 0, M * K, by, 0, bs, 0, bz, 0)
        gemm.encode_float(enc, og.Int8GemmProblem(**p), by, bw, bc, og.Int8Operand(bscale, 0, True),
                          og.Int8Operand(bz, 0))
        device.submit(enc)
        got = bc.read()
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
        assert bs.read()[0].view(np.uint32) == np.float32(wscale).view(np.uint32)
        for v in (bx, by, bs, bz, bw, bscale, bc):
            v.dispose()


def test_dynamic_quantize_near_ties(device):
    """Inputs crowded within a few ulps of half-integer quotients x / scale, the scale fixed by the range's ends,
    for ranges that give zero points at 0, in the middle and at 255; sizes that take the vector and scalar paths."""
    rng = np.random.default_rng(3)
    with og.DynamicQuantizeKernels(device) as dq:
        for lo, hi in ((-1.0, 3.0), (-2.5, 0.75), (0.0, 1.7), (-0.3, 0.0), (-1000.0, 10.0)):
            _, scale, _ = oracle.dynamic_quantize(np.array([lo, hi], np.float32))
            scale = np.float32(scale)
            for count, off in ((1 << 20, 0), (100003, 1)):
                k = rng.integers(int(np.ceil(lo / scale)), int(np.floor(hi / scale)), size=count).astype(np.float64)
                x = ((k + 0.5) * np.float64(scale)).astype(np.float32)
                x = (x.view(np.int32) + rng.integers(-4, 5, size=count).astype(np.int32)).view(np.float32)
                x = np.clip(x, np.float32(lo), np.float32(hi)).astype(np.float32)
                x[:2] = (lo, hi)
                wy, ws, wz = oracle.dynamic_quantize(x)
                assert np.float32(ws) == scale
                bx = device.create_buffer(np.float32, np.concatenate([np.zeros(off, np.float32), x]))
                by = device.create_buffer(np.uint8, count + off + 3)
                bs, bz = device.create_buffer(np.float32, 1), device.create_buffer(np.uint8, 4)
                enc = device.begin_commands()
                dq.encode(enc, bx, off, count, by, off, bs, 0, bz, 0)
                device.submit(enc)
                got = by.read()[off:off + count]
                bad = int(np.count_nonzero(got != wy))
                for v in (bx, by, bs, bz):
                    v.dispose()
                assert bad == 0, f"range [{lo}, {hi}] count {count}: {bad} bytes differ"


def _run_dq(device, dq, x, off_x, off_y):
    """One DynamicQuantizeLinear through the C ABI with sentinel bytes around the output; returns (y, scale, zero
    point, launches recorded, stray bytes)."""
    count = x.size
    bx = device.create_buffer(np.float32, np.concatenate([np.zeros(off_x, np.float32), x]))
    by = device.create_buffer(np.uint8, np.full(off_y + count + 8, 0x3C, np.uint8))
    bs = device.create_buffer(np.float32, 1)
    bz = device.create_buffer(np.uint8, np.full(4, 0xEE, np.uint8))
    try:
        enc = device.begin_commands()
        dq.encode(enc, bx, off_x, count, by, off_y, bs, 0, bz, 0)
        launches = enc.dispatch_count
        device.submit(enc)
        y, s, z = by.read(), bs.read()[0], bz.read()
    finally:
        for v in (bx, by, bs, bz):
            v.dispose()
    stray = int(np.count_nonzero(y[:off_y] != 0x3C)) + int(np.count_nonzero(y[off_y + count:] != 0x3C))
    stray += int(np.count_nonzero(z[1:] != 0xEE))
    return y[off_y:off_y + count], s, int(z[0]), launches, stray


@pytest.mark.parametrize("count", [1 << 18, (1 << 18) + 3, 1_000_003, 4096 * 4096])
def test_dynamic_quantize_single_kernel_is_bit_exact(device, count):
    """Tensors of 2^18 elements and more whose input starts on a 16-byte boundary run as one kernel (range, grid
    barrier, quantize from the copies kept in shared memory and registers, the rest read again): every distribution of
    DynamicQuantizeIsBitExact (Int8Tests.cs:632-647) against the oracle, at the threshold, with a tail of elements past
    the last whole float4, with slices that have a re-read rest, and at config 2's size; misaligned inputs still take
    the two launches."""
    kinds = golden()["tables"]["dq_counts"]["kinds"]
    with og.DynamicQuantizeKernels(device) as dq:
        for seed, kind in enumerate(kinds, start=count % 1000):
            x = oracle.dq_input(count, seed, kind)
            wy, ws, wz = oracle.dynamic_quantize(x)
            for off_x, off_y, launches_want in ((0, 0, 1), (4, 8, 1), (1, 0, 2)):
                y, s, z, launches, stray = _run_dq(device, dq, x, off_x, off_y)
                what = f"kind {kind} offsets {off_x}/{off_y}"
                assert launches == launches_want, what
                assert stray == 0, what
                assert np.array_equal(y, wy), what
                assert np.float32(s).view(np.uint32) == np.float32(ws).view(np.uint32), what
                assert z == wz, what


def test_dynamic_quantize_single_kernel_special_values(device):
    """NaN (skipped by the range, quantized to 0), infinities (an infinite scale: zero point 0) and an all-zero tensor
    (scale 1, zero point 0) through the single kernel."""
    count = 3 * (1 << 18) + 1
    rng = np.random.default_rng(5)
    base = rng.standard_normal(count).astype(np.float32)
    cases = []
    x = base.copy()
    x[rng.choice(count, 1000, replace=False)] = np.nan
    cases.append(x)
    x = base.copy()
    x[[7, count - 1]] = [np.inf, -np.inf]
    cases.append(x)
    cases.append(np.zeros(count, np.float32))
    with og.DynamicQuantizeKernels(device) as dq:
        for i, x in enumerate(cases):
            wy, ws, wz = oracle.dynamic_quantize(x)
            y, s, z, launches, stray = _run_dq(device, dq, x, 0, 0)
            assert launches == 1 and stray == 0, i
            assert np.array_equal(y, wy), i
            assert np.float32(s).view(np.uint32) == np.float32(ws).view(np.uint32), i
            assert z == wz, i
