"""The allocation-free EncodeInt32 (og_int8_gemm_int32_noalloc) against the allocating one.

Some callers cannot call cudaMalloc: code recording work during a CUDA graph capture in the global capture mode, and
hosts that hand all device memory to their own pool. For them the entry point keeps the byte sums of the zero-point
correction in a fixed device array of the library (at most 1,048,576 int32) instead of scratch it allocates. This file
runs last (pytest collects it after the others) so that a failure here leaves every other test already run; it passes
alone in a fresh process and after the other tests alike.
"""
import numpy as np
import pytest

import og_oracle as oracle
import onegpu_cuda as og

pytestmark = pytest.mark.gpu


def run_both(device, p, a, b, za, zb):
    """Runs the product through og_int8_gemm_encode_int32 and through og_int8_gemm_int32_noalloc on the device's
    stream; returns both results."""
    ba = device.create_buffer(np.uint8, a)
    bb = device.create_buffer(np.int8, b.view(np.int8))
    bza = device.create_buffer(np.uint8, za)
    bzb = device.create_buffer(np.int8, zb.view(np.int8))
    count = p.batch * p.m * p.n
    c_ref = device.create_buffer(np.int32, count)
    c_new = device.create_buffer(np.int32, np.full(count, 0x5A5A5A5A, np.int32))
    zpa, zpb = og.Int8Operand(bza, 0), og.Int8Operand(bzb, 0, True)
    with og.Int8Gemm(device) as gemm:
        enc = device.begin_commands()
        gemm.encode_int32(enc, p, ba, bb, c_ref, zpa, zpb)
        kernel = gemm.last_kernel
        device.submit(enc)
    og.int8_gemm_int32_noalloc(device.stream, p, ba, bb, c_new, zpa, zpb)
    device.wait_idle()
    ref, new = c_ref.read(), c_new.read()
    for v in (ba, bb, bza, bzb, c_ref, c_new):
        v.dispose()
    return ref, new, kernel


def test_no_alloc_matches_the_allocating_entry_point_twice(device):
    rng = np.random.default_rng(2024)
    shapes = [og.Int8GemmProblem(640, 528, 384), og.Int8GemmProblem(300, 1040, 256, batch=3, stride_a=300 * 256)]
    for p in shapes:  # two calls in a row: the second reuses the fixed array the first left behind
        a = rng.integers(0, 256, size=p.batch * p.m * p.k, dtype=np.int64).astype(np.uint8)
        b = rng.integers(-128, 128, size=p.k * p.n, dtype=np.int64).astype(np.int8)
        za = np.array([rng.integers(0, 256)], np.uint8)
        zb = rng.integers(-8, 9, size=p.n).astype(np.int8)
        ref, new, kernel = run_both(device, p, a, b, za, zb)
        assert kernel.startswith("tensor-core")  # the path that needs the byte sums
        assert np.array_equal(new, ref)
        # and both equal the definition on a few rows
        rows = [0, p.m - 1]
        want = oracle.int8_gemm(a[:p.m * p.k].reshape(p.m, p.k)[rows], False, b.view(np.uint8), True, za, False,
                                zb.view(np.uint8), True, m=len(rows), n=p.n, k=p.k)
        assert np.array_equal(new.reshape(p.batch, p.m, p.n)[0][rows].reshape(-1), want)


def test_no_alloc_refuses_products_beyond_its_array(device):
    p = og.Int8GemmProblem((1 << 20) + 16, 64, 16)  # row sums of A alone exceed the array by 16
    a = device.create_buffer(np.uint8, p.m * p.k)
    b = device.create_buffer(np.int8, p.k * p.n)
    c = device.create_buffer(np.int32, p.m * p.n)
    zb = device.create_buffer(np.int8, np.ones(p.n, np.int8))
    with pytest.raises(og.GpuUnsupportedException) as e:
        og.int8_gemm_int32_noalloc(device.stream, p, a, b, c, None, og.Int8Operand(zb, 0, True))
    assert e.value.capability == "NoAllocScratch"
    for v in (a, b, c, zb):
        v.dispose()
