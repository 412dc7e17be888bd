"""The allocation-free EncodeInt32 (og_int8_gemm_int32_noalloc) against the allocating one.

Some callers cannot call cudaMalloc while they run products: serving hosts whose own pool holds all of the GPU's
memory, engines whose execution step forbids allocation, latency-bound loops that cannot afford cudaMalloc's implicit
synchronisation. For them the entry point keeps the byte sums of the zero-point correction in a fixed device array of
the library (at most 1,048,576 int32) instead of scratch it allocates. Every product here is compared bit for bit
with og_int8_gemm_encode_int32 on the same inputs (integer sums: the tolerance is zero), on calls made back to back so
that each one reuses the array the previous one left behind. This file runs last (pytest collects it after the
others) so that a failure here leaves every other test already run; it passes alone in a fresh process and after the
other tests alike.
"""
import zlib

import numpy as np
import pytest

import og_oracle as oracle
import onegpu_cuda as og

pytestmark = pytest.mark.gpu


def run_both(device, p, a, b, za, zb, za_vector=False, bias=None):
    """Runs the product through og_int8_gemm_encode_int32 and through og_int8_gemm_int32_noalloc on the device's
    stream (either zero point may be None); returns both results and the allocating path's kernel."""
    ba = device.create_buffer(np.uint8, a)
    bb = device.create_buffer(np.int8, b.view(np.int8))
    extra = []
    zpa = zpb = opb = None
    if za is not None:
        extra.append(device.create_buffer(np.uint8, za))
        zpa = og.Int8Operand(extra[-1], 0, za_vector)
    if zb is not None:
        extra.append(device.create_buffer(np.int8, zb.view(np.int8)))
        zpb = og.Int8Operand(extra[-1], 0, True)
    if bias is not None:
        extra.append(device.create_buffer(np.int32, bias))
        opb = og.Int8Operand(extra[-1], 0, True)
    count = p.batch * p.m * p.n
    c_ref = device.create_buffer(np.int32, count)
    c_new = device.create_buffer(np.int32, np.full(count, 0x5A5A5A5A, np.int32))
    with og.Int8Gemm(device) as gemm:
        enc = device.begin_commands()
        gemm.encode_int32(enc, p, ba, bb, c_ref, zpa, zpb, opb)
        kernel = gemm.last_kernel
        device.submit(enc)
    og.int8_gemm_int32_noalloc(device.stream, p, ba, bb, c_new, zpa, zpb, opb)
    og.int8_gemm_noalloc_status(device.stream)  # no kernel of the call gave up a wait
    device.wait_idle()
    ref, new = c_ref.read(), c_new.read()
    for v in [ba, bb, c_ref, c_new] + extra:
        v.dispose()
    return ref, new, kernel


def operands(rng, p, lda=None):
    rows_a = (p.batch if p.stride_a else 1) * p.m
    a = rng.integers(0, 256, size=rows_a * (lda or p.k), dtype=np.int64).astype(np.uint8)
    b = rng.integers(-128, 128, size=p.k * p.n, dtype=np.int64).astype(np.int8)
    return a, b


def check_rows(new, p, a, b, za, zb, za_vector=False, lda=None, bias=None):
    """Two whole rows of batch 0 against the definition (the oracle)."""
    rows = [0, p.m - 1]
    ld = lda or p.k
    a_rows = np.stack([a[r * ld:r * ld + p.k] for r in rows]).reshape(-1)
    za_rows = None if za is None else (za[rows] if za_vector else za)
    want = oracle.int8_gemm(a_rows, False, b.view(np.uint8), True, za_rows, za_vector,
                            None if zb is None else zb.view(np.uint8), True, m=len(rows), n=p.n, k=p.k)
    if bias is not None:
        want = (want.reshape(len(rows), p.n).astype(np.int64) + bias[None, :]).astype(np.int64)
        want = ((want + 2 ** 31) % 2 ** 32 - 2 ** 31).astype(np.int32).reshape(-1)
    assert np.array_equal(new.reshape(p.batch, p.m, p.n)[0][rows].reshape(-1), want)


def test_no_alloc_matches_the_allocating_entry_point_twice(device):
    rng = np.random.default_rng(2024)
    shapes = [og.Int8GemmProblem(640, 528, 384), og.Int8GemmProblem(300, 1040, 256, batch=3, stride_a=300 * 256)]
    for p in shapes:  # two calls in a row: the second reuses the fixed array the first left behind
        a, b = operands(rng, p)
        za = np.array([rng.integers(0, 256)], np.uint8)
        zb = rng.integers(-8, 9, size=p.n).astype(np.int8)
        ref, new, kernel = run_both(device, p, a, b, za, zb)
        assert kernel.startswith("tensor-core")  # the path that needs the byte sums
        assert np.array_equal(new, ref)
        check_rows(new, p, a, b, za, zb)


@pytest.mark.parametrize("mode", ["a-scalar-only", "a-vector-only", "b-only", "none", "both-bias"])
def test_no_alloc_every_zero_point_mode(device, mode):
    """One zero point, the other, neither, and both with a bias: the fixed array holds only the sums the mode needs
    (row sums of A when B has a zero point, column sums of B when A has one). Each mode runs twice back to back."""
    rng = np.random.default_rng(zlib.crc32(mode.encode()))
    p = og.Int8GemmProblem(520, 784, 448)
    for _ in range(2):
        a, b = operands(rng, p)
        za_vector = mode == "a-vector-only"
        za = (rng.integers(0, 256, size=p.m).astype(np.uint8) if za_vector
              else np.array([rng.integers(0, 256)], np.uint8)) if mode.startswith(("a-", "both")) else None
        zb = (rng.integers(-8, 9, size=p.n).astype(np.int8) if mode in ("b-only",) else
              np.full(p.n, int(rng.integers(-8, 9)), np.int8) if mode.startswith("both") else None)
        bias = rng.integers(-2 ** 31, 2 ** 31, size=p.n, dtype=np.int64).astype(np.int32) if "bias" in mode else None
        ref, new, kernel = run_both(device, p, a, b, za, zb, za_vector, bias)
        assert kernel.startswith("tensor-core")
        assert np.array_equal(new, ref)
        check_rows(new, p, a, b, za, zb, za_vector, bias=None if bias is None else bias.astype(np.int64))


def test_no_alloc_portable_branch(device):
    """Products that the tensor cores do not take: under 2^16 multiply-adds, or an A whose rows are not 16-byte
    aligned (Lda = 100). The allocating entry point stages the latter onto the tensor cores; the allocation-free one
    runs the portable kernel, which needs no byte sums. Both results agree bit for bit, twice in a row."""
    rng = np.random.default_rng(99)
    small = og.Int8GemmProblem(20, 24, 16)
    for _ in range(2):
        a, b = operands(rng, small)
        za = np.array([200], np.uint8)
        zb = rng.integers(-8, 9, size=small.n).astype(np.int8)
        ref, new, kernel = run_both(device, small, a, b, za, zb)
        assert kernel == "portable"
        assert np.array_equal(new, ref)
        check_rows(new, small, a, b, za, zb)
    unaligned = og.Int8GemmProblem(1536, 1024, 100, lda=100)
    for _ in range(2):
        a, b = operands(rng, unaligned, lda=100)
        za = np.array([131], np.uint8)
        zb = rng.integers(-8, 9, size=unaligned.n).astype(np.int8)
        ref, new, _ = run_both(device, unaligned, a, b, za, zb)
        assert np.array_equal(new, ref)
        check_rows(new, unaligned, a, b, za, zb, lda=100)


def test_no_alloc_reports_a_wait_that_gave_up(device):
    """A kernel of an allocation-free product that gives up a bounded wait raises the library's failure word for
    these products; og_int8_gemm_noalloc_status reports it once (GpuCommandFailedException, reason Watchdog) and
    clears it. The self-test kernel makes a wait run out (an mbarrier nobody arrives at): no fault, and the device
    then computes correctly."""
    og.int8_gemm_noalloc_status(device.stream)  # clean to start with
    og.int8_gemm_noalloc_watchdog_selftest(device.stream, 2000)
    with pytest.raises(og.GpuCommandFailedException) as e:
        og.int8_gemm_noalloc_status(device.stream)
    assert e.value.reason == "Watchdog"
    og.int8_gemm_noalloc_status(device.stream)  # cleared
    rng = np.random.default_rng(5)
    p = og.Int8GemmProblem(384, 512, 256)
    a, b = operands(rng, p)
    za = np.array([77], np.uint8)
    zb = rng.integers(-8, 9, size=p.n).astype(np.int8)
    ref, new, _ = run_both(device, p, a, b, za, zb)
    assert np.array_equal(new, ref)


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
