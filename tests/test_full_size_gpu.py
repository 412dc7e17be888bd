"""BASELINE.json's configs at their full sizes, every element against the oracle (the reference's CPU definitions
restated, run threaded on all host cores), as the reference's ModelShapesAreBitExact compares every element
(Int8Tests.cs:285-317):

* config 2: DynamicQuantizeLinear of f32 [4096 x 4096] ~ N(0, 1) (y, scale and zero point bit for bit against
  DynamicReference, Int8Tests.cs:577-615), then u8 x s8 [4096 x 4096] with per-column zero points -8..8, dequantized
  to f32 by a_scale * b_scale[col] (the chain's expectation (float)sum * (a_scale * w_scale[n]), Int8Tests.cs:745);
* config 3: 8192^3 s8 x s8 -> s32 with both operands uniform over -128..127 (the -128 x -128 extreme included), B
  stored K x N and, once more, N x K;
* config 4: A = DynamicQuantizeLinear of N(0, 0.5) over the whole [8, 2048, 4096] tensor (its zero point), times the
  shared s8 B [4096 x 12288] -127..127 with per-column zero points -8..8 -> s32 [8, 2048, 12288];
* config 5: u8 A [16 x 8192] (zero point 128) x s8 B [8192 x 28672] -127..127 with per-column zero points -4..4, as
  int32 sums and dequantized to f32 by a_scale 0.02 * b_scale[col] (0.001..0.02).

Float results are compared bit for bit (the north star's tolerance is 1e-6 relative; the epilogue's two IEEE
roundings with no contraction match the definition exactly)."""
import numpy as np
import pytest

import og_oracle as oracle
import onegpu_cuda as og

pytestmark = pytest.mark.gpu


def bits_equal(got: np.ndarray, want: np.ndarray) -> int:
    """Mismatching elements (float arrays compared by their bits)."""
    if got.dtype == np.float32:
        return int(np.count_nonzero(got.view(np.uint32) != want.view(np.uint32)))
    return int(np.count_nonzero(got != want))


def dql_on_device(device, x: np.ndarray):
    """DynamicQuantizeLinear on the GPU; returns the device buffers (y, scale, zero point) after checking all three
    against the oracle bit for bit."""
    wy, ws, wz = oracle.dynamic_quantize(x)
    bx = device.create_buffer(np.float32, x)
    by = device.create_buffer(np.uint8, x.size)
    bs = device.create_buffer(np.float32, 1)
    bz = device.create_buffer(np.uint8, 4)
    with og.DynamicQuantizeKernels(device) as dq:
        enc = device.begin_commands()
        dq.encode(enc, bx, 0, x.size, by, 0, bs, 0, bz, 0)
        device.submit(enc)
        assert bits_equal(by.read(), wy) == 0
        assert bs.read()[0].view(np.uint32) == np.float32(ws).view(np.uint32)
        assert int(bz.read()[0]) == wz
    bx.dispose()
    return by, bs, bz, wy, np.float32(ws), wz


def test_config_2_chain_every_element(device):
    m = n = k = 4096
    rng = np.random.default_rng(2)
    x = rng.standard_normal(m * k, dtype=np.float32)
    by, bs, bz, wy, ws, wz = dql_on_device(device, x)
    b = rng.integers(-127, 128, size=k * n, dtype=np.int16).astype(np.int8)
    zb = rng.integers(-8, 9, size=n).astype(np.int8)
    b_scale = rng.uniform(0.001, 0.02, size=n).astype(np.float32)
    sums = oracle.int8_gemm(wy, False, b.view(np.uint8), True, np.array([wz], np.uint8), False, zb.view(np.uint8),
                            True, m=m, n=n, k=k)
    want = oracle.float_epilogue(sums, np.tile((ws * b_scale).astype(np.float32), m))
    bufs = [device.create_buffer(np.int8, b), device.create_buffer(np.int8, zb),
            device.create_buffer(np.float32, b_scale), device.create_buffer(np.float32, m * n)]
    with og.Int8Gemm(device) as gemm:
        enc = device.begin_commands()
        gemm.encode_dequantize(enc, og.Int8GemmProblem(m, n, k), by, bufs[0], bufs[3], og.Int8Operand(bs, 0),
                               og.Int8Operand(bufs[2], 0, True), og.Int8Operand(bz, 0), og.Int8Operand(bufs[1], 0, True))
        device.submit(enc)
        got = bufs[3].read()
        assert bits_equal(got, want) == 0, gemm.last_kernel
    for v in bufs + [by, bs, bz]:
        v.dispose()


@pytest.mark.parametrize("trans_b", [False, True])
def test_config_3_every_element(device, trans_b):
    m = n = k = 8192
    rng = np.random.default_rng(3 + trans_b)
    a = rng.integers(-128, 128, size=m * k, dtype=np.int16).astype(np.int8)
    b = rng.integers(-128, 128, size=k * n, dtype=np.int16).astype(np.int8)
    a[:4] = -128  # the extreme product (-128) x (-128) in the first sums
    b[:4] = -128
    want = oracle.int8_gemm(a.view(np.uint8), True, b.view(np.uint8), True, m=m, n=n, k=k, transpose_b=trans_b)
    ba, bb = device.create_buffer(np.int8, a), device.create_buffer(np.int8, b)
    bc = device.create_buffer(np.int32, m * n)
    with og.Int8Gemm(device) as gemm:
        enc = device.begin_commands()
        gemm.encode_int32(enc, og.Int8GemmProblem(m, n, k, transpose_b=trans_b), ba, bb, bc)
        device.submit(enc)
        got = bc.read()
        assert gemm.last_kernel.startswith("tensor-core-2sm")
        assert bits_equal(got, want) == 0, gemm.last_kernel
    for v in (ba, bb, bc):
        v.dispose()


def test_config_4_every_element(device):
    batch, m, n, k = 8, 2048, 12288, 4096
    rng = np.random.default_rng(4)
    x = (rng.standard_normal(batch * m * k, dtype=np.float32) * np.float32(0.5))
    by, bs, bz, wy, ws, wz = dql_on_device(device, x)
    del x
    b = rng.integers(-127, 128, size=k * n, dtype=np.int16).astype(np.int8)
    zb = rng.integers(-8, 9, size=n).astype(np.int8)
    want = oracle.int8_gemm(wy, False, b.view(np.uint8), True, np.array([wz], np.uint8), False, zb.view(np.uint8),
                            True, m=m, n=n, k=k, batch=batch, stride_a=m * k, stride_b=0)
    bufs = [device.create_buffer(np.int8, b), device.create_buffer(np.int8, zb),
            device.create_buffer(np.int32, batch * m * n)]
    with og.Int8Gemm(device) as gemm:
        enc = device.begin_commands()
        gemm.encode_int32(enc, og.Int8GemmProblem(m, n, k, batch=batch, stride_a=m * k), by, bufs[0], bufs[2],
                          og.Int8Operand(bz, 0), og.Int8Operand(bufs[1], 0, True))
        device.submit(enc)
        got = bufs[2].read()
        assert bits_equal(got, want) == 0, gemm.last_kernel
    for v in bufs + [by, bs, bz]:
        v.dispose()


@pytest.mark.parametrize("n", [28672, 14336, 7168, 3584])
def test_config_5_int32_and_dequantized_every_element(device, n):
    """Config 5 whole and as the column shard one GPU computes at 2, 4 and 8 GPUs (the shards split K across the
    workers and meet through records), int32 and dequantized, every element."""
    m, k = 16, 8192
    rng = np.random.default_rng(5 + n)
    a = rng.integers(0, 256, size=m * k, dtype=np.int16).astype(np.uint8)
    b = rng.integers(-127, 128, size=k * n, dtype=np.int16).astype(np.int8)
    zb = rng.integers(-4, 5, size=n).astype(np.int8)
    a_scale = np.array([0.02], np.float32)
    b_scale = rng.uniform(0.001, 0.02, size=n).astype(np.float32)
    za = np.array([128, 0, 0, 0], np.uint8)
    sums = oracle.int8_gemm(a, False, b.view(np.uint8), True, za[:1], False, zb.view(np.uint8), True, m=m, n=n, k=k)
    want_f = oracle.float_epilogue(sums, np.tile((a_scale[0] * b_scale).astype(np.float32), m))
    bufs = [device.create_buffer(np.uint8, a), device.create_buffer(np.int8, b), device.create_buffer(np.uint8, za),
            device.create_buffer(np.int8, zb), device.create_buffer(np.float32, a_scale),
            device.create_buffer(np.float32, b_scale), device.create_buffer(np.int32, m * n),
            device.create_buffer(np.float32, m * n)]
    p = og.Int8GemmProblem(m, n, k)
    zpa, zpb = og.Int8Operand(bufs[2], 0), og.Int8Operand(bufs[3], 0, True)
    with og.Int8Gemm(device) as gemm:
        enc = device.begin_commands()
        gemm.encode_int32(enc, p, bufs[0], bufs[1], bufs[6], zpa, zpb)
        gemm.encode_dequantize(enc, p, bufs[0], bufs[1], bufs[7], og.Int8Operand(bufs[4], 0),
                               og.Int8Operand(bufs[5], 0, True), zpa, zpb)
        device.submit(enc)
        assert gemm.last_kernel == "tensor-core-rows"
        assert bits_equal(bufs[6].read(), sums) == 0
        assert bits_equal(bufs[7].read(), want_f) == 0
    for v in bufs:
        v.dispose()
