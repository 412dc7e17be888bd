"""Work recorded into a CUDA graph (og_device_capture_begin / og_device_capture_end) and replayed with
og_graph_launch, against the oracle: each replay reads the buffers' contents as they are when it is launched. Covers
the few-rows product split across workers (per-tile tickets that every launch must leave at zero), the tensor-core
product with its byte-sums pass, and the DynamicQuantizeLinear -> dequantize-product chain (launches that overlap
through programmatic dependent launch inside the graph; at 2^18 elements the quantization is the single cooperative
kernel with its grid barrier)."""
import numpy as np
import pytest

import og_oracle as oracle
import onegpu_cuda as og
from cases import oracle_shape, problem

pytestmark = pytest.mark.gpu


def _replays(device, record, refresh, expect, launches=3):
    """Runs record(encoder) once as usual (the instances' first encodings allocate their scratch), captures it, then
    for each launch writes new inputs (refresh(i)), replays and checks."""
    refresh(-1)
    enc = device.begin_commands()
    record(enc)
    device.submit(enc)
    expect(-1)
    device.capture_begin()
    enc = device.begin_commands()
    try:
        record(enc)
        device.submit(enc)
    finally:
        graph = device.capture_end()
    try:
        for i in range(launches):
            refresh(i)
            graph.launch()
            expect(i)
    finally:
        graph.dispose()


@pytest.mark.parametrize("m,n,k", [(16, 4096, 2048), (512, 768, 1024)])
def test_products_replay_bit_exact(device, m, n, k):
    """u8 A with a scalar zero point, s8 B with per-column zero points, int32 C, replayed with new A each time."""
    rng = np.random.default_rng(m * 7 + n)
    b = rng.integers(-128, 128, size=k * n, dtype=np.int16).astype(np.int8)
    za = np.array([131, 0, 0, 0], np.uint8)
    zb = rng.integers(-8, 9, size=n, dtype=np.int16).astype(np.int8)
    p = problem(m, n, k)
    with og.Int8Gemm(device) as gemm:
        ba = device.create_buffer(np.uint8, m * k)
        bb, bc = device.create_buffer(np.int8, b), device.create_buffer(np.int32, m * n)
        bza, bzb = device.create_buffer(np.uint8, za), device.create_buffer(np.int8, zb)
        state = {}

        def record(enc):
            gemm.encode_int32(enc, og.Int8GemmProblem(**p), ba, bb, bc, og.Int8Operand(bza, 0),
                              og.Int8Operand(bzb, 0, True))

        def refresh(i):
            a = rng.integers(0, 256, size=m * k, dtype=np.int16).astype(np.uint8)
            ba.write(a)
            state["a"] = a

        def expect(i):
            want = oracle.int8_gemm(state["a"], False, b.view(np.uint8), True, za[:1], False, zb.view(np.uint8), True,
                                    **oracle_shape(p))
            assert np.array_equal(bc.read(), want), f"launch {i} ({gemm.last_kernel})"

        try:
            _replays(device, record, refresh, expect)
        finally:
            for v in (ba, bb, bc, bza, bzb):
                v.dispose()


def test_quantize_and_product_chain_replays_bit_exact(device):
    """DynamicQuantizeLinear, then the dequantize form of the product (scale a_scale * b_scale[n] in the epilogue),
    captured as one graph and replayed with new activations: expected (float)sum * (a_scale * b_scale[n])."""
    m, n, k = 256, 512, 1024
    rng = np.random.default_rng(5)
    w = rng.integers(-127, 128, size=n * k, dtype=np.int16).astype(np.int8)
    zw = rng.integers(-8, 9, size=n, dtype=np.int16).astype(np.int8)
    bscale = rng.uniform(0.001, 0.02, size=n).astype(np.float32)
    p = problem(m, n, k)
    with og.DynamicQuantizeKernels(device) as dq, og.Int8Gemm(device) as gemm:
        bx = device.create_buffer(np.float32, m * k)
        by = device.create_buffer(np.uint8, m * k)
        bs, bz = device.create_buffer(np.float32, 1), device.create_buffer(np.uint8, 4)
        bw, bzw = device.create_buffer(np.int8, w), device.create_buffer(np.int8, zw)
        bbs, bc = device.create_buffer(np.float32, bscale), device.create_buffer(np.float32, m * n)
        state = {}

        def record(enc):
            dq.encode(enc, bx, 0, m * k, by, 0, bs, 0, bz, 0)
            gemm.encode_dequantize(enc, og.Int8GemmProblem(**p), by, bw, bc, og.Int8Operand(bs, 0),
                                   og.Int8Operand(bbs, 0, True), og.Int8Operand(bz, 0), og.Int8Operand(bzw, 0, True))

        def refresh(i):
            x = (rng.standard_normal(m * k) * (0.5 + i)).astype(np.float32)
            bx.write(x)
            state["x"] = x

        def expect(i):
            wy, wscale, wzero = oracle.dynamic_quantize(state["x"])
            sums = oracle.int8_gemm(wy, False, w.view(np.uint8), True, np.array([wzero], np.uint8), False,
                                    zw.view(np.uint8), True, **oracle_shape(p))
            scale_vec = (np.float32(wscale) * bscale).astype(np.float32)
            want = (sums.astype(np.float32) * np.tile(scale_vec, m)).astype(np.float32)
            assert np.array_equal(by.read(), wy), f"launch {i}: quantized activations"
            assert np.array_equal(bc.read().view(np.uint32), want.view(np.uint32)), f"launch {i}: product"

        try:
            _replays(device, record, refresh, expect)
        finally:
            for v in (bx, by, bs, bz, bw, bzw, bbs, bc):
                v.dispose()
