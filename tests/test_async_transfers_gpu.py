"""Asynchronous uploads and readbacks (og_buffer_write_async / og_buffer_read_async): products of consecutive steps
pipelined over two sets of device buffers, each step's inputs uploaded and its result read back while the next step
runs; every result bit-exact against the oracle."""
import numpy as np
import pytest

import og_oracle as oracle
import onegpu_cuda as og


@pytest.mark.gpu
def test_pipelined_steps_are_bit_exact(device):
    m, n, k, steps = 384, 512, 640, 6
    a_host = [oracle.bytes_(m * k, 300 + s) for s in range(steps)]
    b_host = [oracle.bytes_(k * n, 400 + s) for s in range(steps)]
    zb = oracle.bytes_(n, 7)
    wants = [oracle.int8_gemm(a_host[s], False, b_host[s], True, np.array([3], np.uint8), False, zb, True, m=m, n=n,
                              k=k) for s in range(steps)]
    pin_in = og.PinnedHost(steps * (m * k + k * n))
    pin_out = og.PinnedHost(steps * m * n * 4)
    for s in range(steps):
        pin_in.view(np.uint8, m * k, s * (m * k + k * n))[:] = a_host[s]
        pin_in.view(np.uint8, k * n, s * (m * k + k * n) + m * k)[:] = b_host[s]
    a = [device.create_buffer(np.uint8, m * k) for _ in range(2)]
    b = [device.create_buffer(np.int8, k * n) for _ in range(2)]
    c = [device.create_buffer(np.int32, m * n) for _ in range(2)]
    za = device.create_buffer(np.uint8, np.array([3], np.uint8))
    zbb = device.create_buffer(np.int8, zb.view(np.int8))
    gemm = og.Int8Gemm(device)
    tickets = []
    try:
        for s in range(steps):
            j = s % 2
            if s >= 2:
                tickets[s - 2].wait()  # step s - 2 used buffers j: its readback (after its product) is done
            base = pin_in.ptr + s * (m * k + k * n)
            device.write_async(a[j].ptr, base, m * k)
            device.write_async(b[j].ptr, base + m * k, k * n)
            enc = device.begin_commands()
            gemm.encode_int32(enc, og.Int8GemmProblem(m, n, k), a[j], b[j], c[j], og.Int8Operand(za, 0),
                              og.Int8Operand(zbb, 0, True))
            device.submit(enc)
            tickets.append(device.read_async(pin_out.ptr + s * m * n * 4, c[j].ptr, m * n * 4))
        for t in tickets[-2:]:
            t.wait()
        for s in range(steps):
            assert np.array_equal(pin_out.view(np.int32, m * n, s * m * n * 4), wants[s]), s
    finally:
        device.wait_idle()
        for v in a + b + c + [za, zbb]:
            v.dispose()
        gemm.dispose()
        pin_in.dispose()
        pin_out.dispose()


@pytest.mark.gpu
def test_more_readbacks_in_flight_than_pinned_status_words(device):
    """Readbacks take one of the device's 1024 page-locked status words each, and one page-locked on its own once all
    are in flight: 1100 readbacks of distinct words queued before any wait all land, and the words return to the
    device's pool (a second round works the same)."""
    count = 1100
    src = device.create_buffer(np.int32, np.arange(count, dtype=np.int32) * 7 + 1)
    pin = og.PinnedHost(count * 4)
    try:
        for rnd in range(2):
            pin.view(np.int32, count)[:] = -1
            tickets = [device.read_async(pin.ptr + 4 * i, src.ptr + 4 * i, 4) for i in range(count)]
            for t in tickets:
                t.wait()
            assert np.array_equal(pin.view(np.int32, count), np.arange(count, dtype=np.int32) * 7 + 1), rnd
    finally:
        pin.dispose()
        src.dispose()
