"""Failure detection on the GPU without a fault: a kernel whose bounded wait runs out (an mbarrier nobody arrives at)
raises the device's failure word and returns; the host reports GpuCommandFailedException with reason Watchdog, clears
the word, and the same device then computes a product bit-exactly (GpuDevice.cs:337-374 failure kinds)."""
import time

import numpy as np
import pytest

import onegpu_cuda as og
from cases import Case, problem
from gpu_rig import run_int32


@pytest.mark.gpu
def test_a_wait_that_runs_out_fails_the_submission_and_the_device_stays_usable(device):
    device.wait_idle()
    t0 = time.perf_counter()
    device.watchdog_selftest(20000)  # 20 ms
    with pytest.raises(og.GpuCommandFailedException) as info:
        device.wait_idle()
    assert info.value.reason == "Watchdog"
    assert time.perf_counter() - t0 < 5.0
    device.wait_idle()  # the failure word was cleared

    gemm = og.Int8Gemm(device, og.Int8GemmOptions(kernel=og.KERNEL_TENSOR_CORE))
    try:
        c = Case("after watchdog", problem(256, 384, 192), a_signed=False, b_signed=True, za_mode=1, zb_mode=2)
        bad, kernel = run_int32(device, gemm, c, seed=5)
        assert bad == 0
        assert kernel.startswith("tensor-core")
    finally:
        gemm.dispose()


@pytest.mark.gpu
def test_watchdog_limit_is_checked(device):
    with pytest.raises(og.ArgumentOutOfRangeException):
        device.watchdog_selftest(0)
    with pytest.raises(og.ArgumentOutOfRangeException):
        device.watchdog_selftest(2000001)
