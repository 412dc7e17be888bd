"""Helpers of the GPU parity tests: upload a case, run it through the C ABI, compare with the oracle (the reference's
Rig / RunInt32 pattern, Int8Tests.cs:116-175, with sentinel guard bands around every output)."""
from __future__ import annotations

import numpy as np

import og_oracle as oracle
import onegpu_cuda as og
from cases import Case, case_data, oracle_shape

SENTINEL = 0x5A5A5A5A


def base_kernel(kernel: str) -> str:
    """The kernel configuration a product ran on, without the split-tail schedule suffix (int32 products whose last
    wave of tiles is partial split that wave in K; the tile and kernel are the same)."""
    return kernel.replace("-split-tail", "")


def typed(device, data: np.ndarray, signed: bool):
    return device.create_buffer(np.int8 if signed else np.uint8, data.view(np.int8 if signed else np.uint8))


def align_case(c: Case) -> Case:
    """The same product with rows, batches and operands moved to 16-byte boundaries, so the tensor-core kernel can
    load it with TMA (dense strides padded up to a multiple of 16)."""
    p = dict(c.p)
    r16 = lambda v: (v + 15) // 16 * 16
    k, n, m = p["k"], p["n"], p["m"]
    p["lda"] = r16(max(k, 1))
    p["ldb"] = r16(max(k if p["transpose_b"] else n, 1))
    p["offset_a"] = 16 * (p["offset_a"] % 4)
    p["offset_b"] = 16 * (p["offset_b"] % 4)
    if p["batch"] > 1:
        p["stride_a"] = m * p["lda"] if p["stride_a"] else 0
        p["stride_b"] = (n if p["transpose_b"] else k) * p["ldb"] if p["stride_b"] else 0
    return Case(c.name + " aligned", p, c.a_signed, c.b_signed, c.za_mode, c.zb_mode, c.fill)


def run_int32(device, gemm, c: Case, seed: int, want=None, data=None):
    """Runs EncodeInt32 on a case (the reference's generated data, or `data` = (a, b, za, zb)); returns
    (mismatches, kernel used)."""
    p = c.p
    a, b, za, zb = data if data is not None else case_data(c, seed, oracle.bytes_)
    if want is None:
        want = oracle.int8_gemm(a, c.a_signed, b, c.b_signed, za, c.za_mode == 2, zb, c.zb_mode == 2,
                                **oracle_shape(p))
    count = want.size
    init = np.full(p["offset_c"] + count + 2, SENTINEL, dtype=np.int32)
    bufs = [typed(device, a, c.a_signed), typed(device, b, c.b_signed), device.create_buffer(np.int32, init)]
    zpa = zpb = None
    if za is not None:
        bufs.append(typed(device, za, c.a_signed))
        zpa = og.Int8Operand(bufs[-1], 0, c.za_mode == 2)
    if zb is not None:
        bufs.append(typed(device, zb, c.b_signed))
        zpb = og.Int8Operand(bufs[-1], 0, c.zb_mode == 2)
    try:
        enc = device.begin_commands()
        gemm.encode_int32(enc, og.Int8GemmProblem(**p), bufs[0], bufs[1], bufs[2], zpa, zpb)
        kernel = gemm.last_kernel
        device.submit(enc)
        got = bufs[2].read()
    finally:
        for buf in bufs:
            buf.dispose()
    off = p["offset_c"]
    bad = int(np.count_nonzero(got[off:off + count] != want))
    bad += int(np.count_nonzero(got[:off] != SENTINEL)) + int(np.count_nonzero(got[off + count:] != SENTINEL))
    return bad, kernel
