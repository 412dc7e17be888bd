"""The split tail of the tensor-core int32 product, bit for bit against the oracle.

When the tiles of a product leave at least half of the SM pairs (or of the SMs, one-SM tile) idle in the last wave,
the tiles past the last full wave are cut into equal K ranges dealt over the workers. Every piece of a cut tile adds
its sums into C (cleared first) with TMA reductions, the K-block-0 piece with the zero-point terms and the bias;
integer addition modulo 2^32 is exact in any order, so C must equal the definition bit for bit. The cases cover a
partial wave after full ones, fewer tiles than workers, ragged M, N and K edges, every zero-point mode and
signedness, a bias, batched A, B stored N x K, the one-SM tile, the per-shard shapes of the square benchmark product
split over 4 and 8 GPUs, and products recorded back to back (the count of cleared shares goes back to zero at the
end of every launch).
"""
import numpy as np
import pytest

import og_oracle as oracle
import onegpu_cuda as og
from cases import Case, case_data, oracle_shape, problem
from gpu_rig import SENTINEL, align_case, run_int32, typed

pytestmark = pytest.mark.gpu

TC2 = og.Int8GemmOptions(kernel=og.KERNEL_TENSOR_CORE, tile=256)
TC1 = og.Int8GemmOptions(kernel=og.KERNEL_TENSOR_CORE, tile=128)


def wrap32(x: np.ndarray) -> np.ndarray:
    return ((x.astype(np.int64) + 2 ** 31) % 2 ** 32 - 2 ** 31).astype(np.int32)


@pytest.mark.parametrize("opts,m,n,k,batch,trans_b", [
    (TC2, 2048, 2560, 2048, 1, False),   # 80 pair tiles: one full wave, 6 tiles split over the pairs
    (TC2, 2000, 2500, 2000, 1, False),   # the same with ragged M, N and K edges
    (TC2, 1024, 1024, 4096, 1, False),   # 16 tiles, fewer than the pairs: every tile split
    (TC2, 600, 1100, 3000, 2, False),    # batched A, shared B, ragged everything
    (TC2, 1536, 1536, 2560, 1, True),    # B stored N x K
    (TC1, 1664, 3072, 4096, 1, False),   # one-SM tile: 156 tiles over 148 SMs
])
def test_split_tail_is_bit_exact(device, opts, m, n, k, batch, trans_b):
    with og.Int8Gemm(device, opts) as gemm:
        kernels = set()
        for i, (za_mode, zb_mode, a_s, b_s) in enumerate(((1, 2, False, True), (2, 1, True, False), (0, 0, True, True),
                                                          (2, 2, False, False), (0, 2, True, True), (1, 0, False, True))):
            p = problem(m, n, k, batch=batch, trans_b=trans_b, share_b=batch > 1)
            c = align_case(Case("split tail", p, a_s, b_s, za_mode, zb_mode))
            bad, kernel = run_int32(device, gemm, c, 600 + 7 * i)
            kernels.add(kernel)
            assert bad == 0, (c.p, za_mode, zb_mode, a_s, b_s, kernel)
        assert all(kn.endswith("-split-tail") for kn in kernels), kernels


def run_bias(device, gemm, m, n, k, seed):
    """EncodeInt32 with zero points of both operands and a bias per column, against the oracle plus the bias (mod
    2^32)."""
    p = problem(m, n, k)
    c = align_case(Case("bias", p, False, True, 1, 2))
    a, b, za, zb = case_data(c, seed, oracle.bytes_)
    want = oracle.int8_gemm(a, False, b, True, za, False, zb, True, **oracle_shape(c.p))
    bias = oracle.bytes_(4 * n, seed + 9).view(np.int32).copy()
    want = wrap32(want.reshape(m, n).astype(np.int64) + bias[None, :]).reshape(-1)
    bufs = [typed(device, a, False), typed(device, b, True), device.create_buffer(np.int32, np.full(m * n + 8, SENTINEL,
                                                                                                    np.int32)),
            typed(device, za, False), typed(device, zb, True), device.create_buffer(np.int32, bias)]
    enc = device.begin_commands()
    gemm.encode_int32(enc, og.Int8GemmProblem(**c.p), bufs[0], bufs[1], bufs[2], og.Int8Operand(bufs[3], 0),
                      og.Int8Operand(bufs[4], 0, True), og.Int8Operand(bufs[5], 0, True))
    kernel = gemm.last_kernel
    device.submit(enc)
    got = bufs[2].read()
    for v in bufs:
        v.dispose()
    return int(np.count_nonzero(got[:m * n] != want)) + int(np.count_nonzero(got[m * n:] != SENTINEL)), kernel


def test_split_tail_adds_the_bias_once(device):
    with og.Int8Gemm(device, TC2) as gemm:
        for seed in (31, 32):
            bad, kernel = run_bias(device, gemm, 2048, 2560, 2048, seed)
            assert kernel.endswith("-split-tail")
            assert bad == 0


def test_split_tail_products_back_to_back(device):
    """Three split products recorded in one encoder and a fourth in a second submission, on one instance (one set of
    claim words): each launch's generation tells its claims from the previous launch's."""
    with og.Int8Gemm(device) as gemm:
        shapes = [(2048, 2560, 2048, 90), (1024, 1024, 4096, 91), (2048, 2560, 2048, 92)]
        data, bufs = [], []
        enc = device.begin_commands()
        for (m, n, k, seed) in shapes:
            c = align_case(Case("seq", problem(m, n, k), False, True, 1, 2))
            a, b, za, zb = case_data(c, seed, oracle.bytes_)
            want = oracle.int8_gemm(a, False, b, True, za, False, zb, True, **oracle_shape(c.p))
            bs = [typed(device, a, False), typed(device, b, True), device.create_buffer(np.int32, want.size),
                  typed(device, za, False), typed(device, zb, True)]
            gemm.encode_int32(enc, og.Int8GemmProblem(**c.p), bs[0], bs[1], bs[2], og.Int8Operand(bs[3], 0),
                              og.Int8Operand(bs[4], 0, True))
            assert gemm.last_kernel.endswith("-split-tail")
            data.append((bs[2], want))
            bufs += bs
        device.submit(enc)
        try:
            for c_buf, want in data:
                assert np.array_equal(c_buf.read(), want)
        finally:
            for v in bufs:
                v.dispose()
        bad, _ = run_int32(device, gemm, align_case(Case("again", problem(2048, 2560, 2048), True, True, 2, 2)), 93)
        assert bad == 0


def test_whole_tiles_option_does_not_split(device):
    """Option stream_k = 1 keeps whole tiles; both agree with the split product bit for bit."""
    c = align_case(Case("whole", problem(2048, 2560, 2048), False, True, 1, 2))
    with og.Int8Gemm(device, og.Int8GemmOptions(stream_k=1)) as whole, og.Int8Gemm(device) as split:
        bad_w, kw = run_int32(device, whole, c, 77)
        bad_s, ks = run_int32(device, split, c, 77)
        assert bad_w == 0 and bad_s == 0
        assert kw == "tensor-core-2sm" and ks == "tensor-core-2sm-split-tail"


def test_other_outputs_do_not_split(device):
    """The float and requantized forms keep whole tiles (their epilogue is not additive) and agree with the oracle."""
    with og.Int8Gemm(device) as gemm:
        a = device.create_buffer(np.uint8, 2048 * 2048)
        b = device.create_buffer(np.int8, 2048 * 2560)
        y = device.create_buffer(np.uint8, 2048 * 2560)
        f = device.create_buffer(np.float32, 2048 * 2560)
        s = device.create_buffer(np.float32, np.array([0.001], np.float32))
        try:
            enc = device.begin_commands()
            gemm.encode_requantized(enc, og.Int8GemmProblem(2048, 2560, 2048), a, b, y, og.Int8Operand(s, 0), 128)
            assert gemm.last_kernel == "tensor-core-2sm"
            gemm.encode_float(enc, og.Int8GemmProblem(2048, 2560, 2048), a, b, f, og.Int8Operand(s, 0))
            assert gemm.last_kernel == "tensor-core-2sm"
            device.submit(enc)
            device.wait_idle()
        finally:
            for v in (a, b, y, f, s):
                v.dispose()


@pytest.mark.parametrize("shards", [4, 8])
def test_square_product_shards_are_bit_exact(device, shards):
    """The column shard one GPU computes when the square benchmark product (8192^3, s8 x s8, B drawn over the whole
    -128..127 range) is split over 4 or 8 GPUs: 8192 x (8192 / shards) x 8192, every element against the threaded
    oracle, with and without zero points."""
    m = k = 8192
    n = 8192 // shards
    rng = np.random.default_rng(8000 + shards)
    a = rng.integers(-128, 128, size=m * k, dtype=np.int16).astype(np.int8)
    b = rng.integers(-128, 128, size=k * n, dtype=np.int16).astype(np.int8)
    ba, bb = device.create_buffer(np.int8, a), device.create_buffer(np.int8, b)
    bc = device.create_buffer(np.int32, m * n)
    za = np.array([-3], np.int8)
    zb = rng.integers(-8, 9, size=n).astype(np.int8)
    bza, bzb = device.create_buffer(np.int8, za), device.create_buffer(np.int8, zb)
    try:
        with og.Int8Gemm(device) as gemm:
            for zp in (False, True):
                enc = device.begin_commands()
                gemm.encode_int32(enc, og.Int8GemmProblem(m, n, k), ba, bb, bc,
                                  og.Int8Operand(bza, 0) if zp else None, og.Int8Operand(bzb, 0, True) if zp else None)
                kernel = gemm.last_kernel
                device.submit(enc)
                got = bc.read()
                want = oracle.int8_gemm(a.view(np.uint8), True, b.view(np.uint8), True,
                                        za.view(np.uint8) if zp else None, False, zb.view(np.uint8) if zp else None,
                                        True, m=m, n=n, k=k)
                # 4 shards: 256 tiles, a last wave of 34 over 74 pairs (split in halves); 8 shards: 128 tiles, 54
                # past the first wave (left whole)
                assert kernel == ("tensor-core-2sm-split-tail" if shards == 4 else "tensor-core-2sm")
                assert np.array_equal(got, want), f"{int(np.count_nonzero(got != want))} sums differ (zp {zp})"
    finally:
        for v in (ba, bb, bc, bza, bzb):
            v.dispose()
