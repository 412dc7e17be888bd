"""Int8Gemm on the GPU through the C ABI, bit for bit against the oracle.

Mirrors tests/RecursiveAI.OneGpu.Kernels.Tests/Int8Tests.cs (EdgeShapesAreBitExact, ModelShapesAreBitExact,
ForcingTheDotVariantOffChangesNothing, FloatAndRequantizedFormsAreBitExact, RequantizationRoundsHalfToEvenAndSaturates,
BadArgumentsAreRejected), Int8ScratchTests.cs, MultiDeviceTests.cs and ConvIntegerTests.cs:343-392, run on both
kernels (the tcgen05 tensor-core kernel on TMA-aligned copies of each case, and the portable SIMT kernel).
"""
import numpy as np
import pytest

import og_oracle as oracle
import onegpu_cuda as og
from cases import (Case, case_data, edge_cases, float_biases, float_scale, golden, oracle_shape, problem, requant_bias,
                   requant_mult)
from gpu_rig import SENTINEL, align_case, base_kernel, run_int32, typed

pytestmark = pytest.mark.gpu


CONFIGS = {
    "default": og.Int8GemmOptions(),
    "portable": og.Int8GemmOptions(allow_packed_dot=False),
    "tensor-core-1sm": og.Int8GemmOptions(kernel=og.KERNEL_TENSOR_CORE, tile=128),
    "tensor-core-2sm": og.Int8GemmOptions(kernel=og.KERNEL_TENSOR_CORE, tile=256),
    "tensor-core-auto": og.Int8GemmOptions(kernel=og.KERNEL_TENSOR_CORE),  # the few-rows kernel for M <= 16
}


def configs(device, names=None):
    """Every way the product can run: as chosen, the portable kernel, and each tensor-core tile forced (the
    reference's Configs, Int8Tests.cs:24-34)."""
    return [(n, og.Int8Gemm(device, CONFIGS[n])) for n in (names or CONFIGS)]


def test_edge_shapes_are_bit_exact(device):
    cases = edge_cases()
    aligned = [align_case(c) for c in cases]
    total = {}
    for name, gemm in configs(device):
        with gemm:
            kernels = set()
            for seed, c in enumerate(cases + aligned, start=1):
                if name.startswith("tensor-core") and (c.p["k"] == 0 or "aligned" not in c.name):
                    continue
                b, k = run_int32(device, gemm, c, seed)
                kernels.add(base_kernel(k))
                assert b == 0, f"[{name}] {c.name} signed {c.a_signed}/{c.b_signed} zp {c.za_mode}/{c.zb_mode}"
            total[name] = kernels
    assert total["portable"] == {"portable"}
    assert total["tensor-core-1sm"] == {"tensor-core-1sm"}
    assert total["tensor-core-2sm"] == {"tensor-core-2sm"}
    assert "tensor-core-rows" in total["tensor-core-auto"]


def test_model_shapes_are_bit_exact(device):
    """ModelShapesAreBitExact: uint8 activations with a zero point, int8 weights stored N x K."""
    for name, m, n, k in golden()["tables"]["model_shapes"]["shapes"]:
        c = Case(name, problem(m, n, k, trans_b=True), False, True, 1, 0)
        data = case_data(c, m + n + k, oracle.bytes_)
        a, b, za, _ = data
        want = oracle.int8_gemm(a, False, b, True, za, False, **oracle_shape(c.p))
        for cfg, gemm in configs(device):
            with gemm:
                bad, kern = run_int32(device, gemm, c, m + n + k, want, data)
                assert bad == 0, f"{name} [{cfg}] via {kern}"


def test_forcing_the_dot_variant_off_changes_nothing(device):
    with og.Int8Gemm(device) as chosen, og.Int8Gemm(device, og.Int8GemmOptions(allow_packed_dot=False)) as forced:
        c = Case("forced", problem(70, 90, 100), False, True, 1, 2)
        assert run_int32(device, chosen, c, 5)[0] == 0
        assert run_int32(device, forced, c, 5)[0] == 0
        assert chosen.variant.startswith("tcgen05-i8")
        assert forced.variant.startswith("portable")
        assert chosen.bind_groups_created == 0


def float_case(device, gemm, m, n, k, scale_vec, with_ib, with_fb, seed, aligned=False):
    """FloatCase (Int8Tests.cs:334-386)."""
    p = problem(m, n, k)
    if aligned:
        p = align_case(Case("f", p)).p
    a = oracle.bytes_(p["m"] * (p["lda"] or k) + 4 + p["offset_a"], seed)
    b = oracle.bytes_(k * (p["ldb"] or n) + 4 + p["offset_b"], seed + 1)
    za = oracle.bytes_(1, seed + 2)
    zb = oracle.bytes_(n, seed + 3)
    want = oracle.int8_gemm(a, False, b, True, za, False, zb, True, **oracle_shape(p))
    scale = float_scale(n, scale_vec, seed)
    ib, fb = float_biases(n)
    expected = oracle.float_epilogue(want, np.resize(scale, want.size) if not scale_vec else np.tile(scale, m),
                                     np.tile(ib, m) if with_ib else None, np.tile(fb, m) if with_fb else None)
    bufs = dict(a=typed(device, a, False), b=typed(device, b, True), za=typed(device, za, False),
                zb=typed(device, zb, True), s=device.create_buffer(np.float32, scale),
                ib=device.create_buffer(np.int32, ib), fb=device.create_buffer(np.float32, fb),
                c=device.create_buffer(np.float32, np.full(m * n, np.nan, np.float32)))
    try:
        enc = device.begin_commands()
        gemm.encode_float(enc, og.Int8GemmProblem(**p), bufs["a"], bufs["b"], bufs["c"],
                          og.Int8Operand(bufs["s"], 0, scale_vec), og.Int8Operand(bufs["za"], 0),
                          og.Int8Operand(bufs["zb"], 0, True), og.Int8Operand(bufs["fb"], 0, True) if with_fb else None,
                          og.Int8Operand(bufs["ib"], 0, True) if with_ib else None)
        device.submit(enc)
        got = bufs["c"].read()
    finally:
        for v in bufs.values():
            v.dispose()
    return int(np.count_nonzero(got.view(np.uint32) != expected.view(np.uint32)))


def requant_case(device, gemm, m, n, k, mult_vec, unsigned, zero_y, with_bias, seed, a_signed, b_signed,
                 aligned=False):
    """RequantCase (Int8Tests.cs:388-466): odd output offset 3, sentinel bytes 0xA7 around the output."""
    p = problem(m, n, k, off_c=3)
    if aligned:
        p = align_case(Case("q", p)).p
    a = oracle.bytes_(p["m"] * (p["lda"] or k) + 4 + p["offset_a"], seed)
    b = oracle.bytes_(k * (p["ldb"] or n) + 4 + p["offset_b"], seed + 1)
    za = oracle.bytes_(1, seed + 2)
    want = oracle.int8_gemm(a, a_signed, b, b_signed, za, False, **oracle_shape(p))
    mult = requant_mult(n, mult_vec, seed)
    ib = requant_bias(n)
    acc = want.astype(np.int64) + (np.tile(ib, m) if with_bias else 0)
    acc = ((acc + 2 ** 31) % 2 ** 32 - 2 ** 31).astype(np.int32)
    expected = oracle.requant_array(acc, np.tile(mult, m) if mult_vec else np.resize(mult, acc.size), zero_y,
                                    unsigned)
    out = np.full(((3 + m * n + 3 + 3) // 4) * 4 + 4, 0xA7, np.uint8)
    bufs = dict(a=typed(device, a, a_signed), b=typed(device, b, b_signed), za=typed(device, za, a_signed),
                m=device.create_buffer(np.float32, mult), ib=device.create_buffer(np.int32, ib),
                y=typed(device, out, not unsigned))
    try:
        enc = device.begin_commands()
        gemm.encode_requantized(enc, og.Int8GemmProblem(**p), bufs["a"], bufs["b"], bufs["y"],
                                og.Int8Operand(bufs["m"], 0, mult_vec), zero_y, og.Int8Operand(bufs["za"], 0), None,
                                og.Int8Operand(bufs["ib"], 0, True) if with_bias else None)
        device.submit(enc)
        got = bufs["y"].read().view(np.uint8)
    finally:
        for v in bufs.values():
            v.dispose()
    bad = int(np.count_nonzero(got[3:3 + m * n] != expected))
    bad += int(np.count_nonzero(got[:3] != 0xA7)) + int(np.count_nonzero(got[3 + m * n:] != 0xA7))
    return bad


@pytest.mark.parametrize("cfg", list(CONFIGS))
def test_float_and_requantized_forms_are_bit_exact(device, cfg):
    gemm = og.Int8Gemm(device, CONFIGS[cfg])
    aligned = cfg.startswith("tensor-core")
    with gemm:
        bad_f = bad_q = 0
        seed = 10
        shapes = golden()["tables"]["float_requant_shapes"]["shapes"] + [[130, 80, 384], [64, 272, 128], [257, 33, 96]]
        for (m, n, k) in shapes:
            for vec in (False, True):
                for ib, fb in ((False, False), (True, False), (False, True), (True, True)):
                    bad_f += float_case(device, gemm, m, n, k, vec, ib, fb, seed, aligned)
                    seed += 1
            for vec in (False, True):
                for unsigned, zero in golden()["tables"]["requant_output_modes"]["modes"]:
                    bad_q += requant_case(device, gemm, m, n, k, vec, unsigned, zero, (seed & 1) == 0, seed,
                                          (seed & 2) != 0, (seed & 4) != 0, aligned)
                    seed += 1
        assert bad_f == 0 and bad_q == 0


@pytest.mark.parametrize("cfg", list(CONFIGS))
def test_requantization_rounds_half_to_even_and_saturates(device, cfg):
    """Int8Tests.cs:503-547: a 1 x 1 product of K = 1 puts ties, saturation, NaN and infinity through the epilogue
    (for the tensor-core kernels the product is padded to 16 x 16 x 16 with zeros)."""
    gemm = og.Int8Gemm(device, CONFIGS[cfg])
    pad = 16 if cfg.startswith("tensor-core") else 1
    with gemm:
        for c in golden()["tables"]["requant_ties"]["cases"]:
            a = np.zeros(pad * pad + 4, np.int8)
            a[0] = c["a"]
            b = np.zeros(pad * pad + 4, np.int8)
            b[0] = 1
            bufs = [device.create_buffer(np.int8, a), device.create_buffer(np.int8, b),
                    device.create_buffer(np.float32, np.array([c["mult"]], np.float32)),
                    typed(device, np.zeros(pad * pad + 4, np.uint8), not c["unsigned"])]
            try:
                enc = device.begin_commands()
                gemm.encode_requantized(enc, og.Int8GemmProblem(pad, pad, pad), bufs[0], bufs[1], bufs[3],
                                        og.Int8Operand(bufs[2], 0), c["zero"])
                device.submit(enc)
                got = int(bufs[3].read().view(np.uint8)[0])
            finally:
                for v in bufs:
                    v.dispose()
            assert got == c["expected"], c


def test_bad_arguments_are_rejected_on_the_device(device):
    """Int8Tests.cs:549-574 through the encode entry points: raised before anything is recorded."""
    with og.Int8Gemm(device) as gemm:
        a = device.create_buffer(np.uint8, 64)
        b = device.create_buffer(np.int8, 64)
        c = device.create_buffer(np.int32, 64)
        f = device.create_buffer(np.float32, 64)
        fl = device.create_buffer(np.float32, 1)
        enc = device.begin_commands()
        P, Op = og.Int8GemmProblem, og.Int8Operand
        bad = [
            lambda: gemm.encode_int32(enc, P(9, 9, 9), a, b, c),
            lambda: gemm.encode_int32(enc, P(-1, 2, 2), a, b, c),
            lambda: gemm.encode_int32(enc, P(2, 2, 2, batch=0), a, b, c),
            lambda: gemm.encode_int32(enc, P(2, 2, 2, lda=1), a, b, c),
            lambda: gemm.encode_int32(enc, P(2, 2, 2, offset_c=62), a, b, c),
            lambda: gemm.encode_int32(enc, P(8, 8, 8, offset_a=1), a, b, c),
            lambda: gemm.encode_int32(enc, P(2, 2, 2), a, b, c, Op(a, 63, True)),
            lambda: gemm.encode_int32(enc, P(2, 2, 2), f, b, c),
            lambda: gemm.encode_float(enc, P(2, 8, 2), a, b, f, Op(fl, 0, True)),
            lambda: gemm.encode_requantized(enc, P(2, 2, 2), a, b, a, Op(fl, 0), 300),
            lambda: gemm.encode_requantized(enc, P(2, 2, 2), a, b, b, Op(fl, 0), 128),
        ]
        for fn in bad:
            with pytest.raises(og.GpuKernelShapeException):
                fn()
        assert enc.dispatch_count == 0
        with pytest.raises(og.ArgumentNullException):
            gemm.encode_int32(None, P(2, 2, 2), a, b, c)
        device.submit(enc)
        device.wait_idle()
        for v in (a, b, c, f, fl):
            v.dispose()


def test_a_caller_sized_scratch_and_reserved_scratch(device):
    """Int8ScratchTests.cs:27-66: caller-placed and reserved scratch; CUDA builds no bind groups at all."""
    N, K, small, large = 96, 64, 32, 160
    a = device.create_buffer(np.uint8, oracle.bytes_(large * K + 4, 1))
    b = device.create_buffer(np.int8, np.zeros(N * K + 4, np.int8))
    y = device.create_buffer(np.uint8, large * N + 4)
    mult = device.create_buffer(np.float32, np.array([0.001], np.float32))
    need = og.Int8Gemm.scratch_elements(og.Int8GemmProblem(large, N, K))
    assert need == large * N
    scratch = device.create_buffer(np.int32, need)
    for reserve, caller in ((False, True), (True, False), (False, False)):
        with og.Int8Gemm(device) as gemm:
            if reserve:
                gemm.reserve_scratch(need)
            for m in (small, large):
                enc = device.begin_commands()
                gemm.encode_requantized(enc, og.Int8GemmProblem(m, N, K), a, b, y, og.Int8Operand(mult, 0), 3,
                                        scratch=og.Int8Scratch(scratch) if caller else None)
                device.submit(enc)
            got = y.read()[:large * N]
            assert np.all(got == 3)  # B is all zero, so every output is the zero point
            assert gemm.bind_groups_created == 0
    with og.Int8Gemm(device) as gemm:
        with pytest.raises(og.ArgumentOutOfRangeException):
            gemm.reserve_scratch(-1)
        with pytest.raises(og.GpuKernelShapeException) as e:
            gemm.encode_requantized(device.begin_commands(), og.Int8GemmProblem(64, 64, 8), a, b, y,
                                    og.Int8Operand(mult, 0), 0, scratch=og.Int8Scratch(scratch, need - 100))
        assert e.value.argument == "scratch"
    for v in (a, b, y, mult, scratch):
        v.dispose()


def test_multi_device_known_answer():
    """MultiDeviceTests.cs:6-107: every visible device computes the 2 x 3 x 2 known answer, interleaved."""
    n = og.device_count()
    devices = [og.GpuDevice(i) for i in range(n)]
    try:
        gemms = [og.Int8Gemm(d) for d in devices]
        kat = golden()["kat_multidevice"]
        a = [d.create_buffer(np.uint8, np.array(kat["a_u8"], np.uint8)) for d in devices]
        b = [d.create_buffer(np.int8, np.array(kat["b_s8"], np.int8)) for d in devices]
        c = [d.create_buffer(np.int32, 6) for d in devices]
        for _ in range(3):
            for i, d in enumerate(devices):
                enc = d.begin_commands()
                gemms[i].encode_int32(enc, og.Int8GemmProblem(2, 3, 2), a[i], b[i], c[i])
                d.submit(enc)
        for i in range(n):
            assert c[i].read().tolist() == kat["expected"]
        for i in range(n):
            for v in (a[i], b[i], c[i]):
                v.dispose()
            gemms[i].dispose()
    finally:
        for d in devices:
            d.dispose()


def test_products_wider_than_one_grid_axis(device):
    """ConvIntegerTests.cs:343-392: products with millions of columns or rows (k = 5)."""
    for (m, n) in ((3, 4_300_001), (4_300_001, 3), (2, 4_194_241)):
        c = Case(f"{m}x{n}", problem(m, n, 5), False, True, 1, 2)
        for name, gemm in configs(device, ["default", "portable"]):
            with gemm:
                bad, _ = run_int32(device, gemm, c, 11)
                assert bad == 0, f"{m}x{n} [{name}]"


@pytest.mark.parametrize("cfg", ["tensor-core-1sm", "tensor-core-2sm"])
def test_tensor_core_sums_wrap_modulo_2_32(device, cfg):
    """The definition wraps modulo 2^32 (Int8Gemm.cs:103-105): 255 * 255 * K passes 2^32 at K = 66560."""
    m, n, k = 300, 144, 66560
    c = Case("wrap", problem(m, n, k), False, False, 1, 2)
    a = np.full(m * k + 4, 255, np.uint8)
    b = np.full(k * n + 4, 255, np.uint8)
    za = np.zeros(1, np.uint8)
    zb = np.ones(n + 1, np.uint8)
    with og.Int8Gemm(device, CONFIGS[cfg]) as gemm:
        for zpa, zpb in ((None, None), (za, zb)):
            cc = Case("wrap", c.p, False, False, 0 if zpa is None else 1, 0 if zpb is None else 2)
            bad, kern = run_int32(device, gemm, cc, 3, data=(a, b, zpa, zpb))
            assert base_kernel(kern) == cfg
            assert bad == 0


@pytest.mark.parametrize("cfg,m,n,k", [("tensor-core-2sm", 1280, 4096, 512), ("tensor-core-1sm", 1280, 4096, 512),
                                       ("tensor-core-2sm", 1536, 3328, 1152), ("tensor-core-2sm", 1100, 4100, 520)])
def test_stream_k_split_tiles_are_bit_exact(device, cfg, m, n, k):
    """With the stream-K option and a partial last wave of tiles, the (tile, K block) units are split evenly across
    the SMs and a tile cut between two of them is finished by the one holding K block 0 after the other has handed
    over its sums. int32 with both zero-point layouts, the float and requantized forms, and three products
    recorded back to back in one encoder (the hand-over flags are reset between launches)."""
    opts = CONFIGS[cfg]
    gemm = og.Int8Gemm(device, og.Int8GemmOptions(kernel=opts.kernel, tile=opts.tile, stream_k=2))
    with gemm:
        kernels = set()
        for i, (za_mode, zb_mode, a_s, b_s) in enumerate(((1, 2, False, True), (2, 1, True, False), (0, 0, True, True))):
            c = align_case(Case("stream-k", problem(m, n, k), a_signed=a_s, b_signed=b_s, za_mode=za_mode,
                                zb_mode=zb_mode))
            bad, kernel = run_int32(device, gemm, c, 70 + i)
            assert bad == 0, (c.p, kernel)
            kernels.add(kernel)
        assert kernels == {cfg + "-stream-k"}, kernels
        assert float_case(device, gemm, m, n, k, True, True, True, 80, aligned=True) == 0
        assert requant_case(device, gemm, m, n, k, True, False, 3, True, 81, False, True, aligned=True) == 0

        # Three products in one encoder, run in stream order on one instance (and so one hand-over buffer).
        shapes = [(m, n, k, 90), (m, n, 2 * k, 91), (m, n, k, 92)]
        data, bufs = [], []
        enc = device.begin_commands()
        for (mm, nn, kk, seed) in shapes:
            p = align_case(Case("seq", problem(mm, nn, kk), a_signed=False, b_signed=True, za_mode=1, zb_mode=2)).p
            a = oracle.bytes_(p["m"] * p["lda"] + p["offset_a"] + 4, seed)
            b = oracle.bytes_(kk * p["ldb"] + p["offset_b"] + 4, seed + 1)
            za, zb = oracle.bytes_(1, seed + 2), oracle.bytes_(nn, seed + 3)
            want = oracle.int8_gemm(a, False, b, True, za, False, zb, True, **oracle_shape(p))
            bs = [typed(device, a, False), typed(device, b, True), device.create_buffer(np.int32, want.size),
                  typed(device, za, False), typed(device, zb, True)]
            gemm.encode_int32(enc, og.Int8GemmProblem(**p), bs[0], bs[1], bs[2], og.Int8Operand(bs[3], 0),
                              og.Int8Operand(bs[4], 0, True))
            data.append((bs[2], want))
            bufs += bs
        device.submit(enc)
        try:
            for c_buf, want in data:
                assert np.array_equal(c_buf.read(), want)
        finally:
            for v in bufs:
                v.dispose()


@pytest.mark.parametrize("m,n,k,batch,trans_b", [
    (16, 300, 2048, 1, False),    # 3 column tiles over 6 workers: every tile split
    (7, 1000, 4100, 1, False),    # ragged K (the last K block holds 4 bytes), 33 workers
    (1, 128, 2560, 3, False),     # batched B, one row
    (16, 384, 3072, 2, True),     # B stored N x K
    (12, 2048, 8192, 1, False),   # 16 tiles over 128 workers, each tile met by eight segments
])
def test_few_rows_even_split_is_bit_exact(device, m, n, k, batch, trans_b):
    """The few-rows kernel with its (column tile, K block) units split evenly across persistent workers (partial
    segments meet through records and tickets; the segment completing a tile adds the others' dot products, column
    sums of B and row sums of A, then finishes it): int32 with every zero-point mode, the float form and the
    requantized form, against the oracle, twice in a row on one instance (the tickets return to zero)."""
    gemm = og.Int8Gemm(device, CONFIGS["tensor-core-auto"])
    try:
        for rep in range(2):
            for za_mode, zb_mode, a_s, b_s in ((0, 0, True, True), (1, 2, False, True), (2, 1, True, False),
                                               (1, 1, False, False)):
                c = align_case(Case("k-split", problem(m, n, k, batch=batch, trans_b=trans_b), a_s, b_s,
                                    za_mode, zb_mode))
                bad, kernel = run_int32(device, gemm, c, 1000 * rep + 10 * za_mode + zb_mode)
                assert kernel == "tensor-core-rows", kernel
                assert bad == 0, f"zp modes {za_mode}/{zb_mode}: {bad} mismatches"
            if batch == 1 and not trans_b:
                assert float_case(device, gemm, m, n, k, True, True, True, 31 + rep, aligned=True) == 0
                assert requant_case(device, gemm, m, n, k, True, False, 5, True, 41 + rep, True, True,
                                    aligned=True) == 0
    finally:
        gemm.dispose()


@pytest.mark.parametrize("cfg", ["default", "portable", "tensor-core-1sm", "tensor-core-2sm"])
def test_config_1_matmulinteger_is_bit_exact(device, cfg):
    """Config 1 at its size: A u8 [256 x 384] uniform 0..255 with scalar zero point 128, B s8 [384 x 512] uniform
    -128..127 with zero point 0, int32 output, against the oracle (the reference's CPU case)."""
    rng = np.random.default_rng(0)
    m, k, n = 256, 384, 512
    a = rng.integers(0, 256, size=m * k, dtype=np.int16).astype(np.uint8)
    b = rng.integers(-128, 128, size=k * n, dtype=np.int16).astype(np.int8)
    p = problem(m, n, k)
    want = oracle.int8_gemm(a, False, b.view(np.uint8), True, np.array([128], np.uint8), False,
                            np.array([0], np.uint8), False, **oracle_shape(p))
    gemm = og.Int8Gemm(device, CONFIGS[cfg])
    bufs = [device.create_buffer(np.uint8, a), device.create_buffer(np.int8, b),
            device.create_buffer(np.int32, np.full(m * n + 2, SENTINEL, np.int32)),
            device.create_buffer(np.uint8, np.array([128, 0, 0, 0], np.uint8)),
            device.create_buffer(np.int8, np.zeros(4, np.int8))]
    try:
        enc = device.begin_commands()
        gemm.encode_int32(enc, og.Int8GemmProblem(**p), bufs[0], bufs[1], bufs[2], og.Int8Operand(bufs[3], 0),
                          og.Int8Operand(bufs[4], 0))
        device.submit(enc)
        got = bufs[2].read()
        assert np.array_equal(got[:m * n], want), gemm.last_kernel
        assert np.all(got[m * n:] == SENTINEL)
    finally:
        for v in bufs:
            v.dispose()
        gemm.dispose()


@pytest.mark.parametrize("m,n,k,batch,trans_b,off_a,off_b", [
    (512, 640, 1000, 1, False, 0, 0),    # A's rows 1000 bytes apart
    (300, 1000, 1024, 1, False, 0, 0),   # B's rows 1000 bytes apart
    (384, 520, 1000, 1, True, 3, 5),     # both, B stored N x K, bases off 16-byte boundaries
    (256, 512, 999, 3, False, 0, 0),     # batched A and B, dense batches of odd size
    (8, 8192, 3000, 1, False, 1, 0),     # few rows
])
def test_misaligned_operands_take_the_tensor_cores(device, m, n, k, batch, trans_b, off_a, off_b):
    """Products large enough for the tensor cores whose operand rows or batches do not start on 16-byte boundaries:
    the misaligned operands are copied into pitched buffers and the tensor-core product runs on the copies. int32 with
    every zero-point mode, then the float and requantized forms, against the oracle."""
    gemm = og.Int8Gemm(device)
    try:
        kernels = set()
        for za_mode, zb_mode, a_s, b_s in ((1, 2, False, True), (2, 1, True, False), (0, 0, True, True)):
            c = Case("staged", problem(m, n, k, batch=batch, trans_b=trans_b, off_a=off_a, off_b=off_b), a_s, b_s,
                     za_mode, zb_mode)
            bad, kernel = run_int32(device, gemm, c, 300 + za_mode)
            kernels.add(kernel)
            assert bad == 0, f"zp modes {za_mode}/{zb_mode} via {kernel}"
        assert all(kr.startswith("tensor-core") and kr.endswith("-staged") for kr in kernels), kernels
        if batch == 1 and not trans_b and off_a == 0 and off_b == 0:
            assert float_case(device, gemm, m, n, k, True, True, True, 310) == 0
            assert requant_case(device, gemm, m, n, k, True, False, 4, True, 311, True, True) == 0
    finally:
        gemm.dispose()


@pytest.mark.parametrize("cfg", ["tensor-core-1sm", "tensor-core-2sm"])
@pytest.mark.parametrize("m,n,k,batch,trans_b", [
    (200, 600, 8192, 1, False),   # K of 64 whole blocks, split across the sums CTAs
    (200, 600, 8200, 1, False),   # a partial last K block
    (260, 1030, 777, 3, False),   # ragged column tiles, batched A and B, an odd K
    (384, 700, 3000, 2, True),    # B stored N x K
    (150, 530, 5, 1, False),      # K inside one block
])
def test_zero_point_byte_sums_are_bit_exact(device, cfg, m, n, k, batch, trans_b):
    """The byte sums of the zero-point correction (row sums of A, column sums of B, through the tensor-core sums
    kernel and added up by the product's epilogue) for every zero-point mode and signedness, against the oracle."""
    with og.Int8Gemm(device, CONFIGS[cfg]) as gemm:
        for za_mode, zb_mode, a_s, b_s in ((1, 2, False, True), (2, 1, True, False), (2, 2, True, True),
                                           (1, 0, False, True), (0, 2, False, True)):
            c = align_case(Case("sums", problem(m, n, k, batch=batch, trans_b=trans_b), a_s, b_s, za_mode, zb_mode))
            bad, kernel = run_int32(device, gemm, c, 400 + 3 * za_mode + zb_mode)
            assert base_kernel(kernel) == cfg
            assert bad == 0, f"zp modes {za_mode}/{zb_mode} signed {a_s}/{b_s}"
