"""The CPU oracle pinned against the reference's golden vectors and against an independent pure-Python restatement.

Runs without a GPU. The oracle (oracle/og_oracle.c) restates the C# references of the reference's int8 tests; the
literal known answer of MultiDeviceTests.cs and the restatements in tests/golden/make_golden.py must agree with it
bit for bit.
"""
import math

import numpy as np
import pytest

import og_oracle as oracle
from cases import case_data, edge_cases, golden, oracle_shape
from golden import make_golden as restated


def test_generators_match_the_reference_lcg():
    for seed in (0, 1, 7, 123456):
        assert oracle.bytes_(257, seed).tolist() == restated.lcg_bytes(257, seed)
    # Rig.Random (Rig.cs:8-19), first values by hand: s = seed*2654435761 + 12345, then the LCG step.
    s = (3 * 2654435761 + 12345) & 0xFFFFFFFF
    want = []
    for _ in range(5):
        s = (s * 1664525 + 1013904223) & 0xFFFFFFFF
        u = np.float32(s >> 8) / np.float32(16777216)
        want.append(np.float32(np.float32(-3) + np.float32(np.float32(8) * np.float32(u))))
    assert oracle.random(5, 3, -3.0, 5.0).tolist() == [float(w) for w in want]


def test_multidevice_known_answer():
    """MultiDeviceTests.cs:30-31,53-55: [[1 2],[3 4]] x [[1 -1 2],[-2 3 -3]] = [[-3 5 -4],[-5 9 -6]]."""
    kat = golden()["kat_multidevice"]
    a = np.array(kat["a_u8"], dtype=np.uint8)
    b = np.array(kat["b_s8"], dtype=np.int8).view(np.uint8)
    got = oracle.int8_gemm(a, False, b, True, m=2, n=3, k=2)
    assert got.tolist() == kat["expected"] == [-3, 5, -4, -5, 9, -6]


def test_smoke_known_answers():
    """KernelSmoke.cs:199-236: the AOT smoke's int8 product and DynamicQuantizeLinear."""
    g = golden()
    s = g["smoke_gemm"]
    got = oracle.int8_gemm(np.array(s["a_u8"], np.uint8), False, np.array(s["b_s8_bytes"], np.uint8), True,
                           za=np.array([s["za"]], np.uint8), m=s["m"], n=s["n"], k=s["k"])
    assert got.tolist() == s["expected"]
    q = g["smoke_dq"]
    y, scale, zp = oracle.dynamic_quantize(np.array(q["x"], np.float32))
    assert y.tolist() == q["expected_y"]
    assert np.float32(scale).view(np.uint32) == np.float32(q["expected_scale"]).view(np.uint32)
    assert zp == q["expected_zero_point"]


def test_edge_cases_match_the_python_restatement():
    """EdgeShapesAreBitExact's small cases (reference generator, seeds and offsets) against pure Python."""
    for c in golden()["edge_cases_small"]["cases"]:
        from cases import Case
        case = Case(c["name"], c["problem"], c["a_signed"], c["b_signed"], c["za_mode"], c["zb_mode"])
        a, b, za, zb = case_data(case, c["seed"], oracle.bytes_)
        got = oracle.int8_gemm(a, case.a_signed, b, case.b_signed, za, case.za_mode == 2, zb, case.zb_mode == 2,
                               **oracle_shape(case.p))
        assert got.tolist() == c["expected"], c["name"]


@pytest.mark.parametrize("threads", [1, 3])
def test_signed_domain_identity_equals_the_definition(threads):
    """Int8GemmDot.hlsl:4-10: the packed-dot rewrite gives the same sums as the definition, extremes included."""
    cases = [c for c in edge_cases() if c.p["m"] * c.p["n"] * c.p["k"] * c.p["batch"] <= 200_000]
    assert len(cases) > 100
    for seed, c in enumerate(cases, start=1):
        a, b, za, zb = case_data(c, seed, oracle.bytes_)
        args = (a, c.a_signed, b, c.b_signed, za, c.za_mode == 2, zb, c.zb_mode == 2)
        d = oracle.int8_gemm(*args, threads=threads, **oracle_shape(c.p))
        s = oracle.int8_gemm(*args, signed_domain=True, **oracle_shape(c.p))
        assert np.array_equal(d, s), c.name


def test_sums_wrap_modulo_2_32():
    """The sums are defined modulo 2^32 (Int8Gemm.cs:103-105): 255 * 255 * 66050 overflows and must wrap."""
    k = 66050
    a = np.full(k, 255, np.uint8)
    b = np.full(k, 255, np.uint8)
    got = oracle.int8_gemm(a, False, b, False, m=1, n=1, k=k)
    want = (255 * 255 * k) % 2 ** 32
    want = want - 2 ** 32 if want >= 2 ** 31 else want
    assert got.tolist() == [want]


def test_requantization_ties_saturation_nan():
    """RequantizationRoundsHalfToEvenAndSaturates' table (Int8Tests.cs:512) against the pure-Python restatement."""
    t = golden()["tables"]["requant_ties"]
    assert len(t["cases"]) == 9 * 19
    for c in t["cases"]:
        assert oracle.requant(c["a"], c["mult"], c["zero"], c["unsigned"]) & 0xFF == c["expected"], c
    # Hand-checked ties: 3 * 0.5 = 1.5 -> 2, 5 * 0.5 = 2.5 -> 2, -3 * 0.5 = -1.5 -> -2 (half to even).
    assert oracle.requant(3, 0.5, 10, True) == 12
    assert oracle.requant(5, 0.5, 10, True) == 12
    assert oracle.requant(-3, 0.5, -10, False) == -12
    assert oracle.requant(1, float("nan"), 5, True) == 0
    assert oracle.requant(1, float("nan"), 5, False) == -128
    assert oracle.requant(1, float("inf"), 1, False) == 127
    assert oracle.requant(-1, 1e9, 3, True) == 0


def test_float_epilogue_two_roundings():
    rng = np.random.default_rng(5)
    acc = rng.integers(-2 ** 31, 2 ** 31, 2000, dtype=np.int64).astype(np.int32)
    scale = rng.uniform(1e-4, 1e-2, 2000).astype(np.float32)
    ib = rng.integers(-10000, 10000, 2000).astype(np.int32)
    fb = rng.uniform(-2, 2, 2000).astype(np.float32)
    vec = oracle.float_epilogue(acc, scale, ib, fb)
    for i in range(0, 2000, 97):
        s = oracle.float_epilogue_scalar(int(acc[i]), float(scale[i]), int(ib[i]), float(fb[i]))
        assert np.float32(s).view(np.uint32) == vec[i].view(np.uint32)


def test_div_exact_restatement_equals_ieee_division():
    """DivExact.hlsli is a correctly rounded division: it must equal C's float division everywhere it applies."""
    rng = np.random.default_rng(11)
    xs = np.concatenate([rng.standard_normal(3000).astype(np.float32) * np.float32(10.0),
                         (rng.integers(-1016, 1016, 2000) * 0.125).astype(np.float32)])
    ss = np.concatenate([rng.uniform(1e-6, 0.1, 2500).astype(np.float32),
                         np.full(2500, np.float32(4.7) * 2 / np.float32(255), np.float32)])
    for x, s in zip(xs.tolist(), ss.tolist()):
        want = np.float32(np.float32(x) / np.float32(s))
        got = np.float32(oracle.div_exact(x, s))
        assert got.view(np.uint32) == want.view(np.uint32), (x, s)
    assert math.copysign(1.0, oracle.div_exact(-0.0, 3.0)) == -1.0


@pytest.mark.parametrize("kind", range(7))
def test_dynamic_quantize_matches_the_python_restatement(kind):
    """DynamicReference (Int8Tests.cs:577-615) on the test's seven distributions, small counts."""
    for seed, count in enumerate((1, 2, 3, 255, 257, 1025), start=1):
        x = oracle.dq_input(count, seed * 7 + kind, kind)
        y, scale, zp = oracle.dynamic_quantize(x)
        wy, ws, wz = restated.dynamic_reference(x.tolist())
        assert y.tolist() == wy
        assert np.float32(scale).view(np.uint32) == np.float32(ws).view(np.uint32)
        assert zp == wz


def test_dynamic_quantize_edge_values():
    y, s, z = oracle.dynamic_quantize(np.zeros(5, np.float32))
    assert y.tolist() == [0] * 5 and s == 1.0 and z == 0
    y, s, z = oracle.dynamic_quantize(np.array([np.nan, np.nan], np.float32))
    assert y.tolist() == [0, 0] and s == 1.0 and z == 0
    y, s, z = oracle.dynamic_quantize(np.array([0.0, 255.0, np.nan], np.float32))
    assert s == 1.0 and z == 0 and y.tolist() == [0, 255, 0]
    y, s, z = oracle.dynamic_quantize(np.array([-255.0, 0.0, -1.0], np.float32))
    assert s == 1.0 and z == 255 and y.tolist() == [0, 255, 254]
    y, s, z = oracle.dynamic_quantize(np.array([np.inf, 1.0], np.float32))
    assert math.isinf(s) and z == 0 and y.tolist() == [0, 0]


# ---- DequantizeLinear / QuantizeLinear / ConvInteger restatements ----------------------------------------------------

def _sha(a) -> str:
    import hashlib
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def test_half_conversions_match_ieee():
    """The oracle's binary16 conversions against numpy's (IEEE round to nearest even), every half and random
    floats including ties, subnormal results and overflow."""
    h = np.arange(65536, dtype=np.uint16)
    h = h[~np.isnan(h.view(np.float16))]
    got = np.array([oracle.half_to_float(v) for v in h[::7]], np.float32)
    assert np.array_equal(got.view(np.uint32), h[::7].view(np.float16).astype(np.float32).view(np.uint32))
    rng = np.random.default_rng(3)
    f = rng.integers(0, 2**32, size=6000, dtype=np.uint64).astype(np.uint32).view(np.float32)
    f = np.concatenate([f[~np.isnan(f)], np.array([65504, 65519.99, 65520, 2**-25, 2**-24, 3 * 2**-26, 6.1e-5, -0.0],
                                                  np.float32)])
    with np.errstate(over="ignore"):
        want = f.astype(np.float16).view(np.uint16)
    assert [oracle.float_to_half(v) for v in f] == want.tolist()


def test_dequantize_matches_the_python_restatement():
    from cases import axis_params, quantized

    g = golden()["dequantize"]
    off = g["offsets"]
    assert g["dequantize_small"]
    for c in g["dequantize_small"]:
        count, axis_len, inner = axis_params(c["shape"], c["axis"], c["per_axis"])
        x = quantized(c["kind"], count + off["OffX"], c["seed"])
        scale = oracle.random(axis_len + off["OffS"], c["seed"] + 1, 0.001, 2.0)
        zs = quantized(c["kind"], axis_len + off["OffZ"], c["seed"] + 2)
        got = oracle.dequantize(x[off["OffX"]:], c["shape"], c["axis"], c["per_axis"], scale[off["OffS"]:],
                                zs[off["OffZ"]:] if c["with_zero"] else None, c["half"])
        assert _sha(got) == c["sha256"], c


def test_quantize_matches_the_python_restatement():
    from cases import axis_params, quantize_input, quantized

    g = golden()["dequantize"]
    off = g["offsets"]
    assert g["quantize_small"]
    for c in g["quantize_small"]:
        count, axis_len, inner = axis_params(c["shape"], c["axis"], c["per_axis"])
        x = quantize_input(count + off["OffX"], c["seed"])
        if c["half_in"]:
            with np.errstate(over="ignore"):
                x = x.astype(np.float16)
        scale = np.array([c["scales"][i % len(c["scales"])] for i in range(axis_len + off["OffS"])], np.float32)
        zs = quantized("s8" if c["signed"] else "u8", axis_len + off["OffZ"], c["seed"] + 2)
        got = oracle.quantize(x[off["OffX"]:], c["shape"], c["axis"], c["per_axis"], scale[off["OffS"]:],
                              zs[off["OffZ"]:] if c["with_zero"] else None, c["signed"])
        assert _sha(got) == c["sha256"], c


def test_conv_integer_matches_the_python_restatement():
    from cases import conv_case_data

    cases = golden()["conv_integer"]["spread_small"]
    assert len(cases) >= 30
    for c in cases:
        x, w, xz, wz = conv_case_data(c["p"], c["seed"], c["xz_mode"], c["wz_mode"], -1, oracle.bytes_)
        y = oracle.conv_integer(c["p"], x, c["x_signed"], w, c["w_signed"], xz, wz, c["wz_mode"] == 2, threads=2)
        assert _sha(y.astype(np.int32)) == c["sha256"], c["name"]


def test_conv_integer_equals_the_int8_product_of_its_columns():
    """A second route to the same sums: unfold the windows on the host (padding with the zero point of x) and run the
    oracle's int8 product, as the GPU path does."""
    p = dict(batch=2, cin=4, h=7, w=6, cout=6, kh=3, kw=2, stride_h=2, stride_w=1, dilation_h=1, dilation_w=2,
             pad_top=1, pad_left=0, pad_bottom=2, pad_right=1, groups=2, offset_x=0, offset_w=0)
    rng = np.random.default_rng(9)
    x = rng.integers(0, 256, size=2 * 4 * 7 * 6, dtype=np.uint16).astype(np.uint8)
    w = rng.integers(0, 256, size=6 * 2 * 3 * 2, dtype=np.uint16).astype(np.uint8)
    xz, wz = np.array([131], np.uint8), rng.integers(0, 256, size=6, dtype=np.uint16).astype(np.uint8)
    want = oracle.conv_integer(p, x, False, w, True, xz, wz, True, threads=1)
    oh = oracle.conv_out_extent(7, 3, 2, 1, 1, 2)
    ow = oracle.conv_out_extent(6, 2, 1, 2, 0, 1)
    xs = x.reshape(2, 4, 7, 6)
    for n in range(2):
        for g in range(2):
            cols = np.full((2 * 3 * 2, oh * ow), 131, np.uint8)
            for c in range(2):
                for kh in range(3):
                    for kw in range(2):
                        for i in range(oh):
                            for j in range(ow):
                                ih, iw = i * 2 + kh - 1, j + kw * 2
                                if 0 <= ih < 7 and 0 <= iw < 6:
                                    cols[(c * 3 + kh) * 2 + kw, i * ow + j] = xs[n, g * 2 + c, ih, iw]
            a = w.reshape(6, 12)[g * 3:(g + 1) * 3]
            got = oracle.int8_gemm(a.reshape(-1), True, cols.reshape(-1), False, wz[g * 3:(g + 1) * 3], True, xz,
                                   False, threads=1, m=3, n=oh * ow, k=12)
            assert np.array_equal(got.reshape(3, oh, ow), want[n, g * 3:(g + 1) * 3])


def test_tiled_restatement_equals_the_definition():
    """og_oracle_int8_gemm_tiled (the reference portable kernel's 64 x 64 x 16 blocking with float sums folded into
    int32 every 128 k, Int8GemmKernel.hlsl:98-244) against og_oracle_int8_gemm (Int8Tests.Reference): ragged tiles, K
    past one fold and not a multiple of 16, batches, B stored N x K, every zero-point mode and signedness."""
    rng = np.random.default_rng(11)
    for (m, n, k, batch, tb) in [(70, 90, 100, 1, False), (130, 65, 300, 2, False), (64, 64, 16, 1, True),
                                 (200, 129, 1000, 1, True), (1, 1, 1, 1, False), (33, 257, 2047, 3, False)]:
        for (a_s, b_s, zam, zbm) in [(False, True, 1, 2), (True, False, 2, 1), (True, True, 0, 0), (False, False, 2, 2)]:
            a = rng.integers(0, 256, batch * m * k, dtype=np.uint8)
            b = rng.integers(0, 256, batch * k * n, dtype=np.uint8)
            za = None if zam == 0 else rng.integers(0, 256, m if zam == 2 else 1, dtype=np.uint8)
            zb = None if zbm == 0 else rng.integers(0, 256, n if zbm == 2 else 1, dtype=np.uint8)
            shape = dict(m=m, n=n, k=k, batch=batch, transpose_b=tb, stride_a=m * k if batch > 1 else 0,
                         stride_b=k * n if batch > 1 else 0)
            want = oracle.int8_gemm(a, a_s, b, b_s, za, zam == 2, zb, zbm == 2, **shape)
            got = oracle.int8_gemm(a, a_s, b, b_s, za, zam == 2, zb, zbm == 2, tiled=True, threads=3, **shape)
            assert np.array_equal(got, want), (m, n, k, batch, tb, a_s, b_s, zam, zbm)
