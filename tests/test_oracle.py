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
