"""The multiply-first quotient rule of QuantizeLinear's uniform-scale path, restated in numpy float32 and checked
against the correctly rounded division: whenever the rule keeps rint(RN(x * RN(1 / s))), that equals
rint(RN(x / s)). Inputs are crowded within a few ulps of half-integer quotients, over scales from 1e-30 to 1e30.
The device code is checked against the oracle by the GPU tests; this pins the rule's margin itself."""
import numpy as np

F32 = np.float32


def _rule(x: np.ndarray, r: np.float32):
    """(fast value, taken) of the device rule: m = RN(x r), q = rint(m), d = m - q, taken when
    RN(|m| 2^-20 + |d|) < 1/2 - 2^-19."""
    m = (x * r).astype(F32)
    q = np.rint(m)
    d = (m - q).astype(F32)
    t = (np.abs(m).astype(np.float64) * 2.0 ** -20 + np.abs(d).astype(np.float64)).astype(F32)
    return q, t < F32(0.5 - 2.0 ** -19)


def test_multiply_first_rule_matches_division():
    rng = np.random.default_rng(5)
    taken = 0
    for trial in range(60):
        s = F32(np.exp(rng.uniform(np.log(1e-30), np.log(1e30)))) if trial % 3 else F32(rng.uniform(0.001, 10))
        r = F32(1) / s
        if not (np.isfinite(r) and abs(r) >= np.finfo(np.float32).tiny):
            continue
        k = np.concatenate([rng.integers(-300, 300, size=100000),
                            rng.integers(-(1 << 22), 1 << 22, size=50000)]).astype(np.float64)
        base = ((k + 0.5) * np.float64(s)).astype(F32)
        x = (base.view(np.int32) + rng.integers(-6, 7, size=base.size).astype(np.int32)).view(F32)
        x = np.concatenate([x, (rng.standard_normal(50000) * 300 * np.float64(s)).astype(F32)])
        with np.errstate(all="ignore"):
            x = x[np.isfinite(x)]
            exact = np.rint(x / s)
            q, fast = _rule(x, r)
        taken += int(fast.sum())
        assert not np.any(fast & (q != exact)), f"scale {s}"
    assert taken > 1_000_000


def test_rule_declines_ties_nan_and_huge():
    s = F32(0.25)
    r = F32(1) / s
    with np.errstate(all="ignore"):
        _, fast = _rule(np.array([0.125, -0.375, np.nan, np.inf, 3e38, 1.1e6], F32), r)
    assert not fast.any()


def _byte_through_bits(x: np.ndarray, s: np.float32, zp: int):
    """(byte, taken) of DynamicQuantizeLinear's single-kernel path: cz = zp + 1.5 * 2^23, t = RN(RN(x r) + cz); the
    rule's test on m = RN(x r) with d = m - (t - cz); where taken, t's bits clamped to [0x4B400000, 0x4B4000FF] give
    the byte in their low 8 bits, elsewhere clamp(rint(RN(x / s)) + zp) with NaN to 0."""
    r = F32(1) / s
    cz = F32(F32(zp) + F32(12582912.0))
    with np.errstate(all="ignore"):
        m = (x * r).astype(F32)
        t = (m + cz).astype(F32)
        d = (m - (t - cz).astype(F32)).astype(F32)
        test = (np.abs(m).astype(np.float64) * 2.0 ** -20 + np.abs(d).astype(np.float64)).astype(F32)
        taken = (test < F32(0.5 - 2.0 ** -19)) & bool(np.isfinite(r) and abs(r) >= np.finfo(np.float32).tiny)
        bits = np.clip(t.view(np.uint32), 0x4B400000, 0x4B4000FF) & 0xFF
        v = (np.rint((x / s).astype(F32)) + F32(zp)).astype(F32)
        slow = np.where(np.isnan(v), 0, np.clip(v, 0, 255))
    return np.where(taken, bits, slow).astype(np.int64), taken


def test_byte_through_bits_matches_the_definition():
    """clamp(rint(x / s) + zp, 0, 255) with the division correctly rounded, NaN to 0, for DynamicQuantizeLinear's
    scales (range / 255) and zero points, inputs crowded around half-integer quotients, huge quotients, NaN and
    infinities."""
    rng = np.random.default_rng(11)
    taken_total = 0
    for trial in range(120):
        lo = -abs(rng.standard_normal()) * 10 ** rng.uniform(-3, 3)
        hi = abs(rng.standard_normal()) * 10 ** rng.uniform(-3, 3)
        s = F32((F32(hi) - F32(lo)) / F32(255))
        zp = int(np.clip(np.rint(-(F32(lo) / s)), 0, 255))
        k = rng.integers(-300, 300, size=20000).astype(np.float64)
        ties = ((k + 0.5) * np.float64(s)).astype(F32)
        near = (ties.view(np.int32) + rng.integers(-4, 5, size=ties.size).astype(np.int32)).view(F32)
        x = np.concatenate([rng.uniform(lo, hi, 40000).astype(F32), ties, near,
                            (rng.standard_normal(2000) * 1e7 * np.float64(s)).astype(F32),
                            np.array([np.nan, np.inf, -np.inf, 0.0, -0.0], F32)])
        got, taken = _byte_through_bits(x, s, zp)
        with np.errstate(all="ignore"):
            v = (np.rint((x / s).astype(F32)) + F32(zp)).astype(F32)
        want = np.where(np.isnan(v), 0, np.clip(v, 0, 255)).astype(np.int64)
        assert np.array_equal(got, want), f"scale {s} zero point {zp}"
        taken_total += int(taken.sum())
    assert taken_total > 4_000_000
