"""Case tables and data builders of the reference's int8 tests (tests/RecursiveAI.OneGpu.Kernels.Tests/Int8Tests.cs),
loaded from tests/golden/reference_cases.json (read out of the reference's sources by tests/golden/make_golden.py)."""
from __future__ import annotations

import json
import os
from dataclasses import dataclass, field

import numpy as np

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "reference_cases.json")


def golden() -> dict:
    with open(GOLDEN, encoding="utf-8") as f:
        return json.load(f)


def problem(m, n, k, batch=1, trans_b=False, off_a=0, off_b=0, off_c=0, lda_extra=0, ldb_extra=0, share_b=False):
    """Int8Tests.Problem (Int8Tests.cs:198-212) as keyword arguments of Int8GemmProblem."""
    lda = k + lda_extra
    ldb = (k if trans_b else n) + ldb_extra
    stride_a = m * lda
    stride_b = 0 if share_b else (n if trans_b else k) * ldb
    if batch == 1:
        stride_a = stride_b = 0
    return dict(m=m, n=n, k=k, batch=batch, transpose_b=trans_b, lda=lda, ldb=ldb, offset_a=off_a, offset_b=off_b,
                offset_c=off_c, stride_a=stride_a, stride_b=stride_b)


@dataclass
class Case:
    """Int8Tests.Case (Int8Tests.cs:99-106)."""
    name: str
    p: dict
    a_signed: bool = False
    b_signed: bool = False
    za_mode: int = 0  # 0 none, 1 scalar, 2 vector
    zb_mode: int = 0
    fill: int = -1    # 0..255: every byte of A, B and the zero points holds this value
    extra: dict = field(default_factory=dict)


def edge_cases(shapes=None) -> list[Case]:
    """EdgeShapesAreBitExact's cases (Int8Tests.cs:219-259)."""
    g = golden()["tables"]
    cases = []
    for (m, n, k) in (shapes or g["edge_shapes"]["shapes"]):
        for s in range(4):
            for za in range(3):
                zb = (za + s) % 3
                cases.append(Case(f"{m}x{n}x{k}", problem(m, n, k, off_a=za, off_b=1 + zb, off_c=s),
                                  bool(s & 1), bool(s & 2), za, zb))
    cases.append(Case("transposed B", problem(40, 70, 50, trans_b=True, off_a=3, off_b=1), False, True, 1, 2))
    cases.append(Case("padded rows", problem(21, 22, 23, lda_extra=5, ldb_extra=3, off_a=2, off_b=3), True, True, 2, 1))
    cases.append(Case("batch 5 shared B", problem(9, 70, 33, batch=5, share_b=True, off_a=1, off_b=2), False, True, 1,
                      2))
    cases.append(Case("batch 3", problem(70, 9, 33, batch=3, off_a=3, off_b=1, off_c=3), False, False, 2, 1))
    for fill in (0x00, 0x7F, 0x80, 0xFF):
        for s in range(4):
            cases.append(Case(f"extreme {fill:02X}", problem(37, 41, 77, trans_b=bool(s & 1)), bool(s & 1),
                              bool(s & 2), 1 + (s & 1), 2 - (s & 1), fill))
    for fill in (0x00, 0x7F, 0x80, 0xFF):
        for s in range(4):
            for (m, n, k) in g["long_extreme_shapes"]["shapes"]:
                cases.append(Case(f"long extreme {fill:02X} {m}x{n}x{k}", problem(m, n, k, trans_b=bool(s & 1)),
                                  bool(s & 1), bool(s & 2), (s + fill) % 3, (s + 1) % 3, fill))
    return cases


def case_data(c: Case, seed: int, bytes_fn):
    """The inputs of Int8Tests.RunInt32 (Int8Tests.cs:118-133): A, B, zero points (None when absent)."""
    p = c.p
    lda = p["lda"] or p["k"]
    ldb = p["ldb"] or (p["k"] if p["transpose_b"] else p["n"])
    len_a = p["offset_a"] + (p["batch"] - 1) * p["stride_a"] + p["m"] * lda + 4
    len_b = p["offset_b"] + (p["batch"] - 1) * p["stride_b"] + (p["n"] if p["transpose_b"] else p["k"]) * ldb + 4
    a = bytes_fn(len_a, seed)
    b = bytes_fn(len_b, seed + 1)
    za = None if c.za_mode == 0 else bytes_fn(1 + (p["m"] if c.za_mode == 2 else 0), seed + 2)
    zb = None if c.zb_mode == 0 else bytes_fn(1 + (p["n"] if c.zb_mode == 2 else 0), seed + 3)
    if c.fill >= 0:
        a[:] = c.fill
        b[:] = c.fill ^ 0xFF
        if za is not None:
            za[:] = c.fill
        if zb is not None:
            zb[:] = c.fill ^ 0x80
    return a, b, za, zb


def oracle_shape(p: dict) -> dict:
    return {k: p[k] for k in ("m", "n", "k", "batch", "transpose_b", "lda", "ldb", "offset_a", "offset_b", "stride_a",
                              "stride_b")}


def float_scale(n: int, vec: bool, seed: int) -> np.ndarray:
    """FloatCase's scale (Int8Tests.cs:342-346)."""
    i = np.arange(n if vec else 1, dtype=np.int64)
    return (np.float32(0.0007) + (((i * 37) + seed) % 101).astype(np.float32) * np.float32(1.3e-5)).astype(np.float32)


def float_biases(n: int):
    """FloatCase's int and float biases (Int8Tests.cs:348-354)."""
    i = np.arange(n, dtype=np.int64)
    ib = (((i * 7919) % 20001) - 10000).astype(np.int32)
    fb = ((((i * 31) % 201) - 100).astype(np.float32) * np.float32(0.0137)).astype(np.float32)
    return ib, fb


def requant_mult(n: int, vec: bool, seed: int) -> np.ndarray:
    """RequantCase's multiplier (Int8Tests.cs:395-399)."""
    i = np.arange(n if vec else 1, dtype=np.int64)
    return (np.float32(0.00011) + (((i * 13) + seed) % 59).astype(np.float32) * np.float32(2.7e-6)).astype(np.float32)


def requant_bias(n: int) -> np.ndarray:
    """RequantCase's bias (Int8Tests.cs:401-405)."""
    i = np.arange(n, dtype=np.int64)
    return (((i * 6007) % 4001) - 2000).astype(np.int32)


# ---- DequantizeTests / ConvIntegerTests data (DequantizeTests.cs:8-33,150-170; ConvIntegerTests.cs:19-30) -------------

def quantized(kind: str, n: int, seed: int) -> np.ndarray:
    """DequantizeTests.Quantized<T>: int32 values (mostly large, the extremes every 17th / 19th element) or bytes, the
    byte arrays padded to a whole 32-bit word. kind: "u8", "s8" or "i32"."""
    length = n if kind == "i32" else max(n, 1) + (-max(n, 1)) % 4
    h = (seed * 2654435761 + 1) & 0xFFFFFFFF
    raw = np.empty(length, dtype=np.uint32)
    for i in range(length):
        h = (h * 1664525 + 1013904223) & 0xFFFFFFFF
        raw[i] = h
    if kind != "i32":
        b = ((raw >> 16) & 0xFF).astype(np.uint8)
        return b if kind == "u8" else b.view(np.int8)
    i = np.arange(length)
    v = raw.view(np.int32) >> (i % 7).astype(np.int32)
    v[i % 19 == 0] = np.iinfo(np.int32).max
    v[i % 17 == 0] = np.iinfo(np.int32).min
    return v.astype(np.int32)


def quantize_input(n: int, seed: int, special: bool = True) -> np.ndarray:
    """DequantizeTests.QuantizeInput: Rig.Random(n, seed, -40, 40) with ties, saturating values and (special) NaN,
    infinities, a subnormal and signed zeros at fixed positions."""
    import og_oracle as oracle

    x = oracle.random(n, seed, -40.0, 40.0).astype(np.float32)
    i = np.arange(n)
    r = i % 13
    x[r == 3] = ((i[r == 3] % 5 - 2).astype(np.float32) * np.float32(0.25))
    m5 = r == 5
    x[m5] = np.where(i[m5] % 2 == 0, 1, -1).astype(np.float32) * (np.float32(100.0) + i[m5].astype(np.float32))
    x[r == 7] = (i[r == 7] % 9 - 4).astype(np.float32) + np.float32(0.5)
    if special:
        m9 = r == 9
        sp = np.array([np.nan, np.inf, -np.inf, np.float32(1e-42)], dtype=np.float32)
        x[m9] = sp[i[m9] % 4]
        m11 = r == 11
        x[m11] = np.where(i[m11] % 2 == 0, np.float32(0.0), np.float32(-0.0))
    return x


def axis_params(shape, axis: int, per_axis: bool) -> tuple[int, int, int]:
    """(count, axis length, inner) of a tensor seen as [outer, axisLen, inner]."""
    count = int(np.prod(shape)) if len(shape) else 1
    if not per_axis:
        return count, 1, 1
    ax = axis + len(shape) if axis < 0 else axis
    return count, int(shape[ax]), int(np.prod(shape[ax + 1:])) if ax + 1 < len(shape) else 1


def conv_problem_dict(p: dict) -> dict:
    """A golden conv geometry as ConvProblem keyword arguments."""
    return dict(batch=p["batch"], in_channels=p["cin"], height=p["h"], width=p["w"], out_channels=p["cout"],
                kernel_height=p["kh"], kernel_width=p["kw"], stride_height=p["stride_h"], stride_width=p["stride_w"],
                dilation_height=p["dilation_h"], dilation_width=p["dilation_w"], pad_top=p["pad_top"],
                pad_left=p["pad_left"], pad_bottom=p["pad_bottom"], pad_right=p["pad_right"], groups=p["groups"],
                offset_x=p["offset_x"], offset_w=p["offset_w"], offset_y=p["offset_y"])


def conv_case_data(p: dict, seed: int, xz_mode: int, wz_mode: int, fill: int, bytes_fn):
    """ConvIntegerTests.Run's inputs: x = Bytes(xLen, seed), w = Bytes(wLen, seed + 1), zero points from seed + 2 and
    seed + 3, every byte replaced by the fill (w by fill ^ 0xFF, its zero points by fill ^ 0x80) when fill >= 0."""
    cin_g = p["cin"] // p["groups"]
    x_len = p["offset_x"] + p["batch"] * p["cin"] * p["h"] * p["w"] + 4
    w_len = p["offset_w"] + p["cout"] * cin_g * p["kh"] * p["kw"] + 4
    x = bytes_fn(x_len, seed)
    w = bytes_fn(w_len, seed + 1)
    xz = None if xz_mode == 0 else bytes_fn(1, seed + 2)
    wz = None if wz_mode == 0 else bytes_fn(p["cout"] if wz_mode == 2 else 1, seed + 3)
    if fill >= 0:
        x[:] = fill
        w[:] = fill ^ 0xFF
        if xz is not None:
            xz[:] = fill
        if wz is not None:
            wz[:] = fill ^ 0x80
    return x, w, xz, wz
