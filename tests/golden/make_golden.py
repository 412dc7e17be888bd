"""Generates tests/golden/reference_cases.json from the reference repository's own test files.

Run where the reference repository is checked out, with its root as --reference; the GPU box never runs this script,
the tests only read the JSON it wrote.

What it records:
  * the case tables of the reference's int8 tests, read as text from the C# sources (shapes, fills, signedness and
    zero-point mixes, requantization ties, DynamicQuantizeLinear counts), with the file:line each comes from;
  * the literal known-answer test of MultiDeviceTests.cs:30-31,53-55 (2x3x2 product);
  * expected outputs of small cases computed by an independent pure-Python restatement of the reference's C#
    references (big integers wrapped to int32, numpy float32 scalars for the float steps) - a second implementation,
    separate from the C oracle, that the oracle is checked against.

The reference (C#/.NET 10 + a NuGet shader compiler) cannot be built or run here, so these restatements and the
literal known answer are what pins the oracle.
"""
from __future__ import annotations

import argparse
import json
import os
import re

import numpy as np

REF_TESTS = "tests/RecursiveAI.OneGpu.Kernels.Tests"


def read(ref: str, rel: str) -> list[str]:
    with open(os.path.join(ref, rel), encoding="utf-8") as f:
        return f.read().splitlines()


def find(lines: list[str], pattern: str) -> tuple[int, str]:
    for i, line in enumerate(lines):
        if re.search(pattern, line):
            return i + 1, line
    raise LookupError(pattern)


def tuples(text: str, arity: int) -> list[tuple]:
    """The literal tuples of a C# array or collection expression (text after its opening bracket)."""
    cut = [text.find(t) for t in ("= [", "new[] {") if text.find(t) >= 0]
    if cut:
        text = text[min(cut):]
    inner = r"\(" + r",\s*".join([r"([^,()]+)"] * arity) + r"\)"
    return [tuple(x.strip() for x in m.groups()) for m in re.finditer(inner, text)]


def cs_float(tok: str) -> float:
    tok = tok.strip()
    if tok == "float.NaN":
        return float("nan")
    if tok == "float.PositiveInfinity":
        return float("inf")
    if tok == "float.NegativeInfinity":
        return float("-inf")
    return float(np.float32(float(tok.rstrip("f"))))


def cs_bool(tok: str) -> bool:
    return tok.strip() == "true"


# ---- independent restatements (pure Python / numpy scalars) -------------------------------------------------------

def lcg_bytes(length: int, seed: int) -> list[int]:
    """Int8Tests.Bytes (Int8Tests.cs:36-47)."""
    s = (seed * 2654435761 + 7) & 0xFFFFFFFF
    out = []
    for _ in range(length):
        s = (s * 1664525 + 1013904223) & 0xFFFFFFFF
        out.append(s >> 24)
    return out


def wrap32(v: int) -> int:
    v &= 0xFFFFFFFF
    return v - (1 << 32) if v >= (1 << 31) else v


def val(byte: int, signed: bool) -> int:
    return byte - 256 if signed and byte >= 128 else byte


def gemm_reference(p: dict, a: list[int], a_signed: bool, b: list[int], b_signed: bool, za, za_vec, zb, zb_vec):
    """Int8Tests.Reference (Int8Tests.cs:52-82) with Python integers."""
    m_, n_, k_ = p["m"], p["n"], p["k"]
    lda = p["lda"] or k_
    ldb = p["ldb"] or (k_ if p["transpose_b"] else n_)
    out = []
    for bt in range(p["batch"]):
        for m in range(m_):
            z_a = 0 if za is None else val(za[m if za_vec else 0], a_signed)
            for n in range(n_):
                z_b = 0 if zb is None else val(zb[n if zb_vec else 0], b_signed)
                acc = 0
                for k in range(k_):
                    av = val(a[p["offset_a"] + bt * p["stride_a"] + m * lda + k], a_signed) - z_a
                    bi = p["offset_b"] + bt * p["stride_b"] + (n * ldb + k if p["transpose_b"] else k * ldb + n)
                    acc += av * (val(b[bi], b_signed) - z_b)
                out.append(wrap32(acc))
    return out


def requant(acc: int, mult: float, zero: int, unsigned: bool) -> int:
    """Int8Tests.Requant (Int8Tests.cs:84-97)."""
    lo, hi = (0, 255) if unsigned else (-128, 127)
    v = np.float32(np.float32(acc) * np.float32(mult))
    if np.isnan(v):
        return lo
    r = float(round(float(v))) if np.isfinite(v) else float(v)
    r = min(max(r, float(lo - zero)), float(hi - zero))
    return int(r) + zero


def dynamic_reference(x: list[float]):
    """Int8Tests.DynamicReference (Int8Tests.cs:577-615) with numpy float32 scalars."""
    f = np.float32
    mn, mx = f(np.inf), f(-np.inf)
    for v in x:
        v = f(v)
        if v < mn:
            mn = v
        if v > mx:
            mx = v
    lo = mn if mn < 0 else f(0)
    hi = mx if mx > 0 else f(0)
    scale = f(f(hi - lo) / f(255))
    zp = 0
    if scale != 0 and np.isfinite(scale):
        z = round(float(f(f(0) - f(lo / scale))))
        zp = 0 if z < 0 else (255 if z > 255 else int(z))
    if scale == 0:
        return [0] * len(x), 1.0, 0
    y = []
    for v in x:
        q = f(f(round(float(f(f(v) / scale)))) + f(zp))
        y.append(0 if np.isnan(q) else (0 if q < 0 else (255 if q > 255 else int(q))))
    return y, float(scale), zp


def quantized(kind: str, n: int, seed: int) -> list[int]:
    """DequantizeTests.Quantized<T> (DequantizeTests.cs:8-33): int32 values (mostly large, plus the extremes) or bytes;
    byte tensors are padded to a whole 32-bit word."""
    length = n if kind == "i32" else max(n, 1) + (-max(n, 1)) % 4
    h = (seed * 2654435761 + 1) & 0xFFFFFFFF
    out = []
    for i in range(length):
        h = (h * 1664525 + 1013904223) & 0xFFFFFFFF
        if kind == "i32":
            out.append(-2**31 if i % 17 == 0 else 2**31 - 1 if i % 19 == 0 else wrap32(h) >> (i % 7))
        elif kind == "u8":
            out.append((h >> 16) & 0xFF)
        else:
            b = (h >> 16) & 0xFF
            out.append(b - 256 if b >= 128 else b)
    return out


def rig_random(n: int, seed: int, lo: float, hi: float) -> list[float]:
    """Rig.Random (Rig.cs:8-19), every step in binary32."""
    s = (seed * 2654435761 + 12345) & 0xFFFFFFFF
    lo32, hi32 = np.float32(lo), np.float32(hi)
    out = []
    for _ in range(n):
        s = (s * 1664525 + 1013904223) & 0xFFFFFFFF
        u = np.float32(s >> 8) / np.float32(16777216.0)
        out.append(float(lo32 + (hi32 - lo32) * u))
    return out


def quantize_input(n: int, seed: int, special: bool = True) -> list[float]:
    """DequantizeTests.QuantizeInput (DequantizeTests.cs:150-170)."""
    x = rig_random(n, seed, -40.0, 40.0)
    for i in range(n):
        r = i % 13
        if r == 3:
            x[i] = float(np.float32(i % 5 - 2) * np.float32(0.25))
        elif r == 5:
            x[i] = float(np.float32(1 if i % 2 == 0 else -1) * np.float32(100.0 + i))
        elif r == 7:
            x[i] = float(np.float32(i % 9 - 4) + np.float32(0.5))
        elif r == 9 and special:
            x[i] = [float("nan"), float("inf"), float("-inf"), float(np.float32(1e-42))][i % 4]
        elif r == 11 and special:
            x[i] = 0.0 if i % 2 == 0 else -0.0
    return x


def digest(values, dtype) -> str:
    import hashlib
    return hashlib.sha256(np.asarray(values, dtype=dtype).tobytes()).hexdigest()


def dequantize_reference(x, zp, scale, half):
    """DequantizeTests.cs:57-68: (float)unchecked(x - zp) * scale, then (Half) for half outputs."""
    want = np.float32(wrap32(x - zp)) * np.float32(scale)
    return np.float16(want).view(np.uint16).item() if half else np.float32(want).view(np.uint32).item()


def quantize_reference(x: float, scale: float, zp: int, lo: int, hi: int) -> int:
    """DequantizeTests.QuantizeOne (DequantizeTests.cs:138-148)."""
    with np.errstate(all="ignore"):
        v = np.float32(np.rint(np.float32(x) / np.float32(scale))) + np.float32(zp)
    if np.isnan(v):
        return lo
    return lo if v < lo else hi if v > hi else int(v)


def cs_call_args(text: str) -> tuple[list[int], dict]:
    pos, named = [], {}
    for tok in text.split(","):
        tok = tok.strip()
        if ":" in tok:
            k, v = tok.split(":")
            named[k.strip()] = int(v)
        elif tok:
            pos.append(int(tok))
    return pos, named


def conv_p(pos, named) -> dict:
    """ConvIntegerTests.P (ConvIntegerTests.cs:191-203)."""
    batch, cin, h, w, cout, kh, kw = pos
    st, dl, pad = named.get("stride", 1), named.get("dilation", 1), named.get("pad", 0)
    return dict(batch=batch, cin=cin, h=h, w=w, cout=cout, kh=kh, kw=kw, stride_h=st, stride_w=st, dilation_h=dl,
                dilation_w=dl, pad_top=pad, pad_left=pad, pad_bottom=pad, pad_right=pad, groups=named.get("groups", 1),
                offset_x=0, offset_w=0, offset_y=0)


def conv_1d(pos, named) -> dict:
    """ConvProblem.Conv1D: height 1."""
    batch, cin, length, cout, kernel = pos
    return dict(batch=batch, cin=cin, h=1, w=length, cout=cout, kh=1, kw=kernel, stride_h=1,
                stride_w=named.get("stride", 1), dilation_h=1, dilation_w=named.get("dilation", 1), pad_top=0,
                pad_left=named.get("padBegin", 0), pad_bottom=0, pad_right=named.get("padEnd", 0),
                groups=named.get("groups", 1), offset_x=0, offset_w=0, offset_y=0)


CS_PROPS = {"PadTop": "pad_top", "PadBottom": "pad_bottom", "PadLeft": "pad_left", "PadRight": "pad_right",
            "StrideHeight": "stride_h", "StrideWidth": "stride_w", "OffsetX": "offset_x", "OffsetW": "offset_w",
            "OffsetY": "offset_y"}


def conv_extent(inp, k, s, d, pb, pe) -> int:
    span = inp + pb + pe - (d * (k - 1) + 1)
    return 0 if span < 0 else span // s + 1


def conv_reference(p, x, xs, w, ws, xz, wz, wz_vec) -> list[int]:
    """ConvIntegerTests.Reference (ConvIntegerTests.cs:41-88), pure Python."""
    oh = conv_extent(p["h"], p["kh"], p["stride_h"], p["dilation_h"], p["pad_top"], p["pad_bottom"])
    ow = conv_extent(p["w"], p["kw"], p["stride_w"], p["dilation_w"], p["pad_left"], p["pad_right"])
    cin_g, cout_g = p["cin"] // p["groups"], p["cout"] // p["groups"]
    xzv = 0 if xz is None else val(xz[0], xs)
    y = []
    for n in range(p["batch"]):
        for m in range(p["cout"]):
            g = m // cout_g
            wzv = 0 if wz is None else val(wz[m if wz_vec else 0], ws)
            for i in range(oh):
                for j in range(ow):
                    acc = 0
                    for c in range(cin_g):
                        for kh in range(p["kh"]):
                            ih = i * p["stride_h"] + kh * p["dilation_h"] - p["pad_top"]
                            if not 0 <= ih < p["h"]:
                                continue
                            for kw in range(p["kw"]):
                                iw = j * p["stride_w"] + kw * p["dilation_w"] - p["pad_left"]
                                if not 0 <= iw < p["w"]:
                                    continue
                                xi = p["offset_x"] + (((n * p["cin"] + g * cin_g + c) * p["h"] + ih) * p["w"] + iw)
                                wi = p["offset_w"] + (((m * cin_g + c) * p["kh"] + kh) * p["kw"] + kw)
                                acc += (val(x[xi], xs) - xzv) * (val(w[wi], ws) - wzv)
                    y.append(wrap32(acc))
    return y


def problem(m, n, k, batch=1, trans_b=False, off_a=0, off_b=0, off_c=0, lda_extra=0, ldb_extra=0, share_b=False):
    """Int8Tests.Problem (Int8Tests.cs:198-212)."""
    lda = k + lda_extra
    ldb = (k if trans_b else n) + ldb_extra
    stride_a = m * lda
    stride_b = 0 if share_b else (n if trans_b else k) * ldb
    if batch == 1:
        stride_a = stride_b = 0
    return dict(m=m, n=n, k=k, batch=batch, transpose_b=trans_b, lda=lda, ldb=ldb, offset_a=off_a, offset_b=off_b,
                offset_c=off_c, stride_a=stride_a, stride_b=stride_b)


def run_int32_case(case: dict, seed: int) -> dict:
    """The data of Int8Tests.RunInt32 (Int8Tests.cs:116-134) and its expected sums."""
    p = case["problem"]
    lda = p["lda"] or p["k"]
    ldb = p["ldb"] or (p["k"] if p["transpose_b"] else p["n"])
    len_a = p["offset_a"] + (p["batch"] - 1) * p["stride_a"] + p["m"] * lda + 4
    len_b = p["offset_b"] + (p["batch"] - 1) * p["stride_b"] + (p["n"] if p["transpose_b"] else p["k"]) * ldb + 4
    a = lcg_bytes(len_a, seed)
    b = lcg_bytes(len_b, seed + 1)
    za = None if case["za_mode"] == 0 else lcg_bytes(1 + (p["m"] if case["za_mode"] == 2 else 0), seed + 2)
    zb = None if case["zb_mode"] == 0 else lcg_bytes(1 + (p["n"] if case["zb_mode"] == 2 else 0), seed + 3)
    fill = case.get("fill", -1)
    if fill >= 0:
        a = [fill] * len(a)
        b = [fill ^ 0xFF] * len(b)
        za = None if za is None else [fill] * len(za)
        zb = None if zb is None else [fill ^ 0x80] * len(zb)
    want = gemm_reference(p, a, case["a_signed"], b, case["b_signed"], za, case["za_mode"] == 2, zb,
                          case["zb_mode"] == 2)
    return dict(case, seed=seed, expected=want)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="root of the reference repository")
    ap.add_argument("--out", default=os.path.join(os.path.dirname(os.path.abspath(__file__)),
                                                  "reference_cases.json"))
    args = ap.parse_args()
    ref = args.reference
    t8 = read(ref, f"{REF_TESTS}/Int8Tests.cs")
    out: dict = {"source": "recursive-ai-oss/onegpu-csharp test sources, read as text", "tables": {}}
    tables = out["tables"]

    ln, line = find(t8, r"\(int M, int N, int K\)\[\] shapes = \[")
    tables["edge_shapes"] = {"cite": f"{REF_TESTS}/Int8Tests.cs:{ln}",
                             "shapes": [tuple(int(v) for v in t) for t in tuples(line, 3)]}
    ln0, _ = find(t8, r"static readonly \(string Name, int M, int N, int K\)\[\] ModelShapes")
    model = []
    for i in range(ln0, ln0 + 14):
        m = re.search(r'\("([^"]+)",\s*(\d+),\s*(\d+),\s*(\d+)\)', t8[i])
        if m:
            model.append((m.group(1), int(m.group(2)), int(m.group(3)), int(m.group(4))))
    tables["model_shapes"] = {"cite": f"{REF_TESTS}/Int8Tests.cs:{ln0}", "shapes": model}
    ln, line = find(t8, r"foreach \(var \(m, n, k\) in new\[\] \{ \(33, 35, 4096\)")
    tables["long_extreme_shapes"] = {"cite": f"{REF_TESTS}/Int8Tests.cs:{ln}",
                                     "shapes": [tuple(int(v) for v in t) for t in tuples(line, 3)]}
    ln, line = find(t8, r"foreach \(var \(m, n, k\) in new\[\] \{ \(1, 1, 1\), \(5, 7, 9\)")
    tables["float_requant_shapes"] = {"cite": f"{REF_TESTS}/Int8Tests.cs:{ln}",
                                      "shapes": [tuple(int(v) for v in t) for t in tuples(line, 3)]}
    ln, line = find(t8, r"foreach \(var \(unsigned, zero\) in new\[\]")
    tables["requant_output_modes"] = {"cite": f"{REF_TESTS}/Int8Tests.cs:{ln}",
                                      "modes": [(cs_bool(u), int(z)) for u, z in tuples(line, 2)]}
    ln, line = find(t8, r"foreach \(var \(mult, zeroY, unsigned\) in new\[\]")
    ties = [(cs_float(mv), int(z), cs_bool(u)) for mv, z, u in tuples(line, 3)]
    tie_cases = []
    for mult, zero, unsigned in ties:
        for av in range(-9, 10):
            tie_cases.append(dict(a=av, mult=mult, zero=zero, unsigned=unsigned,
                                  expected=requant(av, mult, zero, unsigned) & 0xFF))
    tables["requant_ties"] = {"cite": f"{REF_TESTS}/Int8Tests.cs:{ln}", "table": ties, "cases": tie_cases}
    ln, line = find(t8, r"var counts = new\[\] \{")
    body = line[line.index("{") + 1: line.rindex("}")]
    counts = [int(eval(tok, {"__builtins__": {}})) for tok in body.split(",")]  # integer arithmetic like 128 * 384
    tables["dq_counts"] = {"cite": f"{REF_TESTS}/Int8Tests.cs:{ln}", "counts": counts, "kinds": list(range(7))}

    # Literal known answer: MultiDeviceTests.cs.
    md = read(ref, f"{REF_TESTS}/MultiDeviceTests.cs")
    ln_a, la = find(md, r"CreateBuffer<byte>\(\[")
    ln_b, lb = find(md, r"CreateBuffer<sbyte>\(\[")
    ln_w, lw = find(md, r"Assert\.Equal\(new\[\] \{")
    nums = lambda s: [int(v) for v in re.findall(r"-?\d+", s[s.index("["):] if "[" in s else s)]
    a = nums(la[la.index("<byte>(["):])[:6]
    b = nums(lb[lb.index("<sbyte>(["):])[:6]
    want = [int(v) for v in re.findall(r"-?\d+", lw[lw.index("{"):lw.index("}")])]
    out["kat_multidevice"] = {"cite": f"{REF_TESTS}/MultiDeviceTests.cs:{ln_a},{ln_b},{ln_w}",
                              "m": 2, "n": 3, "k": 2, "a_u8": a, "b_s8": b, "expected": want,
                              "restated": gemm_reference(problem(2, 3, 2), a, False, [v & 0xFF for v in b], True,
                                                         None, False, None, False)}

    # AOT smoke int8 case: KernelSmoke.cs:199-235.
    M, N, K = 5, 6, 7
    sa = [(i * 29) % 251 for i in range(M * K)]
    sb = [((i * 13 % 255) - 127) & 0xFF for i in range(K * N)]
    out["smoke_gemm"] = {"cite": "tests/RecursiveAI.OneGpu.AotSmoke/KernelSmoke.cs:199-216", "m": M, "n": N, "k": K,
                         "za": 17, "a_u8": sa, "b_s8_bytes": sb,
                         "expected": gemm_reference(problem(M, N, K), sa, False, sb, True, [17], False, None, False)}
    q = [float(np.float32(np.float32((i * 37) % 101 - 40) / np.float32(9))) for i in range(300)]
    y, s, z = dynamic_reference(q)
    out["smoke_dq"] = {"cite": "tests/RecursiveAI.OneGpu.AotSmoke/KernelSmoke.cs:218-236", "x": q, "expected_y": y,
                       "expected_scale": s, "expected_zero_point": z}

    # Small EdgeShapesAreBitExact cases (the reference's own generator, seeds and offsets), expected by the
    # pure-Python restatement.
    cases = []
    seed = 1
    for (m, n, k) in tables["edge_shapes"]["shapes"]:
        for s_ in range(4):
            for za_mode in range(3):
                zb_mode = (za_mode + s_) % 3
                c = dict(name=f"{m}x{n}x{k}", problem=problem(m, n, k, off_a=za_mode, off_b=1 + zb_mode, off_c=s_),
                         a_signed=bool(s_ & 1), b_signed=bool(s_ & 2), za_mode=za_mode, zb_mode=zb_mode)
                if m * n * k <= 4096:
                    cases.append(run_int32_case(c, seed))
                seed += 1
    out["edge_cases_small"] = {"cite": f"{REF_TESTS}/Int8Tests.cs:214-232", "cases": cases}

    # DequantizeTests: the case table, offsets and scale sets, and restated results of small cases.
    dq = read(ref, f"{REF_TESTS}/DequantizeTests.cs")
    ln_off, loff = find(dq, r"const int OffX = ")
    offsets = {k: int(v) for k, v in re.findall(r"(Off\w)\s*=\s*(\d+)", loff)}
    ln_c, _ = find(dq, r"\(int\[\] Shape, int Axis, bool PerAxis\)\[\] cases =")
    body = " ".join(dq[ln_c - 1: ln_c + 4])
    qcases = [([int(v) for v in sh.split(",")], int(ax), cs_bool(pa))
              for sh, ax, pa in re.findall(r"\(\[([\d,\s]+)\],\s*(-?\d+),\s*(true|false)\)", body)]
    ln_s, ls = find(dq, r"float\[\]\[\] scaleSets = ")
    sets = []
    for grp in re.findall(r"\[([^\[\]]+)\]", ls[ls.index("= [") + 2:]):
        vals = []
        for tok in grp.split(","):
            tok = tok.strip()
            if "/" in tok:
                num, den = tok.split("/")
                vals.append(float(np.float32(cs_float(num)) / np.float32(cs_float(den))))
            else:
                vals.append(cs_float(tok))
        sets.append(vals)
    dq_expect = []
    for kind, seed0 in (("u8", 1), ("s8", 100), ("i32", 200)):
        seed = seed0
        for shape_, axis, per_axis in qcases:
            for with_zero in (True, False):
                for half in (False, True):
                    n = int(np.prod(shape_))
                    if n <= 64:
                        ax = axis + len(shape_) if axis < 0 else axis
                        axis_len = shape_[ax] if per_axis else 1
                        inner = int(np.prod(shape_[ax + 1:])) if per_axis and ax + 1 < len(shape_) else 1
                        x = quantized(kind, n + offsets["OffX"], seed)
                        sc = rig_random(axis_len + offsets["OffS"], seed + 1, 0.001, 2.0)
                        zs = quantized(kind, axis_len + offsets["OffZ"], seed + 2)
                        out_vals = []
                        for j in range(n):
                            a = (j // inner) % axis_len if per_axis else 0
                            zp = zs[offsets["OffZ"] + a] if with_zero else 0
                            out_vals.append(dequantize_reference(x[offsets["OffX"] + j], zp, sc[offsets["OffS"] + a],
                                                                 half))
                        dq_expect.append(dict(kind=kind, shape=shape_, axis=axis, per_axis=per_axis,
                                              with_zero=with_zero, half=half, seed=seed,
                                              sha256=digest(out_vals, np.uint16 if half else np.uint32)))
                    seed += 1
    q_expect = []
    count = 0
    seed = 1
    for shape_, axis, per_axis in qcases:
        for with_zero in (True, False):
            scales = sets[count % len(sets)]
            for signed, half_in in ((False, False), (True, False), (False, True), (True, True)):
                n = int(np.prod(shape_))
                if n <= 64:
                    ax = axis + len(shape_) if axis < 0 else axis
                    axis_len = shape_[ax] if per_axis else 1
                    inner = int(np.prod(shape_[ax + 1:])) if per_axis and ax + 1 < len(shape_) else 1
                    x = quantize_input(n + offsets["OffX"], seed)
                    if half_in:
                        x = [float(np.float32(np.float16(np.float32(v)))) for v in x]
                    sc = [scales[i % len(scales)] for i in range(axis_len + offsets["OffS"])]
                    zs = quantized("s8" if signed else "u8", axis_len + offsets["OffZ"], seed + 2)
                    lo, hi = (-128, 127) if signed else (0, 255)
                    out_vals = []
                    for j in range(n):
                        a = (j // inner) % axis_len if per_axis else 0
                        zp = zs[offsets["OffZ"] + a] if with_zero else 0
                        out_vals.append(quantize_reference(x[offsets["OffX"] + j], sc[offsets["OffS"] + a], zp, lo, hi)
                                        & 0xFF)
                    q_expect.append(dict(signed=signed, half_in=half_in, shape=shape_, axis=axis, per_axis=per_axis,
                                         with_zero=with_zero, scales=scales, seed=seed,
                                         sha256=digest(out_vals, np.uint8)))
                seed += 1
            count += 4
    out["dequantize"] = {"cite": f"{REF_TESTS}/DequantizeTests.cs:{ln_off},{ln_c},{ln_s}", "offsets": offsets,
                         "cases": qcases, "scale_sets": sets, "dequantize_small": dq_expect,
                         "quantize_small": q_expect}

    # ConvIntegerTests: the geometries of EdgeGeometriesAreBitExact / WhisperStemIsBitExact / ResNetShapesAreBitExact.
    cv = read(ref, f"{REF_TESTS}/ConvIntegerTests.cs")
    spreads, named_p = [], {}
    for i, line in enumerate(cv):
        m = re.search(r'var (\w+) = P\(([^)]*)\);', line)
        if m:
            named_p[m.group(1)] = conv_p(*cs_call_args(m.group(2)))
        m = re.search(r'^\s*(\w+)\.(\w+) = (-?\d+);', line)
        if m and m.group(1) in named_p:
            named_p[m.group(1)][CS_PROPS[m.group(2)]] = int(m.group(3))
        m = re.search(r'Spread\("([^"]+)",\s*(P|ConvProblem\.Conv1D)\(([^)]*)\)\)', line)
        if m:
            maker = conv_p if m.group(2) == "P" else conv_1d
            spreads.append(dict(name=m.group(1), p=maker(*cs_call_args(m.group(3))), line=i + 1))
            continue
        m = re.search(r'Spread\("([^"]+)",\s*(\w+)\)\)', line)
        if m and m.group(2) in named_p:
            spreads.append(dict(name=m.group(1), p=dict(named_p[m.group(2)]), line=i + 1))
    singles = []
    for i, line in enumerate(cv):
        m = re.search(r'Name = (\$?)"([^"]+)", P = (P|ConvProblem\.Conv1D)\(([^)]*)\)(.*)\}', line)
        if not m:
            continue
        maker = conv_p if m.group(3) == "P" else conv_1d
        props = {k: (v == "true" if v in ("true", "false") else v) for k, v in
                 re.findall(r"(\w+) = (true|false|\d+|fill|\(s & \d\) != 0)", m.group(5))}
        singles.append(dict(name=m.group(2), templated=bool(m.group(1)), p=maker(*cs_call_args(m.group(4))),
                            props=props, line=i + 1))
    ln_f, lf = find(cv, r"foreach \(var fill in new\[\] \{")
    fills = [int(v) for v in re.findall(r"\d+", lf[lf.index("{"):])]
    conv_expect = []
    seed = 100
    for sp in spreads:
        for s_ in range(4):
            c = dict(name=f"{sp['name']} s{s_}", p=sp["p"], x_signed=bool(s_ & 1), w_signed=bool(s_ & 2),
                     xz_mode=1 - (s_ & 1), wz_mode=(s_ + 1) % 3, seed=seed)
            p_ = c["p"]
            oh = conv_extent(p_["h"], p_["kh"], p_["stride_h"], p_["dilation_h"], p_["pad_top"], p_["pad_bottom"])
            ow = conv_extent(p_["w"], p_["kw"], p_["stride_w"], p_["dilation_w"], p_["pad_left"], p_["pad_right"])
            macs = p_["batch"] * p_["cout"] * oh * ow * (p_["cin"] // p_["groups"]) * p_["kh"] * p_["kw"]
            if macs <= 60000:
                x_len = p_["offset_x"] + p_["batch"] * p_["cin"] * p_["h"] * p_["w"] + 4
                w_len = p_["offset_w"] + p_["cout"] * (p_["cin"] // p_["groups"]) * p_["kh"] * p_["kw"] + 4
                x = lcg_bytes(x_len, seed)
                w = lcg_bytes(w_len, seed + 1)
                xz = None if c["xz_mode"] == 0 else lcg_bytes(1, seed + 2)
                wz = None if c["wz_mode"] == 0 else lcg_bytes(p_["cout"] if c["wz_mode"] == 2 else 1, seed + 3)
                y = conv_reference(p_, x, c["x_signed"], w, c["w_signed"], xz, wz, c["wz_mode"] == 2)
                c["sha256"] = digest(y, np.int32)
                conv_expect.append(c)
            seed += 1
    out["conv_integer"] = {"cite": f"{REF_TESTS}/ConvIntegerTests.cs:{spreads[0]['line']}-{singles[-1]['line']}",
                           "spreads": spreads, "singles": singles, "fills": fills, "spread_small": conv_expect}

    with open(args.out, "w", encoding="utf-8") as f:
        json.dump(out, f, separators=(",", ":"))
    print(f"wrote {args.out}: {len(cases)} edge cases, {len(tie_cases)} tie cases, {len(dq_expect)} dequantize, "
          f"{len(q_expect)} quantize, {len(conv_expect)} conv cases restated; {len(spreads)} spreads, "
          f"{len(singles)} single conv cases")


if __name__ == "__main__":
    main()
