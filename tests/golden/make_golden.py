"""Generates tests/golden/reference_cases.json from the reference repository's own test files.

Run in a container where the reference is mounted (default /root/reference); the GPU box never runs this script, the
tests only read the JSON it wrote.

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
    ap.add_argument("--reference", default="/root/reference")
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

    with open(args.out, "w", encoding="utf-8") as f:
        json.dump(out, f, separators=(",", ":"))
    print(f"wrote {args.out}: {len(cases)} edge cases, {len(tie_cases)} tie cases")


if __name__ == "__main__":
    main()
